"""torch.ops.mcb200 without a GPU: libmcb200_torch.so loads, the operators carry the boundary's
schemas (kv_append_rope, kv_broadcast, decode_attn, the fused append_attn, kv_advance, and the
decode step's linear and add_rms_norm), and their shape functions answer on meta tensors -- what
torch.compile traces with."""
import torch


def test_the_operators_are_registered_with_their_schemas():
    import modelcore_b200.torch_ops as T
    for name in T.OPS:
        schema = str(getattr(torch.ops.mcb200, name).default._schema)
        assert schema.startswith(f"mcb200::{name}(")
    s = str(torch.ops.mcb200.append_attn.default._schema)
    assert "Tensor(a!) k_cache" in s and "Tensor(b!) v_cache" in s  # written in place
    s = str(torch.ops.mcb200.decode_attn.default._schema)
    assert "(a!)" not in s  # reads its slot only


def test_shape_functions_on_meta_tensors():
    import modelcore_b200.torch_ops  # noqa: F401
    m = dict(device="meta", dtype=torch.bfloat16)
    q = torch.empty(4, 1, 16, 128, **m)
    kc = torch.empty(4, 1024, 4, 128, **m)
    sl = torch.empty(4, device="meta", dtype=torch.int32)
    cos = torch.empty(1, 2048, 1, 64, **m)
    y = torch.ops.mcb200.decode_attn(q, kc, kc, sl, window=100)
    assert y.shape == q.shape and y.dtype == torch.bfloat16 and y.device.type == "meta"
    k = torch.empty(4, 1, 4, 128, **m)
    y = torch.ops.mcb200.append_attn(q, k, k, kc, kc, sl, cos, cos)
    assert y.shape == q.shape
    q2 = torch.ops.mcb200.kv_append_rope(q, None, None, None, None, sl, cos, cos)
    assert q2.shape == q.shape
