"""Window-ring KV slots (position p at index p % capacity) against the full-length layout:
the kernels read the same keys at the same absolute positions, so attention over a ring equals
attention over the full cache bit for bit (every plan: split, cluster-merged split, persistent,
the tensor-core prefill); the fused append writes position p at p % capacity; through
modelcore's API a model whose windowed layers keep rings decodes like the full cache (chunked
prefill: within the bf16 logits tolerance) on a fraction of the memory."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def _ring_of(lin, lens, T, cap):
    """The ring image of a full-length slot: positions [end - cap, end) of each row at p % cap."""
    B = lin.shape[0]
    ring = torch.zeros((B, cap) + tuple(lin.shape[2:]), dtype=lin.dtype, device=lin.device)
    for b in range(B):
        end = int(lens[b]) + T
        pos = torch.arange(max(0, end - cap), end, device=lin.device)
        ring[b, pos % cap] = lin[b, pos]
    return ring


CASES = [  # B, T, Hq, Hkv, D, lengths, window, cap, plans
    (3, 1, 8, 2, 128, [5, 900, 3000], 300, 512, (0, -1, -3, -12, -20, 37)),
    (2, 3, 12, 12, 64, [700, 1600], 400, 512, (0, -2, 5)),
    (2, 130, 4, 1, 128, [0, 1000], 256, 512, (0, -1)),   # T >= 64: the tensor-core prefill plan
    (64, 1, 16, 4, 128, list(range(1000, 1640, 10)), 1024, 1152, (0, 148)),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}D{}w{}cap{}".format(c[0], c[1], c[4], c[6], c[7]))
def test_attention_over_a_ring_equals_the_full_cache(ops, case):
    B, T, Hq, Hkv, D, lens, window, cap, plans = case
    Tlin = max(lens) + T
    g = torch.Generator(device="cuda").manual_seed(B * 7 + T)
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kl = torch.randn(B, Tlin, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vl = torch.randn(B, Tlin, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    kr, vr = _ring_of(kl, lens, T, cap), _ring_of(vl, lens, T, cap)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    for plan in plans:
        want = ops.decode_attn(q, kl, vl, sl, window=window, num_ctas=plan)
        got = ops.decode_attn(q, kr, vr, sl, window=window, num_ctas=plan, ring=True)
        torch.cuda.synchronize()
        assert ops.device_error()[0] == 0
        assert torch.equal(got, want), plan


def test_ring_append_writes_position_p_at_p_mod_capacity(ops):
    B, T, Hq, Hkv, D, cap = 3, 2, 4, 2, 64, 256
    lens = [0, 255, 1000]
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    cos = torch.randn(2048, D // 2, device="cuda", generator=g).to(torch.bfloat16)
    sin = torch.randn(2048, D // 2, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    kl = torch.zeros(B, 1100, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vl = torch.zeros_like(kl)
    kr = torch.zeros(B, cap, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vr = torch.zeros_like(kr)
    q1 = ops.kv_append_rope(q, k, v, kl, vl, sl, cos, sin)
    q2 = ops.kv_append_rope(q, k, v, kr, vr, sl, cos, sin, ring=True)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(q1, q2)
    for b, L in enumerate(lens):
        for t in range(T):
            assert torch.equal(kr[b, (L + t) % cap], kl[b, L + t])
            assert torch.equal(vr[b, (L + t) % cap], vl[b, L + t])


def test_ring_slots_through_modelcore_decode_like_the_full_cache():
    from conftest import have_modelcore
    if not have_modelcore():
        pytest.skip("modelcore not importable")
    import copy
    import modelcore_b200
    from modelcore_b200 import workloads
    cfg = workloads.gqa_window_config(n_layer=4, window=64, sequence_len=1024)
    base = modelcore_b200.ModelManager()
    model = workloads.awaken(base.create_model(cfg, device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    ringm = modelcore_b200.ModelManager()
    ringm.ring_window = True
    prompts = workloads.prompts(3, 800, seed=6).tolist()
    prompts[1] = prompts[1][:333]
    with torch.inference_mode():
        full = base.new_decoder(model, prompts, max_tokens=80, cuda_graph=True)
        ring = ringm.new_decoder(model, prompts, max_tokens=80, cuda_graph=True)
        kc = ring.kv_cache
        assert kc.ring_capacity == 640 and kc.step_limit == 576
        assert [kc.slot_ring(s) for s in range(4)] == [True, True, True, False]
        # K and V, 3 rows, 4 kv heads of 128, bf16: one full slot of 880 positions + 3 rings of 640
        assert kc.cache_bytes() == 2 * 2 * 3 * 4 * 128 * (880 + 3 * 640)
        assert full.kv_cache.cache_bytes() == 2 * 2 * 3 * 4 * 128 * (4 * 880)
        assert ring.kv_cache.cache_seqlens.tolist() == full.kv_cache.cache_seqlens.tolist()
        assert (ring.logits - full.logits).abs().max().item() <= LOGIT_TOL
        for s in range(70):   # rows at 800 + 70 > 640: every ring wraps
            col = [(s * 11 + r) % 700 for r in range(3)]
            a, b = ring.step(col), full.step(col)
            assert (a - b).abs().max().item() <= LOGIT_TOL, s
