"""The KV cache the B200 append writes, compared byte for byte with the cache modelcore itself
writes, at measurement config 2's size, on the GPU.

modelcore's bf16 model (the README quickstart architecture with modelcore's test wake-up, so
every layer's k and v are non-trivial) runs its own forward -- its projections, its rope
(modelcore/components/rotary.py:43-81), its QK-norm through torch's CUDA F.rms_norm
(components/norm.py:43-44), x1.2 (attention.py:147-150) and its SDPA insert
(kernels/flash_attn.py:337-346) -- into its own KVCache over 64 prompts of 512 tokens (one
batched prefill), then 32 greedy decode steps.  Every call of flash_attn_with_kvcache is
intercepted: the raw c_q / c_k / c_v outputs of that layer (forward hooks) go through the B200
append (mcb_kv_append_rope, with the rotary module's own tables and the same cache_seqlens) into
a shadow cache of the same shape, and the rotated q is kept beside modelcore's.

Checked: values bit-exact; keys and queries bit-exact except where the fp32 sum of squares inside
the norm, summed in torch's CUDA reduction order, puts the normed value on the other side of a bf16
rounding boundary: one ulp there, which the x1.2 that follows can round to two; the count of such
elements is printed and bounded (measured on B200: 3.9e-6 of 321M key elements, at most 2 ulp).
"""
import numpy as np
import pytest
import torch

from conftest import have_modelcore

pytestmark = pytest.mark.gpu

ROWS, PROMPT, STEPS, TMAX = 64, 512, 32, 1024
MAX_ULP_RATE = 2e-5  # measured: 3.9e-6 against torch's CUDA order, 6e-6 against its CPU order


def _ulp_diff(a, b):
    """|a - b| in bf16 units in the last place (bit patterns as ordered integers)."""
    def ordered(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)
    return (ordered(a) - ordered(b)).abs()


def test_config2_cache_bytes_equal_modelcores_after_prefill_and_32_steps():
    if not have_modelcore():
        raise RuntimeError("modelcore (the reference package) is not importable: install it into "
                           "baseline/_ref (__graft_entry__.build() does)")
    import modelcore
    from modelcore.kernels.flash_attn import flash_attn as fa_ns
    from modelcore_b200 import ops, workloads

    mgr = modelcore.ModelManager()
    assert mgr.runtime.compute_dtype == torch.bfloat16
    model = mgr.create_model(workloads.quickstart_config(), device=torch.device("cpu"), seed=0)
    workloads.awaken(model)
    model = model.to("cuda").eval()
    blocks = model.body.blocks
    H, D = blocks[0].mixer.n_kv_head, blocks[0].mixer.head_dim
    cache = mgr.new_kv_cache(model, batch_size=ROWS, seq_len=TMAX)
    assert type(cache).__module__.startswith("modelcore.")  # modelcore's own KVCache
    shadow_k, shadow_v = torch.zeros_like(cache.k_cache), torch.zeros_like(cache.v_cache)
    slot_bytes = cache.k_cache[0].nbytes
    rope = blocks[0].mixer.rope
    cos = rope.cos.reshape(-1, D // 2).contiguous()
    sin = rope.sin.reshape(-1, D // 2).contiguous()
    assert cos.dtype == torch.bfloat16

    raw = {}
    hooks = []
    for blk in blocks:
        for name in ("c_q", "c_k", "c_v"):
            mod = getattr(blk.mixer, name)
            hooks.append(mod.register_forward_hook(
                lambda m, i, o, name=name: raw.__setitem__(name, o)))
    stats = {"q_elems": 0, "q_diff": 0, "q_max_ulp": 0, "calls": 0}
    orig = fa_ns.flash_attn_with_kvcache

    def intercept(q, k_cache, v_cache, k=None, v=None, cache_seqlens=None, causal=False,
                  window_size=(-1, -1)):
        B, T, Hq, _ = q.shape
        slot = (k_cache.data_ptr() - cache.k_cache.data_ptr()) // slot_bytes
        rq = raw["c_q"].view(B, T, Hq, D)
        rk, rv = raw["c_k"].view(B, T, H, D), raw["c_v"].view(B, T, H, D)
        q_mine = ops.kv_append_rope(rq, rk, rv, shadow_k[slot], shadow_v[slot], cache_seqlens,
                                    cos, sin)
        d = _ulp_diff(q_mine, q)
        stats["q_elems"] += d.numel()
        stats["q_diff"] += int((d != 0).sum())
        stats["q_max_ulp"] = max(stats["q_max_ulp"], int(d.max()))
        stats["calls"] += 1
        return orig(q, k_cache, v_cache, k=k, v=v, cache_seqlens=cache_seqlens, causal=causal,
                    window_size=window_size)

    fa_ns.flash_attn_with_kvcache = intercept
    try:
        with torch.inference_mode():
            ids = workloads.prompts(ROWS, PROMPT, seed=1).cuda()
            logits = model.forward(ids, kv_cache=cache)[:, -1]
            for _ in range(STEPS):
                nxt = logits.float().argmax(-1, keepdim=True)
                logits = model.forward(nxt, kv_cache=cache)[:, -1]
        torch.cuda.synchronize()
    finally:
        fa_ns.flash_attn_with_kvcache = orig
        for h in hooks:
            h.remove()
    assert stats["calls"] == len(blocks) * (1 + STEPS)
    assert ops.device_error()[0] == 0
    assert cache.cache_seqlens.tolist() == [PROMPT + STEPS] * ROWS
    filled = PROMPT + STEPS
    assert torch.equal(shadow_v[:, :, :filled], cache.v_cache[:, :, :filled])
    dk = _ulp_diff(shadow_k[:, :, :filled], cache.k_cache[:, :, :filled])
    k_diff, k_elems = int((dk != 0).sum()), dk.numel()
    per_slot = [int((dk[s] != 0).sum()) for s in range(dk.shape[0])]
    print(f"config-2 replay: {k_elems:,} key elements, {k_diff} differ from modelcore's cache "
          f"(rate {k_diff / k_elems:.2e}, max {int(dk.max())} ulp; per slot {per_slot}); "
          f"{stats['q_elems']:,} query elements, {stats['q_diff']} differ "
          f"(rate {stats['q_diff'] / stats['q_elems']:.2e}, max {stats['q_max_ulp']} ulp); "
          f"values bit-exact")
    assert int(dk.max()) <= 2 and stats["q_max_ulp"] <= 2
    assert k_diff / k_elems <= MAX_ULP_RATE
    assert stats["q_diff"] / stats["q_elems"] <= MAX_ULP_RATE
    np.testing.assert_equal(cache.k_cache[:, :, filled:].abs().sum().item(), 0.0)
