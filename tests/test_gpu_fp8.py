"""GPU parity of the fp8 (e4m3) KV-cache format (ops.kv_append_rope / ops.decode_attn with a
float8_e4m3fn slot and per-vector scales).

The reference stores its cache in the compute dtype, so there is no reference fp8 to match; the
format is pinned to the CPU oracle instead:
  * the append: every stored byte and scale equals oracle.quantize_fp8 of the bf16 vector the
    bf16 cache gets from the same inputs (bit-exact), and q is unchanged;
  * the attention: within max-abs 2e-2 of a float64 attention over the dequantized cache
    (e4m3 value x scale) -- the same bar as the bf16 kernels against their oracle -- for the
    cluster, workspace and multi-token plans, windows and ring slots;
  * against the bf16 cache the output moves by the quantization only (checked loosely).
"""
import numpy as np
import pytest
import torch

from oracle import kv_path as O

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def tables(rot_len, D):
    ang = torch.arange(rot_len, dtype=torch.float32)[:, None] * \
        (100000.0 ** (-torch.arange(0, D, 2, dtype=torch.float32) / D))[None]
    return ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()


def rand_bf16(g, *shape, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("B,T,Hq,Hkv,D,ring", [(4, 1, 8, 2, 128, False), (3, 5, 12, 12, 64, False),
                                               (2, 3, 32, 8, 128, True), (1, 1, 4, 4, 64, True)])
def test_fp8_append_matches_the_oracle_quantization(ops, B, T, Hq, Hkv, D, ring):
    g = torch.Generator(device="cuda").manual_seed(B * 100 + T * 10 + D)
    Tmax = 256
    q = rand_bf16(g, B, T, Hq, D, scale=2.0)
    k = rand_bf16(g, B, T, Hkv, D, scale=2.0)
    v = rand_bf16(g, B, T, Hkv, D, scale=3.0)
    v[0, 0, 0] = 0.0                                   # an all-zero vector: zeros, scale 0
    cos, sin = tables(1024, D)
    hi = 700 if ring else Tmax - T
    sl = torch.randint(0, hi + 1, (B,), device="cuda", generator=g, dtype=torch.int32)
    kc16 = torch.zeros(B, Tmax, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vc16 = torch.zeros_like(kc16)
    q16 = ops.kv_append_rope(q, k, v, kc16, vc16, sl, cos, sin, ring=ring)
    kc8 = torch.zeros(B, Tmax, Hkv, D, device="cuda", dtype=ops.FP8)
    vc8 = torch.zeros_like(kc8)
    ks, vs = ops.fp8_scales(B, Hkv, Tmax, "cuda"), ops.fp8_scales(B, Hkv, Tmax, "cuda")
    q8 = ops.kv_append_rope(q, k, v, kc8, vc8, sl, cos, sin, ring=ring, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(q8, q16)
    k8, v8 = kc8.view(torch.uint8).cpu().numpy(), vc8.view(torch.uint8).cpu().numpy()
    ksn, vsn = ks.cpu().numpy(), vs.cpu().numpy()
    written = np.zeros((B, Tmax), dtype=bool)
    for b in range(B):
        for t in range(T):
            p = int(sl[b]) + t
            idx = p % Tmax if ring else p
            written[b, idx] = True
            for cache16, c8, sc in ((kc16, k8, ksn), (vc16, v8, vsn)):
                want_b, want_s = O.quantize_fp8(bits(cache16[b, idx]))
                assert np.array_equal(c8[b, idx], want_b)
                assert np.array_equal(sc[b, :, idx], want_s)
    assert not k8[~written].any() and not v8[~written].any()
    assert ksn[:, :, :Tmax].transpose(0, 2, 1)[~written].sum() == 0
    if not ring:
        assert ksn[0, 0, int(sl[0])] > 0 and vsn[0, 0, int(sl[0])] == 0   # the zero vector


def fp8_cache(g, B, Tmax, Hkv, D, scale=1.0):
    """A random bf16 cache and its oracle quantization uploaded as an fp8 slot + scales."""
    c16 = rand_bf16(g, B, Tmax, Hkv, D, scale=scale)
    b8, s = O.quantize_fp8(bits(c16))                  # (B, Tmax, Hkv, D), (B, Tmax, Hkv)
    c8 = torch.from_numpy(b8).cuda().view(torch.float8_e4m3fn)
    sc = torch.zeros(B, Hkv, (Tmax + 63) // 64 * 64, dtype=torch.float32)
    sc[:, :, :Tmax] = torch.from_numpy(s).permute(0, 2, 1)
    return c16, c8, sc.cuda(), O.dequantize_fp8(b8, s)


CASES = [  # B, T, Hq, Hkv, D, Tmax, max_len, window, ring, num_ctas
    (4, 1, 8, 2, 128, 1024, 1000, -1, False, 0),       # short rows: split, one wave
    (2, 1, 32, 8, 128, 8192, 8000, -1, False, 0),      # long rows of few groups: cluster of 16
    (2, 1, 32, 8, 128, 8192, 8000, 1000, False, -20),  # 18 splits: partials, last split merges
    (3, 4, 12, 12, 64, 512, 500, 100, False, 0),       # D 64, several tokens, a window
    (1, 70, 8, 2, 128, 512, 400, -1, False, 0),        # a 70-token chunk (no fp8 tcgen05 path)
    (3, 2, 16, 4, 128, 384, 1500, 200, True, 0),       # ring slot: positions beyond T_max
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}Hq{}Hkv{}D{}w{}r{}n{}".format(
    c[0], c[1], c[2], c[3], c[4], c[7], int(c[8]), c[9]))
def test_fp8_attention_matches_the_dequantized_reference(ops, case):
    B, T, Hq, Hkv, D, Tmax, max_len, window, ring, nc = case
    g = torch.Generator(device="cuda").manual_seed(sum(case[:7]))
    kc16, kc8, ks, kdq = fp8_cache(g, B, Tmax, Hkv, D)
    vc16, vc8, vs, vdq = fp8_cache(g, B, Tmax, Hkv, D, scale=2.0)
    lens = torch.randint(max(0, max_len // 2), max_len - T + 1, (B,), generator=torch.Generator().manual_seed(B))
    sl = lens.to(torch.int32).cuda()
    q = rand_bf16(g, B, T, Hq, D)
    out = ops.decode_attn(q, kc8, vc8, sl, window=window, ring=ring, num_ctas=nc, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    qf = q.float().cpu().numpy().astype(np.float64)
    if ring:  # unroll the ring into absolute positions for the oracle
        P = int(lens.max()) + T
        idx = np.arange(P) % Tmax
        kdq, vdq = kdq[:, idx], vdq[:, idx]
        kc16 = kc16[:, torch.from_numpy(idx).cuda()]
        vc16 = vc16[:, torch.from_numpy(idx).cuda()]
    ref = O.decode_attention(qf, kdq, vdq, lens.numpy(), window=window)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= TOL, err
    # against the bf16 cache the quantization moves the output, but not far
    o16 = O.decode_attention(qf, kc16.float().cpu().numpy(), vc16.float().cpu().numpy(), lens.numpy(),
                             window=window)
    assert np.abs(out.float().cpu().numpy() - o16).max() < 0.25


def test_fp8_rejects_what_it_does_not_cover(ops):
    from modelcore_b200._native import McbError
    B, Tmax, Hkv, D = 2, 128, 2, 32
    kc8 = torch.zeros(B, Tmax, Hkv, D, device="cuda", dtype=ops.FP8)
    ks = ops.fp8_scales(B, Hkv, Tmax, "cuda")
    q = torch.zeros(B, 1, 4, D, device="cuda", dtype=torch.bfloat16)
    sl = torch.zeros(B, dtype=torch.int32, device="cuda")
    with pytest.raises(McbError, match="64 or 128"):
        ops.decode_attn(q, kc8, kc8, sl, k_scale=ks, v_scale=ks)
    kc8 = torch.zeros(B, Tmax, Hkv, 64, device="cuda", dtype=ops.FP8)
    ks = ops.fp8_scales(B, Hkv, Tmax, "cuda")
    q = torch.zeros(B, 1, 4, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(McbError, match="split plan"):
        ops.decode_attn(q, kc8, kc8, sl, k_scale=ks, v_scale=ks, num_ctas=148)
    with pytest.raises(RuntimeError, match="needs"):
        ops.decode_attn(q, kc8, kc8, sl)


def test_fp8_cache_through_the_model_manager():
    """modelcore's Decoder and the CUDA-graph decoder over an fp8 cache (ModelManager.kv_format):
    the prefill (per-prompt and batched), the prefill_row copies (bytes and scales) and the
    decode steps run on the fp8 kernels; the logits stay within the quantization's reach of the
    bf16 cache's, and the graph decoder reproduces the eager fp8 decoder bit for bit."""
    from conftest import have_modelcore
    if not have_modelcore():
        raise RuntimeError("modelcore (the reference package) is not importable")
    import modelcore_b200 as mcb
    from modelcore_b200 import workloads
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    prompts = workloads.prompts(3, 40, seed=1).tolist()
    prompts[1] = prompts[1][:17]
    cols = [[(s * 5 + i) % 1000 for i in range(3)] for s in range(6)]
    with torch.inference_mode():
        d16 = mgr.new_decoder(model, prompts, max_tokens=16)
        mgr.kv_format = "fp8"
        try:
            d8 = mgr.new_decoder(model, prompts, max_tokens=16)
            g8 = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        finally:
            mgr.kv_format = "bf16"
        assert d8.kv_cache.kv_format == "fp8" and d8.kv_cache.k_cache.dtype == torch.float8_e4m3fn
        assert d8.kv_cache.cache_bytes() < 0.55 * d16.kv_cache.cache_bytes()
        worst = 0.0
        for step in range(len(cols) + 1):
            l16, l8, lg = d16.logits.float(), d8.logits.float(), g8.logits.float()
            worst = max(worst, (l8 - l16).abs().max().item() / l16.abs().max().item())
            assert torch.equal(lg, l8)
            if step < len(cols):
                d16.step(cols[step])
                d8.step(cols[step])
                g8.step(cols[step])
        # e4m3 keeps 3 mantissa bits: relative logit deviations of a few percent (7.9% measured
        # at the worst element over 7 steps of this 4-layer model)
        assert worst < 0.15, worst
