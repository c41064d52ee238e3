"""GPU parity of the three kernels, called through the C ABI (modelcore_b200.ops), against the
golden vectors the reference produced and against the CPU oracle on seeded inputs.

Bars: the insert and the cache copies are bit-exact; the fused rope + rms_norm + x1.2 chain is
bit-exact against the oracle (same fp32 reduction order) and against the reference's golden
vectors; decode attention is within max-abs 2e-2 of the fp32 reference (bf16 output)."""
import math

import numpy as np
import pytest
import torch

from conftest import golden_files, load_golden
from oracle import kv_path as O

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-2  # max-abs, bf16 output vs the fp32 reference


@pytest.fixture(scope="module")
def mcb():
    import modelcore_b200
    from modelcore_b200 import ops
    return modelcore_b200, ops


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def no_device_error(ops):
    code, what = ops.device_error()
    assert code == 0, what


# ---------------------------------------------------------------------------------------------
# piece 1: append + rope + QK-norm + scale
@pytest.mark.parametrize("D", [64, 128])
def test_fused_append_matches_the_reference_golden_vectors(mcb, D):
    _, ops = mcb
    z = load_golden(f"rope_norm_D{D}.npz")
    x = dev_bf16(z["x"])                       # (B, T, H, D)
    B, T, H, _ = x.shape
    cos = dev_bf16(z["cos_table"]).view(1, -1, 1, D // 2)
    sin = dev_bf16(z["sin_table"]).view(1, -1, 1, D // 2)
    seqlens = torch.from_numpy(z["seqlens"]).to(torch.int32).cuda()
    Tmax = 128
    kc = torch.zeros(B, Tmax, H, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    v = torch.randn(B, T, H, D, device="cuda").to(torch.bfloat16)
    q_out = ops.kv_append_rope(x, x, v, kc, vc, seqlens, cos, sin)
    torch.cuda.synchronize()
    no_device_error(ops)
    assert np.array_equal(host_bits(q_out), z["out"])
    pos = O.positions(z["seqlens"], T)
    for b in range(B):
        assert np.array_equal(host_bits(kc[b, pos[b]]), z["out"][b])
        assert torch.equal(vc[b, pos[b]], v[b])
    # nothing else in the cache was touched
    mask = torch.ones(B, Tmax, dtype=torch.bool)
    for b in range(B):
        mask[b, pos[b]] = False
    assert kc[mask.cuda()].abs().sum().item() == 0


@pytest.mark.parametrize("D,Hq,Hkv,T", [(16, 4, 4, 1), (32, 4, 2, 3), (64, 12, 12, 1),
                                        (128, 32, 8, 1), (128, 16, 4, 2), (256, 4, 1, 1), (96, 6, 3, 1)])
def test_fused_append_is_bit_exact_against_the_oracle(mcb, D, Hq, Hkv, T):
    _, ops = mcb
    rng = np.random.default_rng(D * 100 + Hq + T)
    B, Tmax, rot = 5, 300, 400
    lens = rng.integers(0, Tmax - T, size=B)
    q = O.f32_to_bf16(rng.standard_normal((B, T, Hq, D)).astype(np.float32) * 3)
    k = O.f32_to_bf16(rng.standard_normal((B, T, Hkv, D)).astype(np.float32) * 3)
    v = O.f32_to_bf16(rng.standard_normal((B, T, Hkv, D)).astype(np.float32))
    cos, sin = O.rotary_tables(rot, D)
    kc = np.zeros((B, Tmax, Hkv, D), np.uint16)
    vc = np.zeros_like(kc)
    q_ref = O.append_rope(q, k, v, kc, vc, lens, cos, sin)
    dkc = torch.zeros(B, Tmax, Hkv, D, dtype=torch.bfloat16, device="cuda")
    dvc = torch.zeros_like(dkc)
    q_out = ops.kv_append_rope(dev_bf16(q), dev_bf16(k), dev_bf16(v), dkc, dvc,
                               torch.from_numpy(lens).to(torch.int32).cuda(),
                               dev_bf16(cos), dev_bf16(sin))
    torch.cuda.synchronize()
    no_device_error(ops)
    assert np.array_equal(host_bits(q_out), q_ref)
    assert np.array_equal(host_bits(dkc), kc)
    assert np.array_equal(host_bits(dvc), vc)


def test_fused_append_reads_strided_projections(mcb):
    """q/k/v arrive as views of one fused projection output (non-contiguous heads)."""
    _, ops = mcb
    B, T, Hq, Hkv, D = 3, 1, 8, 2, 128
    rng = np.random.default_rng(3)
    qkv = O.f32_to_bf16(rng.standard_normal((B, T, Hq + 2 * Hkv, D)).astype(np.float32))
    cos, sin = O.rotary_tables(64, D)
    lens = np.array([1, 7, 30])
    kc = np.zeros((B, 40, Hkv, D), np.uint16)
    vc = np.zeros_like(kc)
    q_ref = O.append_rope(qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:], kc, vc, lens,
                          cos, sin)
    d = dev_bf16(qkv)
    dkc = torch.zeros(B, 40, Hkv, D, dtype=torch.bfloat16, device="cuda")
    dvc = torch.zeros_like(dkc)
    q_out = ops.kv_append_rope(d[:, :, :Hq], d[:, :, Hq:Hq + Hkv], d[:, :, Hq + Hkv:], dkc, dvc,
                               torch.from_numpy(lens).to(torch.int32).cuda(), dev_bf16(cos),
                               dev_bf16(sin))
    assert np.array_equal(host_bits(q_out), q_ref)
    assert np.array_equal(host_bits(dkc), kc) and np.array_equal(host_bits(dvc), vc)


def test_consumer_mode_rotates_only_q(mcb):
    _, ops = mcb
    B, T, Hq, D = 2, 1, 4, 64
    rng = np.random.default_rng(9)
    q = O.f32_to_bf16(rng.standard_normal((B, T, Hq, D)).astype(np.float32))
    cos, sin = O.rotary_tables(32, D)
    lens = np.array([3, 17])
    c, s = O.rope_tables_at(cos, sin, lens, T)
    out = ops.kv_append_rope(dev_bf16(q), None, None, None, None,
                             torch.from_numpy(lens).to(torch.int32).cuda(), dev_bf16(cos),
                             dev_bf16(sin), rotate_q=True, rotate_k=False, write_kv=False)
    assert np.array_equal(host_bits(out), O.rope_norm_scale(q, c, s))


def test_append_past_the_cache_is_reported_not_written(mcb):
    """A row at T_max: the kernel's own bounds check records error 1 and skips the write."""
    _, ops = mcb
    B, Tmax, H, D = 2, 8, 2, 64
    k = torch.randn(B, 1, H, D, device="cuda").to(torch.bfloat16)
    kc = torch.zeros(B, Tmax, H, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    ops.kv_write(k, k, kc, vc, torch.tensor([Tmax, 2], dtype=torch.int32, device="cuda"))
    code, _ = ops.device_error()
    assert code == 1
    assert torch.equal(kc[1, 2], k[1, 0]) and kc[0].abs().sum().item() == 0
    assert ops.device_error()[0] == 0  # reading clears it


@pytest.mark.parametrize("name", golden_files("kv_attn_"))
def test_insert_is_bit_exact_against_the_reference(mcb, name):
    _, ops = mcb
    z = load_golden(name)
    kc, vc = dev_bf16(z["k_cache_before"]), dev_bf16(z["v_cache_before"])
    ops.kv_write(dev_bf16(z["k"]), dev_bf16(z["v"]), kc, vc,
                 torch.from_numpy(z["seqlens"]).to(torch.int32).cuda())
    assert np.array_equal(host_bits(kc), z["k_cache_after"])
    assert np.array_equal(host_bits(vc), z["v_cache_after"])


# ---------------------------------------------------------------------------------------------
# piece 2: prefill broadcast and prefill_row through the KVCache API
def test_prefill_and_prefill_row_are_bit_exact(mcb):
    mod, _ = mcb
    z = load_golden("prefill.npz")
    S, _, P, H, D = z["src_k"].shape
    src = mod.KVCache(1, H, P, D, S, "cuda", torch.bfloat16)
    src.k_cache.copy_(dev_bf16(z["src_k"]))
    src.v_cache.copy_(dev_bf16(z["src_v"]))
    src.advance(P)
    dst = mod.KVCache(4, H, 24, D, S, "cuda", torch.bfloat16)
    dst.prefill(src)
    assert dst.get_pos() == P
    assert dst.cache_seqlens.tolist() == z["bcast_seqlens"].tolist()
    assert np.array_equal(host_bits(dst.k_cache), z["bcast_k"])
    assert np.array_equal(host_bits(dst.v_cache), z["bcast_v"])

    rows = mod.KVCache(3, H, 24, D, S, "cuda", torch.bfloat16)
    for r, key in ((1, "row_a"), (2, "row_b")):
        n = z[f"{key}_k"].shape[2]
        c = mod.KVCache(1, H, n, D, S, "cuda", torch.bfloat16)
        c.k_cache.copy_(dev_bf16(z[f"{key}_k"]))
        c.v_cache.copy_(dev_bf16(z[f"{key}_v"]))
        c.advance(n)
        rows.prefill_row(r, c)
    assert rows.cache_seqlens.tolist() == z["rows_seqlens"].tolist()
    assert rows.uniform_pos() is None
    assert np.array_equal(host_bits(rows.k_cache), z["rows_k"])
    assert np.array_equal(host_bits(rows.v_cache), z["rows_v"])
    with pytest.raises(AssertionError, match="non-empty"):
        rows.prefill_row(1, c)


def test_broadcast_at_config4_size_is_a_faithful_copy(mcb):
    """Config 4's broadcast (12 slots, 4096 positions, 4 x 128 per position) into 64 rows:
    every row equals the source, checked by per-row checksums."""
    mod, _ = mcb
    S, P, H, D, B = 12, 4096, 4, 128, 64
    src = mod.KVCache(1, H, P, D, S, "cuda", torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(4)
    src.k_cache.copy_(torch.randn(src.k_cache.shape, device="cuda", generator=g).to(torch.bfloat16))
    src.v_cache.copy_(torch.randn(src.v_cache.shape, device="cuda", generator=g).to(torch.bfloat16))
    src.advance(P)
    dst = mod.KVCache(B, H, P + 64, D, S, "cuda", torch.bfloat16)
    dst.prefill(src)
    ref_k = src.k_cache[:, 0].view(S, -1).view(torch.int16).to(torch.int64).sum(-1)
    got_k = dst.k_cache[:, :, :P].reshape(S, B, -1).view(torch.int16).to(torch.int64).sum(-1)
    assert torch.equal(got_k, ref_k[:, None].expand(S, B))
    assert torch.equal(dst.v_cache[:, B - 1, :P], src.v_cache[:, 0])
    assert dst.k_cache[:, :, P:].abs().sum().item() == 0
    assert dst.cache_seqlens.tolist() == [P] * B


# ---------------------------------------------------------------------------------------------
# piece 3: decode attention
def _attn_case_to_device(z):
    return (dev_bf16(z["q"]), dev_bf16(z["k_cache_after"]), dev_bf16(z["v_cache_after"]),
            torch.from_numpy(z["seqlens"]).to(torch.int32).cuda(), int(z["window"]))


@pytest.mark.parametrize("splits", [0, 1, 3, 37, -1, -3, -12, -20])
@pytest.mark.parametrize("name", golden_files("kv_attn_"))
def test_attention_matches_the_reference_golden_outputs(mcb, name, splits):
    _, ops = mcb
    z = load_golden(name)
    q, kc, vc, seqlens, window = _attn_case_to_device(z)
    y = ops.decode_attn(q, kc, vc, seqlens, window=window, num_ctas=splits)
    torch.cuda.synchronize()
    no_device_error(ops)
    err = (y.float().cpu().numpy() - z["y"]).__abs__().max()
    assert err <= ATTN_TOL, err


def test_flash_attn_with_kvcache_drop_in_matches_the_reference(mcb):
    mod, _ = mcb
    for name in golden_files("kv_attn_"):
        z = load_golden(name)
        kc, vc = dev_bf16(z["k_cache_before"]), dev_bf16(z["v_cache_before"])
        seqlens = torch.from_numpy(z["seqlens"]).to(torch.int32).cuda()
        y = mod.flash_attn.flash_attn_with_kvcache(
            dev_bf16(z["q"]), kc, vc, k=dev_bf16(z["k"]), v=dev_bf16(z["v"]), cache_seqlens=seqlens,
            causal=True, window_size=(int(z["window"]), 0))
        assert np.array_equal(host_bits(kc), z["k_cache_after"]), name
        assert np.abs(y.float().cpu().numpy() - z["y"]).max() <= ATTN_TOL, name
        assert seqlens.tolist() == z["seqlens"].tolist()  # not advanced


def _random_case(rng, B, T, Hq, Hkv, D, Tmax, lens=None):
    if lens is None:
        lens = rng.integers(0, Tmax - T + 1, size=B)
    q = O.f32_to_bf16(rng.standard_normal((B, T, Hq, D)).astype(np.float32))
    kc = O.f32_to_bf16(rng.standard_normal((B, Tmax, Hkv, D)).astype(np.float32))
    vc = O.f32_to_bf16(rng.standard_normal((B, Tmax, Hkv, D)).astype(np.float32))
    return np.asarray(lens), q, kc, vc


CASES = [
    # B, T, Hq, Hkv, D, Tmax, window
    (3, 1, 4, 4, 16, 200, -1), (2, 4, 8, 2, 32, 150, 5), (4, 1, 12, 12, 64, 700, -1),
    (4, 1, 12, 12, 64, 700, 100), (5, 1, 32, 8, 128, 1500, -1), (5, 1, 32, 8, 128, 1500, 257),
    (3, 2, 16, 4, 128, 400, 64), (2, 1, 8, 1, 128, 300, -1), (2, 1, 4, 1, 256, 330, 40),
    (3, 5, 4, 2, 64, 90, 0), (2, 1, 16, 16, 128, 66, 1), (6, 3, 6, 3, 64, 129, -1),
    # few row groups of long rows: 9-16 splits merge in one (non-portable) cluster
    (1, 1, 32, 8, 128, 2048, -1), (2, 1, 16, 4, 128, 1100, 600),
    # 320 row groups: 12-20 splits are a grid too large for clusters of 16 or for merges in the
    # last CTA of each group -- the partials go to the combine kernel
    (40, 1, 32, 8, 128, 1400, -1),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}Hq{}Hkv{}D{}L{}w{}".format(*c))
def test_attention_matches_the_oracle_on_random_ragged_rows(mcb, case):
    _, ops = mcb
    B, T, Hq, Hkv, D, Tmax, window = case
    rng = np.random.default_rng(abs(hash(case)) % 2**32)
    lens, q, kc, vc = _random_case(rng, B, T, Hq, Hkv, D, Tmax)
    lens[0] = 0
    ref = O.decode_attention(O.bf16_to_f32(q), O.bf16_to_f32(kc), O.bf16_to_f32(vc), lens, window)
    args = (dev_bf16(q), dev_bf16(kc), dev_bf16(vc), torch.from_numpy(lens).to(torch.int32).cuda())
    # -2..-16: cluster merge (above 8 in a non-portable cluster); -20: partials, merged by the
    # split that finishes last (small grids) or by the combine kernel (large grids)
    for splits in (0, 1, 2, 5, 300, -1, -2, -7, -8, -12, -16, -20):
        y = ops.decode_attn(*args, window=window, num_ctas=splits)
        err = np.abs(y.float().cpu().numpy() - ref).max()
        assert err <= ATTN_TOL, (splits, err)
    no_device_error(ops)


def test_stale_kv_beyond_a_rows_content_is_unreachable(mcb):
    """Bit-identical output with garbage past every row's position (test_kernels.py:487-498)."""
    _, ops = mcb
    rng = np.random.default_rng(11)
    B, Hq, Hkv, D, Tmax = 4, 16, 4, 128, 512
    lens, q, kc, vc = _random_case(rng, B, 1, Hq, Hkv, D, Tmax, lens=[4, 170, 311, 9])
    args = dict(window=-1, num_ctas=2)
    dq, dk, dv = dev_bf16(q), dev_bf16(kc), dev_bf16(vc)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    clean = ops.decode_attn(dq, dk, dv, sl, **args)
    for i, L in enumerate(lens):
        dk[i, L + 1:] = 1e4
        dv[i, L + 1:] = -1e4
    assert torch.equal(clean, ops.decode_attn(dq, dk, dv, sl, **args))


def test_batched_rows_equal_each_row_alone(mcb):
    """A ragged batch computes each row as that row alone (test_kernels.py:465-472).  The tile
    partition spans the whole batch, so a row alone is cut at other tile boundaries: the results
    agree up to fp32 summation order (a bf16 ulp or two), and both match the oracle."""
    _, ops = mcb
    rng = np.random.default_rng(5)
    B, Hq, Hkv, D, Tmax = 5, 32, 8, 128, 2000
    lens, q, kc, vc = _random_case(rng, B, 1, Hq, Hkv, D, Tmax)
    dq, dk, dv = dev_bf16(q), dev_bf16(kc), dev_bf16(vc)
    sl = torch.from_numpy(lens).to(torch.int32).cuda()
    for window in (-1, 300):
        ref = O.decode_attention(O.bf16_to_f32(q), O.bf16_to_f32(kc), O.bf16_to_f32(vc), lens, window)
        for ctas in (0, 4, -3):
            batched = ops.decode_attn(dq, dk, dv, sl, window=window, num_ctas=ctas)
            assert np.abs(batched.float().cpu().numpy() - ref).max() <= ATTN_TOL
            for b in range(B):
                alone = ops.decode_attn(dq[b:b + 1].contiguous(), dk[b:b + 1].contiguous(),
                                        dv[b:b + 1].contiguous(), sl[b:b + 1].contiguous(),
                                        window=window, num_ctas=ctas)
                assert (batched[b:b + 1].float() - alone.float()).abs().max().item() <= 2e-3


def test_sliding_window_is_measured_from_each_rows_own_position(mcb):
    """Row 0 at position 3 sees its whole history; row 1 at 20 with window 8 sees [12, 20]
    (test_kernels.py:512-525)."""
    _, ops = mcb
    rng = np.random.default_rng(2)
    lens, q, kc, vc = _random_case(rng, 2, 1, 4, 4, 64, 48, lens=[3, 20])
    dq, dk, dv = dev_bf16(q), dev_bf16(kc), dev_bf16(vc)
    sl = torch.tensor([3, 20], dtype=torch.int32, device="cuda")
    base = ops.decode_attn(dq, dk, dv, sl, window=8)
    k2 = dk.clone()
    k2[1, :10] += 5.0
    assert torch.equal(base[1], ops.decode_attn(dq, k2, dv, sl, window=8)[1])
    k3 = dk.clone()
    k3[0, 0] += 5.0
    assert not torch.equal(base[0], ops.decode_attn(dq, k3, dv, sl, window=8)[0])


def _torch_fp32_reference(q, kc, vc, lens, window):
    """A plain PyTorch fp32 evaluation on the GPU (for sizes beyond the CPU oracle)."""
    B, T, Hq, D = q.shape
    Hkv = kc.shape[2]
    G = Hq // Hkv
    out = torch.empty(B, T, Hq, D, device=q.device, dtype=torch.float32)
    for b in range(B):
        for t in range(T):
            qpos = int(lens[b]) + t
            lo = 0 if window < 0 else max(0, qpos - window)
            K = kc[b, lo:qpos + 1].float().repeat_interleave(G, dim=1)   # (n, Hq, D)
            V = vc[b, lo:qpos + 1].float().repeat_interleave(G, dim=1)
            s = torch.einsum("hd,nhd->hn", q[b, t].float(), K) / math.sqrt(D)
            out[b, t] = torch.einsum("hn,nhd->hd", torch.softmax(s, dim=-1), V)
    return out


@pytest.mark.parametrize("window", [-1, 4096])
def test_attention_at_config5_size(mcb, window):
    """Config 5 (32 q / 8 kv heads, D 128, lengths U[1, 32768] from seed 5) at batch 64 against a
    torch fp32 evaluation on the GPU, and a size-independent property: scaling V by 2 scales
    the output by 2 exactly (linearity in V, bf16-exact factor)."""
    _, ops = mcb
    B, Hq, Hkv, D, Tmax = 64, 32, 8, 128, 32769
    lens = np.random.default_rng(5).integers(1, 32769, size=B) - 1
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.from_numpy(lens).to(torch.int32).cuda()
    y = ops.decode_attn(q, kc, vc, sl, window=window)
    ref = _torch_fp32_reference(q, kc, vc, lens, window)
    assert (y.float() - ref).abs().max().item() <= ATTN_TOL
    y2 = ops.decode_attn(q, kc, vc * 2, sl, window=window)
    assert torch.equal(y2.float(), 2 * y.float())
    no_device_error(ops)


def test_attention_at_config2_size_single_wave_kernel(mcb):
    """Config 2's step shape (64 rows x 12 kv heads of 64: 768 split CTAs) runs the 2-stage split
    kernel whose grid is resident in one wave; it matches the fp32 reference and the persistent
    plan."""
    _, ops = mcb
    B, Hq, Hkv, D, Tmax = 64, 12, 12, 64, 1024
    g = torch.Generator(device="cuda").manual_seed(21)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    lens = torch.randint(500, 1000, (B,), device="cuda", generator=g, dtype=torch.int32)
    y = ops.decode_attn(q, kc, vc, lens)
    y_p = ops.decode_attn(q, kc, vc, lens, num_ctas=296)
    torch.cuda.synchronize()
    no_device_error(ops)
    ref = _torch_fp32_reference(q, kc, vc, lens.tolist(), -1)
    assert (y.float() - ref).abs().max().item() <= ATTN_TOL
    assert (y.float() - y_p.float()).abs().max().item() <= 2e-3
