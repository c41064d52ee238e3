"""The CPU oracle (oracle/kv_path.py) against golden vectors the reference itself produced
(tests/golden/make_golden.py).  This pins the oracle before any GPU test trusts it."""
import numpy as np
import pytest

from conftest import golden_files, load_golden
from oracle import kv_path as O


@pytest.mark.parametrize("D", [64, 128])
def test_rope_is_bit_exact_against_the_reference(D):
    z = load_golden(f"rope_norm_D{D}.npz")
    c, s = O.rope_tables_at(z["cos_table"], z["sin_table"], z["seqlens"], z["x"].shape[1])
    assert np.array_equal(O.rope(z["x"], c, s), z["rope"])


@pytest.mark.parametrize("D", [64, 128])
def test_rope_norm_scale_matches_the_reference(D):
    """rms_norm's fp32 sum order is torch's implementation detail; the oracle fixes the CUDA
    kernel's order.  Against the reference that may move a rare element by one bf16 ulp; on
    these vectors it matches exactly."""
    z = load_golden(f"rope_norm_D{D}.npz")
    out = O.rms_norm_scale(z["rope"])
    diff = np.abs(out.astype(np.int32) - z["out"].astype(np.int32))
    assert diff.max() <= 1
    assert (diff != 0).mean() <= 1e-3
    assert np.array_equal(out, z["out"])
    # the fused chain straight from x
    c, s = O.rope_tables_at(z["cos_table"], z["sin_table"], z["seqlens"], z["x"].shape[1])
    assert np.array_equal(O.rope_norm_scale(z["x"], c, s), z["out"])


@pytest.mark.parametrize("D", [64, 128])
def test_rotary_tables_match_the_reference_modules_buffers(D):
    """numpy's fp32 sin/cos may differ from torch's by an fp32 ulp, which can move a bf16
    rounding on a handful of entries; the CUDA path reads the module's own buffers."""
    z = load_golden(f"rope_norm_D{D}.npz")
    cos, sin = O.rotary_tables(z["cos_table"].shape[0], D)
    assert (cos != z["cos_table"]).mean() < 1e-3
    assert (sin != z["sin_table"]).mean() < 1e-3
    d = np.abs(O.bf16_to_f32(sin) - O.bf16_to_f32(z["sin_table"]))
    assert d.max() <= 2.0 ** -8


def test_kernel_order_sum_of_squares_is_a_sum_of_squares():
    rng = np.random.default_rng(0)
    y = rng.standard_normal((50, 128)).astype(np.float32)
    np.testing.assert_allclose(O.sum_squares_kernel_order(y), (y.astype(np.float64) ** 2).sum(-1),
                               rtol=1e-5)


@pytest.mark.parametrize("name", golden_files("kv_attn_"))
def test_insert_and_attention_match_the_reference_sdpa_path(name):
    z = load_golden(name)
    kc, vc = z["k_cache_before"].copy(), z["v_cache_before"].copy()
    kf = O.bf16_to_f32(kc)
    vf = O.bf16_to_f32(vc)
    k, v = O.bf16_to_f32(z["k"]), O.bf16_to_f32(z["v"])
    y = O.flash_attn_with_kvcache(O.bf16_to_f32(z["q"]), kf, vf, k, v, z["seqlens"],
                                  int(z["window"]))
    assert np.array_equal(O.f32_to_bf16(kf), z["k_cache_after"])
    assert np.array_equal(O.f32_to_bf16(vf), z["v_cache_after"])
    np.testing.assert_allclose(y, z["y"], atol=2e-6, rtol=1e-5)


def test_prefill_broadcast_and_prefill_row_match_the_reference():
    z = load_golden("prefill.npz")
    S, _, P, H, D = z["src_k"].shape
    dk = np.zeros(z["bcast_k"].shape, np.uint16)
    dv = np.zeros_like(dk)
    O.prefill_broadcast(dk, dv, z["src_k"], z["src_v"], P)
    assert np.array_equal(dk, z["bcast_k"]) and np.array_equal(dv, z["bcast_v"])
    rk = np.zeros(z["rows_k"].shape, np.uint16)
    rv = np.zeros_like(rk)
    O.prefill_row(rk, rv, 1, z["row_a_k"], z["row_a_v"], z["row_a_k"].shape[2])
    O.prefill_row(rk, rv, 2, z["row_b_k"], z["row_b_v"], z["row_b_k"].shape[2])
    assert np.array_equal(rk, z["rows_k"]) and np.array_equal(rv, z["rows_v"])
    assert z["bcast_seqlens"].tolist() == [P] * z["bcast_k"].shape[1]
    assert z["rows_seqlens"].tolist() == [0, z["row_a_k"].shape[2], z["row_b_k"].shape[2]]


def test_visible_range_is_the_ragged_mask_of_the_reference():
    """flash_attn.py:246-264: col <= q_pos and (window < 0 or q_pos - col <= window)."""
    for L in (0, 1, 5, 40):
        for t in (0, 2):
            for w in (-1, 0, 1, 8, 100):
                lo, hi = O.visible_range(L, t, w)
                qpos = L + t
                cols = [c for c in range(qpos + 5) if c <= qpos and (w < 0 or qpos - c <= w)]
                assert cols == list(range(lo, hi + 1))


def test_kv_read_bytes_counts_exact_keys():
    # window 4: a row at position 10 reads keys 6..10 (5 keys); at position 2, keys 0..2
    assert O.kv_read_bytes([10, 2], 1, Hkv=8, D=128, window=4) == (5 + 3) * 2 * 8 * 128 * 2
    assert O.kv_read_bytes([10], 1, Hkv=1, D=64, window=-1) == 11 * 2 * 64 * 2


def test_decode_golden_streams_are_well_formed():
    z = load_golden("decode_cfg1.npz")
    assert z["prompts"].shape == (2, 16)
    for v in ("random", "awake"):
        assert z[f"{v}_tokens"].shape == (2, 64)
        assert (z[f"{v}_tokens"] >= 0).all() and (z[f"{v}_tokens"] < 32768).all()


@pytest.mark.parametrize("C", [40, 768, 2048, 4096])
def test_add_rms_norm_matches_the_reference_block(C):
    """Block's residual add is one bf16 rounding and matches exactly; RMSNorm's fp32 sum order is
    torch's detail, so the oracle (the CUDA kernel's order) may move a rare element by one ulp."""
    z = load_golden("step_fused.npz")
    s, h = O.add_rms_norm(z[f"x_C{C}"], z[f"delta_C{C}"])
    assert np.array_equal(s, z[f"sum_C{C}"])
    for got, want in ((h, z[f"norm_C{C}"]), (O.add_rms_norm(z[f"x_C{C}"])[1], z[f"norm_only_C{C}"])):
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1
        assert (diff != 0).mean() <= 2e-3


def test_gated_silu_matches_the_reference_mlp():
    """silu(gate) * up in bf16: torch's CPU exp and numpy's may differ by an fp32 ulp, which can
    move a bf16 rounding of silu; everything else is one rounding per op."""
    z = load_golden("step_fused.npz")
    got = O.gated_silu(z["gate"], z["up"])
    diff = np.abs(got.astype(np.int32) - z["gated"].astype(np.int32))
    assert diff.max() <= 1
    assert (diff != 0).mean() <= 1e-3


def test_embed_rms_norm_matches_the_reference_token_embedding():
    z = load_golden("step_fused.npz")
    x, h = O.embed_rms_norm(z["ids"], z["wte"])
    assert np.array_equal(x, z["embed_x"])
    assert np.array_equal(h, z["embed_h"])


def _f32_ulps(a, b):
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))


def test_softcap_and_greedy_pick_match_the_reference_lm_head():
    """The crop and .float() are exact; the softcap differs from the reference's CPU evaluation by
    at most a few fp32 ulps (exact division and torch's vectorised tanh on the CPU, the reciprocal
    multiply of torch's CUDA path and numpy's tanh here); the greedy pick agrees."""
    z = load_golden("step_fused.npz")
    assert np.array_equal(O.softcap_logits(z["head_logits_bf16"], 1000, None), z["head_out_nocap"])
    y = O.softcap_logits(z["head_logits_bf16"], 1000, 15)
    assert y.shape == z["head_out"].shape
    assert _f32_ulps(y, z["head_out"]).max() <= 4
    assert np.array_equal(O.greedy_pick(y), np.argmax(z["head_out"], axis=-1))


@pytest.mark.parametrize("top_k,T", [(50, 1.0), (7, 0.6), (None, 1.3)])
def test_sampling_candidates_match_the_reference_topk_softmax(top_k, T):
    """The oracle's candidates and probabilities against the reference's own torch ops
    (sample_next_token, modelcore/generate.py:25-33: topk, / temperature, softmax) on the CPU."""
    import torch
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(4, 3000, generator=g) * 4
    for r in range(4):
        order, p = O.sample_candidates(logits[r].numpy(), T, top_k)
        if top_k:
            vals, idx = torch.topk(logits[r], top_k)
            probs = F.softmax(vals / T, dim=-1)
            assert np.array_equal(order, idx.numpy())
        else:
            probs = F.softmax(logits[r] / T, dim=-1)
        assert np.allclose(p, probs.double().numpy(), rtol=1e-5, atol=1e-9)
    # ties at the cut keep the smallest indices
    x = np.zeros(100, dtype=np.float32)
    x[[3, 50, 77]] = 1.0
    order, _ = O.sample_candidates(x, 1.0, 5)
    assert order.tolist() == [3, 50, 77, 0, 1]


def test_e4m3_rounding_matches_torch_float8():
    """The oracle's e4m3 encoding (round to nearest even, saturating at 448; the fp8 cache's
    format) agrees with torch's float8_e4m3fn conversion across normals, subnormals and ties,
    and its known values: 448, 1, the smallest subnormal, ties to even, saturation."""
    import torch
    rng = np.random.default_rng(0)
    y = (rng.standard_normal(200000) * np.exp2(rng.integers(-12, 9, 200000))).astype(np.float32)
    y = np.clip(y, -448, 448)
    want = torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_bits(y), want)
    x = np.array([448, -448, 1.0, 2 ** -9, 0.0, 500, 1.0625, 2 ** -10, 3 * 2 ** -10, 232], dtype=np.float32)
    assert O.e4m3_bits(x).tolist() == [0x7E, 0xFE, 0x38, 0x01, 0x00, 0x7E, 0x38, 0x00, 0x02, 0x76]
    assert np.array_equal(O.e4m3_value(O.e4m3_bits(y)), torch.from_numpy(want).view(torch.float8_e4m3fn).float().numpy())
    b, s = O.quantize_fp8(O.f32_to_bf16(np.array([[0.5, -3.0, 1.25], [0.0, 0.0, 0.0]], dtype=np.float32)))
    assert s.tolist() == [np.float32(3.0) / np.float32(448.0), 0.0] and b[0, 1] == 0xFE and not b[1].any()
