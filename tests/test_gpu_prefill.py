"""GPU parity of the tensor-core prefill attention (mcb_prefill_attn, and mcb_decode_attn's
automatic prefill plan for T_new >= 64), through the C ABI, against the reference's golden outputs,
the CPU oracle (float64) and a torch fp32 evaluation on the GPU.

Bar: max-abs 2e-2 against the fp32 reference (bf16 output; P is rounded to bf16 before the P.V
product, as in every flash-attention kernel)."""
import math

import numpy as np
import pytest
import torch

from conftest import golden_files, load_golden
from oracle import kv_path as O

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-2


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _torch_ref(q, kc, vc, lens, window):
    """fp32 attention on the GPU with the reference's visibility rule."""
    B, T, Hq, D = q.shape
    Hkv = kc.shape[2]
    G = Hq // Hkv
    out = torch.empty(B, T, Hq, D, device=q.device)
    for b in range(B):
        L = int(lens[b])
        k = kc[b, :L + T].float().repeat_interleave(G, dim=1)   # (keys, Hq, D)
        v = vc[b, :L + T].float().repeat_interleave(G, dim=1)
        s = torch.einsum("thd,chd->htc", q[b].float(), k) / math.sqrt(D)
        pos = L + torch.arange(T, device=q.device)[:, None]
        c = torch.arange(L + T, device=q.device)[None, :]
        vis = c <= pos
        if window >= 0:
            vis &= (pos - c) <= window
        s = s.masked_fill(~vis[None], float("-inf"))
        out[b] = torch.einsum("htc,chd->thd", torch.softmax(s, -1), v)
    return out


@pytest.mark.parametrize("name", [n for n in golden_files("kv_attn_") if "_d64_" in n or "_d128_" in n])
def test_prefill_kernel_matches_the_reference_golden_outputs(ops, name):
    """The reference's own SDPA outputs (T_new 1 and 2, ragged rows, windows) through the prefill
    kernel: it serves any T."""
    z = load_golden(name)
    kc, vc = _bf16(z["k_cache_after"]), _bf16(z["v_cache_after"])
    q = _bf16(z["q"])
    seqlens = torch.from_numpy(z["seqlens"]).to(torch.int32).cuda()
    y = ops.prefill_attn(q, kc, vc, seqlens, window=int(z["window"]))
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    err = float(np.abs(y.float().cpu().numpy() - z["y"]).max())
    assert err <= ATTN_TOL, err


CASES = [
    # B, T, Hq, Hkv, D, prefix lengths, window, Tmax
    (1, 128, 1, 1, 64, [0], -1, 128),         # one exact tile, cache exactly full
    (1, 129, 2, 2, 64, [0], -1, 256),         # a one-query second tile
    (2, 200, 4, 2, 64, [0, 37], -1, 512),
    (2, 300, 4, 1, 128, [5, 130], 100, 512),  # GQA 4, window smaller than a tile
    (3, 64, 8, 2, 128, [0, 1000, 333], 257, 1100),
    (1, 513, 12, 12, 64, [0], -1, 1024),      # config 2's prompt length
    (2, 97, 16, 4, 128, [4000, 7], 1024, 4100),
    # head size 64 takes one query tile an item, two CTAs an SM: more items than CTAs, ragged
    # prefixes, GQA, a window
    (8, 640, 16, 4, 64, [0, 3, 129, 700, 1, 0, 64, 900], -1, 1600),
    (4, 700, 12, 12, 64, [0, 10, 500, 1000], 300, 2048),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}T{}Hq{}Hkv{}D{}w{}".format(c[0], c[1], c[2], c[3], c[4], c[6]))
def test_prefill_kernel_against_the_oracle_and_torch(ops, case):
    B, T, Hq, Hkv, D, lens, window, Tmax = case
    g = torch.Generator(device="cuda").manual_seed(T * 31 + D)
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    y = ops.prefill_attn(q, kc, vc, sl, window=window)
    y_auto = ops.decode_attn(q, kc, vc, sl, window=window)         # the automatic plan
    y_split = ops.decode_attn(q, kc, vc, sl, window=window, num_ctas=-2)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    ref = _torch_ref(q, kc, vc, lens, window)
    assert (y.float() - ref).abs().max().item() <= ATTN_TOL
    if T >= 64:
        assert torch.equal(y_auto, y)
    assert (y_split.float() - ref).abs().max().item() <= ATTN_TOL
    if B * T * Hq * D <= 200_000:   # the float64 oracle on the smaller cases
        f = lambda t: t.float().cpu().numpy()
        o = O.decode_attention(f(q), f(kc), f(vc), np.array(lens), window)
        assert float(np.abs(f(y) - o).max()) <= ATTN_TOL


def test_prefill_kernel_never_reads_past_a_rows_positions(ops):
    """Keys past L_b + T (stale or garbage cache contents) do not reach the output."""
    B, T, Hq, Hkv, D, Tmax = 2, 150, 4, 4, 64, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.tensor([10, 200], dtype=torch.int32, device="cuda")
    y0 = ops.prefill_attn(q, kc, vc, sl)
    kc2, vc2 = kc.clone(), vc.clone()
    for b, L in enumerate([10, 200]):
        kc2[b, L + T:] = float("nan")
        vc2[b, L + T:] = 1e4
    y1 = ops.prefill_attn(q, kc2, vc2, sl)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


def test_prefill_positions_past_the_cache_are_reported(ops):
    B, T, Hq, D, Tmax = 1, 100, 2, 64, 128
    q = torch.zeros(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(B, Tmax, Hq, D, device="cuda", dtype=torch.bfloat16)
    sl = torch.tensor([60], dtype=torch.int32, device="cuda")    # 60 + 100 > 128
    ops.prefill_attn(q, kc, kc, sl)
    code, _ = ops.device_error()
    assert code == 1


@pytest.mark.parametrize("window", [-1, 1024])
def test_prefill_kernel_at_config3_prompt_size(ops, window):
    """Config 3's longest prompt: 8192 tokens, 16 q / 4 kv heads of 128, against torch fp32 on a
    sample of query positions (the full fp32 reference would hold 4 GB of scores)."""
    T, Hq, Hkv, D = 8192, 16, 4, 128
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(1, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(1, T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(1, T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.decode_attn(q, kc, vc, sl, window=window)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    rows = torch.tensor([0, 1, 127, 128, 1000, 4095, 4096, 8000, 8191], device="cuda")
    k = kc[0].float().repeat_interleave(Hq // Hkv, dim=1)
    v = vc[0].float().repeat_interleave(Hq // Hkv, dim=1)
    s = torch.einsum("rhd,chd->hrc", q[0, rows].float(), k) / math.sqrt(D)
    c = torch.arange(T, device="cuda")[None, :]
    vis = c <= rows[:, None]
    if window >= 0:
        vis &= (rows[:, None] - c) <= window
    s = s.masked_fill(~vis[None], float("-inf"))
    ref = torch.einsum("hrc,chd->rhd", torch.softmax(s, -1), v)
    assert (y[0, rows].float() - ref).abs().max().item() <= ATTN_TOL
