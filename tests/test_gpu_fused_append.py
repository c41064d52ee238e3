"""GPU parity of the fused append (ops.append_attn / mcb_decode_attn with fuse_append): one launch
that ropes, norms and scales the raw query and key of a decode step, writes the key and value into
the slot and attends over it must give exactly what the two launches give (mcb_kv_append_rope,
then mcb_decode_attn): the same cache bytes and the same attention output, bit for bit, on every
split plan (one split, a cluster merge, partials) and on the persistent plan (row groups cut
between CTAs and merged by the last to arrive, several row groups a CTA, two query blocks a
row), with windows, ring slots, GQA groups and layers that read another layer's slot."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def tables(rot_len, D):
    ang = torch.arange(rot_len, dtype=torch.float32)[:, None] * \
        (10000.0 ** (-torch.arange(0, D, 2, dtype=torch.float32) / D))[None]
    return ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()


CASES = [  # B, Hq, Hkv, D, Tmax, max_len, window, ring, produces_kv, num_ctas
    (64, 12, 12, 64, 1024, 900, -1, False, True, 0),    # config 2's shape: one split per row group
    (4, 32, 8, 128, 2048, 2000, -1, False, True, 0),    # few groups: splits merged in a cluster
    (3, 16, 4, 128, 1024, 1000, 300, False, True, -12), # a window, 12 splits
    (40, 32, 8, 128, 1400, 1390, -1, False, True, -20), # partials and the combine kernel
    (2, 8, 2, 64, 512, 1500, 200, True, True, 0),       # a ring slot
    (5, 16, 4, 128, 1024, 1000, -1, False, False, 0),   # a layer that reads another's slot
    # the persistent plan (num_ctas > 0 or many groups of long rows)
    (64, 32, 8, 128, 2560, 2500, -1, False, True, 0),   # chosen by the planner (512 long groups)
    (6, 16, 4, 64, 1024, 1000, -1, False, True, 16),    # groups cut between CTAs, merged last
    (8, 16, 4, 128, 2048, 2000, 700, False, True, 20),  # a window
    (3, 8, 2, 64, 512, 1500, 200, True, True, 6),       # a ring slot
    (5, 16, 4, 128, 1024, 1000, -1, False, False, 8),   # a layer that reads another's slot
    (4, 32, 2, 128, 1024, 1000, -1, False, True, 12),   # 16 query rows a group (two n-tiles)
    (2, 64, 2, 64, 512, 500, -1, False, True, 4),       # two query blocks a row
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}Hq{}Hkv{}D{}w{}r{}kv{}n{}".format(
    c[0], c[1], c[2], c[3], c[6], int(c[7]), int(c[8]), c[9]))
def test_fused_append_equals_append_then_attention(ops, case):
    B, Hq, Hkv, D, Tmax, max_len, window, ring, produces, nc = case
    g = torch.Generator(device="cuda").manual_seed(B * 7 + Hq + D)
    qkv = (torch.randn(B, 1, Hq + 2 * Hkv, D, device="cuda", generator=g) * 2).to(torch.bfloat16)
    q, k, v = qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:]  # strided views, as packed
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    hi = max_len - 1
    sl = torch.randint(hi // 2, hi + 1, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = tables(max(Tmax, max_len) + 8, D)
    kc2, vc2 = kc.clone(), vc.clone()
    # two launches
    if produces:
        qa = ops.kv_append_rope(q, k, v, kc, vc, sl, cos, sin, eps=1e-6, scale=1.2, ring=ring)
    else:
        qa = ops.kv_append_rope(q, None, None, None, None, sl, cos, sin, rotate_q=True, rotate_k=False,
                                write_kv=False, eps=1e-6, scale=1.2)
    want = ops.decode_attn(qa, kc, vc, sl, window=window, ring=ring, num_ctas=nc)
    # one launch (num_ctas as above: the same split plan)
    args = ops._attn_args(q, kc2, vc2, sl, window, None, nc, None, ring)
    from modelcore_b200 import _native
    assert _native.load().mcb_decode_attn_fusable(__import__("ctypes").byref(args)) == 1
    got = fused(ops, q, k if produces else None, v if produces else None, kc2, vc2, sl, cos, sin,
                window, ring, nc)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)
    assert torch.equal(got, want)


def fused(ops, q, k, v, kc, vc, sl, cos, sin, window, ring, nc):
    """ops.append_attn with an explicit split count (the tests pin the plan)."""
    import ctypes
    from modelcore_b200 import _native
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    args = ops._attn_args(q, kc, vc, sl, window, None, nc, out, ring)
    args.fuse_append = 1
    if k is not None:
        args.k_new, args.v_new = k.data_ptr(), v.data_ptr()
        args.k_new_stride[:] = ops._bthd_strides("k", k)
        args.v_new_stride[:] = ops._bthd_strides("v", v)
    D = q.size(3)
    args.rot_cos, args.rot_sin = cos.data_ptr(), sin.data_ptr()
    args.rot_len = cos.numel() // (D // 2)
    args.rotate_k = 1
    args.norm_eps = 1e-6
    args.qk_scale = 1.2
    lib = _native.load()
    need = int(lib.mcb_decode_attn_workspace_size(ctypes.byref(args)))
    ncount = int(lib.mcb_decode_attn_counter_count(ctypes.byref(args)))
    if need:
        ws = ops.attn_workspace(q.device, need)
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    if ncount:
        cnt = ops.attn_counters(q.device, ncount)
        args.counters, args.counter_count = cnt.data_ptr(), cnt.numel()
    _native.check(lib.mcb_decode_attn(ctypes.byref(args), ops._stream(q)))
    return out


def test_append_attn_picks_the_fused_launch_and_falls_back(ops):
    """ops.append_attn: one launch on a fusable plan, two (append + attention) otherwise -- the same
    results either way."""
    B, Hq, Hkv, D, Tmax = 8, 16, 4, 128, 8192
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    sl = torch.randint(100, 8000, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = tables(Tmax + 8, D)
    for window in (1000, -1):  # rows of 1,001 keys: split; 8k keys in 32 groups: split (few groups)
        kc1, vc1, kc2, vc2 = kc.clone(), vc.clone(), kc.clone(), vc.clone()
        n0 = ops.launch_count()
        got = ops.append_attn(q, k, v, kc1, vc1, sl, cos, sin, eps=1e-6, window=window)
        launches = ops.launch_count() - n0
        qa = ops.kv_append_rope(q, k, v, kc2, vc2, sl, cos, sin, eps=1e-6, scale=1.2)
        want = ops.decode_attn(qa, kc2, vc2, sl, window=window)
        torch.cuda.synchronize()
        assert launches == 1
        assert torch.equal(kc1, kc2) and torch.equal(got, want)
    # a persistent plan (many groups of long rows) fuses too
    B2 = 64
    q2 = q.repeat(B2 // B, 1, 1, 1)
    k2, v2 = k.repeat(B2 // B, 1, 1, 1), v.repeat(B2 // B, 1, 1, 1)
    kc3 = kc.repeat(B2 // B, 1, 1, 1)
    vc3 = vc.repeat(B2 // B, 1, 1, 1)
    sl2 = sl.repeat(B2 // B)
    kc4, vc4 = kc3.clone(), vc3.clone()
    n0 = ops.launch_count()
    got = ops.append_attn(q2, k2, v2, kc3, vc3, sl2, cos, sin, eps=1e-6)
    assert ops.launch_count() - n0 == 1
    qa = ops.kv_append_rope(q2, k2, v2, kc4, vc4, sl2, cos, sin, eps=1e-6, scale=1.2)
    want = ops.decode_attn(qa, kc4, vc4, sl2)
    torch.cuda.synchronize()
    assert torch.equal(kc3, kc4) and torch.equal(got, want)
    # head_dim 32 has no fused kernel: the two launches
    D3 = 32
    q3 = torch.randn(B, 1, Hq, D3, device="cuda", generator=g).to(torch.bfloat16)
    k3 = torch.randn(B, 1, Hkv, D3, device="cuda", generator=g).to(torch.bfloat16)
    v3 = torch.randn(B, 1, Hkv, D3, device="cuda", generator=g).to(torch.bfloat16)
    kc5 = torch.randn(B, 1024, Hkv, D3, device="cuda", generator=g).to(torch.bfloat16)
    vc5 = torch.randn_like(kc5)
    kc6, vc6 = kc5.clone(), vc5.clone()
    sl3 = torch.randint(10, 1000, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos3, sin3 = tables(1032, D3)
    n0 = ops.launch_count()
    got = ops.append_attn(q3, k3, v3, kc5, vc5, sl3, cos3, sin3, eps=1e-6)
    assert ops.launch_count() - n0 == 2
    qa = ops.kv_append_rope(q3, k3, v3, kc6, vc6, sl3, cos3, sin3, eps=1e-6, scale=1.2)
    want = ops.decode_attn(qa, kc6, vc6, sl3)
    torch.cuda.synchronize()
    assert torch.equal(kc5, kc6) and torch.equal(got, want)


# cluster merge; window + 12 splits; a reading layer; persistent: cut groups, a window, two
# query blocks a row
ORACLE_CASES = [CASES[1], CASES[2], CASES[5], CASES[7], CASES[8], CASES[12]]


@pytest.mark.parametrize("case", ORACLE_CASES, ids=lambda c: "B{}Hq{}D{}w{}kv{}n{}".format(
    c[0], c[1], c[3], c[6], int(c[8]), c[9]))
def test_fused_append_matches_the_oracle(ops, case):
    """The one-launch step against the CPU oracle (oracle/kv_path.py), not only against the
    two-launch CUDA path: the cache bytes after the append are bit-exact (the new key roped,
    normed and scaled; the value copied), the attention within the bf16 tolerance 2e-2 of a
    float64 attention over the oracle's own q and cache."""
    import numpy as np
    from oracle import kv_path as O
    B, Hq, Hkv, D, Tmax, max_len, window, ring, produces, nc = case
    g = torch.Generator(device="cuda").manual_seed(B * 11 + Hq + D)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).mul(2).to(torch.bfloat16)
    k = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).mul(2).to(torch.bfloat16)
    v = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    hi = max_len - 1
    sl = torch.randint(hi // 2, hi + 1, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = tables(max(Tmax, max_len) + 8, D)

    def bits(t):
        return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

    qb, kb, vb, kcb, vcb = bits(q), bits(k), bits(v), bits(kc), bits(vc)
    lens = sl.cpu().numpy()
    got = fused(ops, q, k if produces else None, v if produces else None, kc, vc, sl, cos, sin,
                window, ring, nc)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    if produces:
        q_ref = O.append_rope(qb, kb, vb, kcb, vcb, lens, bits(cos), bits(sin), eps=1e-6, scale=1.2)
    else:
        q_ref = O.append_rope(qb, None, None, None, None, lens, bits(cos), bits(sin), rotate_k=False,
                              write_kv=False, eps=1e-6, scale=1.2)
    assert np.array_equal(bits(kc), kcb) and np.array_equal(bits(vc), vcb)
    y_ref = O.decode_attention(O.bf16_to_f32(q_ref), O.bf16_to_f32(kcb), O.bf16_to_f32(vcb), lens,
                               window)
    err = float(np.abs(got.float().cpu().numpy() - y_ref).max())
    assert err <= 2e-2, f"fused step vs oracle: max-abs {err}"


def test_fused_append_rejects_new_keys_with_the_wrong_head_count(ops):
    """k / v of the fused path must carry the slot's Hkv heads; fewer would be read past their end
    by the kernel, so the host rejects them (as the two-launch path does)."""
    B, Hq, Hkv, D, Tmax = 2, 16, 4, 128, 256
    q = torch.zeros(B, 1, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(B, 1, Hkv - 2, D, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(B, Tmax, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    sl = torch.full((B,), 10, device="cuda", dtype=torch.int32)
    cos, sin = tables(Tmax + 8, D)
    with pytest.raises(RuntimeError, match="Hkv"):
        ops.append_attn(q, k, k.clone(), kc, vc, sl, cos, sin, eps=1e-6)


PAIR_CASES = [  # B, H, Tmax, lengths, window, ring, produces_kv
    (64, 12, 1024, (500, 1000), -1, False, True),   # config 2's shape
    (32, 8, 1024, (10, 1000), 300, False, True),     # a window
    (16, 4, 512, (600, 1500), 200, True, True),      # a ring slot
    (24, 12, 1024, (100, 900), -1, False, False),    # a layer that reads another's slot
]


@pytest.mark.parametrize("case", PAIR_CASES, ids=lambda c: "B{}H{}w{}r{}kv{}".format(c[0], c[1], c[4], int(c[5]),
                                                                                     int(c[6])))
def test_head_pairs_equal_the_one_head_kernel(ops, case):
    """Head size 64 with one query head a kv head runs, on its one-split plan, as kv heads of 128
    holding two real heads (the split kernel's pair mode): bit for bit the one-head kernel's output
    (num_ctas = -1 keeps that kernel), fused with the append or not, cache bytes included."""
    B, H, Tmax, (lo, hi), window, ring, produces = case
    D = 64
    g = torch.Generator(device="cuda").manual_seed(B + H + Tmax)
    qkv = (torch.randn(B, 1, 3 * H, D, device="cuda", generator=g) * 2).to(torch.bfloat16)
    q, k, v = qkv[:, :, :H], qkv[:, :, H:2 * H], qkv[:, :, 2 * H:]
    kc = torch.randn(B, Tmax, H, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    sl = torch.randint(lo, hi, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = tables(max(Tmax, hi) + 8, D)
    kc1, vc1, kc2, vc2 = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    # unfused: the append, then the attention paired (auto plan) and one-head (num_ctas = -1)
    if produces:
        qa = ops.kv_append_rope(q, k, v, kc1, vc1, sl, cos, sin, eps=1e-6, scale=1.2, ring=ring)
    else:
        qa = ops.kv_append_rope(q, None, None, None, None, sl, cos, sin, rotate_q=True, rotate_k=False,
                                write_kv=False, eps=1e-6, scale=1.2)
    paired = ops.decode_attn(qa, kc1, vc1, sl, window=window, ring=ring)
    name = ops.last_attn_kernel()
    single = ops.decode_attn(qa, kc1, vc1, sl, window=window, ring=ring, num_ctas=-1)
    # fused: one launch, paired
    got = fused(ops, q, k if produces else None, v if produces else None, kc2, vc2, sl, cos, sin,
                window, ring, 0)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert "<128,1,16," in name, name
    assert torch.equal(paired, single) and torch.equal(got, single)
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
