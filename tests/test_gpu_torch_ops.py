"""GPU parity of torch.ops.mcb200 (C++ over the libmcb200 C ABI) with the ctypes entry points of
modelcore_b200.ops: the same library does the work, so cache bytes and outputs must be equal bit
for bit -- eagerly, captured in a CUDA graph, and inside a torch.compile'd function."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import modelcore_b200.torch_ops  # noqa: F401
    from modelcore_b200 import ops
    return ops


def _tables(rot_len, D):
    ang = torch.arange(rot_len, dtype=torch.float32)[:, None] * \
        (10000.0 ** (-torch.arange(0, D, 2, dtype=torch.float32) / D))[None]
    return ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()


def _case(B, Hq, Hkv, D, Tmax, lo, hi, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn(B, 1, Hq + 2 * Hkv, D, device="cuda", generator=g).mul(2).to(torch.bfloat16)
    q, k, v = qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:]
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    sl = torch.randint(lo, hi, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = _tables(Tmax + 8, D)
    return q, k, v, kc, vc, sl, cos, sin


CASES = [  # B, Hq, Hkv, D, Tmax, lengths, window
    (64, 12, 12, 64, 1024, (500, 1000), -1),    # config 2's shape: the split plan, append fused
    (64, 32, 8, 128, 2560, (1000, 2500), -1),   # many long groups: the persistent plan
    (3, 16, 4, 128, 1024, (300, 1000), 200),    # a window, few groups
    (4, 8, 8, 32, 512, (10, 500), -1),          # head size 32: no fused kernel, two launches
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}Hq{}D{}w{}".format(c[0], c[1], c[3], c[6]))
def test_torch_ops_equal_the_ctypes_entry_points(env, case):
    ops = env
    B, Hq, Hkv, D, Tmax, (lo, hi), window = case
    q, k, v, kc, vc, sl, cos, sin = _case(B, Hq, Hkv, D, Tmax, lo, hi, B + D)
    kc2, vc2 = kc.clone(), vc.clone()
    want = ops.append_attn(q, k, v, kc, vc, sl, cos, sin, eps=1e-6, window=window)
    got = torch.ops.mcb200.append_attn(q, k, v, kc2, vc2, sl, cos, sin, eps=1e-6, window=window)
    torch.cuda.synchronize()
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc) and torch.equal(got, want)
    # the two halves on their own: the append (processed q, the insert) and the attention
    kc3, vc3 = kc.clone(), vc.clone()
    qa = torch.ops.mcb200.kv_append_rope(q, k, v, kc3, vc3, sl, cos, sin, eps=1e-6)
    qb = ops.kv_append_rope(q, k, v, kc.clone(), vc.clone(), sl, cos, sin, eps=1e-6, scale=1.2)
    y1 = torch.ops.mcb200.decode_attn(qa, kc3, vc3, sl, window=window)
    y2 = ops.decode_attn(qa, kc3, vc3, sl, window=window)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and torch.equal(y1, y2)
    # a layer that reads another layer's slot: q only
    y3 = torch.ops.mcb200.append_attn(q, None, None, kc3, vc3, sl, cos, sin, eps=1e-6, window=window)
    y4 = ops.append_attn(q, None, None, kc3, vc3, sl, cos, sin, eps=1e-6, window=window)
    assert torch.equal(y3, y4)
    assert ops.device_error()[0] == 0


def test_broadcast_and_advance(env):
    ops = env
    g = torch.Generator(device="cuda").manual_seed(4)
    src_k = torch.randn(3, 1, 300, 4, 64, device="cuda", generator=g).to(torch.bfloat16)
    src_v = torch.randn_like(src_k)
    dk1 = torch.zeros(3, 8, 512, 4, 64, device="cuda", dtype=torch.bfloat16)
    dv1, dk2, dv2 = torch.zeros_like(dk1), torch.zeros_like(dk1), torch.zeros_like(dk1)
    s1 = torch.zeros(8, device="cuda", dtype=torch.int32)
    s2 = s1.clone()
    torch.ops.mcb200.kv_broadcast(src_k, src_v, dk1, dv1, 0, 2, 5, 257, s1)
    ops.kv_copy_rows(dk2, dv2, src_k, src_v, src_row=0, dst_row_begin=2, dst_row_count=5, n_pos=257,
                     dst_seqlens=s2)
    torch.ops.mcb200.kv_advance(s1, 3)
    ops.kv_advance(s2, 3)
    torch.cuda.synchronize()
    assert torch.equal(dk1, dk2) and torch.equal(dv1, dv2) and torch.equal(s1, s2)
    assert s1.tolist() == [3, 3, 260, 260, 260, 260, 260, 3]


def test_in_a_cuda_graph_and_under_torch_compile(env):
    ops = env
    q, k, v, kc, vc, sl, cos, sin = _case(64, 12, 12, 64, 1024, 500, 1000, 7)

    def step(q, k, v, kc, vc, sl):
        y = torch.ops.mcb200.append_attn(q, k, v, kc, vc, sl, cos, sin, eps=1e-6)
        torch.ops.mcb200.kv_advance(sl, 1)
        return y * 1.0

    kc1, vc1, sl1 = kc.clone(), vc.clone(), sl.clone()
    want = [step(q, k, v, kc1, vc1, sl1) for _ in range(3)]
    # captured
    kc2, vc2, sl2 = kc.clone(), vc.clone(), sl.clone()
    step(q, k, v, kc2, vc2, sl2)  # warm-up (counters, workspace) outside the capture
    kc2.copy_(kc), vc2.copy_(vc), sl2.copy_(sl)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        out = step(q, k, v, kc2, vc2, sl2)
    torch.cuda.current_stream().wait_stream(side)
    for i in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want[i])
    assert torch.equal(kc2, kc1) and torch.equal(sl2, sl1)
    # compiled: the operators are opaque nodes whose shapes come from the registered functions
    kc3, vc3, sl3 = kc.clone(), vc.clone(), sl.clone()
    compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
    for i in range(3):
        assert torch.equal(compiled(q, k, v, kc3, vc3, sl3), want[i])
    assert torch.equal(kc3, kc1) and torch.equal(sl3, sl1)


def test_linear_and_add_rms_norm_ops_equal_the_ctypes_entry_points(env):
    """torch.ops.mcb200.linear (plain, residual, gated, norm out) and add_rms_norm against
    ops.linear / ops.add_rms_norm: the same library, the same bits."""
    ops = env
    from modelcore_b200 import step
    g = torch.Generator(device="cuda").manual_seed(11)
    r = lambda *s, sc=1.0: (torch.randn(*s, device="cuda", generator=g) * sc).to(torch.bfloat16)
    x, w_qkv, w_o, w_gu, w_d = r(64, 768), r(2304, 768, sc=0.03), r(768, 768, sc=0.03), \
        r(4096, 768, sc=0.03), r(768, 2048, sc=0.02)
    res = r(64, 768, sc=4.0)
    out = torch.empty(64, 2304, device="cuda", dtype=torch.bfloat16)
    torch.ops.mcb200.linear(x, w_qkv, out)
    assert torch.equal(out, ops.linear(x, w_qkv))
    y1, h1 = res.clone(), torch.empty_like(res)
    torch.ops.mcb200.linear(x, w_o, y1, y1, None, 1e-6, False, True)
    assert torch.equal(y1, ops.linear(x, w_o, res=res))
    if ops.linear_supported(x, w_o, out=y1, res=y1, h_out=h1):
        y2, y3, h2, h3 = res.clone(), res.clone(), torch.empty_like(res), torch.empty_like(res)
        torch.ops.mcb200.linear(x, w_o, y2, y2, h2, 1e-6)
        ops.linear(x, w_o, out=y3, res=y3, h_out=h3, eps=1e-6)
        assert torch.equal(y2, y3) and torch.equal(h2, h3)
    a = torch.empty(64, 2048, device="cuda", dtype=torch.bfloat16)
    torch.ops.mcb200.linear(x, w_gu, a, gated=True)
    assert torch.equal(a, ops.linear(x, w_gu, gated=True))
    f = torch.empty(64, 768, device="cuda", dtype=torch.bfloat16)
    torch.ops.mcb200.linear(a, w_d, f)
    assert torch.equal(f, ops.linear(a, w_d))
    xa, ha = res.clone(), torch.empty_like(res)
    torch.ops.mcb200.add_rms_norm(xa, f, xa, ha, 1e-6)
    xb, hb = ops.add_rms_norm(res.clone(), f, eps=1e-6)
    assert torch.equal(xa, xb) and torch.equal(ha, hb)
    hc = torch.empty_like(res)
    torch.ops.mcb200.add_rms_norm(res, None, None, hc)
    assert torch.equal(hc, ops.add_rms_norm(res)[1])
    # the decode step with and without the operators: the same bits (step.USE_TORCH_OPS)
    assert step.USE_TORCH_OPS
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0


def test_decode_step_bits_do_not_depend_on_the_binding(env):
    """The fused decode step through the torch.ops operators (the default) and through ctypes
    (step.USE_TORCH_OPS / integration.USE_TORCH_OPS off) give identical logits and caches."""
    import modelcore_b200
    from modelcore_b200 import integration, step, workloads
    mgr = modelcore_b200.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    prompts = workloads.prompts(5, 40, seed=3).tolist()
    outs = []
    for use in (True, False):
        step.USE_TORCH_OPS = integration.USE_TORCH_OPS = use
        try:
            with torch.inference_mode():
                dec = mgr.new_decoder(model, prompts, max_tokens=8)
                logits = [dec.step([1, 2, 3, 4, 5]) for _ in range(3)]
                outs.append((torch.stack(logits), dec.kv_cache.k_cache.clone()))
        finally:
            step.USE_TORCH_OPS = integration.USE_TORCH_OPS = True
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
