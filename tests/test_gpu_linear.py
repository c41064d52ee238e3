"""GPU parity of the decode projection (mcb_linear: one CTA per slice of output features over all
of K, warp-level tensor-core MMAs, programmatic dependent launch) and of the Block ops fused into
it (the residual add and the RMSNorm in front, the residual add behind).

Bars: the product against a torch fp32 evaluation of F.linear on the same bf16 operand,
|y - ref| <= 2^-8 |ref| + 1e-3 max|ref| (fp32 accumulation orders differ; one output rounding).
The fused ops are bit-exact: against an identity weight the normed projection returns
mcb_add_rms_norm's h bit for bit, the fused add writes mcb_add_rms_norm's x + delta, and the
residual form returns bf16(res + bf16(product))."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def _check(y, x, w):
    ref = F.linear(x.float(), w.float())
    tol = 2 ** -8 * ref.abs() + 1e-3 * ref.abs().max() + 1e-6
    assert bool(((y.float() - ref).abs() <= tol).all()), (y.float() - ref).abs().max().item()


def _rand(g, *shape, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


SHAPES = [  # R, N, K: the quickstart's projections, ragged R / N, the largest K, 32-wide slices
    (64, 2304, 768), (64, 768, 768), (64, 4096, 768), (1, 768, 768), (37, 300, 640),
    (17, 96, 64), (64, 1001, 768), (64, 768, 1408), (3, 5000, 512), (64, 8, 128),
    (64, 768, 2048), (40, 768, 2048), (20, 96, 2048),  # down_proj: two CTAs a 64-row block
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "R{}N{}K{}".format(*s))
def test_linear_matches_torch(ops, shape):
    R, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(R * 131 + N + K)
    x = _rand(g, R, K)
    w = _rand(g, N, K, scale=K ** -0.5)
    y = ops.linear(x, w)
    y_pdl = ops.linear(x, w, pdl=True)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    _check(y, x, w)
    assert torch.equal(y, y_pdl)  # the same summation order every launch


@pytest.mark.parametrize("shape", [(64, 2048, 768), (3, 2048, 768), (37, 96, 640), (64, 16, 64)],
                         ids=lambda s: "R{}H{}K{}".format(*s))
def test_gated_projection_is_silu_times_up_of_the_plain_one(ops, shape):
    """gated=True on the packed [Wg; Wu]: each output feature's sum is the same warp-ordered
    reduction as the plain projection's, so the result equals mcb_gated_silu over the plain
    projection's two halves -- and torch's F.silu(gate) * up on them -- bit for bit."""
    R, H, K = shape
    g = torch.Generator(device="cuda").manual_seed(R * 7 + H + K)
    x = _rand(g, R, K)
    w = _rand(g, 2 * H, K, scale=K ** -0.5)
    a = ops.linear(x, w, gated=True)
    a_pdl = ops.linear(x, w, gated=True, pdl=True)
    gu = ops.linear(x, w)
    want = ops.gated_silu(gu[:, :H], gu[:, H:])
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert a.shape == (R, H)
    assert torch.equal(a, want) and torch.equal(a_pdl, want)
    assert torch.equal(want, F.silu(gu[:, :H]) * gu[:, H:])


def test_linear_rejects_what_it_does_not_cover(ops):
    from modelcore_b200._native import McbError
    x = torch.zeros(65, 768, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(McbError, match="at most 64"):
        ops.linear(x, torch.zeros(64, 768, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(McbError, match="shared memory"):
        ops.linear(x[:64].new_zeros(64, 3840), torch.zeros(64, 3840, device="cuda", dtype=torch.bfloat16))


def test_linear_reads_strided_rows_and_writes_strided_output(ops):
    g = torch.Generator(device="cuda").manual_seed(4)
    big = _rand(g, 64, 3 * 768)
    x = big[:, 768:1536]
    w = _rand(g, 512, 768, scale=0.04)
    out_big = torch.zeros(64, 1024, device="cuda", dtype=torch.bfloat16)
    y = ops.linear(x, w, out=out_big[:, 256:768])
    torch.cuda.synchronize()
    _check(y, x, w)
    assert not out_big[:, :256].any() and not out_big[:, 768:].any()


@pytest.mark.parametrize("R,K", [(64, 768), (1, 768), (5, 384), (64, 1024), (33, 64)])
def test_norm_is_bit_exact(ops, R, K):
    """Against an identity weight the normed product is h itself, bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(R + K)
    x = _rand(g, R, K, scale=3.0)
    eye = torch.eye(K, device="cuda", dtype=torch.bfloat16)
    _, h = ops.add_rms_norm(x, None, eps=1e-5)
    y = ops.linear(x, eye, norm=True, eps=1e-5)
    y0 = ops.linear(x, eye, norm=True)            # eps None: fp32 machine epsilon
    _, h0 = ops.add_rms_norm(x, None)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(y, h) and torch.equal(y0, h0)


@pytest.mark.parametrize("R,K", [(64, 768), (1, 768), (7, 256), (40, 512)])
def test_add_norm_is_bit_exact(ops, R, K):
    """x' = x + delta written out and its norm: mcb_add_rms_norm's two outputs bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(R * 3 + K)
    x = _rand(g, R, K, scale=3.0)
    d = _rand(g, R, K)
    eye = torch.eye(K, device="cuda", dtype=torch.bfloat16)
    xs, h = ops.add_rms_norm(x, d, eps=1e-5)
    xo, y = ops.linear(x, eye, norm=True, delta=d, eps=1e-5, pdl=True)
    torch.cuda.synchronize()
    assert torch.equal(xo, xs) and torch.equal(y, h)


@pytest.mark.parametrize("R,N,K", [(64, 2304, 768), (64, 4096, 768), (1, 768, 768), (50, 1000, 1024)])
def test_norm_linear_matches_torch(ops, R, N, K):
    g = torch.Generator(device="cuda").manual_seed(R * 7 + N)
    x = _rand(g, R, K, scale=2.0)
    w = _rand(g, N, K, scale=K ** -0.5)
    _, h = ops.add_rms_norm(x, None)
    y = ops.linear(x, w, norm=True, pdl=True)
    torch.cuda.synchronize()
    _check(y, h, w)
    if K <= 768:
        d = _rand(g, R, K)
        _, h2 = ops.add_rms_norm(x, d)
        _, y2 = ops.linear(x, w, norm=True, delta=d)
        _check(y2, h2, w)


@pytest.mark.parametrize("R,N,K", [(64, 768, 768), (64, 768, 1024), (7, 200, 128), (64, 4096, 512)])
def test_residual_epilogue(ops, R, N, K):
    """res + product, each rounded to bf16 as torch's `x + F.linear(a, w)` rounds them; in place
    (out = res) and out of place give the same bits; against an identity weight exactly
    bf16(res + a)."""
    g = torch.Generator(device="cuda").manual_seed(R + N + K)
    a = _rand(g, R, K)
    w = _rand(g, N, K, scale=K ** -0.5)
    res = _rand(g, R, N, scale=4.0)
    want = res + ops.linear(a, w)
    got = ops.linear(a, w, res=res)
    inplace = res.clone()
    ops.linear(a, w, out=inplace, res=inplace, pdl=True)
    eye = torch.eye(K, device="cuda", dtype=torch.bfloat16)
    res_k = _rand(g, R, K, scale=4.0)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and torch.equal(inplace, want)
    assert torch.equal(ops.linear(a, eye, res=res_k), res_k + a)


def test_pdl_chain_in_a_cuda_graph(ops):
    """The fused step's order -- add + norm -> q|k|v, c_proj + residual, norm -> gate|up --
    launched with programmatic dependent launch, captured in a graph and replayed: equal to the
    eager launches without PDL."""
    g = torch.Generator(device="cuda").manual_seed(8)
    x0 = _rand(g, 64, 768)
    d0 = _rand(g, 64, 768)
    w_qkv = _rand(g, 2304, 768, scale=0.03)
    w_o = _rand(g, 768, 768, scale=0.03)
    w_gu = _rand(g, 4096, 768, scale=0.03)
    x1 = torch.empty_like(x0)

    def layer(pdl):
        _, qkv = ops.linear(x0, w_qkv, norm=True, delta=d0, x_out=x1, pdl=pdl)
        ops.linear(qkv[:, :768].contiguous(), w_o, out=x1, res=x1, pdl=pdl)
        gu = ops.linear(x1, w_gu, norm=True, pdl=pdl)
        return x1.clone(), gu

    want = layer(False)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=side):
        got = layer(True)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])


NORM_OUT_SHAPES = [  # R, N, K: config 2's c_proj (clusters of 12), ragged rows, the widest
    (64, 768, 768), (40, 768, 768), (1, 768, 768), (64, 1024, 512), (7, 128, 256), (64, 576, 1024),
    (17, 64, 64),
]


@pytest.mark.parametrize("shape", NORM_OUT_SHAPES, ids=lambda s: "R{}N{}K{}".format(*s))
def test_norm_out_is_the_residual_projection_then_add_rms_norm(ops, shape):
    """h_out: the CTAs of one output row form a cluster and meet in distributed shared memory for
    the norm.  y and h equal, bit for bit, the residual projection followed by mcb_add_rms_norm
    over its output -- in place (out = res) and out of place, with and without PDL."""
    R, N, K = shape
    if not ops.linear_supported(torch.empty(R, K, device="cuda", dtype=torch.bfloat16),
                                torch.empty(N, K, device="cuda", dtype=torch.bfloat16),
                                h_out=torch.empty(R, N, device="cuda", dtype=torch.bfloat16)):
        pytest.skip(f"the device does not schedule clusters of {N // 64}")
    g = torch.Generator(device="cuda").manual_seed(R * 3 + N + K)
    a = _rand(g, R, K)
    w = _rand(g, N, K, scale=K ** -0.5)
    res = _rand(g, R, N, scale=4.0)
    want_y = ops.linear(a, w, res=res)
    want_h = torch.empty_like(want_y)
    ops.add_rms_norm(want_y, eps=1e-6, h_out=want_h)
    y = torch.empty_like(res)
    h = torch.empty_like(res)
    ops.linear(a, w, out=y, res=res, h_out=h, eps=1e-6)
    y2 = res.clone()
    h2 = torch.full_like(res, 7.0)
    ops.linear(a, w, out=y2, res=y2, h_out=h2, eps=1e-6, pdl=True)
    # without a residual: h = rms_norm(bf16(a @ w^T))
    y3 = torch.empty_like(res)
    h3 = torch.empty_like(res)
    ops.linear(a, w, out=y3, h_out=h3, eps=1e-6)
    want_h3 = torch.empty_like(res)
    ops.add_rms_norm(ops.linear(a, w), eps=1e-6, h_out=want_h3)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(y, want_y) and torch.equal(h, want_h)
    assert torch.equal(y2, want_y) and torch.equal(h2, want_h)
    assert torch.equal(h3, want_h3)


def test_norm_out_rejects_what_it_does_not_cover(ops):
    """N a multiple of 64 up to 1024 and no other flag; h_out apart from x, y and res."""
    from modelcore_b200._native import McbError
    a = torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16)
    for N in (96, 1088):
        w = torch.zeros(N, 128, device="cuda", dtype=torch.bfloat16)
        with pytest.raises(McbError, match="multiple of 64"):
            ops.linear(a, w, h_out=torch.empty(8, N, device="cuda", dtype=torch.bfloat16))
    w = torch.zeros(128, 128, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(8, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(McbError, match="h_out must not overlap"):
        ops.linear(a, w, out=y, h_out=y)
    with pytest.raises(McbError, match="no other flag"):
        ops.linear(a, w, norm=True, h_out=torch.empty(8, 128, device="cuda", dtype=torch.bfloat16))


def test_norm_out_in_a_pdl_chain_in_a_cuda_graph(ops):
    """The default decode layer's chain -- q|k|v, c_proj with the residual add and the norm,
    gate|up with silu * up, down_proj, add + norm -- launched with programmatic dependent launch
    and replayed in a graph: equal to the eager launches without PDL."""
    g = torch.Generator(device="cuda").manual_seed(9)
    h0 = _rand(g, 64, 768)
    x0 = _rand(g, 64, 768, scale=4.0)
    w_qkv = _rand(g, 2304, 768, scale=0.03)
    w_o = _rand(g, 768, 768, scale=0.03)
    w_gu = _rand(g, 4096, 768, scale=0.03)
    w_d = _rand(g, 768, 2048, scale=0.02)
    h = h0.clone()
    x = x0.clone()
    probe = ops.linear_supported(h0, w_o, out=x, res=x, h_out=h)
    if not probe:
        pytest.skip("the device does not schedule clusters of 12")

    def layer(pdl):
        h.copy_(h0)
        x.copy_(x0)
        qkv = ops.linear(h, w_qkv, pdl=pdl)
        ops.linear(qkv[:, :768].contiguous(), w_o, out=x, res=x, h_out=h, eps=1e-6, pdl=pdl)
        act = ops.linear(h, w_gu, gated=True, pdl=pdl)
        f = ops.linear(act, w_d, pdl=pdl)
        ops.add_rms_norm(x, f, eps=1e-6, x_out=x, h_out=h)
        return x.clone(), h.clone()

    want = layer(False)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=side):
        got = layer(True)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
