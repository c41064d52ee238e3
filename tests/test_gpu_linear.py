"""GPU parity of the decode projection (mcb_linear: tcgen05 MMAs with TMEM accumulators, split-K
over a thread-block cluster with a distributed-shared-memory reduction, programmatic dependent
launch) and of its fused prologues (residual add + RMSNorm, gated silu).

Bars: the product against a torch fp32 evaluation of F.linear on the same bf16 operand,
|y - ref| <= 2^-8 |ref| + 1e-3 max|ref| (fp32 accumulation orders differ; one output rounding).
The fused operand itself is bit-exact: against an identity weight the projection returns the
operand unchanged, and that equals mcb_add_rms_norm's h / mcb_gated_silu's product bit for bit;
the fused residual x + delta equals mcb_add_rms_norm's."""
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


SHAPES = [  # R, N, K, split
    (64, 2304, 768, 0), (64, 768, 768, 0), (64, 4096, 768, 0), (64, 768, 2048, 0),
    (64, 768, 384, 1), (64, 768, 2048, 8), (64, 768, 768, 5), (128, 768, 768, 9),
    (1, 768, 768, 0), (37, 300, 640, 0), (128, 1024, 3072, 0), (100, 4096, 2048, 0),
    (17, 96, 64, 0), (64, 1001, 768, 0), (64, 768, 4096, 0),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "R{}N{}K{}s{}".format(*s))
def test_linear_matches_torch(ops, shape):
    R, N, K, split = shape
    g = torch.Generator(device="cuda").manual_seed(R * 131 + N + K)
    x = _rand(g, R, K)
    w = _rand(g, N, K, scale=K ** -0.5)
    y = ops.linear(x, w, split=split)
    y_pdl = ops.linear(x, w, split=split, pdl=True)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    _check(y, x, w)
    assert torch.equal(y, y_pdl)  # the same reduction order every launch


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


@pytest.mark.parametrize("R,K,split", [(64, 768, 0), (64, 768, 2), (64, 768, 12), (5, 384, 1),
                                       (128, 768, 0), (64, 2048, 16), (64, 2048, 0), (33, 1024, 3)])
def test_add_norm_prologue_is_bit_exact(ops, R, K, split):
    """Against an identity weight the product is h itself: the cluster's panel-ordered sum of
    squares gives mcb_add_rms_norm's bits whatever the split; x' = x + delta is written once."""
    g = torch.Generator(device="cuda").manual_seed(R + K + split)
    x = _rand(g, R, K, scale=3.0)
    d = _rand(g, R, K)
    eye = torch.eye(K, device="cuda", dtype=torch.bfloat16)
    x_ref, h_ref = ops.add_rms_norm(x, d, eps=1e-5)
    xo, y = ops.add_norm_linear(x, d, eye, eps=1e-5, split=split)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert torch.equal(xo, x_ref)
    assert torch.equal(y, h_ref)
    # no delta: h = rms_norm(x), the residual is x itself
    _, h0 = ops.add_rms_norm(x, None, eps=1e-5)
    same, y0 = ops.add_norm_linear(x, None, eye, eps=1e-5, split=split)
    assert same is x and torch.equal(y0, h0)


@pytest.mark.parametrize("R,N,K", [(64, 2304, 768), (64, 4096, 768), (1, 768, 768), (100, 1000, 1024)])
def test_add_norm_linear_matches_torch(ops, R, N, K):
    g = torch.Generator(device="cuda").manual_seed(R * 7 + N)
    x = _rand(g, R, K, scale=2.0)
    d = _rand(g, R, K)
    w = _rand(g, N, K, scale=K ** -0.5)
    _, h = ops.add_rms_norm(x, d)
    xo, y = ops.add_norm_linear(x, d, w, pdl=True)
    torch.cuda.synchronize()
    _check(y, h, w)


@pytest.mark.parametrize("R,H,split", [(64, 2048, 0), (64, 2048, 8), (7, 384, 1), (128, 1536, 0)])
def test_gated_silu_prologue_is_bit_exact(ops, R, H, split):
    g = torch.Generator(device="cuda").manual_seed(R + H)
    gu = _rand(g, R, 2 * H, scale=3.0)
    gate, up = gu[:, :H], gu[:, H:]
    eye = torch.eye(H, device="cuda", dtype=torch.bfloat16)
    a = ops.gated_silu(gate, up)
    y = ops.silu_linear(gate, up, eye, split=split)
    torch.cuda.synchronize()
    assert torch.equal(y, a)
    w = _rand(g, 768, H, scale=H ** -0.5)
    _check(ops.silu_linear(gate, up, w, pdl=True), a, w)


def test_pdl_chain_in_a_cuda_graph(ops):
    """The fused step's order -- add+norm -> projection, projection, add+norm -> projection,
    silu -> projection -- launched with programmatic dependent launch, captured in a graph and
    replayed: equal to the eager launches without PDL."""
    g = torch.Generator(device="cuda").manual_seed(8)
    x0 = _rand(g, 64, 768)
    d0 = _rand(g, 64, 768)
    w_qkv = _rand(g, 2304, 768, scale=0.03)
    w_o = _rand(g, 768, 768, scale=0.03)
    w_gu = _rand(g, 4096, 768, scale=0.03)
    w_d = _rand(g, 768, 2048, scale=0.03)
    bufs = [torch.empty_like(x0), torch.empty_like(x0)]

    def layer(pdl):
        x1, qkv = ops.add_norm_linear(x0, d0, w_qkv, x_out=bufs[0], pdl=pdl)
        o = ops.linear(qkv[:, :768].contiguous(), w_o, pdl=pdl)
        x2, gu = ops.add_norm_linear(x1, o, w_gu, x_out=bufs[1], pdl=pdl)
        return x2.clone(), ops.silu_linear(gu[:, :2048], gu[:, 2048:], w_d, pdl=pdl)

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
