"""GPU parity of the decode projection (mcb_linear: tcgen05, TMEM accumulators, split-K over a
cluster with a distributed-shared-memory reduction, programmatic dependent launch) against a
torch fp32 evaluation of F.linear on the same bf16 inputs.

Bar: |y - ref| <= 1e-2 * max|ref| + one bf16 rounding of ref (the only rounding is the output's;
fp32 accumulation orders differ)."""
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


SHAPES = [  # R, N, K, split
    (64, 2304, 768, 0), (64, 768, 768, 0), (64, 4096, 768, 0), (64, 768, 2048, 0),
    (64, 768, 768, 1), (64, 768, 2048, 8), (64, 768, 768, 3),
    (1, 768, 768, 0), (37, 300, 640, 0), (128, 1024, 5632, 0), (256, 512, 1024, 0),
    (200, 4096, 2048, 0), (17, 96, 64, 0),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "R{}N{}K{}s{}".format(*s))
def test_linear_matches_torch(ops, shape):
    R, N, K, split = shape
    g = torch.Generator(device="cuda").manual_seed(R * 131 + N + K)
    x = torch.randn(R, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    y = ops.linear(x, w, split=split)
    y_pdl = ops.linear(x, w, split=split, pdl=True)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    _check(y, x, w)
    assert torch.equal(y, y_pdl)


def test_linear_reads_strided_rows_and_writes_strided_output(ops):
    g = torch.Generator(device="cuda").manual_seed(4)
    big = torch.randn(64, 3 * 768, device="cuda", generator=g).to(torch.bfloat16)
    x = big[:, 768:1536]
    w = (torch.randn(512, 768, device="cuda", generator=g) * 0.04).to(torch.bfloat16)
    out_big = torch.zeros(64, 1024, device="cuda", dtype=torch.bfloat16)
    y = ops.linear(x, w, out=out_big[:, 256:768])
    torch.cuda.synchronize()
    _check(y, x, w)
    assert not out_big[:, :256].any() and not out_big[:, 768:].any()


def test_pdl_chain_in_a_cuda_graph(ops):
    """Projections launched with programmatic dependent launch, back to back and captured in a
    graph, each reading the previous one's output: the chain equals the eager, unchained one."""
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(64, 768, device="cuda", generator=g).to(torch.bfloat16)
    ws = [(torch.randn(768, 768, device="cuda", generator=g) * 0.03).to(torch.bfloat16) for _ in range(6)]
    def chain(pdl):
        h = x
        for w in ws:
            h = ops.linear(h, w, pdl=pdl)
        return h
    want = chain(False)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=side):
        got = chain(True)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(got, want)
