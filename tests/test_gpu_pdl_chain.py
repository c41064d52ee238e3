"""Decode steps made only of this library's kernels, launched back to back with programmatic
dependent launch, must equal the same steps with the device synchronised after every launch.

Every kernel of the library lets the next one start only after its own griddepcontrol.wait has
returned, and the advance never lets it start early; the decode attention reads cache_seqlens and
the key tiles of earlier steps before its own wait.  In a chain of append -> attention -> advance
-> append -> ... with nothing else between the launches, that order is what keeps those early
reads off data a still-running kernel writes (in the model's step, cuBLAS projections sit between
the launches and serialise them anyway).  The chain runs three ways -- synchronised after every
launch, back to back on one stream, and as one CUDA graph -- and the attention outputs, the cache
bytes and the lengths must agree bit for bit.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 24

CASES = [  # B, Hq, Hkv, D, Tmax, window, fused, num_ctas (two-launch path only)
    (16, 12, 12, 64, 512, -1, True, 0),      # config 2's layout, one split per row group
    (1, 32, 8, 128, 4096, -1, True, 0),      # batch 1, long rows: splits merged in a cluster
    (4, 16, 4, 128, 1024, 300, True, 0),     # a window
    (2, 32, 8, 128, 2048, -1, False, -20),   # two launches; partials merged by the last split
    (16, 32, 8, 128, 2048, -1, False, -20),  # two launches; partials and the combine kernel
    (64, 12, 12, 64, 1024, -1, False, 0),    # two launches, the append kernel ahead of each attention
]


def _tables(rot_len, D):
    ang = torch.arange(rot_len, dtype=torch.float32)[:, None] * \
        (10000.0 ** (-torch.arange(0, D, 2, dtype=torch.float32) / D))[None]
    return ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()


def _steps(ops, case, state, inputs, sync):
    B, Hq, Hkv, D, Tmax, window, fused, nc = case
    kc, vc, sl = state
    cos, sin = inputs["tables"]
    outs = []
    for s in range(STEPS):
        q, k, v = inputs["q"][s], inputs["k"][s], inputs["v"][s]
        if fused:
            outs.append(ops.append_attn(q, k, v, kc, vc, sl, cos, sin, window=window))
            if sync:
                torch.cuda.synchronize()
        else:
            qr = ops.kv_append_rope(q, k, v, kc, vc, sl, cos, sin)
            if sync:
                torch.cuda.synchronize()
            outs.append(ops.decode_attn(qr, kc, vc, sl, window=window, num_ctas=nc))
            if sync:
                torch.cuda.synchronize()
        ops.kv_advance(sl, 1)
        if sync:
            torch.cuda.synchronize()
    return outs


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}Hq{}Hkv{}D{}w{}{}n{}".format(
    c[0], c[1], c[2], c[3], c[5], "fused" if c[6] else "two", c[7]))
def test_back_to_back_steps_equal_synchronised_steps(case):
    from modelcore_b200 import ops
    B, Hq, Hkv, D, Tmax, window, fused, nc = case
    g = torch.Generator(device="cuda").manual_seed(B * 31 + Hq + D)
    kc0 = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc0 = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    lo, hi = Tmax // 4, Tmax // 2
    sl0 = torch.randint(lo, hi, (B,), device="cuda", generator=g, dtype=torch.int32)
    inputs = {
        "q": [torch.randn(B, 1, Hq, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(STEPS)],
        "k": [torch.randn(B, 1, Hkv, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(STEPS)],
        "v": [torch.randn(B, 1, Hkv, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(STEPS)],
        "tables": _tables(Tmax + STEPS, D),
    }

    def fresh():
        return kc0.clone(), vc0.clone(), sl0.clone()

    ref_state = fresh()
    ref = _steps(ops, case, ref_state, inputs, sync=True)
    eager_state = fresh()
    eager = _steps(ops, case, eager_state, inputs, sync=False)
    torch.cuda.synchronize()

    graph_state = fresh()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        captured = _steps(ops, case, graph_state, inputs, sync=False)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()

    for name, (outs, state) in (("back to back", (eager, eager_state)), ("graph", (captured, graph_state))):
        for s in range(STEPS):
            assert torch.equal(outs[s], ref[s]), f"{name}: attention output of step {s} differs"
        assert torch.equal(state[0], ref_state[0]) and torch.equal(state[1], ref_state[1]), f"{name}: cache"
        assert torch.equal(state[2], ref_state[2]), f"{name}: cache_seqlens"
    assert torch.equal(ref_state[2], sl0 + STEPS)
    assert ops.device_error()[0] == 0
    del graph
