"""mcb_decode_attn_noalloc: decode attention for callers that cannot allocate device memory.

A host that owns all of its device memory up front (a serving engine with pre-carved pools) or a
binding with no device allocator cannot hand mcb_decode_attn a workspace; this entry point keeps
the split partials in the library's static 8 MiB per-GPU scratch instead.  These tests call it
through the C ABI twice in a row, on new inputs each time (the scratch keeps the previous call's
contents), and compare each result with the existing entry point's (mcb_decode_attn with a
workspace) within the attention tolerance of the other tests.  The file sorts last so a run that
stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from modelcore_b200 import _native, ops

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-2  # max-abs, bf16 output, as in test_gpu_kernels.py


def _inputs(seed, B, Hq, Hkv, D, Tmax):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lens = np.random.default_rng(seed).integers(0, Tmax, size=B)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Tmax, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    return q, kc, vc, torch.from_numpy(lens).to(torch.int32).cuda()


def _call_noalloc(q, kc, vc, sl, out, window, num_ctas):
    """One call of the new entry point through the C ABI (ctypes, raw pointers, current stream)."""
    args = ops._attn_args(q, kc, vc, sl, window, None, num_ctas, out)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _native.load().mcb_decode_attn_noalloc(ctypes.byref(args), stream)


SHAPES = [
    # B, Hq, Hkv, D, Tmax, window, num_ctas (0: automatic plan, persistent for these rows --
    # long, and more than 128 row groups;
    # > 0 persistent grid; < 0 split plan with that many key splits -- more than 16, so its
    # partials go through memory: up to 16 splits merge inside a cluster and need none)
    (32, 32, 8, 128, 8192, -1, 0),
    (4, 12, 12, 64, 3000, 100, 24),
    (4, 12, 12, 64, 1000, -1, -20),
    # two row groups of one long row cut into 19 splits: a small grid, so the split that arrives
    # last merges the partials through the arrival counters, which each call clears first
    (1, 16, 2, 128, 8192, -1, -20),
]


@pytest.mark.parametrize("shape", SHAPES, ids=["cfg5-like-auto", "mha-d64-window-24-ctas",
                                               "mha-d64-17-splits", "gqa-d128-19-splits-counters"])
def test_noalloc_matches_the_allocating_entry_point_on_two_calls_in_a_row(shape):
    B, Hq, Hkv, D, Tmax, window, splits = shape
    for call, seed in enumerate((11, 12)):
        q, kc, vc, sl = _inputs(seed, B, Hq, Hkv, D, Tmax)
        need = ops.decode_attn_workspace_bytes(q, kc, vc, sl, window=window, num_ctas=splits)
        assert 0 < need <= _native.NOALLOC_SCRATCH_BYTES  # partials live in the scratch
        if shape == SHAPES[3]:
            assert ops.decode_attn_counter_count(q, kc, vc, sl, window=window, num_ctas=splits) > 0
        expected = ops.decode_attn(q, kc, vc, sl, window=window, num_ctas=splits)
        out = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = _call_noalloc(q, kc, vc, sl, out, window, splits)
        assert st == _native.MCB_OK, _native.last_error()
        torch.cuda.synchronize()
        if call == 1:  # after the first call has set up the scratch address on this device
            assert torch.cuda.mem_get_info()[0] >= free_before - (2 << 20)
        err = (out.float() - expected.float()).abs().max().item()
        assert err <= ATTN_TOL, (call, err)
        assert ops.device_error()[0] == 0


def test_noalloc_rejects_a_grid_whose_partials_exceed_its_scratch():
    B, Hq, Hkv, D, Tmax = 64, 32, 8, 128, 4096
    q, kc, vc, sl = _inputs(3, B, Hq, Hkv, D, Tmax)
    assert ops.decode_attn_workspace_bytes(q, kc, vc, sl, num_ctas=4096) > _native.NOALLOC_SCRATCH_BYTES
    out = torch.zeros_like(q)
    st = _call_noalloc(q, kc, vc, sl, out, -1, 4096)
    assert st == _native.MCB_ERR_WORKSPACE
    assert "static scratch" in _native.last_error() and "persistent CTAs" in _native.last_error()
    # a split plan whose partials do not fit: the message asks for fewer splits
    assert _call_noalloc(q, kc, vc, sl, out, -1, -64) == _native.MCB_ERR_WORKSPACE
    assert "key splits" in _native.last_error() and "fewer splits" in _native.last_error()
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0  # nothing was enqueued
    # with fewer CTAs the same shape fits and matches
    out2 = ops.decode_attn_noalloc(q, kc, vc, sl, num_ctas=64)
    ref = ops.decode_attn(q, kc, vc, sl, num_ctas=64)
    assert (out2.float() - ref.float()).abs().max().item() <= ATTN_TOL


def test_cluster_merged_splits_need_no_scratch():
    """Up to 8 key splits of a row group merge through distributed shared memory: the plan needs
    no partials at all, so the no-alloc entry point serves it without touching the scratch."""
    q, kc, vc, sl = _inputs(3, 4, 12, 12, 64, 1000)
    assert ops.decode_attn_workspace_bytes(q, kc, vc, sl, num_ctas=-3) == 0
    out = torch.empty_like(q)
    assert _call_noalloc(q, kc, vc, sl, out, -1, -3) == _native.MCB_OK
    expected = ops.decode_attn(q, kc, vc, sl, num_ctas=-12)
    torch.cuda.synchronize()
    assert (out.float() - expected.float()).abs().max().item() <= ATTN_TOL
