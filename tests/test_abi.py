"""The C-ABI library on the CPU: it loads without a GPU, exports every symbol include/mcb200.h
declares, its ctypes structures match the C layout (checked against gcc), and host-side argument
checks reject bad input with a status and a message before anything touches a device."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO
from modelcore_b200 import _native
from modelcore_b200._native import (AddNormArgs, AppendArgs, AttnArgs, CopyArgs, EmbedArgs,
                                    GatedSiluArgs, LinearArgs, SampleArgs, SoftcapArgs)

HEADER = os.path.join(REPO, "include", "mcb200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|uint64_t)\s+(mcb_\w+)\s*\(", text, re.M)))


def test_library_loads_and_reports_its_abi_version():
    lib = _native.load()
    assert lib.mcb_abi_version() == _native.ABI_VERSION == 9


def test_every_declared_symbol_is_exported():
    lib = _native.load()
    declared = declared_functions()
    assert len(declared) >= 9
    assert sorted(_native.EXPORTED_SYMBOLS) == declared
    for name in declared:
        assert hasattr(lib, name), name


def _c_layout(struct, fields):
    src = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
           f'printf("%zu\\n", sizeof({struct}));']
    src += [f'printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    src += ["return 0;}"]
    tmp = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"mcb_layout_{struct}_{os.getpid()}")
    with open(tmp + ".c", "w") as fh:
        fh.write("\n".join(src))
    subprocess.run(["gcc", "-O0", "-o", tmp, tmp + ".c"], check=True)
    out = subprocess.run([tmp], check=True, capture_output=True, text=True).stdout.split()
    os.unlink(tmp)
    os.unlink(tmp + ".c")
    return [int(x) for x in out]


@pytest.mark.parametrize("cls,cname", [(AppendArgs, "mcb_append_args"), (CopyArgs, "mcb_copy_args"),
                                       (AttnArgs, "mcb_attn_args"), (AddNormArgs, "mcb_add_norm_args"),
                                       (GatedSiluArgs, "mcb_gated_silu_args"), (EmbedArgs, "mcb_embed_args"),
                                       (SoftcapArgs, "mcb_softcap_args"), (SampleArgs, "mcb_sample_args"),
                                       (LinearArgs, "mcb_linear_args")])
def test_ctypes_structures_match_the_c_layout(cls, cname):
    fields = [f for f, _ in cls._fields_]
    c = _c_layout(cname, fields)
    assert c[0] == ctypes.sizeof(cls)
    assert c[1:] == [getattr(cls, f).offset for f in fields]


def _err(status):
    return status, _native.last_error()


def test_append_rejects_bad_arguments_on_the_host():
    lib = _native.load()
    st, msg = _err(lib.mcb_kv_append_rope(None, None))
    assert st == _native.MCB_ERR_INVALID_ARG and "NULL" in msg
    a = AppendArgs()
    a.B, a.T, a.D = 1, 1, 64
    a.flags = 0
    st, msg = _err(lib.mcb_kv_append_rope(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "flags 0" in msg
    a.flags = _native.MCB_APPEND_ROTATE_K
    st, msg = _err(lib.mcb_kv_append_rope(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "WRITE_KV" in msg
    a.flags = 1 << 7
    st, msg = _err(lib.mcb_kv_append_rope(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "unknown flags" in msg
    a.flags = _native.MCB_APPEND_WRITE_KV
    a.cache_seqlens = 16
    st, msg = _err(lib.mcb_kv_append_rope(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "WRITE_KV needs" in msg


def test_copy_rejects_out_of_range_rows_and_lengths():
    lib = _native.load()
    a = CopyArgs()
    a.n_slots, a.src_batch, a.src_row, a.src_tmax = 2, 1, 0, 8
    a.dst_batch, a.dst_row_begin, a.dst_row_count, a.dst_tmax = 4, 3, 2, 16
    a.n_pos, a.row_elems = 4, 64
    st, msg = _err(lib.mcb_kv_copy_rows(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "out of range" in msg
    a.dst_row_begin, a.dst_row_count, a.n_pos = 0, 4, 9
    st, msg = _err(lib.mcb_kv_copy_rows(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "exceed cache length" in msg
    a.n_pos, a.row_elems = 4, 12
    st, msg = _err(lib.mcb_kv_copy_rows(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_ALIGNMENT


def _attn(**kw):
    a = AttnArgs()
    a.B, a.T, a.Hq, a.Hkv, a.D, a.Tmax, a.window = 2, 1, 8, 2, 128, 64, -1
    a.softmax_scale = 0.088
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_attention_rejects_unsupported_shapes_without_a_device():
    lib = _native.load()
    a = _attn(D=48)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "head_dim 48" in msg
    assert lib.mcb_decode_attn_workspace_size(ctypes.byref(a)) == 0
    a = _attn(Hq=6, Hkv=4)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "divisible" in msg
    a = _attn()  # NULL pointers
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "NULL" in msg


def test_attention_workspace_is_per_persistent_cta_not_per_length():
    lib = _native.load()
    r256 = lambda x: (x + 255) // 256 * 256
    # rows = 8 (T=1, G=4), D=128: per CTA two partial slots of 8 rows x (128 + 1) fp32; the grid
    # is whole groups of Hkv (= 2) CTAs, at least one group
    for asked, ctas in ((1, 2), (4, 4), (5, 4), (300, 300)):
        want = r256(ctas * 2 * 8 * 128 * 4) + r256(ctas * 2 * 8 * 4)
        for tmax in (64, 4096):
            a = _attn(num_ctas=asked, Tmax=tmax)
            assert lib.mcb_decode_attn_workspace_size(ctypes.byref(a)) == want
            assert lib.mcb_decode_attn_counter_count(ctypes.byref(a)) == 2 * 1 * 2  # B x blocks x Hkv
    # 16 rows per group when T * G > 8: T=3, G=4 -> 12 rows -> one query block
    a = _attn(num_ctas=2, T=3)
    assert lib.mcb_decode_attn_workspace_size(ctypes.byref(a)) == r256(2 * 2 * 16 * 128 * 4) + r256(2 * 2 * 16 * 4)
    # T=5, G=4 -> 20 rows -> two query blocks of 16
    assert lib.mcb_decode_attn_counter_count(ctypes.byref(_attn(num_ctas=2, T=5))) == 2 * 2 * 2


def test_split_plan_counters_only_for_partials_through_memory():
    """A split plan merged inside a cluster (up to 8 splits without a device, 16 where the device
    schedules clusters of 16) needs no workspace and no counters; more splits publish partials and
    count arrivals per row group."""
    lib = _native.load()
    for splits, partials in ((4, False), (8, False), (20, True), (40, True)):
        a = _attn(num_ctas=-splits, Tmax=4096)
        ws = lib.mcb_decode_attn_workspace_size(ctypes.byref(a))
        cnt = lib.mcb_decode_attn_counter_count(ctypes.byref(a))
        assert (ws > 0) == partials and cnt == (2 * 1 * 2 if partials else 0), (splits, ws, cnt)


def test_attention_checks_the_workspace_before_launching():
    lib = _native.load()
    a = _attn(num_ctas=4, q=0x1000, k_cache=0x2000, v_cache=0x3000, out=0x4000,
              cache_seqlens=0x5000)
    a.q_stride[:] = (8 * 128, 8 * 128, 128)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_WORKSPACE and "workspace" in msg
    a.workspace, a.workspace_bytes = 0x100000, 1 << 20  # enough partials, no counters
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_WORKSPACE and "counters" in msg
    a.q_stride[:] = (8 * 128, 8 * 128, 100)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_ALIGNMENT


def test_advance_rejects_null():
    lib = _native.load()
    st, _ = _err(lib.mcb_kv_advance(None, 4, 1, None))
    assert st == _native.MCB_ERR_INVALID_ARG


def test_step_kernels_validate_on_the_host():
    """Shape and alignment errors are reported before any launch (no device needed)."""
    lib = _native.load()
    MCB_ERR_UNSUPPORTED, MCB_ERR_ALIGNMENT = _native.MCB_ERR_UNSUPPORTED, _native.MCB_ERR_ALIGNMENT
    MCB_ERR_INVALID_ARG = _native.MCB_ERR_INVALID_ARG
    a = AddNormArgs()
    a.x, a.h_out, a.rows, a.C = 16, 32, 4, 12
    assert lib.mcb_add_rms_norm(ctypes.byref(a), None) == MCB_ERR_UNSUPPORTED
    a.C = 4104
    assert lib.mcb_add_rms_norm(ctypes.byref(a), None) == MCB_ERR_UNSUPPORTED
    a.C, a.x = 64, 18
    assert lib.mcb_add_rms_norm(ctypes.byref(a), None) == MCB_ERR_ALIGNMENT
    a.x, a.delta = 16, 48          # delta without x_out
    assert lib.mcb_add_rms_norm(ctypes.byref(a), None) == MCB_ERR_INVALID_ARG
    g = GatedSiluArgs()
    g.gate, g.up, g.out, g.rows, g.H = 16, 32, 48, 2, 20
    assert lib.mcb_gated_silu(ctypes.byref(g), None) == MCB_ERR_UNSUPPORTED
    g.H, g.gate_stride, g.up_stride, g.out_stride = 16, 20, 16, 16
    assert lib.mcb_gated_silu(ctypes.byref(g), None) == MCB_ERR_ALIGNMENT
    g.gate_stride, g.rows = 16, 0
    assert lib.mcb_gated_silu(ctypes.byref(g), None) == 0   # nothing to do, nothing launched


def test_embedding_and_lm_head_epilogue_validate_on_the_host():
    lib = _native.load()
    e = EmbedArgs()
    e.ids, e.table, e.x_out, e.rows, e.C, e.V = 16, 32, 48, 2, 20, 100
    assert lib.mcb_embed_rms_norm(ctypes.byref(e), None) == _native.MCB_ERR_UNSUPPORTED
    e.C, e.V = 64, 0
    assert lib.mcb_embed_rms_norm(ctypes.byref(e), None) == _native.MCB_ERR_INVALID_ARG
    e.V, e.table_stride, e.x_stride = 100, 68, 64
    assert lib.mcb_embed_rms_norm(ctypes.byref(e), None) == _native.MCB_ERR_ALIGNMENT
    s = SoftcapArgs()
    s.logits, s.rows, s.V, s.logits_stride = 16, 2, 1000, 999
    s.argmax = 64
    assert lib.mcb_softcap_argmax(ctypes.byref(s), None) == _native.MCB_ERR_INVALID_ARG
    s.logits_stride, s.argmax = 1024, None
    assert lib.mcb_softcap_argmax(ctypes.byref(s), None) == _native.MCB_ERR_INVALID_ARG


def test_sampler_validates_on_the_host():
    lib = _native.load()
    a = SampleArgs()
    a.logits, a.uniforms, a.out, a.rows, a.V, a.logits_stride = 16, 32, 48, 2, 1000, 1000
    a.temperature = 0.0
    assert lib.mcb_sample(ctypes.byref(a), None) == _native.MCB_ERR_INVALID_ARG
    a.temperature = 1.0
    a.V, a.logits_stride, a.top_k, a.rows = 5000, 5000, 2000, 0  # any top_k < V is accepted
    assert lib.mcb_sample(ctypes.byref(a), None) == 0
    a.top_k, a.logits = 50, None
    assert lib.mcb_sample(ctypes.byref(a), None) == _native.MCB_ERR_INVALID_ARG


def test_ring_slots_are_validated_on_the_host():
    """A ring slot must hold every visible key: window >= 0, window + T <= Tmax, Tmax a multiple
    of 128 (so no 64- or 128-key tile wraps)."""
    lib = _native.load()
    for kw in (dict(window=-1, Tmax=1024), dict(window=1000, T=30, Tmax=1024),
               dict(window=100, Tmax=1000)):
        a = _attn(**kw)
        a.ring = 1
        st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
        assert st == _native.MCB_ERR_INVALID_ARG and "ring" in msg


def test_linear_rejects_bad_arguments_on_the_host():
    """Every case fails in the host checks, before any launch (the pointers are never read)."""
    lib = _native.load()
    base = 1 << 20

    def args(**kw):
        a = LinearArgs()
        a.x, a.w, a.y = base, base + (1 << 20), base + (2 << 20)
        a.x_stride = a.w_stride = a.y_stride = 768
        a.R, a.N, a.K = 64, 768, 768
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=8)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "flags" in msg
    assert lib.mcb_linear_supported(ctypes.byref(args())) == 1
    assert lib.mcb_linear_supported(ctypes.byref(args(flags=8))) == 0
    # the norm out: N a multiple of 64 up to 1024, no other flag, h_out given, aligned and apart
    nout, h = _native.LINEAR_NORM_OUT, base + (3 << 20)
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=nout | _native.LINEAR_GATED, h_out=h,
                                                    h_out_stride=768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "no other flag" in msg
    for n in (96, 1088):
        st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=nout, N=n, y_stride=n, h_out=h,
                                                        h_out_stride=n)), None))
        assert st == _native.MCB_ERR_UNSUPPORTED and "multiple of 64" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=nout)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "NULL" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=nout, h_out=h + 8, h_out_stride=768)), None))
    assert st == _native.MCB_ERR_ALIGNMENT and "h_out" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=nout, h_out=base + (2 << 20) + 64,
                                                    h_out_stride=768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "h_out must not overlap" in msg
    assert lib.mcb_linear_supported(ctypes.byref(args(flags=nout, h_out=h + 8, h_out_stride=768))) == 0
    # the gated projection stands alone: no norm, delta or res, and N a multiple of 16
    gated = _native.LINEAR_GATED
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=gated | _native.LINEAR_NORM)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "GATED" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=gated, res=base + (3 << 20), res_stride=768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "GATED" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=gated, N=24, y_stride=24)), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "multiple of 16" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(K=96, x_stride=96, w_stride=96)), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "multiple of 64" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(R=65)), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "at most 64" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(delta=base + (3 << 20), delta_stride=768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "delta needs" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=_native.LINEAR_NORM, delta=base + (3 << 20),
                                                    delta_stride=768, x_out=base + 1024, x_out_stride=768)),
                                  None))
    assert st == _native.MCB_ERR_INVALID_ARG and "overlap" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(flags=_native.LINEAR_NORM, K=1088, x_stride=1088,
                                                    w_stride=1088)), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "1024" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(x=base + 8)), None))
    assert st == _native.MCB_ERR_ALIGNMENT
    # every CTA reads all of x: the output must not overlap it
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(y=base + 64 * 768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "overlap" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(res=base + (2 << 20) + 16, res_stride=768)), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "res" in msg
    st, msg = _err(lib.mcb_linear(ctypes.byref(args(K=64 * 400, x_stride=64 * 400, w_stride=64 * 400,
                                                    x=base, w=base + (8 << 20), y=base + (16 << 20))),
                                  None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "shared memory" in msg


def test_fused_append_is_offered_only_where_the_decode_kernels_can_do_it():
    """mcb_decode_attn_fusable decides from the shapes on the host: one new token a row, a bf16
    slot, head size 64 or 128 and the split or persistent plan; a fused call outside that is
    rejected before any launch (the pointers are never read)."""
    lib = _native.load()
    fusable = lambda **kw: lib.mcb_decode_attn_fusable(ctypes.byref(_attn(**kw)))
    assert fusable() == 1                                     # 2 rows, 64-position slot: split
    assert fusable(D=64, Hq=4, Hkv=4) == 1
    assert fusable(B=200, Tmax=65536) == 1                    # many groups of long rows: persistent
    assert fusable(num_ctas=16) == 1                          # persistent, a given grid
    assert fusable(T=2) == 0                                  # several new tokens
    assert fusable(T=64) == 0                                 # the prefill plan
    assert fusable(D=32) == 0
    assert fusable(k_scale=1 << 20, v_scale=1 << 21, scale_tmax=64) == 0   # an fp8 slot
    a = _attn(T=2, q=0x1000, k_cache=0x2000, v_cache=0x3000, out=0x4000, cache_seqlens=0x5000,
              fuse_append=1, rot_cos=0x6000, rot_sin=0x7000, rot_len=64)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_UNSUPPORTED and "fuses only" in msg
    a = _attn(q=0x1000, k_cache=0x2000, v_cache=0x3000, out=0x4000, cache_seqlens=0x5000,
              fuse_append=1, rot_len=64)
    st, msg = _err(lib.mcb_decode_attn(ctypes.byref(a), None))
    assert st == _native.MCB_ERR_INVALID_ARG and "rot_cos" in msg
