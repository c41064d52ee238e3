"""ctypes binding of libmcb200.so (the C ABI declared in include/mcb200.h).

The structures below mirror the header field for field.  Loading fails loudly: there is no
Python or CPU fallback for any entry point, so a missing or stale library is an error, not a
slower path.
"""
import ctypes
import os
import threading

from .build import LIB_PATH

MCB_OK = 0
MCB_ERR_INVALID_ARG = -1
MCB_ERR_UNSUPPORTED = -2
MCB_ERR_ALIGNMENT = -3
MCB_ERR_WORKSPACE = -4
MCB_ERR_CUDA = -5
STATUS_NAMES = {
    MCB_ERR_INVALID_ARG: "MCB_ERR_INVALID_ARG",
    MCB_ERR_UNSUPPORTED: "MCB_ERR_UNSUPPORTED",
    MCB_ERR_ALIGNMENT: "MCB_ERR_ALIGNMENT",
    MCB_ERR_WORKSPACE: "MCB_ERR_WORKSPACE",
    MCB_ERR_CUDA: "MCB_ERR_CUDA",
}

MCB_APPEND_ROTATE_Q = 1
MCB_APPEND_ROTATE_K = 2
MCB_APPEND_WRITE_KV = 4

DEVICE_ERRORS = {
    0: "none",
    1: "position beyond the cache length (Tmax)",
    2: "position beyond the rotary table",
    3: "pipeline wait timed out",
    4: "token id outside the embedding table",
}

ABI_VERSION = 9

# Size of the static scratch behind mcb_decode_attn_noalloc (MCB_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 8 << 20

# Every entry point include/mcb200.h declares.
EXPORTED_SYMBOLS = (
    "mcb_abi_version",
    "mcb_last_error",
    "mcb_kv_append_rope",
    "mcb_kv_copy_rows",
    "mcb_kv_advance",
    "mcb_decode_attn_workspace_size",
    "mcb_decode_attn_counter_count",
    "mcb_decode_attn_fusable",
    "mcb_decode_attn",
    "mcb_decode_attn_noalloc",
    "mcb_add_rms_norm",
    "mcb_gated_silu",
    "mcb_embed_rms_norm",
    "mcb_prefill_attn",
    "mcb_sample",
    "mcb_linear",
    "mcb_linear_supported",
    "mcb_softcap_argmax",
    "mcb_device_error",
    "mcb_launch_count",
    "mcb_last_attn_kernel",
)

_i64x3 = ctypes.c_int64 * 3


class AppendArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("q_stride", _i64x3), ("k_stride", _i64x3), ("v_stride", _i64x3),
        ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("cache_seqlens", ctypes.c_void_p),
        ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32), ("D", ctypes.c_int32), ("Tmax", ctypes.c_int32),
        ("rot_len", ctypes.c_int32),
        ("eps", ctypes.c_float), ("scale", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("ring", ctypes.c_int32),
        ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p),
        ("scale_tmax", ctypes.c_int32),
    ]


class CopyArgs(ctypes.Structure):
    _fields_ = [
        ("dst_k", ctypes.c_void_p), ("dst_v", ctypes.c_void_p),
        ("src_k", ctypes.c_void_p), ("src_v", ctypes.c_void_p),
        ("n_slots", ctypes.c_int32),
        ("src_batch", ctypes.c_int32), ("src_row", ctypes.c_int32), ("src_tmax", ctypes.c_int32),
        ("dst_batch", ctypes.c_int32), ("dst_row_begin", ctypes.c_int32),
        ("dst_row_count", ctypes.c_int32), ("dst_tmax", ctypes.c_int32),
        ("n_pos", ctypes.c_int32), ("row_elems", ctypes.c_int32),
        ("dst_seqlens", ctypes.c_void_p),
    ]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("q_stride", _i64x3),
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("cache_seqlens", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32), ("D", ctypes.c_int32), ("Tmax", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("num_ctas", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("counters", ctypes.c_void_p), ("counter_count", ctypes.c_size_t),
        ("ring", ctypes.c_int32),
        ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p),
        ("scale_tmax", ctypes.c_int32),
        ("fuse_append", ctypes.c_int32),
        ("k_new", ctypes.c_void_p), ("v_new", ctypes.c_void_p),
        ("k_new_stride", _i64x3), ("v_new_stride", _i64x3),
        ("rot_cos", ctypes.c_void_p), ("rot_sin", ctypes.c_void_p),
        ("rot_len", ctypes.c_int32), ("rotate_k", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("qk_scale", ctypes.c_float),
    ]


class AddNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("x_out", ctypes.c_void_p),
        ("h_out", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64), ("delta_stride", ctypes.c_int64),
        ("x_out_stride", ctypes.c_int64), ("h_stride", ctypes.c_int64),
        ("rows", ctypes.c_int32), ("C", ctypes.c_int32), ("eps", ctypes.c_float),
    ]


class GatedSiluArgs(ctypes.Structure):
    _fields_ = [
        ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("gate_stride", ctypes.c_int64), ("up_stride", ctypes.c_int64), ("out_stride", ctypes.c_int64),
        ("rows", ctypes.c_int32), ("H", ctypes.c_int32),
    ]


class EmbedArgs(ctypes.Structure):
    _fields_ = [
        ("ids", ctypes.c_void_p), ("table", ctypes.c_void_p), ("x_out", ctypes.c_void_p),
        ("h_out", ctypes.c_void_p),
        ("table_stride", ctypes.c_int64), ("x_stride", ctypes.c_int64), ("h_stride", ctypes.c_int64),
        ("V", ctypes.c_int64), ("rows", ctypes.c_int32), ("C", ctypes.c_int32), ("eps", ctypes.c_float),
    ]


class SoftcapArgs(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("out", ctypes.c_void_p), ("argmax", ctypes.c_void_p),
        ("logits_stride", ctypes.c_int64), ("out_stride", ctypes.c_int64),
        ("argmax_stride", ctypes.c_int64),
        ("rows", ctypes.c_int32), ("V", ctypes.c_int32), ("softcap", ctypes.c_float),
    ]


class SampleArgs(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("uniforms", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("logits_stride", ctypes.c_int64), ("out_stride", ctypes.c_int64),
        ("rows", ctypes.c_int32), ("V", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("temperature", ctypes.c_float),
    ]


LINEAR_NORM = 1
LINEAR_GATED = 2
LINEAR_NORM_OUT = 4


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("res", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("x_out", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64), ("w_stride", ctypes.c_int64), ("y_stride", ctypes.c_int64),
        ("res_stride", ctypes.c_int64), ("delta_stride", ctypes.c_int64),
        ("x_out_stride", ctypes.c_int64),
        ("R", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32),
        ("flags", ctypes.c_int32), ("eps", ctypes.c_float), ("pdl", ctypes.c_int32),
        ("h_out", ctypes.c_void_p), ("h_out_stride", ctypes.c_int64),
    ]


class McbError(RuntimeError):
    """A C-ABI call returned a non-zero mcb_status."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P = ctypes.POINTER
    lib.mcb_abi_version.restype = ctypes.c_int
    lib.mcb_abi_version.argtypes = []
    lib.mcb_last_error.restype = ctypes.c_int
    lib.mcb_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.mcb_kv_append_rope.restype = ctypes.c_int
    lib.mcb_kv_append_rope.argtypes = [P(AppendArgs), ctypes.c_void_p]
    lib.mcb_kv_copy_rows.restype = ctypes.c_int
    lib.mcb_kv_copy_rows.argtypes = [P(CopyArgs), ctypes.c_void_p]
    lib.mcb_kv_advance.restype = ctypes.c_int
    lib.mcb_kv_advance.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
    lib.mcb_decode_attn_workspace_size.restype = ctypes.c_size_t
    lib.mcb_decode_attn_workspace_size.argtypes = [P(AttnArgs)]
    lib.mcb_decode_attn_counter_count.restype = ctypes.c_size_t
    lib.mcb_decode_attn_fusable.restype = ctypes.c_int
    lib.mcb_decode_attn_fusable.argtypes = [P(AttnArgs)]
    lib.mcb_decode_attn_counter_count.argtypes = [P(AttnArgs)]
    lib.mcb_decode_attn.restype = ctypes.c_int
    lib.mcb_decode_attn.argtypes = [P(AttnArgs), ctypes.c_void_p]
    lib.mcb_decode_attn_noalloc.restype = ctypes.c_int
    lib.mcb_decode_attn_noalloc.argtypes = [P(AttnArgs), ctypes.c_void_p]
    lib.mcb_add_rms_norm.restype = ctypes.c_int
    lib.mcb_add_rms_norm.argtypes = [P(AddNormArgs), ctypes.c_void_p]
    lib.mcb_gated_silu.restype = ctypes.c_int
    lib.mcb_gated_silu.argtypes = [P(GatedSiluArgs), ctypes.c_void_p]
    lib.mcb_linear.restype = ctypes.c_int
    lib.mcb_linear.argtypes = [P(LinearArgs), ctypes.c_void_p]
    lib.mcb_linear_supported.restype = ctypes.c_int
    lib.mcb_linear_supported.argtypes = [P(LinearArgs)]
    lib.mcb_sample.restype = ctypes.c_int
    lib.mcb_sample.argtypes = [P(SampleArgs), ctypes.c_void_p]
    lib.mcb_prefill_attn.restype = ctypes.c_int
    lib.mcb_prefill_attn.argtypes = [P(AttnArgs), ctypes.c_void_p]
    lib.mcb_embed_rms_norm.restype = ctypes.c_int
    lib.mcb_embed_rms_norm.argtypes = [P(EmbedArgs), ctypes.c_void_p]
    lib.mcb_softcap_argmax.restype = ctypes.c_int
    lib.mcb_softcap_argmax.argtypes = [P(SoftcapArgs), ctypes.c_void_p]
    lib.mcb_device_error.restype = ctypes.c_int
    lib.mcb_device_error.argtypes = [P(ctypes.c_int32), ctypes.c_void_p]
    lib.mcb_launch_count.restype = ctypes.c_uint64
    lib.mcb_launch_count.argtypes = []
    lib.mcb_last_attn_kernel.restype = ctypes.c_int
    lib.mcb_last_attn_kernel.argtypes = [ctypes.c_char_p, ctypes.c_size_t]


def lib_path():
    return os.environ.get("MCB200_LIBRARY", LIB_PATH)


def load():
    """Returns the loaded library; raises if it is missing, stale or of another ABI version."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"libmcb200.so not found at {path}: build it with `python -m modelcore_b200.build` "
                "(the KV decode path has no fallback without it)")
        lib = ctypes.CDLL(path)
        missing = [n for n in EXPORTED_SYMBOLS if not hasattr(lib, n)]
        if missing:
            raise RuntimeError(f"{path} is stale (missing {', '.join(missing)}); rebuild it with "
                               "`python -m modelcore_b200.build`")
        _declare(lib)
        ver = lib.mcb_abi_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"{path} has ABI version {ver}, expected {ABI_VERSION}; rebuild it")
        _lib = lib
        return lib


def last_error():
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.mcb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status):
    if status != MCB_OK:
        raise McbError(status, last_error())
