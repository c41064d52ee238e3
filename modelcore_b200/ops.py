"""Torch-facing wrappers of the C-ABI entry points.

Each wrapper checks device, dtype, shape and layout on the host (no device sync), passes raw
pointers and the current CUDA stream to libmcb200 and returns.  All of them are safe inside
CUDA-graph capture: they only enqueue kernels; the attention workspace is a cached per-device
buffer (allocated the first time, outside capture when the first call is eager).  None has a
CPU path: non-CUDA or non-bf16 tensors raise.
"""
import ctypes
import math

import torch

from . import _native
from ._native import (AddNormArgs, AppendArgs, AttnArgs, CopyArgs, EmbedArgs, GatedSiluArgs,
                      LINEAR_GATED, LINEAR_NORM, LINEAR_NORM_OUT, LinearArgs, SampleArgs,
                      SoftcapArgs, check)


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need(name, t, ndim=None, dtype=torch.bfloat16):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: modelcore_b200 has no CPU path (got {t.device})")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise RuntimeError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")


def _bthd_strides(name, t):
    if t.stride(3) != 1:
        raise RuntimeError(f"{name} must have unit stride on head_dim, got strides {t.stride()}")
    return (t.stride(0), t.stride(1), t.stride(2))


FP8 = torch.float8_e4m3fn


def fp8_scale_tmax(Tmax):
    """Positions per (row, kv head) in an fp8 cache's scale arrays: T_max rounded up to 64 (a key
    tile's scales are read as one 256-byte block)."""
    return (int(Tmax) + 63) // 64 * 64


def fp8_scales(B, Hkv, Tmax, device, n_slots=None):
    """Zeroed per-vector scales for an fp8 (e4m3) cache slot: (B, Hkv, fp8_scale_tmax(Tmax))
    fp32, or (n_slots, B, Hkv, ...) for a whole cache."""
    shape = (B, Hkv, fp8_scale_tmax(Tmax))
    if n_slots is not None:
        shape = (n_slots,) + shape
    return torch.zeros(shape, dtype=torch.float32, device=device)


def _check_fp8_scales(name, sc, k_cache):
    B, Tmax, Hkv, _ = k_cache.shape
    _need(name, sc, 3, torch.float32)
    if tuple(sc.shape) != (B, Hkv, fp8_scale_tmax(Tmax)) or not sc.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous ({B}, {Hkv}, {fp8_scale_tmax(Tmax)}) float32 tensor")
    if sc.data_ptr() % 256:
        raise RuntimeError(f"{name} must be 256-byte aligned")


def _check_slot_cache(name, c, B, Hkv, D):
    _need(name, c, 4, c.dtype if isinstance(c, torch.Tensor) and c.dtype == FP8 else torch.bfloat16)
    if not c.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous (B, T_max, H_kv, D) cache slot")
    if c.size(0) != B or c.size(2) != Hkv or c.size(3) != D:
        raise RuntimeError(f"{name} has shape {tuple(c.shape)}, expected ({B}, T_max, {Hkv}, {D})")
    if c.data_ptr() % 16:
        raise RuntimeError(f"{name} must be 16-byte aligned")


def _check_seqlens(cache_seqlens, B, device):
    _need("cache_seqlens", cache_seqlens, 1, torch.int32)
    if cache_seqlens.numel() != B or not cache_seqlens.is_contiguous():
        raise RuntimeError(f"cache_seqlens must be a contiguous ({B},) int32 tensor")
    if cache_seqlens.device != device:
        raise RuntimeError("cache_seqlens is on another device")


def rms_norm_eps(eps):
    """The epsilon torch's F.rms_norm applies to bf16 input: fp32 machine epsilon when None
    (the opmath type's epsilon), otherwise the given value in fp32."""
    return torch.finfo(torch.float32).eps if eps is None else float(eps)


def kv_append_rope(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin, *, rotate_q=True,
                   rotate_k=True, write_kv=True, eps=None, scale=1.2, q_out=None, ring=False,
                   k_scale=None, v_scale=None):
    """Fused rope + QK-norm + scale for q (and k), and the insert of k, v at each row's position.

    q: (B, T, Hq, D) bf16 or None; k, v: (B, T, Hkv, D) bf16 or None; k_cache/v_cache: one slot
    (B, T_max, Hkv, D); cos/sin: the rotary buffers (1, rot_len, 1, D/2) bf16 of
    modelcore.components.rotary.RotaryEmbedding.  Returns the rotated q (a new (B, T, Hq, D)
    tensor, or q_out) when rotate_q, else None.  cache_seqlens is not advanced.

    An fp8 slot (k_cache/v_cache of dtype float8_e4m3fn, D 64 or 128) stores each new vector as
    e4m3 with a per-vector scale in k_scale / v_scale (fp8_scales): the bf16 vector x a bf16
    cache would hold, as e4m3(x * 448 / max|x|) and scale max|x| / 448."""
    flags = 0
    ref = q if rotate_q else k
    if ref is None:
        raise RuntimeError("kv_append_rope: nothing to do")
    _need("q" if rotate_q else "k", ref, 4)
    B, T = ref.shape[0], ref.shape[1]
    D = ref.shape[3]
    args = AppendArgs()
    if rotate_q:
        flags |= _native.MCB_APPEND_ROTATE_Q
        Hq = q.shape[2]
        if q_out is None:
            q_out = torch.empty((B, T, Hq, D), dtype=torch.bfloat16, device=q.device)
        else:
            _need("q_out", q_out, 4)
            if tuple(q_out.shape) != (B, T, Hq, D) or not q_out.is_contiguous():
                raise RuntimeError("q_out must be a contiguous tensor shaped like q")
        args.q = q.data_ptr()
        args.q_stride[:] = _bthd_strides("q", q)
        args.q_out = q_out.data_ptr()
        args.Hq = Hq
    if rotate_k:
        flags |= _native.MCB_APPEND_ROTATE_K
    if write_kv:
        flags |= _native.MCB_APPEND_WRITE_KV
        _need("k", k, 4)
        _need("v", v, 4)
        Hkv = k.shape[2]
        if tuple(k.shape) != (B, T, Hkv, D) or tuple(v.shape) != (B, T, Hkv, D):
            raise RuntimeError(f"k and v must be ({B}, {T}, H_kv, {D}), got {tuple(k.shape)}, {tuple(v.shape)}")
        _check_slot_cache("k_cache", k_cache, B, Hkv, D)
        _check_slot_cache("v_cache", v_cache, B, Hkv, D)
        if v_cache.size(1) != k_cache.size(1):
            raise RuntimeError("k_cache and v_cache lengths differ")
        args.k = k.data_ptr()
        args.v = v.data_ptr()
        args.k_stride[:] = _bthd_strides("k", k)
        args.v_stride[:] = _bthd_strides("v", v)
        args.k_cache = k_cache.data_ptr()
        args.v_cache = v_cache.data_ptr()
        args.Hkv = Hkv
        args.Tmax = k_cache.size(1)
        if (k_cache.dtype == FP8) != (v_cache.dtype == FP8):
            raise RuntimeError("k_cache and v_cache must both be bf16 or both fp8")
        if k_cache.dtype == FP8:
            if k_scale is None or v_scale is None:
                raise RuntimeError("an fp8 cache slot needs k_scale and v_scale")
            _check_fp8_scales("k_scale", k_scale, k_cache)
            _check_fp8_scales("v_scale", v_scale, k_cache)
            args.k_scale, args.v_scale = k_scale.data_ptr(), v_scale.data_ptr()
            args.scale_tmax = k_scale.size(2)
    elif rotate_k:
        raise RuntimeError("rotate_k requires write_kv")
    _check_seqlens(cache_seqlens, B, ref.device)
    if rotate_q or rotate_k:
        for name, tab in (("cos", cos), ("sin", sin)):
            _need(name, tab)
            if not tab.is_contiguous() or tab.shape[-1] != D // 2:
                raise RuntimeError(f"rotary {name} table must be contiguous with D/2={D // 2} columns")
        args.cos = cos.data_ptr()
        args.sin = sin.data_ptr()
        args.rot_len = cos.numel() // (D // 2)
    args.cache_seqlens = cache_seqlens.data_ptr()
    args.B, args.T, args.D = B, T, D
    args.eps = rms_norm_eps(eps)
    args.scale = scale
    args.flags = flags
    args.ring = int(bool(ring))
    check(_native.load().mcb_kv_append_rope(ctypes.byref(args), _stream(ref)))
    return q_out


def kv_write(k, v, k_cache, v_cache, cache_seqlens):
    """Inserts already-processed k, v (B, T, Hkv, D) at rows' positions [L_b, L_b + T): the
    in-place cache write of flash_attn_with_kvcache (modelcore/kernels/flash_attn.py:337-346)."""
    kv_append_rope(None, k, v, k_cache, v_cache, cache_seqlens, None, None, rotate_q=False,
                   rotate_k=False, write_kv=True)


def kv_copy_rows(dst_k, dst_v, src_k, src_v, *, src_row, dst_row_begin, dst_row_count, n_pos,
                 dst_seqlens=None):
    """Copies positions [0, n_pos) of source row src_row, every slot, into destination rows
    [dst_row_begin, dst_row_begin + dst_row_count); optionally sets dst_seqlens for those rows.
    Caches are full (n_slots, B, T_max, Hkv, D) tensors."""
    if dst_k.dtype == FP8:  # e4m3 bytes move as pairs: the same kernel on a bf16 view
        if not all(t.dtype == FP8 for t in (dst_v, src_k, src_v)):
            raise RuntimeError("k and v caches must all be fp8 or all bf16")
        dst_k, dst_v, src_k, src_v = (t.view(torch.bfloat16) for t in (dst_k, dst_v, src_k, src_v))
    for name, t in (("dst_k", dst_k), ("dst_v", dst_v), ("src_k", src_k), ("src_v", src_v)):
        _need(name, t, 5)
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
    if dst_k.shape != dst_v.shape or src_k.shape != src_v.shape:
        raise RuntimeError("k and v caches must have equal shapes")
    S, Bd, Td, H, D = dst_k.shape
    Ss, Bs, Ts, Hs, Ds = src_k.shape
    if (S, H, D) != (Ss, Hs, Ds):
        raise RuntimeError(f"cache layouts differ: dst {tuple(dst_k.shape)} vs src {tuple(src_k.shape)}")
    args = CopyArgs()
    args.dst_k, args.dst_v = dst_k.data_ptr(), dst_v.data_ptr()
    args.src_k, args.src_v = src_k.data_ptr(), src_v.data_ptr()
    args.n_slots = S
    args.src_batch, args.src_row, args.src_tmax = Bs, src_row, Ts
    args.dst_batch, args.dst_row_begin, args.dst_row_count, args.dst_tmax = Bd, dst_row_begin, dst_row_count, Td
    args.n_pos = n_pos
    args.row_elems = H * D
    if dst_seqlens is not None:
        _check_seqlens(dst_seqlens, Bd, dst_k.device)
        args.dst_seqlens = dst_seqlens.data_ptr()
    check(_native.load().mcb_kv_copy_rows(ctypes.byref(args), _stream(dst_k)))


def kv_advance(cache_seqlens, n):
    """cache_seqlens += n on the device (KVCache.advance, modelcore/cache.py:71)."""
    _need("cache_seqlens", cache_seqlens, 1, torch.int32)
    check(_native.load().mcb_kv_advance(ctypes.c_void_p(cache_seqlens.data_ptr()),
                                        cache_seqlens.numel(), int(n), _stream(cache_seqlens)))


def _attn_args(q, k_cache, v_cache, cache_seqlens, window, softmax_scale, num_ctas, out, ring=False,
               k_scale=None, v_scale=None):
    _need("q", q, 4)
    B, T, Hq, D = q.shape
    Hkv = k_cache.shape[2] if k_cache.dim() == 4 else -1
    _check_slot_cache("k_cache", k_cache, B, Hkv, D)
    _check_slot_cache("v_cache", v_cache, B, Hkv, D)
    if v_cache.shape != k_cache.shape:
        raise RuntimeError("k_cache and v_cache shapes differ")
    _check_seqlens(cache_seqlens, B, q.device)
    if Hq % Hkv:
        raise RuntimeError(f"n_head ({Hq}) must be divisible by n_kv_head ({Hkv})")
    args = AttnArgs()
    args.q = q.data_ptr()
    args.q_stride[:] = _bthd_strides("q", q)
    args.k_cache, args.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    args.cache_seqlens = cache_seqlens.data_ptr()
    args.out = out.data_ptr() if out is not None else 0
    args.B, args.T, args.Hq, args.Hkv, args.D, args.Tmax = B, T, Hq, Hkv, D, k_cache.shape[1]
    args.window = -1 if window is None or window < 0 else int(window)
    args.softmax_scale = (1.0 / math.sqrt(D)) if softmax_scale is None else float(softmax_scale)
    args.num_ctas = int(num_ctas)
    args.ring = int(bool(ring))
    if k_cache.dtype == FP8:
        if v_cache.dtype != FP8 or k_scale is None or v_scale is None:
            raise RuntimeError("an fp8 cache slot needs fp8 k_cache and v_cache, k_scale and v_scale")
        _check_fp8_scales("k_scale", k_scale, k_cache)
        _check_fp8_scales("v_scale", v_scale, k_cache)
        args.k_scale, args.v_scale = k_scale.data_ptr(), v_scale.data_ptr()
        args.scale_tmax = k_scale.size(2)
    return args


def decode_attn_counter_count(q, k_cache, v_cache, cache_seqlens, *, window=-1, num_ctas=0,
                              ring=False):
    """Arrival counters the launch plan needs: one per row group for the persistent plan and for
    a split plan on a small grid whose partials go through memory (its last split to finish
    merges them); 0 for a split plan merged in a cluster or by the combine kernel."""
    args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, None, num_ctas, None, ring)
    return int(_native.load().mcb_decode_attn_counter_count(ctypes.byref(args)))


def decode_attn_workspace_bytes(q, k_cache, v_cache, cache_seqlens, *, window=-1, num_ctas=0,
                                ring=False):
    args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, None, num_ctas, None, ring)
    return int(_native.load().mcb_decode_attn_workspace_size(ctypes.byref(args)))


_WORKSPACES = {}  # device index -> partial-result buffers (grown on demand)
_COUNTERS = {}    # device index -> zero-initialised arrival-counter arrays (grown on demand)


def _grow(cache, device, n, dtype, zero):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    bufs = cache.setdefault(idx, [])
    if not bufs or bufs[-1].numel() < n:
        make = torch.zeros if zero else torch.empty
        bufs.append(make(max(n, 1 << 16), dtype=dtype, device=device))  # older ones stay alive:
    return bufs[-1]                                                     # a CUDA graph may hold them


def attn_workspace(device, nbytes):
    """The per-device partials buffer decode_attn uses when none is passed."""
    return _grow(_WORKSPACES, device, nbytes, torch.uint8, zero=False)


def attn_counters(device, count):
    """The per-device arrival counters decode_attn uses when none are passed: allocated
    zero-filled; every completed call leaves the counters it used at zero again, so one array
    serves every call on the device, CUDA-graph replays included.  Calls that can overlap on the
    GPU must pass their own workspace and counters."""
    return _grow(_COUNTERS, device, count, torch.int32, zero=True)


def reset_counters():
    """Zero the cached counter arrays again (after a call that reported a device error)."""
    for bufs in _COUNTERS.values():
        for b in bufs:
            b.zero_()


def decode_attn(q, k_cache, v_cache, cache_seqlens, *, window=-1, softmax_scale=None,
                num_ctas=0, out=None, workspace=None, counters=None, ring=False, k_scale=None,
                v_scale=None):
    """softmax(q . K^T * scale) . V over each row's visible keys of one cache slot.

    q: (B, T, Hq, D) bf16; k_cache/v_cache: (B, T_max, Hkv, D) bf16 slot; query t of row b sits at
    cache_seqlens[b] + t and sees keys c <= that position within `window` (< 0: all).  The new
    tokens must already be in the cache.  num_ctas: 0 picks the launch plan; > 0 a persistent grid
    of that many CTAs dividing all key tiles; < 0 one CTA per row group and key split, -num_ctas
    splits (every plan gives the same result up to fp32 summation order).  workspace: uint8
    partials buffer; counters: int32 arrival counters, zero before their first use (defaults:
    the cached per-device ones).  ring: the slot is a ring of T_max positions (key c at index
    c % T_max; needs window >= 0 and window + T <= T_max, T_max a multiple of 128).  An fp8 slot
    (float8_e4m3fn, with the k_scale / v_scale kv_append_rope filled) is read as e4m3 * scale, on
    the split plan.  Returns out (B, T, Hq, D) bf16."""
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    else:
        _need("out", out, 4)
        if out.shape != q.shape or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous tensor shaped like q")
    args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, softmax_scale, num_ctas, out, ring,
                      k_scale, v_scale)
    lib = _native.load()
    need = int(lib.mcb_decode_attn_workspace_size(ctypes.byref(args)))
    ncount = int(lib.mcb_decode_attn_counter_count(ctypes.byref(args)))
    if need:
        if workspace is None:
            workspace = attn_workspace(q.device, need)
        elif workspace.numel() < need:
            raise RuntimeError(f"workspace of {workspace.numel()} bytes, {need} needed")
        args.workspace = workspace.data_ptr()
        args.workspace_bytes = workspace.numel()
    if ncount:
        if counters is None:
            counters = attn_counters(q.device, ncount)
        elif counters.dtype != torch.int32 or counters.numel() < ncount:
            raise RuntimeError(f"counters must be >= {ncount} zero-initialised int32")
        args.counters = counters.data_ptr()
        args.counter_count = counters.numel()
    check(lib.mcb_decode_attn(ctypes.byref(args), _stream(q)))
    return out


def append_attn(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin, *, eps=None, scale=1.2,
                rotate_k=True, window=-1, ring=False, out=None, k_scale=None, v_scale=None):
    """kv_append_rope followed by decode_attn -- one decode step of an attention layer from its
    RAW projections q (B, T, Hq, D), k, v (B, T, Hkv, D; None for a layer that reads another
    layer's slot) -- in ONE launch where the plan allows it (T = 1, a bf16 slot, D = 64 or 128,
    the split or persistent plan: mcb_decode_attn_fusable), with the same bits as the two
    launches; otherwise the two launches.  cache_seqlens is not advanced.  Returns the
    attention output."""
    T, D = q.size(1), q.size(3)
    fusable = k_cache.dtype == torch.bfloat16 and T == 1 and D in (64, 128)
    if fusable:
        if out is None:
            out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
        args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, None, 0, out, ring)
        lib = _native.load()
        fusable = bool(lib.mcb_decode_attn_fusable(ctypes.byref(args)))
    if not fusable:
        if k is not None:
            q = kv_append_rope(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin, rotate_q=True,
                               rotate_k=rotate_k, write_kv=True, eps=eps, scale=scale, ring=ring,
                               k_scale=k_scale, v_scale=v_scale)
        else:
            q = kv_append_rope(q, None, None, None, None, cache_seqlens, cos, sin, rotate_q=True,
                               rotate_k=False, write_kv=False, eps=eps, scale=scale)
        return decode_attn(q, k_cache, v_cache, cache_seqlens, window=window, ring=ring, out=out,
                           k_scale=k_scale, v_scale=v_scale)
    if not out.is_contiguous() or out.shape != q.shape:
        raise RuntimeError("out must be a contiguous tensor shaped like q")
    args.fuse_append = 1
    if k is not None:
        _need("k", k, 4)
        _need("v", v, 4)
        if (k.shape != v.shape or k.shape[0] != q.shape[0] or k.shape[1] != 1
                or k.shape[2] != k_cache.shape[2] or k.shape[3] != D):
            raise RuntimeError("k and v must be (B, 1, Hkv, D) like the slot")
        args.k_new, args.v_new = k.data_ptr(), v.data_ptr()
        args.k_new_stride[:] = _bthd_strides("k", k)
        args.v_new_stride[:] = _bthd_strides("v", v)
    for name, tab in (("cos", cos), ("sin", sin)):
        _need(name, tab)
        if not tab.is_contiguous() or tab.shape[-1] != D // 2:
            raise RuntimeError(f"rotary {name} table must be contiguous with D/2={D // 2} columns")
    args.rot_cos, args.rot_sin = cos.data_ptr(), sin.data_ptr()
    args.rot_len = cos.numel() // (D // 2)
    args.rotate_k = int(bool(rotate_k))
    args.norm_eps = rms_norm_eps(eps)
    args.qk_scale = scale
    need = int(lib.mcb_decode_attn_workspace_size(ctypes.byref(args)))
    ncount = int(lib.mcb_decode_attn_counter_count(ctypes.byref(args)))
    if need:
        ws = attn_workspace(q.device, need)
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    if ncount:
        cnt = attn_counters(q.device, ncount)
        args.counters, args.counter_count = cnt.data_ptr(), cnt.numel()
    check(lib.mcb_decode_attn(ctypes.byref(args), _stream(q)))
    return out


def prefill_attn(q, k_cache, v_cache, cache_seqlens, *, window=-1, softmax_scale=None, out=None,
                 ring=False):
    """decode_attn's semantics on the tensor-core prefill kernel (mcb_prefill_attn), for any T:
    128-query tiles, S = Q K^T and O += P V as tcgen05 MMAs with TMEM accumulators.  head_dim 64
    or 128.  decode_attn picks this plan itself for T >= 64 with num_ctas=0."""
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    else:
        _need("out", out, 4)
        if out.shape != q.shape or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous tensor shaped like q")
    args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, softmax_scale, 0, out, ring)
    check(_native.load().mcb_prefill_attn(ctypes.byref(args), _stream(q)))
    return out


def decode_attn_noalloc(q, k_cache, v_cache, cache_seqlens, *, window=-1, softmax_scale=None,
                        num_ctas=0, out=None):
    """decode_attn through mcb_decode_attn_noalloc: for callers that cannot allocate device
    memory (a host whose HBM is all carved into its own pools, or a binding without a device
    allocator).  The partials go to the library's static 8 MiB per-GPU scratch instead of a
    workspace; a grid whose partials need more raise McbError(MCB_ERR_WORKSPACE).  Calls that
    can overlap on the GPU share that scratch and race: keep them on one stream.  `out` must be
    given by such a caller; when it is None this wrapper allocates it (torch), for tests."""
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    else:
        _need("out", out, 4)
        if out.shape != q.shape or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous tensor shaped like q")
    args = _attn_args(q, k_cache, v_cache, cache_seqlens, window, softmax_scale, num_ctas, out)
    check(_native.load().mcb_decode_attn_noalloc(ctypes.byref(args), _stream(q)))
    return out


def _rows2d(name, t):
    _need(name, t, 2)
    if t.stride(1) != 1:
        raise RuntimeError(f"{name} must have unit stride on its last dim")
    return t.stride(0)


def add_rms_norm(x, delta=None, *, eps=None, x_out=None, h_out=None):
    """x' = x + delta (bf16), h = rms_norm(x') (bf16): Block's residual add fused with the next
    norm (modelcore/components/block.py:57-59, norm.py:43-44).  x, delta: (rows, C) bf16.
    Returns (x', h); with delta None returns (x, rms_norm(x)).  x_out may be x (in place)."""
    rows, C = x.shape
    args = AddNormArgs()
    args.x = x.data_ptr()
    args.x_stride = _rows2d("x", x)
    if h_out is None:
        h_out = torch.empty((rows, C), dtype=torch.bfloat16, device=x.device)
    args.h_out = h_out.data_ptr()
    args.h_stride = _rows2d("h_out", h_out)
    if delta is not None:
        if tuple(delta.shape) != (rows, C):
            raise RuntimeError(f"delta must be ({rows}, {C}), got {tuple(delta.shape)}")
        args.delta = delta.data_ptr()
        args.delta_stride = _rows2d("delta", delta)
        if x_out is None:
            x_out = torch.empty((rows, C), dtype=torch.bfloat16, device=x.device)
        args.x_out = x_out.data_ptr()
        args.x_out_stride = _rows2d("x_out", x_out)
    else:
        x_out = x
    args.rows, args.C = rows, C
    args.eps = rms_norm_eps(eps)
    check(_native.load().mcb_add_rms_norm(ctypes.byref(args), _stream(x)))
    return x_out, h_out


def embed_rms_norm(ids, table, *, eps=None, second_norm=True, x_out=None, h_out=None):
    """TokenEmbedding without smear (wte lookup + norm, modelcore/components/embedding.py:71-75)
    and, with second_norm, the first block's norm of its output, in one launch.  ids: int64 of
    any shape; table: (V, C) bf16.  Returns (x, h) shaped ids.shape + (C,) (h None without
    second_norm).  An id outside [0, V) sets device error 4 and yields zeros."""
    if ids.dtype != torch.int64 or not ids.is_cuda:
        raise RuntimeError("ids must be an int64 CUDA tensor")
    V, C = table.shape
    flat = ids.reshape(-1)
    if not flat.is_contiguous():
        flat = flat.contiguous()
    rows = flat.numel()
    if x_out is None:
        x_out = torch.empty((rows, C), dtype=torch.bfloat16, device=ids.device)
    if second_norm and h_out is None:
        h_out = torch.empty((rows, C), dtype=torch.bfloat16, device=ids.device)
    args = EmbedArgs()
    args.ids = flat.data_ptr()
    args.table, args.table_stride = table.data_ptr(), _rows2d("table", table)
    args.x_out, args.x_stride = x_out.data_ptr(), _rows2d("x_out", x_out)
    if second_norm:
        args.h_out, args.h_stride = h_out.data_ptr(), _rows2d("h_out", h_out)
    args.V, args.rows, args.C = V, rows, C
    args.eps = rms_norm_eps(eps)
    check(_native.load().mcb_embed_rms_norm(ctypes.byref(args), _stream(table)))
    shape = tuple(ids.shape) + (C,)
    return x_out.view(shape), (h_out.view(shape) if second_norm else None)


def softcap_argmax(logits, vocab_size, softcap, *, out=None, want_logits=True, argmax_out=None):
    """LMHead's epilogue (modelcore/components/unembedding.py:52-56): crop the (..., V_padded)
    bf16 logits to vocab_size, .float(), and cap * tanh(x / cap) (softcap None: no cap); with
    argmax_out (an int64 tensor holding one id per row), also the greedy pick of
    sample_next_token(temperature=0) (modelcore/generate.py:23-24).  Returns the fp32 logits
    shaped (..., vocab_size), or None when want_logits is False."""
    _need("logits", logits)
    lead = tuple(logits.shape[:-1])
    lg = logits.reshape(-1, logits.shape[-1])
    if lg.stride(-1) != 1:
        raise RuntimeError("logits must have unit stride on the vocab dim")
    rows = lg.shape[0]
    args = SoftcapArgs()
    args.logits, args.logits_stride = lg.data_ptr(), lg.stride(0)
    if want_logits:
        if out is None:
            out = torch.empty(lead + (vocab_size,), dtype=torch.float32, device=logits.device)
        o2 = out.view(rows, vocab_size)
        args.out, args.out_stride = o2.data_ptr(), o2.stride(0)
    if argmax_out is not None:
        if argmax_out.dtype != torch.int64 or argmax_out.numel() != rows:
            raise RuntimeError(f"argmax_out must hold {rows} int64 ids")
        args.argmax = argmax_out.data_ptr()
        args.argmax_stride = argmax_out.reshape(-1).stride(0)
    args.rows, args.V = rows, vocab_size
    args.softcap = float(softcap) if softcap is not None else 0.0
    check(_native.load().mcb_softcap_argmax(ctypes.byref(args), _stream(logits)))
    return out if want_logits else None


def sample(logits, uniforms, *, temperature=1.0, top_k=None, out=None):
    """One token per row of fp32 logits (B, V): sample_next_token (modelcore/generate.py:19-34)
    for temperature > 0 with the draw at the given uniforms (B,) in [0, 1) -- the inverse CDF over
    the top_k candidates in descending-logit order (ties by index), or over the whole row in index
    order.  temperature == 0 is the greedy pick (top_k = 1).  Returns out (B, 1) int64."""
    _need("logits", logits, 2, dtype=torch.float32)
    rows, V = logits.shape
    if logits.stride(1) != 1:
        raise RuntimeError("logits must have unit stride on the vocab dim")
    if uniforms.dtype != torch.float32 or uniforms.numel() != rows or not uniforms.is_cuda:
        raise RuntimeError(f"uniforms must be {rows} float32 values on the GPU")
    if out is None:
        out = torch.empty((rows, 1), dtype=torch.int64, device=logits.device)
    args = SampleArgs()
    args.logits, args.logits_stride = logits.data_ptr(), logits.stride(0)
    u = uniforms.reshape(-1)
    if not u.is_contiguous():
        u = u.contiguous()
    args.uniforms = u.data_ptr()
    args.out, args.out_stride = out.data_ptr(), out.reshape(-1).stride(0)
    args.rows, args.V = rows, V
    if temperature == 0:
        args.top_k, args.temperature = 1, 1.0
    else:
        if temperature < 0:
            raise RuntimeError("temperature must be non-negative")
        args.top_k = int(top_k) if top_k is not None and top_k > 0 else 0
        args.temperature = float(temperature)
    check(_native.load().mcb_sample(ctypes.byref(args), _stream(logits)))
    return out


LINEAR_MAX_ROWS = 64


def _linear_args(x, weight, out, res, norm, delta, x_out, eps, pdl, gated, h_out):
    R, K = x.shape
    N = weight.shape[0] // 2 if gated else weight.shape[0]
    args = LinearArgs()
    args.x, args.x_stride = x.data_ptr(), _rows2d("x", x)
    args.w, args.w_stride = weight.data_ptr(), _rows2d("weight", weight)
    args.y, args.y_stride = out.data_ptr(), _rows2d("out", out)
    if res is not None:
        if tuple(res.shape) != (R, N):
            raise RuntimeError(f"res must be ({R}, {N}), got {tuple(res.shape)}")
        args.res, args.res_stride = res.data_ptr(), _rows2d("res", res)
    if delta is not None:
        if tuple(delta.shape) != (R, K):
            raise RuntimeError(f"delta must be ({R}, {K}), got {tuple(delta.shape)}")
        args.delta, args.delta_stride = delta.data_ptr(), _rows2d("delta", delta)
        args.x_out, args.x_out_stride = x_out.data_ptr(), _rows2d("x_out", x_out)
    if h_out is not None:
        if tuple(h_out.shape) != (R, N):
            raise RuntimeError(f"h_out must be ({R}, {N}), got {tuple(h_out.shape)}")
        args.h_out, args.h_out_stride = h_out.data_ptr(), _rows2d("h_out", h_out)
    args.R, args.N, args.K = R, N, K
    args.flags = ((LINEAR_NORM if norm else 0) | (LINEAR_GATED if gated else 0)
                  | (LINEAR_NORM_OUT if h_out is not None else 0))
    args.eps = rms_norm_eps(eps)
    args.pdl = int(bool(pdl))
    return args


def linear_supported(x, weight, *, out=None, res=None, norm=False, delta=None, eps=None,
                     gated=False, h_out=None):
    """Whether linear() with these arguments runs on the current device (mcb_linear_supported:
    the same host-side checks, nothing launched)."""
    R, K = x.shape
    N = weight.shape[0] // 2 if gated else weight.shape[0]
    if out is None:
        out = torch.empty((R, N), dtype=torch.bfloat16, device=x.device)
    x_out = torch.empty((R, K), dtype=torch.bfloat16, device=x.device) if delta is not None else None
    args = _linear_args(x, weight, out, res, norm, delta, x_out, eps, False, gated, h_out)
    return bool(_native.load().mcb_linear_supported(ctypes.byref(args)))


def linear(x, weight, *, out=None, res=None, norm=False, delta=None, x_out=None, eps=None,
           pdl=False, gated=False, h_out=None):
    """F.linear(x, weight) without bias (modelcore/components/linear.py:14) for the decode step's
    rows -- x (R, K) with R <= 64 and K a multiple of 64, weight (N, K), bf16, fp32 accumulation
    -- with the Block's elementwise ops around it fused in:

      norm=True   rms_norm(x, eps) @ weight^T (modelcore/components/norm.py:43-44; the bits of
                  add_rms_norm's h), K <= 1024;
      delta       (with norm) x' = x + delta is written to x_out (allocated when None) and
                  normed: the residual add of the previous block's MLP, K <= 768;
      res         res + (x @ weight^T), each rounded to bf16 (the residual add after c_proj,
                  modelcore/components/block.py:58); out may be res (in place);
      gated=True  weight is the packed [Wg; Wu] (2H, K) and out (R, H) = silu(x @ Wg^T) *
                  (x @ Wu^T) with mcb_gated_silu's rounding (GatedMLP, modelcore/components/
                  mlp.py:89-90); H a multiple of 16, no norm, delta or res;
      h_out       also h_out (R, N) = rms_norm(out, eps): c_proj's residual add and the Block's
                  next norm (block.py:58-59) in one launch, the bits of add_rms_norm over out;
                  N a multiple of 64 up to 1024, no norm, delta or gated (linear_supported says
                  whether the device schedules it).

    pdl: launch with programmatic stream serialization (the weight slice streams in while the
    previous kernel finishes).  Returns out (R, N), or (x_out, out) with delta."""
    R, K = x.shape
    N = weight.shape[0]
    if gated:
        if N % 2 or norm or delta is not None or res is not None:
            raise RuntimeError("gated: weight must be [Wg; Wu] (2H rows); no norm, delta or res")
        N //= 2
    if weight.shape[1] != K:
        raise RuntimeError(f"weight must be (N, {K}), got {tuple(weight.shape)}")
    if out is None:
        out = torch.empty((R, N), dtype=torch.bfloat16, device=x.device)
    if delta is not None and x_out is None:
        x_out = torch.empty((R, K), dtype=torch.bfloat16, device=x.device)
    args = _linear_args(x, weight, out, res, norm, delta, x_out, eps, pdl, gated, h_out)
    check(_native.load().mcb_linear(ctypes.byref(args), _stream(x)))
    return (x_out, out) if delta is not None else out


def gated_silu(gate, up, out=None):
    """silu(gate) * up in bf16 (GatedMLP with activation "silu", modelcore/components/mlp.py:89-90);
    gate, up: (rows, H) bf16, e.g. the two halves of one fused gate|up projection."""
    rows, H = gate.shape
    if tuple(up.shape) != (rows, H):
        raise RuntimeError("gate and up must have equal shapes")
    if out is None:
        out = torch.empty((rows, H), dtype=torch.bfloat16, device=gate.device)
    args = GatedSiluArgs()
    args.gate, args.up, args.out = gate.data_ptr(), up.data_ptr(), out.data_ptr()
    args.gate_stride = _rows2d("gate", gate)
    args.up_stride = _rows2d("up", up)
    args.out_stride = _rows2d("out", out)
    args.rows, args.H = rows, H
    check(_native.load().mcb_gated_silu(ctypes.byref(args), _stream(gate)))
    return out


def device_error(device=None):
    """Reads and clears the library's device error word (synchronises the current stream).
    Returns (code, description)."""
    code = ctypes.c_int32(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    check(_native.load().mcb_device_error(ctypes.byref(code), stream))
    return code.value, _native.DEVICE_ERRORS.get(code.value, "unknown")


def launch_count():
    """Kernels libmcb200 has enqueued in this process."""
    return int(_native.load().mcb_launch_count())


def last_attn_kernel():
    """The attention kernel (template instance, as the profiler names it) this thread enqueued
    last through libmcb200; '' before the first."""
    buf = ctypes.create_string_buffer(96)
    check(_native.load().mcb_last_attn_kernel(buf, len(buf)))
    return buf.value.decode()
