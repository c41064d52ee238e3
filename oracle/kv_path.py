"""CPU oracle for modelcore's KV-cache decode path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it.  The product path (modelcore_b200) never calls it and
has no CPU fallback.

It restates, in numpy, what modelcore computes on the decode path (file:line cited per function,
relative to the modelcore project root).  bf16 values travel as uint16 bit patterns; every
place where the reference rounds a tensor op's result to bf16, this code rounds with IEEE
round-to-nearest-even.  Parity is pinned by tests/test_oracle_golden.py against golden vectors
that tests/golden/make_golden.py produced by running the reference itself.

The one place where bit-exactness against torch is not defined is the fp32 sum of squares
inside rms_norm: torch's reduction order is an implementation detail.  `rms_norm_scale` fixes the
order the CUDA kernels use (per-lane partial sums over pairs (i, i + D/2), then an xor butterfly;
see `sum_squares_kernel_order`), so the kernels match this oracle bit for bit and the reference to
within one bf16 ulp on rare elements.
"""
import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------------------------
# bf16 <-> fp32
def bf16_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """float32 -> uint16 bf16 bits, IEEE round-to-nearest-even (what torch's .to(bfloat16) and
    every bf16 tensor op's output store do)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> 16) & np.uint32(1)
    return ((u + np.uint32(0x7FFF) + lsb) >> 16).astype(np.uint16)


def round_bf16(x):
    """float32 -> float32 rounded to the nearest bf16 value."""
    return bf16_to_f32(f32_to_bf16(x))


# ---------------------------------------------------------------------------------------------
# Rotary tables: modelcore/components/rope.py:15-27
def rotary_tables(seq_len, head_dim, base=100000):
    """(cos, sin) bf16 bits of shape (seq_len, head_dim/2): theta_{t,i} = t * base^(-2i/D) in
    fp32, cos/sin in fp32, then rounded to bf16 (rope.py:19-25).  numpy's fp32 cos/sin may differ
    from torch's by one fp32 ulp, which can move a bf16 rounding; the CUDA path never recomputes
    the tables (it reads the RotaryEmbedding module's own buffers)."""
    ch = np.arange(0, head_dim, 2, dtype=np.float32)
    inv_freq = (F32(1.0) / (F32(base) ** (ch / F32(head_dim)))).astype(np.float32)
    t = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    return f32_to_bf16(np.cos(freqs)), f32_to_bf16(np.sin(freqs))


# ---------------------------------------------------------------------------------------------
# apply_rotary_emb: modelcore/components/rope.py:4-12
def rope(x_bits, cos_bits, sin_bits):
    """x (..., D) bf16 bits; cos/sin (..., D/2) bf16 bits broadcastable to x's halves.
    y1 = x1*cos + x2*sin, y2 = x1*(-sin) + x2*cos, every product and sum rounded to bf16."""
    x = bf16_to_f32(x_bits)
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c, s = bf16_to_f32(cos_bits), bf16_to_f32(sin_bits)
    y1 = round_bf16(round_bf16(x1 * c) + round_bf16(x2 * s))
    y2 = round_bf16(round_bf16(x1 * (-s)) + round_bf16(x2 * c))
    return f32_to_bf16(np.concatenate([y1, y2], axis=-1))


# ---------------------------------------------------------------------------------------------
# RMSNorm + scale: modelcore/components/norm.py:43-44 (F.rms_norm, eps=None -> the fp32 machine
# epsilon for bf16 input) and modelcore/components/attention.py:149-150 (x 1.2)
def sum_squares_kernel_order(y):
    """fp32 sum of y^2 over the last axis in the CUDA kernels' fixed order.

    D a power of two in [16, 256] (the vectorised kernel): L = D/16 lanes; lane i adds y1^2 then
    y2^2 for its pairs 8i .. 8i+7 (pair p = (y[p], y[p + D/2])) in increasing order; the L lane
    sums combine by an xor butterfly over masks L/2 .. 1.  Other D (one warp per vector): lane l
    adds y1^2 then y2^2 for its pairs l, l+32, ..; the 32 lane sums combine over masks 16 .. 1."""
    y = np.asarray(y, dtype=np.float32)
    D = y.shape[-1]
    half = D // 2
    lead = y.shape[:-1]
    if D in (16, 32, 64, 128, 256):
        lanes = D // 16
        pairs = [[8 * i + j for j in range(8)] for i in range(lanes)]
        masks = [m for m in (8, 4, 2, 1) if m < lanes]
    else:
        lanes = 32
        pairs = [[lane + 32 * u for u in range(4) if lane + 32 * u < half] for lane in range(32)]
        masks = [16, 8, 4, 2, 1]
    acc = np.zeros(lead + (lanes,), dtype=np.float32)
    for lane in range(lanes):
        for i in pairs[lane]:
            a = y[..., i]
            b = y[..., i + half]
            acc[..., lane] = acc[..., lane] + a * a
            acc[..., lane] = acc[..., lane] + b * b
    for m in masks:
        acc = acc + acc[..., np.arange(lanes) ^ m]
    return acc[..., 0]


def rms_norm_scale(y_bits, eps=None, scale=1.2):
    """bf16(bf16(y * rsqrt(mean(y^2) + eps)) * scale) with fp32 arithmetic; rsqrt correctly
    rounded; the mean's sum in the kernel's order."""
    y = bf16_to_f32(y_bits)
    D = y.shape[-1]
    e = F32(np.finfo(np.float32).eps if eps is None else eps)
    ms = (sum_squares_kernel_order(y) / F32(D)).astype(np.float32)
    v = (ms + e).astype(np.float32)
    r = (np.longdouble(1.0) / np.sqrt(v.astype(np.longdouble))).astype(np.float32)
    z = round_bf16((y * r[..., None]).astype(np.float32))
    return f32_to_bf16((z * F32(scale)).astype(np.float32))


def rope_norm_scale(x_bits, cos_bits, sin_bits, eps=None, scale=1.2):
    """The fused chain of modelcore/components/attention.py:147-150 for one tensor."""
    return rms_norm_scale(rope(x_bits, cos_bits, sin_bits), eps=eps, scale=scale)


def positions(cache_seqlens, T):
    """(B, T) absolute positions cache_seqlens[b] + t (rotary.py:60-67, flash_attn.py:341-346)."""
    return np.asarray(cache_seqlens, dtype=np.int64)[:, None] + np.arange(T)[None, :]


def rope_tables_at(cos_bits, sin_bits, cache_seqlens, T):
    """Per-row table rows gathered at each row's own positions: (B, T, 1, D/2)."""
    pos = positions(cache_seqlens, T)
    return cos_bits[pos][:, :, None, :], sin_bits[pos][:, :, None, :]


# ---------------------------------------------------------------------------------------------
# The decode step either side of attention
def _row_rms_norm(x, eps):
    """bf16-representable fp32 rows x (..., C) -> bf16(x * rsqrt(sum(x^2)/C + eps)) as fp32, the sum
    in the step kernels' order (step_fused.cuh row_rms_rsqrt, decode_proj.cuh's fused norm): the
    squares added element by element within each 8-element chunk, a pairwise tree over the 8
    chunks of each 64-column panel ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)) (absent chunks of a short
    last panel count 0), then the panels in order."""
    C = x.shape[-1]
    nchunk = C // 8
    npanel = (nchunk + 7) // 8
    s = np.zeros(x.shape[:-1] + (npanel * 8,), dtype=np.float32)
    for c in range(nchunk):
        for i in range(8):
            v = x[..., 8 * c + i]
            s[..., c] = s[..., c] + v * v
    for m in (1, 2, 4):
        s = s + s[..., np.arange(npanel * 8) ^ m]
    acc = np.zeros(x.shape[:-1], dtype=np.float32)
    for p in range(npanel):
        acc = acc + s[..., 8 * p]
    e = F32(np.finfo(np.float32).eps if eps is None else eps)
    v = ((acc / F32(C)).astype(np.float32) + e).astype(np.float32)
    r = (np.longdouble(1.0) / np.sqrt(v.astype(np.longdouble))).astype(np.float32)
    return round_bf16((x * r[..., None]).astype(np.float32))


def add_rms_norm(x_bits, delta_bits=None, eps=None):
    """Block's residual add then norm (modelcore/components/block.py:57-59, norm.py:43-44):
    x' = bf16(x + delta), h = bf16(x' * rsqrt(sum(x'^2)/C + eps)), the fp32 sum in the kernel's
    order (_row_rms_norm).  Returns (x' bits, h bits)."""
    x = bf16_to_f32(x_bits)
    if delta_bits is not None:
        x = round_bf16((x + bf16_to_f32(delta_bits)).astype(np.float32))
    return f32_to_bf16(x), f32_to_bf16(_row_rms_norm(x, eps))


def embed_rms_norm(ids, table_bits, eps=None):
    """TokenEmbedding without smear (modelcore/components/embedding.py:71-75: wte lookup, norm)
    and the first block's norm of its output (block.py:57).  Returns (x bits, h bits)."""
    x = _row_rms_norm(bf16_to_f32(table_bits[np.asarray(ids)]), eps)
    return f32_to_bf16(x), f32_to_bf16(_row_rms_norm(x, eps))


def softcap_logits(logits_bits, vocab_size, softcap):
    """LMHead.forward's epilogue (modelcore/components/unembedding.py:52-56): crop the padded
    bf16 logits to vocab_size, .float(), softcap * tanh(x / softcap) in fp32, with the division
    as torch performs it on CUDA for a Python-number divisor: x * fp32(1 / softcap).  On the CPU
    torch divides exactly and uses its own vectorised tanh; numpy's float32 tanh differs from
    both by an ulp or two on some elements (tests bound it)."""
    x = bf16_to_f32(logits_bits[..., :vocab_size])
    if softcap is None:
        return x
    c = F32(softcap)
    inv = (F32(1.0) / c).astype(np.float32)
    return (c * np.tanh((x * inv).astype(np.float32)).astype(np.float32)).astype(np.float32)


def greedy_pick(logits):
    """sample_next_token(temperature=0) (modelcore/generate.py:23-24): the first index of each
    row's maximum."""
    return np.argmax(logits, axis=-1)


def gated_silu(gate_bits, up_bits):
    """GatedMLP's silu(gate) * up (modelcore/components/mlp.py:89-90): silu in fp32 as
    g / (1 + exp(-g)) rounded to bf16, the product rounded to bf16.  numpy's exp may differ from
    the device's expf by an fp32 ulp, which can move a bf16 rounding (tests allow one bf16 ulp)."""
    g = bf16_to_f32(gate_bits)
    u = bf16_to_f32(up_bits)
    s = round_bf16((g / (F32(1.0) + np.exp(-g))).astype(np.float32))
    return f32_to_bf16((s * u).astype(np.float32))


# ---------------------------------------------------------------------------------------------
# The insert of flash_attn_with_kvcache: modelcore/kernels/flash_attn.py:337-346
def kv_insert(k_cache, v_cache, k, v, cache_seqlens):
    """In place: row b's new tokens land at [cache_seqlens[b], cache_seqlens[b] + T)."""
    T = k.shape[1]
    pos = positions(cache_seqlens, T)
    for b in range(k.shape[0]):
        k_cache[b, pos[b]] = k[b]
        v_cache[b, pos[b]] = v[b]


def append_rope(q, k, v, k_cache, v_cache, cache_seqlens, cos_bits, sin_bits, *, rotate_q=True,
                rotate_k=True, write_kv=True, eps=None, scale=1.2):
    """Restatement of one producer layer's decode-side chain (attention.py:147-153 + the insert):
    returns the processed q (bf16 bits) and writes the processed k and raw v into the caches."""
    T = (q if q is not None else k).shape[1]
    c, s = rope_tables_at(cos_bits, sin_bits, cache_seqlens, T)
    q_out = rope_norm_scale(q, c, s, eps, scale) if rotate_q else None
    if write_kv:
        k_new = rope_norm_scale(k, c, s, eps, scale) if rotate_k else k
        kv_insert(k_cache, v_cache, k_new, v, cache_seqlens)
    return q_out


# ---------------------------------------------------------------------------------------------
# fp8 (e4m3) cache vectors: a cache format this build adds (the reference stores the compute
# dtype).  Each (row, position, kv head) vector x -- the bf16 values a bf16 cache would hold -- is
# stored as e4m3(x * fp32(448 / amax)) with scale fp32(amax / 448), amax = max |x|; amax = 0 gives
# zeros and scale 0.  e4m3 ("fn": 1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no
# infinities, max finite 448, subnormal step 2^-9) rounded to nearest even and saturated to 448.
def e4m3_bits(x):
    """float32 values -> e4m3 bit patterns (uint8), round to nearest even, saturating at 448."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    neg = np.signbit(x)
    a = np.minimum(np.abs(x), 448.0)
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.clip(e, -6, 8)
    step = np.exp2(e - 3)                      # 3 mantissa bits; binade -6 also spans subnormals
    q = np.minimum(np.round(a / step) * step, 448.0)   # np.round: half to even
    qe = np.floor(np.log2(np.where(q > 0, q, 1.0)))
    normal = q >= 2.0 ** -6
    exp_field = np.where(normal, qe + 7, 0)
    man = np.where(normal, q / np.exp2(qe) * 8 - 8, q / 2.0 ** -9)
    bits = (exp_field.astype(np.int64) << 3) | np.round(man).astype(np.int64)
    bits = np.where(q == 0, 0, bits) | (neg.astype(np.int64) << 7)
    return bits.astype(np.uint8)


def e4m3_value(bits):
    """e4m3 bit patterns -> float32 values (exact; 0x7f / 0xff, the NaNs, are not produced)."""
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    ef = (b >> 3) & 0xF
    m = b & 7
    v = np.where(ef == 0, m * 2.0 ** -9, (1 + m / 8.0) * np.exp2(ef - 7.0))
    return (sign * v).astype(np.float32)


def quantize_fp8(x_bits):
    """bf16 vectors (..., D) -> (e4m3 bytes (..., D), fp32 scales (...)) as the fp8 cache's append
    stores them."""
    x = bf16_to_f32(x_bits)
    amax = np.abs(x).max(axis=-1).astype(np.float32)
    pos = amax > 0
    inv = np.where(pos, F32(448.0) / np.where(pos, amax, F32(1.0)), F32(0.0)).astype(np.float32)
    scale = np.where(pos, amax / F32(448.0), F32(0.0)).astype(np.float32)
    y = (x * inv[..., None]).astype(np.float32)
    return e4m3_bits(y), scale


def dequantize_fp8(bytes_, scale):
    """The values an fp8 cache vector stands for: e4m3 value x scale (float64)."""
    return e4m3_value(bytes_).astype(np.float64) * np.asarray(scale, dtype=np.float64)[..., None]


# ---------------------------------------------------------------------------------------------
# KVCache.prefill / prefill_row: modelcore/cache.py:75-90, :92-119
def prefill_broadcast(dst_k, dst_v, src_k, src_v, n_pos):
    """dst[:, :, :n_pos] = src[:, :, :n_pos] with src batch 1 broadcast (cache.py:84-85)."""
    dst_k[:, :, :n_pos] = src_k[:, :, :n_pos]
    dst_v[:, :, :n_pos] = src_v[:, :, :n_pos]


def prefill_row(dst_k, dst_v, row, src_k, src_v, n_pos):
    """dst[:, row, :n_pos] = src[:, 0, :n_pos] (cache.py:106-107)."""
    dst_k[:, row, :n_pos] = src_k[:, 0, :n_pos]
    dst_v[:, row, :n_pos] = src_v[:, 0, :n_pos]


# ---------------------------------------------------------------------------------------------
# Decode attention: modelcore/kernels/flash_attn.py:348-366 with _ragged_decode_mask (:246-264)
def visible_range(L, t, window):
    """Keys c visible to query t of a row at L: c <= L + t and (window < 0 or L + t - c <= window)."""
    qpos = L + t
    lo = 0 if window is None or window < 0 else max(0, qpos - window)
    return lo, qpos


def decode_attention(q, k_cache, v_cache, cache_seqlens, window=-1, scale=None):
    """float64 attention of q (B, T, Hq, D) over each row's visible cache keys; k/v caches
    (B, Tmax, Hkv, D) as float arrays; q head h reads kv head h // (Hq // Hkv) (SDPA enable_gqa);
    scale defaults to 1/sqrt(D) (SDPA's default, flash_attn.py:364)."""
    q = np.asarray(q, dtype=np.float64)
    kc = np.asarray(k_cache, dtype=np.float64)
    vc = np.asarray(v_cache, dtype=np.float64)
    B, T, Hq, D = q.shape
    Hkv = kc.shape[2]
    G = Hq // Hkv
    sc = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((B, T, Hq, D), dtype=np.float64)
    for b in range(B):
        L = int(cache_seqlens[b])
        for t in range(T):
            lo, hi = visible_range(L, t, window)
            K = kc[b, lo:hi + 1]            # (n, Hkv, D)
            V = vc[b, lo:hi + 1]
            Kg = np.repeat(K, G, axis=1)    # (n, Hq, D)
            Vg = np.repeat(V, G, axis=1)
            s = np.einsum("hd,nhd->hn", q[b, t], Kg) * sc
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[b, t] = np.einsum("hn,nhd->hd", p, Vg)
    return out


def flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens, window=-1):
    """Insert then attend, as the reference's SDPA path does (flash_attn.py:330-366); the caller
    advances cache_seqlens."""
    if k is not None and v is not None:
        kv_insert(k_cache, v_cache, k, v, cache_seqlens)
    return decode_attention(q, k_cache, v_cache, cache_seqlens, window)


def kv_read_bytes(cache_seqlens, T, Hkv, D, window, itemsize=2):
    """Algorithmic KV bytes one attention call reads: 2 * Hkv * D * itemsize per visible key,
    keys counted exactly (n_keys = min(pos + 1, window + 1)), per row for its last query token
    (the union of its queries' ranges).  The reference's own model of this number is
    modelcore/stats.py:98-107."""
    total = 0
    for L in np.asarray(cache_seqlens).tolist():
        lo, _ = visible_range(L, 0, window)
        hi = L + T - 1
        total += (hi - lo + 1)
    return total * 2 * Hkv * D * itemsize


# ---------------------------------------------------------------------------------------------
# Sampling: sample_next_token, modelcore/generate.py:19-34
def sample_candidates(logits, temperature, top_k):
    """The reference's candidates and their probabilities for one row of fp32 logits: with
    1 <= top_k < V the top_k largest (torch.topk, generate.py:26-27; ties here by ascending
    index) in descending order, else the whole row in index order; probabilities
    softmax(x / T) (generate.py:28-29, 32-33) with x / T as x * fp32(1 / T), in float64."""
    x = np.asarray(logits, dtype=np.float32)
    V = x.shape[-1]
    if top_k is not None and 1 <= top_k < V:
        order = np.lexsort((np.arange(V), -x.astype(np.float64)))[:top_k]
    else:
        order = np.arange(V)
    inv = (F32(1.0) / F32(temperature)).astype(np.float32)
    xs = (x[order] * inv).astype(np.float32).astype(np.float64)
    w = np.exp(xs - xs.max())
    return order, w / w.sum()


def sample_token(logits, u, temperature, top_k):
    """The draw at uniform u: the first candidate whose inclusive cumulative probability exceeds
    u (the inverse CDF; torch.multinomial, generate.py:30 and :34, draws from the same
    distribution with its own generator).  Returns (index, distance of u to the nearest CDF
    boundary) -- the second lets tests skip draws that fp32 rounding can move (and, above 1024
    candidates, the kernel's fixed-point weights: at most top_k * 2^-41 of the total)."""
    order, p = sample_candidates(logits, temperature, top_k)
    c = np.cumsum(p)
    i = int(np.searchsorted(c, u, side="right"))
    i = min(i, len(order) - 1)
    return int(order[i]), float(np.min(np.abs(c - u)))
