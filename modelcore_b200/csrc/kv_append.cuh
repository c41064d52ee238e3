// Piece 1: the per-step K/V append fused with rotary, QK-norm and the 1.2 scale.
//
// One warp per (row b, token t, head vector).  Warp w of the grid handles vector index
//   w = ((b * T) + t) * (nq + 2 * nkv) + j
// where j < nq are query heads, nq <= j < nq + nkv key heads and the rest value heads.
//
// Arithmetic, element for element, in the order the reference applies it:
//   rope   (modelcore/components/rope.py:4-12, rotation by -theta on the halves [0,D/2), [D/2,D)):
//            y1 = bf16(bf16(x1*cos) + bf16(x2*sin)),  y2 = bf16(bf16(x1*(-sin)) + bf16(x2*cos))
//          with cos/sin the bf16 table rows at position cache_seqlens[b] + t
//          (RotaryEmbedding._cos_sin, modelcore/components/rotary.py:43-67)
//   norm   (F.rms_norm, modelcore/components/norm.py:43-44): fp32 sum of squares, then
//            z = bf16(y * rsqrt(sum/D + eps)),  eps = fp32 machine epsilon when None
//   scale  (modelcore/components/attention.py:149-150): out = bf16(z * 1.2f)
// Two kernels, one arithmetic.  For D a power of two in [16, 256] (every head size modelcore
// configs use) kv_append_rope_vec_kernel gives each vector L = D/16 lanes that move 16-byte
// chunks: lane i owns the pairs 8i .. 8i+7, and the fp32 sum of squares adds, per lane, y1^2 then
// y2^2 for its pairs in increasing order, then combines the L lane sums by an xor butterfly over
// masks L/2, .., 1.  For other D kv_append_rope_kernel uses one warp per vector: lane l adds
// y1^2 then y2^2 for its pairs i = l, l+32, ... in increasing i, then a butterfly over masks
// 16 .. 1.  The CPU oracle restates both orders, so kernel and oracle agree bit for bit; against
// torch's own reduction order the result can differ by one bf16 ulp in rare elements (reduction
// order only).
#pragma once

#include "common.cuh"

namespace mcb {

struct AppendParams {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  int64_t qs[3], ks[3], vs[3];
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  const int32_t* cache_seqlens;
  const uint16_t* cos;
  const uint16_t* sin;
  int B, T, Hq, Hkv, D, Tmax, rot_len;
  float eps, scale;
  int nq;     // query vectors per (b, t): Hq when rotating q, else 0
  int nk;     // key vectors per (b, t): Hkv when writing kv, else 0
  bool rotate_k;
  long long total_vectors;
  int ring;   // the slot is a ring of Tmax positions: position p at index p % Tmax
  // fp8 cache (kv_append_rope_vec_kernel<D, true>): k_cache / v_cache hold e4m3 bytes and every
  // (row, position, head) vector has its scale at k_scale / v_scale[(b * Hkv + h) * scale_tmax + index]
  float* k_scale;
  float* v_scale;
  int scale_tmax;
};

constexpr int kAppendWarpsPerBlock = 4;

__global__ void __launch_bounds__(kAppendWarpsPerBlock * 32)
    kv_append_rope_kernel(const AppendParams p) {
  pdl_wait();               // q, k, v come from the projection ahead
  pdl_launch_dependents();  // after the wait: see pdl_launch_dependents in common.cuh
  const int lane = threadIdx.x & 31;
  const long long w = static_cast<long long>(blockIdx.x) * kAppendWarpsPerBlock + (threadIdx.x >> 5);
  if (w >= p.total_vectors) return;
  const int per_bt = p.nq + 2 * p.nk;
  const int j = static_cast<int>(w % per_bt);
  const long long bt = w / per_bt;
  const int t = static_cast<int>(bt % p.T);
  const int b = static_cast<int>(bt / p.T);
  const int pos = p.cache_seqlens[b] + t;
  const int half = p.D >> 1;

  // Value heads: a plain copy into the cache.
  if (j >= p.nq + p.nk) {
    const int h = j - p.nq - p.nk;
    if (pos < 0 || (!p.ring && pos >= p.Tmax)) {
      if (lane == 0) record_error(kErrPositionBeyondCache);
      return;
    }
    const uint16_t* src = p.v + b * p.vs[0] + t * p.vs[1] + h * p.vs[2];
    const int idx = p.ring ? pos % p.Tmax : pos;
    uint16_t* dst = p.v_cache + ((static_cast<long long>(b) * p.Tmax + idx) * p.Hkv + h) * p.D;
    for (int d = lane; d < p.D; d += 32) dst[d] = src[d];
    return;
  }

  const bool is_q = j < p.nq;
  const int h = is_q ? j : j - p.nq;
  const uint16_t* src = is_q ? p.q + b * p.qs[0] + t * p.qs[1] + h * p.qs[2]
                             : p.k + b * p.ks[0] + t * p.ks[1] + h * p.ks[2];
  uint16_t* dst;
  if (is_q) {
    dst = p.q_out + ((static_cast<long long>(b) * p.T + t) * p.Hq + h) * p.D;
  } else {
    if (pos < 0 || (!p.ring && pos >= p.Tmax)) {
      if (lane == 0) record_error(kErrPositionBeyondCache);
      return;
    }
    dst = p.k_cache + ((static_cast<long long>(b) * p.Tmax + (p.ring ? pos % p.Tmax : pos)) * p.Hkv + h) * p.D;
  }

  if (!is_q && !p.rotate_k) {  // raw key insert
    for (int d = lane; d < p.D; d += 32) dst[d] = src[d];
    return;
  }
  if (pos < 0 || pos >= p.rot_len) {
    if (lane == 0) record_error(kErrPositionBeyondRotary);
    return;
  }

  // Rope on the pairs (i, i + D/2) this lane owns; at most 4 pairs per lane (D <= 256).
  const uint16_t* cos_row = p.cos + static_cast<long long>(pos) * half;
  const uint16_t* sin_row = p.sin + static_cast<long long>(pos) * half;
  float y1[4], y2[4];
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = lane + 32 * u;
    y1[u] = 0.f;
    y2[u] = 0.f;
    if (i < half) {
      const float x1 = bf16_bits_to_float(src[i]);
      const float x2 = bf16_bits_to_float(src[i + half]);
      const float c = bf16_bits_to_float(cos_row[i]);
      const float s = bf16_bits_to_float(sin_row[i]);
      // Products of two bf16 values are exact in fp32; each is rounded to bf16 as torch does.
      const float a = round_bf16(__fmul_rn(x1, c));
      const float bb = round_bf16(__fmul_rn(x2, s));
      const float cc = round_bf16(__fmul_rn(x1, -s));
      const float dd = round_bf16(__fmul_rn(x2, c));
      y1[u] = round_bf16(__fadd_rn(a, bb));
      y2[u] = round_bf16(__fadd_rn(cc, dd));
      acc = __fadd_rn(acc, __fmul_rn(y1[u], y1[u]));
      acc = __fadd_rn(acc, __fmul_rn(y2[u], y2[u]));
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
  const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.D)), p.eps));
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = lane + 32 * u;
    if (i < half) {
      const float z1 = round_bf16(__fmul_rn(y1[u], r));
      const float z2 = round_bf16(__fmul_rn(y2[u], r));
      dst[i] = float_to_bf16_bits(__fmul_rn(z1, p.scale));
      dst[i + half] = float_to_bf16_bits(__fmul_rn(z2, p.scale));
    }
  }
}

// 8 bf16 (one 16-byte chunk) <-> 8 floats
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}

// The e4m3 quantization of one cache vector (fp8 cache): amax = max |x| over the vector's D
// values (x the bf16 values a bf16 cache would hold), scale = amax / 448 and x8 =
// e4m3(x * (448 / amax)) rounded to nearest even and saturated to +-448 (both quotients correctly
// rounded fp32; amax = 0 stores zeros with scale 0).  cvt packs its first source in the upper byte.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint2 e4m3x8(const float* x, float inv) {
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    w[i] = static_cast<uint32_t>(e4m3x2(__fmul_rn(x[4 * i], inv), __fmul_rn(x[4 * i + 1], inv))) |
           (static_cast<uint32_t>(e4m3x2(__fmul_rn(x[4 * i + 2], inv), __fmul_rn(x[4 * i + 3], inv))) << 16);
  return make_uint2(w[0], w[1]);
}

// One head vector's rope + rms_norm + scale, by a group of L = D/16 lanes (lane `sub` of the
// group holds the pairs 8 sub .. 8 sub + 7 of the halves x1 = [0, D/2) and x2 = [D/2, D)): the
// arithmetic of the append, shared by kv_append_rope_vec_kernel and the decode attention that
// fuses the append, so both give the same bits.  Every lane of the warp calls it (the sum of
// squares is an xor butterfly over the group's lanes); with rotate false o1 / o2 are x1 / x2 and
// the lane adds nothing to its group's sum.
// Packed arithmetic for the vector path.  Every result is the bf16 (or fp32) value the scalar
// recipe gives: a product of two bf16 values is exact in fp32, so fp32-multiply-then-round equals
// mul.rn.bf16x2; a sum of two bf16 values is exact in fp32 whenever rounding to bf16 can depend
// on its low bits (operand exponents within 15 of each other; farther apart the smaller one is
// below a quarter ulp of the larger and both roundings return the larger), so
// fp32-add-then-round equals add.rn.bf16x2; f32x2 multiplies round each lane as __fmul_rn does.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// (lo, hi) bf16 pair -> the two values as an fp32 pair (exact)
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) {
  return static_cast<uint64_t>(w << 16) | (static_cast<uint64_t>(w & 0xffff0000u) << 32);
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// fp32 pair -> bf16 pair, each rounded to nearest even
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  uint32_t d;
  asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}"
      : "=r"(d)
      : "l"(v));
  return d;
}

template <int D>
__device__ __forceinline__ void rope_norm_vec_tab(const uint4& x1v, const uint4& x2v, const uint4& cv,
                                                  const uint4& sv, bool rotate, float eps, float scale,
                                                  uint4& w1, uint4& w2) {
  constexpr int L = D / 16;
  uint32_t y1[4], y2[4];
  float acc = 0.f;
  if (rotate) {
    const uint32_t X1[4] = {x1v.x, x1v.y, x1v.z, x1v.w}, X2[4] = {x2v.x, x2v.y, x2v.z, x2v.w};
    const uint32_t C[4] = {cv.x, cv.y, cv.z, cv.w}, S[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // elements 2k, 2k+1 of the lane's 8 pairs
      y1[k] = badd2(bmul2(X1[k], C[k]), bmul2(X2[k], S[k]));
      y2[k] = badd2(bmul2(X1[k], S[k] ^ 0x80008000u), bmul2(X2[k], C[k]));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // element order: y1[i]^2 then y2[i]^2, i increasing
      const float a0 = __uint_as_float(y1[k] << 16), a1 = __uint_as_float(y1[k] & 0xffff0000u);
      const float b0 = __uint_as_float(y2[k] << 16), b1 = __uint_as_float(y2[k] & 0xffff0000u);
      acc = __fadd_rn(acc, __fmul_rn(a0, a0));
      acc = __fadd_rn(acc, __fmul_rn(b0, b0));
      acc = __fadd_rn(acc, __fmul_rn(a1, a1));
      acc = __fadd_rn(acc, __fmul_rn(b1, b1));
    }
  }
#pragma unroll
  for (int m = L / 2; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
  if (rotate) {
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(D)), eps));
    const uint64_t rr = static_cast<uint64_t>(__float_as_uint(r)) * 0x100000001ull;
    const uint64_t ss = static_cast<uint64_t>(__float_as_uint(scale)) * 0x100000001ull;
    uint32_t o1[4], o2[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o1[k] = f2_to_bf2(fmul2(bf2_to_f2(f2_to_bf2(fmul2(bf2_to_f2(y1[k]), rr))), ss));
      o2[k] = f2_to_bf2(fmul2(bf2_to_f2(f2_to_bf2(fmul2(bf2_to_f2(y2[k]), rr))), ss));
    }
    w1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
    w2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
  } else {
    w1 = x1v;
    w2 = x2v;
  }
}

// The same with the lane's cos / sin chunks read from the tables at row `pos`.
template <int D>
__device__ __forceinline__ void rope_norm_vec(const uint4& x1v, const uint4& x2v, const uint16_t* cos,
                                              const uint16_t* sin, int pos, int sub, bool rotate, float eps,
                                              float scale, uint4& w1, uint4& w2) {
  uint4 cv = make_uint4(0, 0, 0, 0), sv = make_uint4(0, 0, 0, 0);
  if (rotate) {
    const long long trow = static_cast<long long>(pos) * (D / 2) + 8 * sub;
    cv = *reinterpret_cast<const uint4*>(cos + trow);
    sv = *reinterpret_cast<const uint4*>(sin + trow);
  }
  rope_norm_vec_tab<D>(x1v, x2v, cv, sv, rotate, eps, scale, w1, w2);
}

// Vectorised variant: L = D/16 lanes per vector, 16-byte loads and stores, 32/L vectors per warp.
// Requires 16-byte aligned rows (checked on the host).  FP8: the cache vectors are stored as
// e4m3 with a per-vector scale (e4m3x8 above), 8-byte stores.
//
// A grid-stride loop (the grid is four 256-thread CTAs per SM) over groups of vectors: each
// iteration a warp loads a group's positions and 16-byte chunks, then the rotary table chunks at
// those positions, computes and stores.  The arithmetic is packed (bf16x2 / f32x2, see
// rope_norm_vec_tab): the kernel was bound by instruction issue, not by bytes in flight (config
// 2's prefill append: 0.37 of the copy peak with scalar arithmetic and one vector group per
// 128-thread CTA, 0.61 with packed arithmetic here; batching two or four groups per iteration for
// more loads in flight measured slower, 0.58 and 0.55: more registers, fewer warps).
constexpr int kAppendVecThreads = 256;

struct AppendVecLoad {
  int b, t, j, pos;
  bool active, rotate, ok;
  uint4 x1v, x2v, cv, sv;
};

template <int D>
__device__ __forceinline__ void append_vec_load(const AppendParams& p, long long w, int sub, AppendVecLoad& r) {
  constexpr int HALF = D / 2;
  r.active = w < p.total_vectors;
  const unsigned wv = r.active ? static_cast<unsigned>(w) : 0u;  // total_vectors < 2^31 (host)
  const unsigned per_bt = static_cast<unsigned>(p.nq + 2 * p.nk);
  r.j = static_cast<int>(wv % per_bt);
  const unsigned bt = wv / per_bt;
  r.t = static_cast<int>(bt % static_cast<unsigned>(p.T));
  r.b = static_cast<int>(bt / static_cast<unsigned>(p.T));
  const bool is_v = r.j >= p.nq + p.nk;
  const bool is_q = r.j < p.nq;
  const int h = is_q ? r.j : (is_v ? r.j - p.nq - p.nk : r.j - p.nq);
  const uint16_t* src = is_q ? p.q + r.b * p.qs[0] + r.t * p.qs[1] + h * p.qs[2]
                             : (is_v ? p.v + r.b * p.vs[0] + r.t * p.vs[1] + h * p.vs[2]
                                     : p.k + r.b * p.ks[0] + r.t * p.ks[1] + h * p.ks[2]);
  r.pos = p.cache_seqlens[r.b] + r.t;
  r.x1v = *reinterpret_cast<const uint4*>(src + 8 * sub);
  r.x2v = *reinterpret_cast<const uint4*>(src + HALF + 8 * sub);
  r.rotate = is_q || (!is_v && p.rotate_k);
}

// The position checks, then the lane's rotary table chunks (rotating vectors only).
template <int D>
__device__ __forceinline__ void append_vec_tables(const AppendParams& p, int sub, AppendVecLoad& r) {
  const bool is_q = r.j < p.nq;
  r.ok = r.active;
  if (!is_q && (r.pos < 0 || (!p.ring && r.pos >= p.Tmax))) {
    if (r.active && sub == 0) record_error(kErrPositionBeyondCache);
    r.ok = false;
  }
  if (r.ok && r.rotate && (r.pos < 0 || r.pos >= p.rot_len)) {
    if (sub == 0) record_error(kErrPositionBeyondRotary);
    r.ok = false;
  }
  r.cv = r.sv = make_uint4(0, 0, 0, 0);
  if (r.ok && r.rotate) {
    const long long trow = static_cast<long long>(r.pos) * (D / 2) + 8 * sub;
    r.cv = *reinterpret_cast<const uint4*>(p.cos + trow);
    r.sv = *reinterpret_cast<const uint4*>(p.sin + trow);
  }
}

template <int D, bool FP8>
__device__ __forceinline__ void append_vec_store(const AppendParams& p, const AppendVecLoad& v, int sub) {
  constexpr int L = D / 16;
  constexpr int HALF = D / 2;
  const int b = v.b, t = v.t, j = v.j, pos = v.pos;
  const bool is_v = j >= p.nq + p.nk;
  const bool is_q = j < p.nq;
  const int h = is_q ? j : (is_v ? j - p.nq - p.nk : j - p.nq);
  const bool ok = v.ok, rotate = v.rotate;
  long long cache_off = 0;   // element offset of the cache vector
  long long scale_off = 0;
  uint16_t* dst = nullptr;
  if (is_q) {
    dst = p.q_out + ((static_cast<long long>(b) * p.T + t) * p.Hq + h) * D;
  } else if (ok) {
    const int idx = p.ring ? pos % p.Tmax : pos;
    cache_off = ((static_cast<long long>(b) * p.Tmax + idx) * p.Hkv + h) * D;
    scale_off = (static_cast<long long>(b) * p.Hkv + h) * p.scale_tmax + idx;
    if (!FP8) dst = (is_v ? p.v_cache : p.k_cache) + cache_off;
  }
  if (!FP8 && !rotate) {  // value heads and raw key inserts: a copy
    if (ok) {
      *reinterpret_cast<uint4*>(dst + 8 * sub) = v.x1v;
      *reinterpret_cast<uint4*>(dst + HALF + 8 * sub) = v.x2v;
    }
    // lanes of a rotating vector in this warp still take part in the butterfly below
  }
  uint4 w1, w2;  // the output vector's bf16 chunks
  rope_norm_vec_tab<D>(v.x1v, v.x2v, v.cv, v.sv, rotate && ok, p.eps, p.scale, w1, w2);
  if (rotate && ok && (!FP8 || is_q)) {  // q always goes out as bf16; fp8 cache vectors below
    *reinterpret_cast<uint4*>(dst + 8 * sub) = w1;
    *reinterpret_cast<uint4*>(dst + HALF + 8 * sub) = w2;
  }
  if constexpr (FP8) {
    float o1[8], o2[8];
    unpack8(w1, o1);
    unpack8(w2, o2);
    // every lane takes part in the amax butterfly; q vectors and idle lanes contribute nothing
    float amax = 0.f;
    if (ok && !is_q)
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fmaxf(fabsf(o1[i]), fabsf(o2[i])));
#pragma unroll
    for (int m = L / 2; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    if (ok && !is_q) {
      const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
      uint8_t* d8 = static_cast<uint8_t*>(static_cast<void*>(is_v ? p.v_cache : p.k_cache)) + cache_off;
      *reinterpret_cast<uint2*>(d8 + 8 * sub) = e4m3x8(o1, inv);
      *reinterpret_cast<uint2*>(d8 + HALF + 8 * sub) = e4m3x8(o2, inv);
      if (sub == 0) (is_v ? p.v_scale : p.k_scale)[scale_off] = amax > 0.f ? __fdiv_rn(amax, 448.f) : 0.f;
    }
  }
}

template <int D, bool FP8>
__global__ void __launch_bounds__(kAppendVecThreads, 4)
    kv_append_rope_vec_kernel(const AppendParams p) {
  pdl_wait();               // q, k, v come from the projection ahead
  pdl_launch_dependents();  // after the wait: see pdl_launch_dependents in common.cuh
  constexpr int L = D / 16;        // lanes per vector
  constexpr int VPW = 32 / L;      // vectors per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;        // chunk index within the half
  const long long warps = static_cast<long long>(gridDim.x) * (kAppendVecThreads / 32);
  const long long stride = warps * VPW;  // vectors per sweep of the grid
  const long long first = (static_cast<long long>(blockIdx.x) * (kAppendVecThreads / 32) + (threadIdx.x >> 5)) * VPW;
  // two vector groups a sweep, both groups' loads issued before either's arithmetic and stores:
  // twice the bytes in flight a warp (a group past the end loads vector 0 and stores nothing);
  // one for an fp8 cache, whose scale butterfly would spill at the 64-register cap
  constexpr int U = FP8 ? 1 : 2;
  for (long long base = first; base < p.total_vectors; base += U * stride) {  // warp-uniform
    AppendVecLoad v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) append_vec_load<D>(p, base + u * stride + lane / L, sub, v[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) append_vec_tables<D>(p, sub, v[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) append_vec_store<D, FP8>(p, v[u], sub);
  }
}

}  // namespace mcb
