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
// The fp32 sum of squares has a fixed order: lane l adds y1^2 then y2^2 for its pairs
// i = l, l+32, ... in increasing i, then the 32 lane sums are combined by an xor butterfly over
// lane masks 16, 8, 4, 2, 1.  The CPU oracle restates exactly that order, so kernel and oracle
// agree bit for bit; against torch's own reduction order the result can differ by one bf16 ulp
// in rare elements (reduction order only).
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
};

constexpr int kAppendWarpsPerBlock = 4;

__global__ void __launch_bounds__(kAppendWarpsPerBlock * 32)
    kv_append_rope_kernel(const AppendParams p) {
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
    if (pos < 0 || pos >= p.Tmax) {
      if (lane == 0) record_error(kErrPositionBeyondCache);
      return;
    }
    const uint16_t* src = p.v + b * p.vs[0] + t * p.vs[1] + h * p.vs[2];
    uint16_t* dst = p.v_cache + ((static_cast<long long>(b) * p.Tmax + pos) * p.Hkv + h) * p.D;
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
    if (pos < 0 || pos >= p.Tmax) {
      if (lane == 0) record_error(kErrPositionBeyondCache);
      return;
    }
    dst = p.k_cache + ((static_cast<long long>(b) * p.Tmax + pos) * p.Hkv + h) * p.D;
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

}  // namespace mcb
