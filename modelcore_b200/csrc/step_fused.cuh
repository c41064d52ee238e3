// The decode step around attention, one (rows, C) bf16 activation block per launch:
//
//   add_rms_norm:    x' = bf16(x + delta)                   (Block: x = x + mixer(..) / ffn(..),
//                    h  = bf16(x' * rsqrt(mean(x'^2) + eps)) modelcore/components/block.py:57-59,
//                                                            then norm, modelcore/components/norm.py:43-44)
//   embed_rms_norm:  x = norm(wte[id]), h = norm(x)          (TokenEmbedding.forward,
//                                                            modelcore/components/embedding.py:71-75,
//                                                            then the first block's norm)
//   gated_silu:      out = bf16(bf16(silu(gate)) * up)       (GatedMLP.forward, modelcore/components/mlp.py:89-90)
//   softcap_argmax:  y = cap * tanh(float(x) / cap), argmax  (LMHead.forward's epilogue,
//                                                            modelcore/components/unembedding.py:52-56,
//                                                            and greedy sample_next_token)
//
// Rounding follows torch's ops: the add is computed in fp32 and rounded once; rms_norm
// accumulates the sum of squares in fp32 in one fixed order (row_rms_rsqrt: within 8-element
// chunks, a pairwise tree over the 8 chunks of each 64-column panel, then the panels in order),
// and rounds once; silu is computed in fp32 as g / (1 + exp(-g)) and rounded, the
// product in fp32 and rounded; the softcap multiplies by the fp32 reciprocal of the cap (as torch's
// CUDA division by a Python number does), then tanhf, then an fp32 multiply.  The
// CPU oracle restates the same order.
#pragma once

#include "common.cuh"

namespace mcb {

struct AddNormParams {
  const uint16_t* x;
  const uint16_t* delta;  // may be null: h = rms_norm(x)
  uint16_t* x_out;        // may be null when delta is null
  uint16_t* h_out;
  long long xs, ds, xos, hs;  // row strides (elements)
  int rows, C;
  float eps;
};

// A row of C bf16 values held by one warp as v[u][0..7] = elements 8c .. 8c+7 of chunk
// c = lane + 32u (CPL 16-byte chunks per lane).
template <int CPL>
__device__ __forceinline__ void load_row_chunks(const uint16_t* row, int lane, int nchunk,
                                                float (&v)[CPL][8]) {
#pragma unroll
  for (int u = 0; u < CPL; ++u) {
    const int c = lane + 32 * u;
    if (c < nchunk) {
      const uint4 w = *reinterpret_cast<const uint4*>(row + 8 * c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[u][2 * i] = __uint_as_float(ws[i] << 16);
        v[u][2 * i + 1] = __uint_as_float(ws[i] & 0xffff0000u);
      }
    }
  }
}

template <int CPL>
__device__ __forceinline__ void store_row_chunks(uint16_t* row, int lane, int nchunk,
                                                 const float (&v)[CPL][8]) {
#pragma unroll
  for (int u = 0; u < CPL; ++u) {
    const int c = lane + 32 * u;
    if (c < nchunk) {
      uint4 o;
      o.x = pack_bf16x2(v[u][0], v[u][1]);
      o.y = pack_bf16x2(v[u][2], v[u][3]);
      o.z = pack_bf16x2(v[u][4], v[u][5]);
      o.w = pack_bf16x2(v[u][6], v[u][7]);
      *reinterpret_cast<uint4*>(row + 8 * c) = o;
    }
  }
}

// rsqrt(mean(v^2) + eps) of the warp's row.  The fp32 sum of squares has one fixed order, shared
// with mcb_linear's fused norm (decode_proj.cuh), which holds a row as 64-column panels spread
// over the CTAs of a cluster: squares added element by element within each 8-element chunk
// (chunk c = lane + 32u), a pairwise tree over the 8 chunks of each 64-column panel (lanes 8g ..
// 8g + 7: xor shuffles 1, 2, 4), then the panels in order, from 0.
template <int CPL>
__device__ __forceinline__ float row_rms_rsqrt(const float (&v)[CPL][8], int lane, int nchunk,
                                               int C, float eps) {
  float s[CPL];
#pragma unroll
  for (int u = 0; u < CPL; ++u) {
    s[u] = 0.f;
    if (lane + 32 * u < nchunk) {
#pragma unroll
      for (int i = 0; i < 8; ++i) s[u] = __fadd_rn(s[u], __fmul_rn(v[u][i], v[u][i]));
    }
    s[u] = __fadd_rn(s[u], __shfl_xor_sync(0xffffffffu, s[u], 1));
    s[u] = __fadd_rn(s[u], __shfl_xor_sync(0xffffffffu, s[u], 2));
    s[u] = __fadd_rn(s[u], __shfl_xor_sync(0xffffffffu, s[u], 4));
  }
  const int npanel = (nchunk + 7) / 8;
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < CPL; ++u)
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float t = __shfl_sync(0xffffffffu, s[u], 8 * g);  // panel 4u + g
      if (4 * u + g < npanel) acc = __fadd_rn(acc, t);
    }
  return __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(C)), eps));
}

// v <- bf16(v * r)
template <int CPL>
__device__ __forceinline__ void scale_round(float (&v)[CPL][8], float r) {
#pragma unroll
  for (int u = 0; u < CPL; ++u)
#pragma unroll
    for (int i = 0; i < 8; ++i) v[u][i] = round_bf16(__fmul_rn(v[u][i], r));
}

// One warp per row (any number of warps per block); C a multiple of 8 with C <= 256 * CPL; rows
// 16-byte aligned.
template <int CPL>
__global__ void __launch_bounds__(128) add_rms_norm_kernel(const AddNormParams p) {
  pdl_wait();  // inputs come from the kernel ahead (programmatic dependent launch)
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nchunk = p.C / 8;
  float v[CPL][8];
  load_row_chunks<CPL>(p.x + static_cast<long long>(row) * p.xs, lane, nchunk, v);
  if (p.delta) {
    const uint16_t* dr = p.delta + static_cast<long long>(row) * p.ds;
#pragma unroll
    for (int u = 0; u < CPL; ++u) {
      const int c = lane + 32 * u;
      if (c < nchunk) {
        const uint4 w = *reinterpret_cast<const uint4*>(dr + 8 * c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[u][2 * i] = round_bf16(__fadd_rn(v[u][2 * i], __uint_as_float(ws[i] << 16)));
          v[u][2 * i + 1] =
              round_bf16(__fadd_rn(v[u][2 * i + 1], __uint_as_float(ws[i] & 0xffff0000u)));
        }
      }
    }
    store_row_chunks<CPL>(p.x_out + static_cast<long long>(row) * p.xos, lane, nchunk, v);
  }
  const float r = row_rms_rsqrt<CPL>(v, lane, nchunk, p.C, p.eps);
  scale_round<CPL>(v, r);
  store_row_chunks<CPL>(p.h_out + static_cast<long long>(row) * p.hs, lane, nchunk, v);
}

struct EmbedNormParams {
  const int64_t* ids;
  const uint16_t* table;  // (V, C) bf16
  uint16_t* x_out;        // norm(table[id])
  uint16_t* h_out;        // norm(x_out), or null
  long long ts, xs, hs;   // row strides (elements)
  long long V;
  int rows, C;
  float eps;
};

// TokenEmbedding (wte lookup + norm) and the first block's norm in one pass: one warp per row.
// An id outside [0, V) records kErrTokenOutOfRange and writes zeros.
template <int CPL>
__global__ void __launch_bounds__(128) embed_rms_norm_kernel(const EmbedNormParams p) {
  pdl_wait();  // inputs come from the kernel ahead (programmatic dependent launch)
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nchunk = p.C / 8;
  const long long id = p.ids[row];
  float v[CPL][8];
  uint16_t* xo = p.x_out + static_cast<long long>(row) * p.xs;
  uint16_t* ho = p.h_out ? p.h_out + static_cast<long long>(row) * p.hs : nullptr;
  if (id < 0 || id >= p.V) {
    if (lane == 0) record_error(kErrTokenOutOfRange);
#pragma unroll
    for (int u = 0; u < CPL; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    store_row_chunks<CPL>(xo, lane, nchunk, v);
    if (ho) store_row_chunks<CPL>(ho, lane, nchunk, v);
    return;
  }
  load_row_chunks<CPL>(p.table + id * p.ts, lane, nchunk, v);
  scale_round<CPL>(v, row_rms_rsqrt<CPL>(v, lane, nchunk, p.C, p.eps));
  store_row_chunks<CPL>(xo, lane, nchunk, v);
  if (ho) {
    scale_round<CPL>(v, row_rms_rsqrt<CPL>(v, lane, nchunk, p.C, p.eps));
    store_row_chunks<CPL>(ho, lane, nchunk, v);
  }
}

struct GatedActParams {
  const uint16_t* gate;
  const uint16_t* up;
  uint16_t* out;
  long long gs, us, os;  // row strides (elements)
  int rows, H;
};

// bf16(bf16(silu(g)) * u) for bf16 values g and u held as floats: silu in fp32 as
// g / (1 + exp(-g)), rounded to bf16, then the product rounded -- torch's F.silu(g) * u on bf16
// tensors.  Shared by gated_silu_kernel and the gated projection (decode_proj.cuh).
__device__ __forceinline__ float silu_mul_bf16(float g, float u) {
  const float s = round_bf16(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))));
  return round_bf16(__fmul_rn(s, u));
}

// One thread per 8 elements (a 16-byte chunk); H a multiple of 8.
__global__ void __launch_bounds__(256) gated_silu_kernel(const GatedActParams p) {
  pdl_wait();  // inputs come from the kernel ahead (programmatic dependent launch)
  pdl_launch_dependents();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nchunk = p.H / 8;
  if (i >= static_cast<long long>(p.rows) * nchunk) return;
  const int row = static_cast<int>(i / nchunk);
  const int c = static_cast<int>(i - static_cast<long long>(row) * nchunk);
  const uint4 gv = *reinterpret_cast<const uint4*>(p.gate + row * p.gs + 8 * c);
  const uint4 uv = *reinterpret_cast<const uint4*>(p.up + row * p.us + 8 * c);
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t ow[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float g[2] = {__uint_as_float(gw[k] << 16), __uint_as_float(gw[k] & 0xffff0000u)};
    float u[2] = {__uint_as_float(uw[k] << 16), __uint_as_float(uw[k] & 0xffff0000u)};
    ow[k] = pack_bf16x2(silu_mul_bf16(g[0], u[0]), silu_mul_bf16(g[1], u[1]));
  }
  *reinterpret_cast<uint4*>(p.out + row * p.os + 8 * c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

struct SoftcapParams {
  const uint16_t* logits;  // (rows, V) bf16, row stride ls
  float* out;              // (rows, V) fp32, row stride os, or null
  int64_t* argmax;         // (rows,) int64 at stride as, or null
  long long ls, os, as;
  int rows, V;
  float cap;               // > 0: cap * tanh(x * inv_cap); otherwise x
  float inv_cap;           // 1 / cap in fp32
  int vec;                 // rows 16-byte aligned and V % 8 == 0: 16-byte loads, 32-byte stores
  int cs;                  // CTAs per row: one thread-block cluster of cs CTAs (1: no cluster)
};

constexpr int kSoftcapThreads = 256;

// torch evaluates `logits / cap` with a Python-number cap as logits * (1 / cap) on CUDA (the
// reciprocal rounded to fp32 once), then tanh, then `cap * t`.
__device__ __forceinline__ float softcap_value(float x, float cap, float inv_cap) {
  return cap > 0.f ? __fmul_rn(cap, tanhf(__fmul_rn(x, inv_cap))) : x;
}

// (a, ia) beats (b, ib) under torch.argmax's order: NaN above everything, then the larger value,
// then the smaller index.
__device__ __forceinline__ bool argmax_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

__device__ __forceinline__ void argmax_warp(float& best, int& bi) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (argmax_better(ob, oi, best, bi)) { best = ob; bi = oi; }
  }
}

// LMHead's epilogue, modelcore/components/unembedding.py:52-56 (crop to V, .float(), softcap),
// fused with the greedy pick of sample_next_token(temperature=0), modelcore/generate.py:23-24.
// A row is split over the cs CTAs of one cluster (cs consecutive blocks of the grid), each taking
// a contiguous range of 16-byte chunks (or elements); the per-CTA picks meet in rank 0 through
// distributed shared memory.  The pick does not depend on the split: argmax_better is a total
// order on (value, index).
__global__ void __launch_bounds__(kSoftcapThreads) softcap_argmax_kernel(const SoftcapParams p) {
  pdl_wait();  // inputs come from the kernel ahead (programmatic dependent launch)
  pdl_launch_dependents();
  const int row = blockIdx.x / p.cs;
  const int part = blockIdx.x % p.cs;
  const uint16_t* in = p.logits + static_cast<long long>(row) * p.ls;
  float* out = p.out ? p.out + static_cast<long long>(row) * p.os : nullptr;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int units = p.vec ? p.V / 8 : p.V;
  const int per = (units + p.cs - 1) / p.cs;
  const int u0 = part * per;
  const int u1 = min(units, u0 + per);
  if (p.vec) {
    for (int c = u0 + threadIdx.x; c < u1; c += kSoftcapThreads) {
      const uint4 w = *reinterpret_cast<const uint4*>(in + 8 * c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      float y[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        y[2 * i] = softcap_value(__uint_as_float(ws[i] << 16), p.cap, p.inv_cap);
        y[2 * i + 1] = softcap_value(__uint_as_float(ws[i] & 0xffff0000u), p.cap, p.inv_cap);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (argmax_better(y[i], 8 * c + i, best, bi)) { best = y[i]; bi = 8 * c + i; }
      if (out) {
        float4* o = reinterpret_cast<float4*>(out + 8 * c);
        o[0] = make_float4(y[0], y[1], y[2], y[3]);
        o[1] = make_float4(y[4], y[5], y[6], y[7]);
      }
    }
  } else {
    for (int j = u0 + threadIdx.x; j < u1; j += kSoftcapThreads) {
      const float y = softcap_value(bf16_bits_to_float(in[j]), p.cap, p.inv_cap);
      if (argmax_better(y, j, best, bi)) { best = y; bi = j; }
      if (out) out[j] = y;
    }
  }
  if (!p.argmax) return;  // uniform over the grid: no CTA of a cluster waits below
  argmax_warp(best, bi);
  constexpr int kWarps = kSoftcapThreads / 32;
  __shared__ float sb[kWarps];
  __shared__ int si[kWarps];
  __shared__ float cb;  // this CTA's pick, read by rank 0 of the cluster
  __shared__ int ci;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < kWarps ? sb[lane] : -INFINITY;
    bi = lane < kWarps ? si[lane] : 0x7fffffff;
    argmax_warp(best, bi);
    if (lane == 0) { cb = best; ci = bi; }
  }
  if (p.cs == 1) {
    if (threadIdx.x == 0) p.argmax[static_cast<long long>(row) * p.as] = ci;
    return;
  }
  cluster_sync();  // every CTA's pick is in its shared memory
  if (part == 0 && warp == 0) {
    best = -INFINITY;
    bi = 0x7fffffff;
    if (lane < p.cs) {
      best = ld_dsmem_f32(map_to_rank(&cb, lane));
      bi = __float_as_int(ld_dsmem_f32(map_to_rank(&ci, lane)));
    }
    argmax_warp(best, bi);
    if (lane == 0) p.argmax[static_cast<long long>(row) * p.as] = bi;
  }
  cluster_sync();  // rank 0 has read every CTA's shared memory before any of them exits
}

}  // namespace mcb
