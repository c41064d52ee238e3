// The decode step either side of attention: the residual add fused with the next RMSNorm, and
// GatedMLP's act(gate) * up, for one (rows, C) bf16 activation block per launch.
//
//   add_rms_norm:  x' = bf16(x + delta)                    (Block: x = x + mixer(..) / ffn(..),
//                  h  = bf16(x' * rsqrt(mean(x'^2) + eps))  modelcore/components/block.py:57-59,
//                                                            then norm, modelcore/components/norm.py:43-44)
//   gated_silu:    out = bf16(bf16(silu(gate)) * up)        (GatedMLP.forward, modelcore/components/mlp.py:89-90)
//
// Rounding follows torch's bf16 ops: the add is computed in fp32 and rounded once; rms_norm
// accumulates the sum of squares in fp32, in this kernel's fixed order (lane l adds the squares of
// its 16-byte chunks c = l, l+32, .. in order, element by element, then an xor butterfly over
// masks 16 .. 1), and rounds once; silu is computed in fp32 as g / (1 + exp(-g)) and rounded, the
// product in fp32 and rounded.  The CPU oracle restates the same order.
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

// One warp per row; C a multiple of 8 with C <= 256 * CPL (CPL 16-byte chunks per lane); rows
// 16-byte aligned.
template <int CPL>
__global__ void __launch_bounds__(128) add_rms_norm_kernel(const AddNormParams p) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nchunk = p.C / 8;
  const uint16_t* xr = p.x + static_cast<long long>(row) * p.xs;
  const uint16_t* dr = p.delta ? p.delta + static_cast<long long>(row) * p.ds : nullptr;
  uint16_t* xo = p.x_out ? p.x_out + static_cast<long long>(row) * p.xos : nullptr;
  uint16_t* ho = p.h_out + static_cast<long long>(row) * p.hs;
  constexpr int MAXC = CPL;
  float v[MAXC][8];
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < MAXC; ++u) {
    const int c = lane + 32 * u;
    if (c < nchunk) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + 8 * c);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      uint32_t dw[4] = {0, 0, 0, 0};
      if (dr) {
        const uint4 dv = *reinterpret_cast<const uint4*>(dr + 8 * c);
        dw[0] = dv.x; dw[1] = dv.y; dw[2] = dv.z; dw[3] = dv.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a0 = __uint_as_float(xw[i] << 16), a1 = __uint_as_float(xw[i] & 0xffff0000u);
        if (dr) {
          a0 = round_bf16(__fadd_rn(a0, __uint_as_float(dw[i] << 16)));
          a1 = round_bf16(__fadd_rn(a1, __uint_as_float(dw[i] & 0xffff0000u)));
        }
        v[u][2 * i] = a0;
        v[u][2 * i + 1] = a1;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(v[u][i], v[u][i]));
      if (xo) {
        uint4 o;
        o.x = pack_bf16x2(v[u][0], v[u][1]);
        o.y = pack_bf16x2(v[u][2], v[u][3]);
        o.z = pack_bf16x2(v[u][4], v[u][5]);
        o.w = pack_bf16x2(v[u][6], v[u][7]);
        *reinterpret_cast<uint4*>(xo + 8 * c) = o;
      }
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
  const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.C)), p.eps));
#pragma unroll
  for (int u = 0; u < MAXC; ++u) {
    const int c = lane + 32 * u;
    if (c < nchunk) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(v[u][i], r);
      uint4 ov;
      ov.x = pack_bf16x2(o[0], o[1]);
      ov.y = pack_bf16x2(o[2], o[3]);
      ov.z = pack_bf16x2(o[4], o[5]);
      ov.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(ho + 8 * c) = ov;
    }
  }
}

struct GatedActParams {
  const uint16_t* gate;
  const uint16_t* up;
  uint16_t* out;
  long long gs, us, os;  // row strides (elements)
  int rows, H;
};

// One thread per 8 elements (a 16-byte chunk); H a multiple of 8.
__global__ void __launch_bounds__(256) gated_silu_kernel(const GatedActParams p) {
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
    float o[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float s = round_bf16(__fdiv_rn(g[e], __fadd_rn(1.f, expf(-g[e]))));
      o[e] = __fmul_rn(s, u[e]);
    }
    ow[k] = pack_bf16x2(o[0], o[1]);
  }
  *reinterpret_cast<uint4*>(p.out + row * p.os + 8 * c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

}  // namespace mcb
