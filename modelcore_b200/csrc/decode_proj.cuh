// The decode step's projections, with the Block's elementwise ops around them fused:
//
//   plain:       Y = X W^T
//   norm:        Y = rms_norm(X) W^T           (the Block's norm in front of the packed q|k|v or
//                                               gate|up projection, modelcore/components/block.py
//                                               :57-59, norm.py:43-44; the bits of
//                                               mcb_add_rms_norm's h)
//   add + norm:  X' = bf16(X + delta) is written out, Y = rms_norm(X') W^T   (the residual add
//                                               of the previous block's MLP, then the norm)
//   residual:    Y = bf16(res + bf16(X W^T))   (the residual add after c_proj, block.py:58; res
//                                               may be Y itself: in place)
//   norm out:    Y = bf16(res + bf16(X W^T)), H = rms_norm(Y)   (c_proj's residual add and the
//                                               Block's next norm, block.py:58-59: one output row
//                                               spans the CTAs of a thread-block cluster, each
//                                               holding one 64-column panel; the per-row panel
//                                               sums of squares meet in distributed shared memory
//                                               -- the bits of mcb_add_rms_norm over Y)
//   gated:       Y = silu(X Wg^T) * (X Wu^T)   (GatedMLP's gate|up projection and act(gate) * up,
//                                               modelcore/components/mlp.py:89-90, with W the
//                                               packed [Wg; Wu]: each CTA takes F/2 gate rows
//                                               and the matching F/2 up rows, and its epilogue
//                                               rounds both sums to bf16 and applies
//                                               silu_mul_bf16 -- the bits of mcb_gated_silu over
//                                               the plain projection)
//
// At decode a projection multiplies R <= 64 rows (one token per sequence) by an N x K weight: the
// work is streaming W from HBM once; the activation block (64 x K bf16, about 100 KB) sits in L2.
// Each CTA takes a slice of F = 16 or 32 output features and ALL of K, so no CTA needs another's
// partial sums and the norm sees whole rows:
//
//   * the W slice (F x K) is requested by TMA at entry, before griddepcontrol.wait: under
//     programmatic dependent launch the weight stream overlaps the kernel ahead; the activation
//     panels (64 columns each, 128-byte swizzled) follow once the kernel ahead has completed;
//   * the products run on warp-level tensor-core MMAs (mma.sync m16n8k16, fp32 accumulate): the
//     8 warps split K, each warp covering all 64 rows x F features of its K range, then the 8
//     partial tiles are summed in warp order.  For these shapes -- 64 x 16 outputs, K in
//     hundreds -- the per-instruction cost of tcgen05.mma with M = 128, N = 16 (measured about
//     0.38 us per 64 columns of K) exceeds the whole product on mma.sync (about 2 clocks per
//     m16n8k16 per SM, 0.4 us for 64 x 16 x 768);
//   * norm: once all panels are resident the 8 warps take all 64 rows at once (four lanes a row)
//     and compute their fp32 sums of squares in the fixed order mcb_add_rms_norm uses
//     (step_fused.cuh row_rms_rsqrt: chunk, 8-chunk panel tree, panels in order), then rescale
//     them in place;
//   * epilogue: round once to bf16 (residual: add the residual row, round again, as torch's
//     `x + y` does) and store 16 bytes a thread.
//
// Every mbarrier wait is bounded; a timeout raises the CTA's abort flag, skips the stores and
// waits (bounded) for the CTA's copies in flight before it exits.
#pragma once

#include "common.cuh"
#include "step_fused.cuh"  // the norm's summation order (row_rms_rsqrt)

namespace mcb {

constexpr int kProjThreads = 256;
constexpr int kProjWarps = kProjThreads / 32;
constexpr int kProjRows = 64;        // rows of the activation block (R <= 64)
constexpr int kProjNormCpl = 4;      // the norm takes K <= 4 * 4 * 64 (as mcb_add_rms_norm's limit)
constexpr int kProjPanel = kProjRows * 128;  // one 64-column activation panel, bytes

struct ProjParams {
  const uint16_t* res;   // residual (R, N) added to the product, or null
  uint16_t* y;           // (R, N)
  uint16_t* x_out;       // add + norm: X + delta (R, K), written by CTA 0
  uint16_t* h_out;       // norm out: rms_norm(Y) (R, N)
  long long ress, ys, xos, hs;  // row strides (elements)
  int R, N, K;
  int panels;            // K / 64
  int vec_out;           // y (and res) rows 16-byte aligned, N % 8 == 0
  float eps;             // norm
};

// Shared memory, from a 1024-byte aligned base (offsets in bytes):
//   W       panels x (F rows x 128 B): the CTA's weight slice, 128-byte swizzled K-major
//   X       panels x 8 KB: the activation panels (64 rows x 128 B, swizzled); after the MMAs the
//           8 warps' fp32 partial tiles [8][64][F]
//   delta   add + norm: panels x 8 KB
//   bars    full[panels] (X, and delta), w_full, abort flag
__host__ __device__ __forceinline__ int proj_x_offset(int F, int panels) {
  return (panels * F * 128 + 1023) & ~1023;
}
// rb: the rows of one CTA's activation block (64; 32 when a row block splits over two CTAs)
__host__ __device__ __forceinline__ int proj_x_bytes(int F, int panels, int rb = kProjRows) {
  const int a = panels * rb * 128, b = kProjWarps * rb * F * 4;
  return a > b ? a : b;
}
__host__ __device__ __forceinline__ int proj_bar_offset(int F, int panels, bool add, int rb = kProjRows) {
  return proj_x_offset(F, panels) + proj_x_bytes(F, panels, rb) + (add ? panels * rb * 128 : 0);
}
__host__ __device__ __forceinline__ int proj_smem_bytes(int F, int panels, bool add, int rb = kProjRows) {
  return proj_bar_offset(F, panels, add, rb) + (panels + 2) * 8 + 1024;
}

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// RB = 32: the 64-row block is split over two CTAs (grid.y), each with all of K -- for the wide-K
// projections (down_proj: K = the MLP width) whose 64-row activation block would not fit; every
// output's sum is the same warp-ordered reduction over K as with RB = 64.  RB = 16 (norm out):
// four row blocks, each a cluster of N / 64 CTAs of 64 features.
template <int F, bool NORM, bool ADD, bool GATED = false, int RB = kProjRows, bool NOUT = false>
__global__ void __launch_bounds__(kProjThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ CUtensorMap dmap, const ProjParams p) {
  static_assert(!ADD || NORM, "the add is fused only in front of the norm");
  static_assert(!GATED || (!NORM && F % 16 == 0), "the gated epilogue stands alone, F/2 a multiple of 8");
  constexpr int NT = F / 8;  // n-tiles of 8 features (of the W slice)
  constexpr int FO = GATED ? F / 2 : F;  // output features a CTA
  static_assert(RB == kProjRows || ((RB == 32 || RB == 16) && !NORM), "row-split blocks: no norm in front");
  static_assert(!NOUT || (F == 64 && !NORM && !GATED && RB * 8 <= kProjThreads),
                "norm out: one 64-column panel a CTA, eight threads a row");
  constexpr int PANEL = RB * 128;        // one 64-column activation panel of the CTA's rows, bytes
  constexpr int MT = RB / 16;            // m-tiles of 16 rows
  const int row0 = static_cast<int>(blockIdx.y) * RB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int panels = p.panels;
  const int n0 = static_cast<int>(blockIdx.x) * FO;
  uint8_t* wsm = smem;
  uint8_t* xsm = smem + proj_x_offset(F, panels);
  uint8_t* dsm = xsm + proj_x_bytes(F, panels, RB);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + proj_bar_offset(F, panels, ADD, RB));
  uint64_t* w_full = full + panels;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(w_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i <= panels; ++i) mbar_init(full + i, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    // the weights do not depend on the kernel ahead: request them before griddepcontrol.wait
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    if (ADD) prefetch_tensormap(&dmap);
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(panels * F * 128));
    for (int i = 0; i < panels; ++i) {
      // gated: the gate rows n0 .. n0 + F/2 - 1, then the up rows N + n0 .. (boxes of F/2 rows;
      // the second starts at a 1024-byte boundary of the panel, so the swizzle phase holds)
      tma_load_4d(wsm + i * F * 128, &wmap, w_full, i * 64, n0, 0, 0, pol);
      if (GATED) tma_load_4d(wsm + i * F * 128 + FO * 128, &wmap, w_full, i * 64, p.N + n0, 0, 0, pol);
    }
  }
  __syncthreads();  // barriers initialised
  pdl_wait();       // the activations and the residual come from the kernels ahead
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < panels; ++i) {
      mbar_arrive_expect_tx(&full[i], ADD ? 2 * PANEL : PANEL);
      tma_load_4d(xsm + i * PANEL, &xmap, &full[i], i * 64, row0, 0, 0, 0ull);
      if (ADD) tma_load_4d(dsm + i * PANEL, &dmap, &full[i], i * 64, row0, 0, 0, 0ull);
    }
  }
  __syncwarp();  // lane 0 of warp 0 rejoins before its warp waits on anything

  bool ok = true;
  if constexpr (NORM) {
    for (int i = 0; i < panels; ++i) ok = ok && mbar_wait_or_abort(&full[i], 0, abort_flag);
    ok = __syncthreads_and(ok);
    // All 64 rows in one pass: warp w takes rows 8w .. 8w+7, four lanes a row; lane `sub` holds
    // chunks 2 sub and 2 sub + 1 of every 64-column panel.  The fp32 sum of squares keeps
    // row_rms_rsqrt's order (step_fused.cuh): each chunk element by element, the panel's
    // pairwise tree -- its first level in the lane, the next two over xor 1 and 2 among the four
    // lanes -- and the panels in order, which every lane of the row adds identically.  Chunks
    // {2 sub, 2 sub + 1} of two consecutive rows land in disjoint swizzled slots: no bank
    // conflicts.  add + norm first writes X' = X + delta (CTA 0 also to x_out).
    const int r = warp * 8 + (lane >> 2), sub = lane & 3;
    const uint32_t xs_addr = smem_u32(xsm), ds_addr = smem_u32(dsm);
    float acc = 0.f;
    for (int pl = 0; pl < panels; ++pl) {
      float part[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 2 * sub + h;
        const uint32_t off = pl * kProjPanel + swz128(r, c);
        uint4 xv = ok ? lds128(xs_addr + off) : make_uint4(0, 0, 0, 0);
        uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        if (ADD && ok) {
          const uint4 dv = lds128(ds_addr + off);
          const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k)
            xw[k] = pack_bf16x2(__fadd_rn(__uint_as_float(xw[k] << 16), __uint_as_float(dw[k] << 16)),
                                __fadd_rn(__uint_as_float(xw[k] & 0xffff0000u), __uint_as_float(dw[k] & 0xffff0000u)));
          xv = make_uint4(xw[0], xw[1], xw[2], xw[3]);
          sts128(xs_addr + off, xv);
          if (blockIdx.x == 0 && r < p.R)
            *reinterpret_cast<uint4*>(p.x_out + static_cast<long long>(r) * p.xos + pl * 64 + c * 8) = xv;
        }
        float sq = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float e0 = __uint_as_float(xw[k] << 16), e1 = __uint_as_float(xw[k] & 0xffff0000u);
          sq = __fadd_rn(sq, __fmul_rn(e0, e0));
          sq = __fadd_rn(sq, __fmul_rn(e1, e1));
        }
        part[h] = sq;
      }
      float t = __fadd_rn(part[0], part[1]);
      t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
      t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
      acc = __fadd_rn(acc, t);
    }
    const float sc = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.K)), p.eps));
    for (int pl = 0; ok && pl < panels; ++pl) {  // h = bf16(X' * scale) in place
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t a = xs_addr + pl * kProjPanel + swz128(r, 2 * sub + h);
        const uint4 v = lds128(a);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = pack_bf16x2(__fmul_rn(__uint_as_float(w[k] << 16), sc),
                             __fmul_rn(__uint_as_float(w[k] & 0xffff0000u), sc));
        sts128(a, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
    __syncthreads();
  }
  ok = mbar_wait_or_abort(w_full, 0, abort_flag) && ok;

  // ---------------- products: warp w takes K steps [ks0, ks1) of 16 columns ----------------
  float acc[MT][NT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
  const int KS = panels * 4;
  const int ks0 = warp * KS / kProjWarps, ks1 = (warp + 1) * KS / kProjWarps;
  const uint32_t xb = smem_u32(xsm), wb = smem_u32(wsm);
  for (int ks = ks0; ks < ks1; ++ks) {
    const int pnl = ks >> 2;
    if (!NORM && ok && (ks == ks0 || (ks & 3) == 0)) ok = mbar_wait_or_abort(&full[pnl], 0, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform: ldmatrix and mma are collective
    const int kc = (ks & 3) * 2;  // first 8-column chunk of the step within the panel
    uint32_t a[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int row = mt * 16 + (lane & 15);
      ldsm_x4(xb + pnl * PANEL + swz128(row, kc + (lane >> 4)), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
    }
    uint32_t b[NT][2];
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      const int f = np * 16 + (lane & 7) + ((lane >> 4) << 3);
      ldsm_x4(wb + pnl * F * 128 + swz128(f, kc + ((lane >> 3) & 1)), b[2 * np][0], b[2 * np][1],
              b[2 * np + 1][0], b[2 * np + 1][1]);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        mma_16816(acc[mt][nt], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[nt][0], b[nt][1]);
  }
  __syncthreads();  // every warp is done reading X: its bytes take the partial tiles
  float* red = reinterpret_cast<float*>(xsm);  // [warp][RB][F]
  {
    const int g = lane >> 2, cq = (lane & 3) * 2;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint32_t a0 = smem_u32(red + (warp * RB + mt * 16 + g) * F + nt * 8 + cq);
        asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a0), "f"(acc[mt][nt][0]), "f"(acc[mt][nt][1]) : "memory");
        asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a0 + 32 * F), "f"(acc[mt][nt][2]), "f"(acc[mt][nt][3])
                     : "memory");
      }
  }
  __syncthreads();
  const bool have = !*abort_flag;
  if constexpr (NOUT) {
    // ---------------- epilogue, norm out: thread (row, chunk) = (tid / 8, tid % 8) ----------------
    // y = bf16(res + bf16(sum of the warps' partials in order)); the chunk's fp32 sum of squares
    // element by element, the panel's pairwise tree over the row's eight lanes (xor 1, 2, 4), the
    // panels -- one a CTA, cluster rank = panel -- added in order from 0: row_rms_rsqrt's order.
    float* psum = reinterpret_cast<float*>(wsm);  // [RB] this panel's row sums (W is consumed)
    const int lrow = threadIdx.x >> 3, c = threadIdx.x & 7;
    const int row = row0 + lrow;
    const bool act = threadIdx.x < RB * 8;      // whole warps: RB * 8 is a multiple of 32
    const bool live = act && have && row < p.R;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (live) {
#pragma unroll
      for (int w = 0; w < kProjWarps; ++w) {
        const uint32_t ra = smem_u32(red + (w * RB + lrow) * F + c * 8);
        const uint4 lo = lds128(ra), hi = lds128(ra + 16);
        const float t[8] = {__uint_as_float(lo.x), __uint_as_float(lo.y), __uint_as_float(lo.z), __uint_as_float(lo.w),
                            __uint_as_float(hi.x), __uint_as_float(hi.y), __uint_as_float(hi.z), __uint_as_float(hi.w)};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = w == 0 ? t[i] : __fadd_rn(v[i], t[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = round_bf16(v[i]);
      if (p.res != nullptr) {
        const uint4 w = *reinterpret_cast<const uint4*>(p.res + static_cast<long long>(row) * p.ress + n0 + c * 8);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = round_bf16(__fadd_rn(__uint_as_float(ws[i] << 16), v[2 * i]));
          v[2 * i + 1] = round_bf16(__fadd_rn(__uint_as_float(ws[i] & 0xffff0000u), v[2 * i + 1]));
        }
      }
      *reinterpret_cast<uint4*>(p.y + static_cast<long long>(row) * p.ys + n0 + c * 8) =
          make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                     pack_bf16x2(v[6], v[7]));
    }
    if (act) {
      float sq = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) sq = __fadd_rn(sq, __fmul_rn(v[i], v[i]));
      sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 1));
      sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 2));
      sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 4));
      if (c == 0) psum[lrow] = sq;
    }
    cluster_sync();  // every CTA's panel sums are published
    if (live) {
      float acc = 0.f;
      const int npanel = static_cast<int>(gridDim.x);  // the cluster spans the row
      for (int q = 0; q < npanel; ++q) acc = __fadd_rn(acc, ld_dsmem_f32(map_to_rank(psum + lrow, q)));
      const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.N)), p.eps));
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = pack_bf16x2(__fmul_rn(v[2 * i], r), __fmul_rn(v[2 * i + 1], r));
      *reinterpret_cast<uint4*>(p.h_out + static_cast<long long>(row) * p.hs + n0 + c * 8) =
          make_uint4(h[0], h[1], h[2], h[3]);
    }
    cluster_sync();  // no CTA leaves while another still reads its panel sums
  }
  // ---------------- epilogue: 8 features a thread, warps summed in order ----------------
  for (int it = threadIdx.x; !NOUT && have && it < RB * (FO / 8); it += kProjThreads) {
    const int lrow = it / (FO / 8), f8 = (it % (FO / 8)) * 8;
    const int row = row0 + lrow;
    if (row >= p.R) continue;
    float o[8], ou[8];  // ou: the matching up features (gated)
#pragma unroll
    for (int w = 0; w < kProjWarps; ++w) {
      const uint32_t ra = smem_u32(red + (w * RB + lrow) * F + f8);
      const uint4 lo = lds128(ra), hi = lds128(ra + 16);
      const float t[8] = {__uint_as_float(lo.x), __uint_as_float(lo.y), __uint_as_float(lo.z), __uint_as_float(lo.w),
                          __uint_as_float(hi.x), __uint_as_float(hi.y), __uint_as_float(hi.z), __uint_as_float(hi.w)};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = w == 0 ? t[i] : __fadd_rn(o[i], t[i]);
      if constexpr (GATED) {
        const uint4 ulo = lds128(ra + FO * 4), uhi = lds128(ra + FO * 4 + 16);
        const float tu[8] = {__uint_as_float(ulo.x), __uint_as_float(ulo.y), __uint_as_float(ulo.z),
                             __uint_as_float(ulo.w), __uint_as_float(uhi.x), __uint_as_float(uhi.y),
                             __uint_as_float(uhi.z), __uint_as_float(uhi.w)};
#pragma unroll
        for (int i = 0; i < 8; ++i) ou[i] = w == 0 ? tu[i] : __fadd_rn(ou[i], tu[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = round_bf16(o[i]);
    if constexpr (GATED) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = silu_mul_bf16(o[i], round_bf16(ou[i]));
    }
    uint16_t* yr = p.y + static_cast<long long>(row) * p.ys + n0 + f8;
    const uint16_t* rr = p.res ? p.res + static_cast<long long>(row) * p.ress + n0 + f8 : nullptr;
    if (p.vec_out && n0 + f8 + 8 <= p.N) {
      if (rr != nullptr) {
        const uint4 w = *reinterpret_cast<const uint4*>(rr);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[2 * i] = __fadd_rn(__uint_as_float(ws[i] << 16), o[2 * i]);
          o[2 * i + 1] = __fadd_rn(__uint_as_float(ws[i] & 0xffff0000u), o[2 * i + 1]);
        }
      }
      *reinterpret_cast<uint4*>(yr) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                 pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (n0 + f8 + i < p.N)
          yr[i] = float_to_bf16_bits(rr != nullptr ? __fadd_rn(bf16_bits_to_float(rr[i]), o[i]) : o[i]);
    }
  }
  if (threadIdx.x == 0 && *abort_flag) {  // copies in flight land before the CTA exits
    mbar_wait(w_full, 0);
    for (int i = 0; i < panels; ++i) mbar_wait(&full[i], 0);
  }
}

}  // namespace mcb
