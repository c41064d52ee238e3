// The decode step's projections on the tensor cores, with the elementwise op before each one
// fused into its operand load:
//
//   none:        Y = X W^T
//   add + norm:  x' = bf16(x + delta), h = rms_norm(x'), Y = h W^T   (Block's residual add and the
//                next norm, modelcore/components/block.py:57-59 and norm.py:43-44, in front of the
//                packed q|k|v or gate|up projection; x' is written out as the new residual)
//   gated silu:  a = bf16(bf16(silu(gate)) * up), Y = a W^T          (GatedMLP.forward,
//                modelcore/components/mlp.py:89-90, in front of down_proj)
//
// At decode a projection multiplies R <= 128 rows (one token per sequence) by an N x K weight:
// the work is streaming W from HBM once.  The kernel spreads W over about one CTA per SM:
//
//   * CTA = 128 output features (the MMA's M, rows of W as nn.Linear stores them) x a range of
//     64-column K panels; the `split` CTAs that share an output tile form one thread-block
//     cluster and cut K between them (uneven when the panels do not divide);
//   * every W panel of the CTA is issued by TMA at entry, before griddepcontrol.wait: under
//     programmatic dependent launch the weight stream overlaps the kernel ahead;
//   * after the wait all threads load the CTA's activation columns (RN = 64 or 128 rows, zero
//     past R), apply the prologue and store the operand into shared memory in the 128-byte
//     swizzled K-major layout the MMA descriptor reads;
//   * one thread issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N RN, K 16 each), fp32 in TMEM;
//   * split > 1: each CTA parks its fp32 partial tile in shared memory and bulk-copies each
//     rank's share of the rows into that rank's shared memory (cp.async.bulk shared::cta ->
//     shared::cluster, counted on the receiver's mbarrier); rank q sums the split partials of its
//     rows in rank order, rounds once to bf16 and writes them -- no workspace, no atomics, the
//     same bits every run.  Two cluster barriers, each split into arrive and wait: the first
//     (mbarriers initialised) is waited for only before the first send, the second (everything a
//     rank is sent has landed) only before exit, so a CTA never leaves while its shared memory is
//     still being copied out.
//
// The norm needs a statistic of the whole row while a CTA holds only its K panels.  Its fp32 sum
// of squares has one fixed order, the one mcb_add_rms_norm uses too (step_fused.cuh): squares
// summed element by element within each 8-element chunk, a pairwise tree over the 8 chunks of a
// 64-column panel, then the panels in order.  Each CTA computes its panels' partials and
// bulk-copies them to every rank of the cluster; every CTA then adds all panels of each row in
// panel order -- h is bit-identical to the stand-alone kernel's.
//
// Every mbarrier wait is bounded; a timeout raises the CTA's abort flag, the CTA skips its
// stores, waits (bounded) for copies in flight, frees TMEM and still reaches every cluster
// barrier, so no CTA of a cluster waits for one that gave up.
#pragma once

#include "common.cuh"
#include "prefill_attn.cuh"  // tcgen05 helpers

namespace mcb {

constexpr int kProjFeat = 128;       // output features per CTA (MMA M)
constexpr int kProjThreads = 256;
constexpr int kProjMaxPanels = 6;    // 64-column K panels per CTA (RN 128: at most 3)
constexpr int kProjMaxSplit = 16;
constexpr int kProjBatch = 8;        // operand chunks a thread loads in flight together

enum ProjPrologue { kProNone = 0, kProAddNorm = 1, kProGatedSilu = 2 };

struct ProjParams {
  const uint16_t* a;   // none: X; add + norm: the residual x; gated silu: gate       (R, K)
  const uint16_t* b;   // add + norm: delta, or null (h = rms_norm(x)); gated silu: up  (R, K)
  uint16_t* a_out;     // add + norm with delta: x + delta (R, K), written by the first tile's CTAs
  uint16_t* y;         // (R, N)
  long long as, bs, aos, ys;   // row strides (elements)
  int R, N, K;
  int panels;          // K / 64
  int split;           // CTAs per output tile (cluster size)
  int max_np;          // largest panel count of a CTA (sizes the shared-memory layout)
  int vec_out;         // y 16-byte aligned, ys and N multiples of 8: 16-byte stores
  float eps;
};

// Panels [p0, p1) of rank q of `split`.
__host__ __device__ __forceinline__ int proj_panel0(int q, int panels, int split) {
  return static_cast<int>((static_cast<long long>(q) * panels) / split);
}

// Shared memory, from a 1024-byte aligned base (offsets in bytes):
//   operand   W panels (16 KB each: 128 rows x 128 B), then the activation panels (RN x 128 B
//             each); once the MMAs are done the same bytes hold this CTA's fp32 partial tile
//             [RN][128] and the staged bf16 output rows [RN][128]
//   recv      split > 1: the partial rows every rank sends this one, [split][per][128] fp32
//   ops_all   add + norm: every panel's partial sums of squares, [panels][RN] fp32
//   ops_loc   add + norm: this CTA's panels' partial sums, [np][RN] fp32
//   scale     the rows' 1 / rms, [RN]
//   bars      w_full, mma_done, recv_full, ops_full, TMEM slot, abort flag
struct ProjSmem {
  int recv, ops_all, ops_loc, scale, bars, total;
};
__host__ __device__ __forceinline__ ProjSmem proj_smem(int RN, int max_np, int split, int panels, bool norm) {
  ProjSmem L;
  const int operand = max_np * (16384 + RN * 128);
  const int reuse = RN * kProjFeat * 4 + RN * kProjFeat * 2;
  const int per = (RN + split - 1) / split;
  L.recv = ((operand > reuse ? operand : reuse) + 1023) & ~1023;
  L.ops_all = L.recv + (split > 1 ? split * per * kProjFeat * 4 : 0);
  L.ops_loc = L.ops_all + (norm ? panels * RN * 4 : 0);
  L.scale = L.ops_loc + (norm ? kProjMaxPanels * RN * 4 : 0);
  L.bars = L.scale + RN * 4;
  L.total = L.bars + 64 + 1024;  // + alignment slack of the dynamic shared memory base
  return L;
}

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int RN, int PRO>
__global__ void __launch_bounds__(kProjThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap wmap, const ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr bool kNorm = PRO == kProAddNorm;
  const int split = p.split;
  const int tile = static_cast<int>(blockIdx.x) / split;
  const int rank = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int p0 = proj_panel0(rank, p.panels, split);
  const int np = proj_panel0(rank + 1, p.panels, split) - p0;
  const int n0 = tile * kProjFeat;
  const ProjSmem L = proj_smem(RN, p.max_np, split, p.panels, kNorm);
  constexpr int kXPanel = RN * 128;
  uint8_t* wsm = smem;
  uint8_t* xsm = smem + p.max_np * 16384;
  float* part = reinterpret_cast<float*>(smem);                                   // [RN][128]
  uint16_t* staged = reinterpret_cast<uint16_t*>(smem + RN * kProjFeat * 4);       // [RN][128]
  float* recv = reinterpret_cast<float*>(smem + L.recv);
  float* ops_all = reinterpret_cast<float*>(smem + L.ops_all);
  float* ops_loc = reinterpret_cast<float*>(smem + L.ops_loc);
  float* rowscale = reinterpret_cast<float*>(smem + L.scale);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* w_full = bars;
  uint64_t* mma_done = bars + 1;
  uint64_t* recv_full = bars + 2;
  uint64_t* ops_full = bars + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 5);
  // output rows [r0, r1) are reduced and written by this rank
  const int per = (RN + split - 1) / split;
  const int r0 = rank * per < RN ? rank * per : RN;
  const int r1 = r0 + per < RN ? r0 + per : RN;

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(recv_full, 1);
    mbar_init(ops_full, 1);
    *abort_flag = 0;
    // the bytes the other ranks will send, armed before any of them may (cluster barrier below)
    if (split > 1) mbar_arrive_expect_tx(recv_full, static_cast<uint32_t>(split * (r1 - r0) * kProjFeat * 4));
    if (kNorm && split > 1) mbar_arrive_expect_tx(ops_full, static_cast<uint32_t>(p.panels * RN * 4));
    fence_mbarrier_init();
    // the weights do not depend on the kernel ahead: issue them before griddepcontrol.wait
    prefetch_tensormap(&wmap);
    const uint64_t pol = l2_policy_evict_first();
    mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(np) * 16384u);
    for (int i = 0; i < np; ++i)
      tma_load_4d(wsm + i * 16384, &wmap, w_full, (p0 + i) * 64, n0, 0, 0, pol);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, RN);
    tmem_relinquish();
  }
  if (split > 1) cluster_arrive_relaxed();  // phase 1: this CTA's mbarriers are initialised
  pdl_wait();  // the activations come from the kernel ahead

  // ---------------- operand: RN rows x np panels, 16-byte chunks, prologue applied ----------------
  // item = (row * np + panel) * 8 + chunk: eight consecutive lanes hold the eight chunks of one
  // row's panel (the norm's per-panel tree runs over them with xor shuffles).
  const int items = RN * np * 8;
  for (int it0 = 0; it0 < items; it0 += kProjThreads * kProjBatch) {
    uint4 va[kProjBatch], vb[kProjBatch];
#pragma unroll
    for (int j = 0; j < kProjBatch; ++j) {  // all loads of the batch in flight together
      const int it = it0 + j * kProjThreads + static_cast<int>(threadIdx.x);
      va[j] = make_uint4(0, 0, 0, 0);
      vb[j] = make_uint4(0, 0, 0, 0);
      const int r = it / (np * 8);
      if (it < items && r < p.R) {
        const int col = (p0 + (it / 8) % np) * 64 + (it & 7) * 8;
        va[j] = *reinterpret_cast<const uint4*>(p.a + static_cast<long long>(r) * p.as + col);
        if (PRO == kProGatedSilu || (kNorm && p.b != nullptr))
          vb[j] = *reinterpret_cast<const uint4*>(p.b + static_cast<long long>(r) * p.bs + col);
      }
    }
#pragma unroll
    for (int j = 0; j < kProjBatch; ++j) {
      const int it = it0 + j * kProjThreads + static_cast<int>(threadIdx.x);
      const int r = it / (np * 8);
      const int pl = (it / 8) % np, c = it & 7;
      uint4 o = va[j];
      if (PRO == kProGatedSilu) {
        const uint32_t gw[4] = {va[j].x, va[j].y, va[j].z, va[j].w};
        const uint32_t uw[4] = {vb[j].x, vb[j].y, vb[j].z, vb[j].w};
        uint32_t ow[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float g[2] = {__uint_as_float(gw[k] << 16), __uint_as_float(gw[k] & 0xffff0000u)};
          float u[2] = {__uint_as_float(uw[k] << 16), __uint_as_float(uw[k] & 0xffff0000u)};
          float s[2];
#pragma unroll
          for (int e = 0; e < 2; ++e)
            s[e] = __fmul_rn(round_bf16(__fdiv_rn(g[e], __fadd_rn(1.f, expf(-g[e])))), u[e]);
          ow[k] = pack_bf16x2(s[0], s[1]);
        }
        o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      } else if (kNorm) {
        const uint32_t xw[4] = {va[j].x, va[j].y, va[j].z, va[j].w};
        const uint32_t dw[4] = {vb[j].x, vb[j].y, vb[j].z, vb[j].w};
        uint32_t ow[4];
        float sq = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float v0 = __uint_as_float(xw[k] << 16), v1 = __uint_as_float(xw[k] & 0xffff0000u);
          if (p.b != nullptr) {
            v0 = round_bf16(__fadd_rn(v0, __uint_as_float(dw[k] << 16)));
            v1 = round_bf16(__fadd_rn(v1, __uint_as_float(dw[k] & 0xffff0000u)));
          }
          sq = __fadd_rn(sq, __fmul_rn(v0, v0));
          sq = __fadd_rn(sq, __fmul_rn(v1, v1));
          ow[k] = pack_bf16x2(v0, v1);
        }
        o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        // the panel's pairwise tree over its 8 chunks (lanes 8g .. 8g + 7)
        sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 1));
        sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 2));
        sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 4));
        if (it < items) {
          if (c == 0) ops_loc[pl * RN + r] = sq;
          if (p.a_out != nullptr && tile == 0 && r < p.R)
            *reinterpret_cast<uint4*>(p.a_out + static_cast<long long>(r) * p.aos + (p0 + pl) * 64 + c * 8) = o;
        }
      }
      if (it < items) *reinterpret_cast<uint4*>(xsm + pl * kXPanel + swz128(r, c)) = o;
    }
  }

  if (kNorm) {
    // every rank's panel partials, then each row's total in panel order 0 .. panels-1
    const float* tot = ops_loc;
    if (split > 1) {
      fence_proxy_async_shared();  // ops_loc is read by the bulk copies below
      __syncthreads();
      cluster_wait();              // phase 1: every rank's mbarriers are initialised
      if (threadIdx.x < split)
        bulk_copy_to_peer(map_to_rank(ops_all + p0 * RN, threadIdx.x), ops_loc,
                          static_cast<uint32_t>(np * RN * 4), map_to_rank(ops_full, threadIdx.x));
      mbar_wait_or_abort(ops_full, 0, abort_flag);
      tot = ops_all;
    } else {
      __syncthreads();
    }
    if (threadIdx.x < RN) {
      float acc = 0.f;
      for (int q = 0; q < p.panels; ++q) acc = __fadd_rn(acc, tot[q * RN + threadIdx.x]);
      rowscale[threadIdx.x] = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.K)), p.eps));
    }
    __syncthreads();
    for (int it = threadIdx.x; it < items; it += kProjThreads) {  // h = bf16(x' * scale)
      const int r = it / (np * 8);
      const int pl = (it / 8) % np, c = it & 7;
      uint4* q = reinterpret_cast<uint4*>(xsm + pl * kXPanel + swz128(r, c));
      const uint4 v = *q;
      const float s = rowscale[r];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = pack_bf16x2(__fmul_rn(__uint_as_float(w[k] << 16), s),
                           __fmul_rn(__uint_as_float(w[k] & 0xffff0000u), s));
      *q = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  fence_proxy_async_shared();  // the operand's generic-proxy stores, visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---------------- MMA: one thread ----------------
  if (threadIdx.x == 32) {
    constexpr uint32_t idesc = umma_idesc_bf16(kProjFeat, RN, 0);
    if (mbar_wait_or_abort(w_full, 0, abort_flag)) {
      tc_fence_after();
      const uint32_t wb = smem_u32(wsm), xb = smem_u32(xsm);
      for (int i = 0; i < np; ++i)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ss(tmem, smem_desc_sw128(wb + i * 16384 + kk * 32, 16, 1024),
                  smem_desc_sw128(xb + i * kXPanel + kk * 32, 16, 1024), idesc,
                  (i > 0 || kk > 0) ? 1u : 0u);
    }
    umma_commit(mma_done);  // arrives when the MMAs above (if any) completed
  }

  // ---------------- epilogue ----------------
  // warp w reads TMEM lanes 32 (w % 4) .. (feature = lane), columns (rows) of half w / 4
  const bool have = mbar_wait_or_abort(mma_done, 0, abort_flag) && !*abort_flag;
  const int quarter = warp & 3, half = warp >> 2;
  const int feat = quarter * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  tc_fence_after();
  if (split > 1) {
    // partial tile [row][feature] fp32 into the (now free) operand bytes, then rank q's rows
    // [q * per, (q + 1) * per) to rank q's recv slot of this rank, by bulk copy
    if (have) {
#pragma unroll
      for (int c = 0; c < RN / 64; ++c) {
        uint32_t v[32];
        const int col = half * (RN / 2) + c * 32;
        tmem_ld32(tmem + lane_off + col, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) part[(col + i) * kProjFeat + feat] = __uint_as_float(v[i]);
      }
    }
    fence_proxy_async_shared();
    __syncthreads();
    if (!kNorm) cluster_wait();  // phase 1 (the norm waited for it before its own exchange)
    if (threadIdx.x < split) {
      const int q = threadIdx.x;
      const int q0 = q * per < RN ? q * per : RN;
      const int q1 = q0 + per < RN ? q0 + per : RN;
      if (q1 > q0)
        bulk_copy_to_peer(map_to_rank(recv + rank * per * kProjFeat, q), part + q0 * kProjFeat,
                          static_cast<uint32_t>((q1 - q0) * kProjFeat * 4), map_to_rank(recv_full, q));
    }
    mbar_wait_or_abort(recv_full, 0, abort_flag);
    cluster_arrive_relaxed();  // phase 2: everything sent to this CTA has landed
    // sum the ranks' partials in rank order, round once
    const int nrow = r1 - r0;
    for (int idx = threadIdx.x; idx < nrow * kProjFeat; idx += kProjThreads) {
      float acc = recv[idx];
      for (int q = 1; q < split; ++q) acc = __fadd_rn(acc, recv[q * per * kProjFeat + idx]);
      staged[idx] = float_to_bf16_bits(acc);
    }
  } else if (have) {
#pragma unroll
    for (int c = 0; c < RN / 64; ++c) {
      uint32_t v[32];
      const int col = half * (RN / 2) + c * 32;
      tmem_ld32(tmem + lane_off + col, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) staged[(col + i) * kProjFeat + feat] = float_to_bf16_bits(__uint_as_float(v[i]));
    }
  }
  __syncthreads();  // the staged rows are complete
  const int rows = (r1 < p.R ? r1 : p.R) - r0;
  if (have && rows > 0) {
    if (p.vec_out) {  // 16 bytes = 8 features a thread; a row of 128 features is 16 chunks
      for (int idx = threadIdx.x; idx < rows * 16; idx += kProjThreads) {
        const int r = idx >> 4, ch = idx & 15;
        const int n = n0 + ch * 8;
        if (n < p.N)
          *reinterpret_cast<uint4*>(p.y + static_cast<long long>(r0 + r) * p.ys + n) =
              *reinterpret_cast<const uint4*>(staged + r * kProjFeat + ch * 8);
      }
    } else {
      for (int idx = threadIdx.x; idx < rows * kProjFeat; idx += kProjThreads) {
        const int r = idx >> 7, f = idx & 127;
        if (n0 + f < p.N) p.y[static_cast<long long>(r0 + r) * p.ys + n0 + f] = staged[r * kProjFeat + f];
      }
    }
  }
  // phase 2: every rank has received all its rows, so the bulk copies out of this CTA's shared
  // memory are complete before it exits
  if (split > 1) cluster_wait();
  if (*abort_flag && threadIdx.x == 0) mbar_wait(w_full, 0);  // copies in flight land first
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, RN);
  }
}

}  // namespace mcb
