// The decode step's projections on the tensor cores: Y = X W^T for a handful of rows.
//
// At decode a projection multiplies R rows (one token per sequence: 64 in config 2) by a weight
// of N x K: the work is streaming W from HBM once, and a library GEMM launched per projection
// spends most of its few microseconds on launch and pipeline ramp.  This kernel is built for that
// shape and for programmatic dependent launch (PDL):
//
//   * swap-AB: the MMA's M = 128 output features (rows of W, K-major as nn.Linear stores them),
//     its N = R (rows of X, padded to the instantiated RN), K in 64-column panels; one
//     tcgen05.mma.cta_group::1.kind::f16 per 16 columns, fp32 accumulator in TMEM (RN columns);
//   * the W tiles do not depend on the previous kernel, so the producer issues the first ring's
//     worth of W loads, then griddepcontrol.wait, then the X tiles: under PDL the weight stream
//     overlaps the tail of the kernel before; every CTA calls griddepcontrol.launch_dependents at
//     once so the kernel after can do the same;
//   * split-K across a thread-block cluster of `split` CTAs (N = 768 projections have only six
//     128-feature tiles): each CTA reduces its K range into TMEM and parks the partial tile in its
//     shared memory; rank q then sums its share of the tile's columns over every rank through
//     distributed shared memory (fixed order rank 0, 1, ..) and writes those rows of Y -- no
//     workspace, no atomics;
//   * epilogue: 4 warps, thread = output feature (TMEM lane), bf16 rounding once.
//
// Every mbarrier wait is bounded; a timeout raises the CTA's abort flag, the MMA issuer waits
// (bounded) for its committed MMAs, TMEM is freed, and the cluster barriers are still reached so
// no CTA of a cluster waits for one that gave up.
#pragma once

#include "common.cuh"
#include "prefill_attn.cuh"  // tcgen05 helpers

namespace mcb {

constexpr int kLinTile = 128;    // output features per CTA (MMA M)
constexpr int kLinThreads = 192;

struct LinearParams {
  uint16_t* y;         // (R, N) bf16, row stride ys
  long long ys;
  int R, N, K;
  int steps_per_cta;   // 64-column K panels per CTA (K / 64 / split)
  int split;           // CTAs of a cluster sharing one output tile
  int vec_out;         // y 16-byte aligned, ys and N multiples of 8: 16-byte stores
};

template <int RN, int STAGES>
struct LinearConfig {
  static constexpr int kWBytes = kLinTile * 128;            // 128 rows x 64 bf16
  static constexpr int kXBytes = RN * 128;                  // RN rows x 64 bf16
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kBarOff = STAGES * kStageBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr uint32_t kTmemCols = RN <= 32 ? 32 : (RN <= 64 ? 64 : (RN <= 128 ? 128 : 256));
  // split-K partials (padded rows) plus the staged bf16 rows of one rank (at most RN / 2 rows)
  static_assert(kLinTile * (RN + 4) * 4 + (RN / 2) * kLinTile * 2 <= kBarOff, "epilogue must fit in the ring");
};

template <int RN, int STAGES>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                  const LinearParams p) {
  using Cfg = LinearConfig<RN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;                  // [STAGES]
  uint64_t* empty = bars + STAGES;        // [STAGES]
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* drained = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drained + 2);

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = p.split;
  const int tile = static_cast<int>(blockIdx.x) / split;
  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  const int n0 = tile * kLinTile;
  const int step0 = static_cast<int>(rank) * p.steps_per_cta;
  const int nsteps = p.steps_per_cta;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * STAGES + 2; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t base = smem_u32(smem);

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    const uint64_t pol_w = l2_policy_evict_first();
    const int pre = nsteps < STAGES ? nsteps : STAGES;
    // weights first: they do not depend on the kernel before this one
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], Cfg::kStageBytes);
      tma_load_4d(smem + i * Cfg::kStageBytes, &wmap, &full[i], (step0 + i) * 64, n0, 0, 0, pol_w);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_4d(smem + i * Cfg::kStageBytes + Cfg::kWBytes, &xmap, &full[i], (step0 + i) * 64, 0, 0,
                  0, 0ull);
    int issued = pre;
    for (int i = STAGES; i < nsteps; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait_or_abort(&empty[s], ((i / STAGES) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
      tma_load_4d(smem + s * Cfg::kStageBytes, &wmap, &full[s], (step0 + i) * 64, n0, 0, 0, pol_w);
      tma_load_4d(smem + s * Cfg::kStageBytes + Cfg::kWBytes, &xmap, &full[s], (step0 + i) * 64, 0, 0,
                  0, 0ull);
      issued = i + 1;
    }
    if (*abort_flag)  // copies still in flight land before the CTA can exit
      for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
        mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(kLinTile, RN, 0);
    bool ok = true;
    for (int i = 0; i < nsteps; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait_or_abort(&full[s], (i / STAGES) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t wb = base + s * Cfg::kStageBytes, xb = wb + Cfg::kWBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_ss(tmem, smem_desc_sw128(wb + kk * 32, 16, 1024), smem_desc_sw128(xb + kk * 32, 16, 1024),
                idesc, (i > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    if (ok) umma_commit(acc_full);
    umma_commit(drained);
    mbar_wait(drained, 0);
  }

  // ---------------- epilogue: warps 2-5, thread = output feature ----------------
  const bool epi = warp >= 2;
  const int quarter = warp & 3;
  const int feat = quarter * 32 + lane;  // TMEM lane
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  bool have = false;
  if (epi) have = __all_sync(0xffffffffu, mbar_wait_or_abort(acc_full, 0, abort_flag));
  // The ring is free once the accumulator is complete.  Split-K partial tiles go there as
  // [feature][row] fp32 with a padded row (RN + 4 floats: conflict-free float4 access by
  // consecutive features); the bf16 output rows a CTA writes are staged as [row][128 features]
  // and copied out 16 bytes a thread.
  constexpr int PSTR = RN + 4;
  float* part = reinterpret_cast<float*>(smem);
  uint16_t* staged;
  int r0 = 0, r1 = RN;
  if (split > 1) {
    if (epi && have) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < RN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(part + feat * PSTR + c * 32 + i) =
              make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                          __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
      }
    }
    cluster_sync();  // every partial tile written and visible to the cluster
    // rank q sums rows [q * per, (q + 1) * per) of the tile over all ranks, in rank order, 8 rows
    // at a time with every rank's loads in flight together
    const int per = ((RN + split - 1) / split + 7) & ~7;
    r0 = static_cast<int>(rank) * per;
    r1 = r0 + per < RN ? r0 + per : RN;
    staged = reinterpret_cast<uint16_t*>(smem + kLinTile * PSTR * 4);
    if (epi) {
      for (int c = r0; c < r1; c += 8) {
        float4 v[8][2];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q < split) {
            const uint32_t a = map_to_rank(part + feat * PSTR + c, static_cast<uint32_t>(q));
            v[q][0] = ld_dsmem_f4(a);
            v[q][1] = ld_dsmem_f4(a + 16);
          }
        }
        float acc[8] = {v[0][0].x, v[0][0].y, v[0][0].z, v[0][0].w,
                        v[0][1].x, v[0][1].y, v[0][1].z, v[0][1].w};
#pragma unroll
        for (int q = 1; q < 8; ++q) {
          if (q < split) {
            acc[0] += v[q][0].x; acc[1] += v[q][0].y; acc[2] += v[q][0].z; acc[3] += v[q][0].w;
            acc[4] += v[q][1].x; acc[5] += v[q][1].y; acc[6] += v[q][1].z; acc[7] += v[q][1].w;
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (c + i < r1) staged[(c + i - r0) * kLinTile + feat] = float_to_bf16_bits(acc[i]);
      }
    }
    cluster_sync();  // every rank has read the partials it needs before any CTA exits
  } else {
    staged = reinterpret_cast<uint16_t*>(smem);
    if (epi && have) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < RN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) staged[(c * 32 + i) * kLinTile + feat] = float_to_bf16_bits(__uint_as_float(v[i]));
      }
    }
  }
  if (epi) {
    named_barrier(1, 128);  // the staged rows are complete
    const int rows = (r1 < p.R ? r1 : p.R) - r0;
    if (have && rows > 0) {
      const int t = threadIdx.x - 64;
      if (p.vec_out) {  // 16 bytes = 8 features a thread, a row of 128 features is 16 chunks
        for (int idx = t; idx < rows * 16; idx += 128) {
          const int r = idx >> 4, ch = idx & 15;
          const int n = n0 + ch * 8;
          if (n < p.N)
            *reinterpret_cast<uint4*>(p.y + static_cast<long long>(r0 + r) * p.ys + n) =
                *reinterpret_cast<const uint4*>(staged + r * kLinTile + ch * 8);
        }
      } else {
        for (int idx = t; idx < rows * kLinTile; idx += 128) {
          const int r = idx >> 7, f = idx & 127;
          if (n0 + f < p.N) p.y[static_cast<long long>(r0 + r) * p.ys + n0 + f] = staged[r * kLinTile + f];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace mcb
