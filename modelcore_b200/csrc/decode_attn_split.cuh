// Piece 3, short-row variant: decode attention with one CTA per (row, kv head, query block, key
// split) -- no persistent loop, no tile-space scan, no cross-CTA publishing.  The host picks it
// when a row can hold at most a few thousand keys (min(Tmax, window + T) <= 32 tiles of 64): there
// the persistent kernel's fixed costs (the start-up scan over every row's length and the merges
// of rows cut between CTAs) are not amortised, and short independent CTAs in waves stream better.
//
// Semantics are those of decode_attn.cuh.  Per CTA: a producer warp streams its K/V tiles by TMA
// into a STAGES-deep ring; four consumer warps each take 16 keys of every 64-key tile; the same
// tensor-core contraction with keys on the M side (S^T = K Q^T, O^T += V^T P^T via
// ldmatrix.trans / movmatrix.trans); the warps merge through shared memory.  With one split per
// row the CTA writes the bf16 output; the splits of a row group merge inside a thread-block
// cluster through distributed shared memory, or -- too many splits for a cluster -- write
// (O/l, log2-sum-exp) partials that the split that finishes last merges (split_publish; small
// grids) or decode_attn_split_combine_kernel merges after the launch (large grids).
#pragma once

#include <math_constants.h>

#include "common.cuh"
#include "decode_attn.cuh"
#include "kv_append.cuh"

namespace mcb {

struct SplitAttnParams {
  const uint16_t* q;
  long long qs[3];
  const int32_t* cache_seqlens;
  uint16_t* out;
  float* part_o;    // [((b*T + t)*Hq + h)*nsplit + s][D]
  float* part_lse;  // [((b*T + t)*Hq + h)*nsplit + s]
  int B, T, Hq, Hkv, G, Tmax, window;
  float scale_log2;  // softmax_scale * log2(e)
  int nsplit, tiles_per_split, nqb;
  int row_cuts;      // cut each row by its own length (small grids) instead of tiles_per_split
  int cluster;       // the nsplit (<= 16) CTAs of a row group form a cluster and merge in DSMEM
  int* counters;     // otherwise, on small grids: [row group] arrivals, zero on entry and on exit
                     // (null: decode_attn_split_combine_kernel merges the partials afterwards)
  int ring;          // the slot is a ring of Tmax positions (key c at index c % Tmax)
  // fp8 cache (decode_attn_split_kernel<.., true>): e4m3 K/V with per-vector fp32 scales at
  // [(b * Hkv + h) * scale_tmax + index]
  const float* k_scale;
  const float* v_scale;
  int scale_tmax;
  // fused append (bf16 cache, one new token a row): q is the raw query projection; each CTA
  // ropes, norms and scales its query heads, and the CTA whose keys reach the row's position
  // also writes the new key (roped, normed, scaled unless raw) and value into the slot and into
  // its own copy of that tile -- kv_append_rope_vec_kernel's arithmetic, the same bits
  int fuse;
  // head pairs (D = 128 instance only, one split, bf16): the slot holds kv heads of 64 as pairs,
  // kv "head" j = real heads 2j, 2j + 1 side by side (the same bytes), and query row r of row
  // group j is real q head 2j + r (G = 2) -- its 64 dimensions in half r of a 128-dimension row,
  // zeros in the other, so the dot product with the pair's key reads only its own head; the
  // output keeps half r of row r and goes to the real (B, T, Hq, 64) layout.  q, k_new and v_new
  // are the real 64-dimension heads (their strides), and the fused rope and norm work on them.
  int pair;
  const uint16_t* k_new;       // (B, 1, Hkv, D) raw key / value projections; null: q only
  const uint16_t* v_new;
  long long kns[3], vns[3];
  uint16_t* kc_out;            // the slot (B, Tmax, Hkv, D) the new key and value go to
  uint16_t* vc_out;
  const uint16_t* rot_cos;     // rotary tables (rot_len, D/2) bf16
  const uint16_t* rot_sin;
  int rot_len, rotate_k;
  float norm_eps, qk_scale;
};


// The most key splits of a row group that merge inside one thread-block cluster (clusters above
// the portable 8 need the non-portable size, which the host checks the device schedules).
constexpr int kMaxClusterSplits = 16;

// The receive rows a cluster merge by push needs: split q's partial of the owner's j-th row goes to
// slot q * ceil(kRows / ns) + j, so up to max over ns of ns * ceil(kRows / ns) slots.
__host__ __device__ constexpr int split_recv_rows(int rows) {
  int best = 0;
  for (int ns = 2; ns <= kMaxClusterSplits; ++ns) {
    const int v = ns * ((rows + ns - 1) / ns);
    best = v > best ? v : best;
  }
  return best;
}

template <int D, int NQT, int KPW, int STAGES, bool FP8 = false>
struct SplitAttnConfig {
  static constexpr int kRows = 8 * NQT;                      // query rows per CTA
  static constexpr int TK = KPW * kAttnConsumerWarps;        // keys per stage
  static constexpr int PANEL = D < 64 ? D : 64;              // columns per swizzled panel
  static constexpr int NPANEL = D / PANEL;
  static constexpr int ROW_BYTES = PANEL * 2;                // 32, 64 or 128
  static constexpr int SWZ_MASK = ROW_BYTES == 128 ? 7 : (ROW_BYTES == 64 ? 3 : 1);
  static constexpr int PANEL_BYTES = TK * ROW_BYTES;
  static constexpr int TILE_BYTES = NPANEL * PANEL_BYTES;    // one K (or V) tile
  // fp8: a stage holds the e4m3 K and V tiles (TK rows of D bytes, one swizzled panel) and the
  // tile's K and V scales; each consumer warp converts its KPW value rows to f16 in its own
  // scratch, laid out as a bf16 tile of KPW rows (same panels, same swizzle); its keys go from
  // the stage to registers
  static constexpr int F8_ROW = D;
  static constexpr int F8_MASK = D == 128 ? 7 : 3;
  static constexpr int F8_TILE = TK * D;
  static constexpr int F8_SCALES = 2 * TK * 4;
  static constexpr int STAGE_BYTES = FP8 ? ((2 * F8_TILE + F8_SCALES + 1023) & ~1023) : 2 * TILE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int SCR_PANEL = KPW * ROW_BYTES;          // one warp's scratch panel
  static constexpr int SCR_WARP = FP8 ? NPANEL * SCR_PANEL : 0;  // the warp's values in f16
  static constexpr int OPITCH = D + 4;                       // merge buffer row pitch (floats)
  static constexpr int MERGE_BYTES = kAttnConsumerWarps * kRows * OPITCH * 4;
  // cluster merge: this CTA's merged partial [kRows][D], its per-row log2-sum-exp and the
  // per-row weights of up to kMaxClusterSplits ranks, after the per-warp merge buffer
  static constexpr int CL_OFFSET = (MERGE_BYTES + 15) & ~15;
  static constexpr int CL_BYTES = kRows * D * 4 + kRows * 4 + kRows * kMaxClusterSplits * 4;
  static constexpr int BODY_BYTES =
      RING_BYTES > CL_OFFSET + CL_BYTES ? RING_BYTES : CL_OFFSET + CL_BYTES;
  static constexpr int SCR_OFFSET = BODY_BYTES;
  // barriers (full + empty per stage) then per-warp row statistics
  static constexpr int BAR_OFFSET = SCR_OFFSET + kAttnConsumerWarps * SCR_WARP;
  static constexpr int STAT_OFFSET = BAR_OFFSET + 2 * STAGES * 8;
  static constexpr int STAT_BYTES = 2 * kAttnConsumerWarps * kRows * 4;  // per-warp row max, sum
  static constexpr int CTL_OFFSET = STAT_OFFSET + STAT_BYTES;  // the "last arrival" flag
  // fused append: the CTA's query rows [kRows][D] and the new key and value [2][D], bf16
  static constexpr int FUSE_OFFSET = CTL_OFFSET + 16;
  static constexpr int FUSE_BYTES = FP8 ? 0 : (kRows + 2) * D * 2;
  // cluster merge by push (bf16 copies of 3-4 stages with 8-row groups, D <= 128, where the extra
  // shared memory keeps the CTAs per SM): every split stores its partial rows and log-sum-exps
  // straight into the owning rank's receive buffer -- its own region, never part of the ring,
  // because a split that finishes early writes while its owner may still be streaming -- and
  // one cluster barrier later the owner merges from its own shared memory.  The 2-stage copies
  // (sized for residency) and the fp8 ones pull the partials through DSMEM loads instead.
  static constexpr bool PUSH = !FP8 && STAGES >= 3 && NQT == 1 && D <= 128;
  static constexpr int RECV_ROWS = split_recv_rows(kRows);
  static constexpr int RECV_OFFSET = (FUSE_OFFSET + FUSE_BYTES + 15) & ~15;
  static constexpr int RECV_BYTES = PUSH ? RECV_ROWS * (D + 1) * 4 : 0;  // [RECV_ROWS][D], then lse
  static constexpr int SMEM_BYTES = RECV_OFFSET + RECV_BYTES + 1024;  // + alignment slack
  // 16-byte vector accesses: the query rows (FUSE) and the receive buffer; 8-byte mbarriers
  static_assert(FUSE_OFFSET % 16 == 0 && RECV_OFFSET % 16 == 0 && BAR_OFFSET % 8 == 0, "alignment");
  static_assert(D % 16 == 0 && D >= 16 && D <= 256, "head_dim");
  static_assert(KPW % 16 == 0, "keys per warp");
  static_assert(PANEL_BYTES % 1024 == 0 || ROW_BYTES < 128, "panel alignment");
  static_assert(!FP8 || D == 64 || D == 128, "fp8 cache: head_dim 64 or 128");
};

// 4 e4m3 bytes (memory order) -> two f16x2 words (exact)
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// c[0..3] += A(16x16, row) * B(16x8, col), f16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 1-D bulk copy global -> this CTA's shared memory (bytes a multiple of 16, both 16-byte
// aligned), counted on the mbarrier as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Merges the nsplit partials of output row `row` (one warp): weights from the partials'
// log2-sum-exps, then the weighted sum of their O rows.  Reads through L2 (the partials were
// written by other CTAs of this launch).
template <int D>
__device__ __forceinline__ void merge_split_row(const SplitAttnParams& p, long long row, int lane) {
  const float* lse = p.part_lse + row * p.nsplit;
  float mmax = -CUDART_INF_F;
  for (int s = lane; s < p.nsplit; s += 32) mmax = fmaxf(mmax, __ldcg(lse + s));
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, m));
  float wsum = 0.f;
  for (int s = lane; s < p.nsplit; s += 32) {
    const float ls = __ldcg(lse + s);
    wsum += (ls == -CUDART_INF_F) ? 0.f : fast_exp2(ls - mmax);
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, m);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  constexpr int PER_LANE = (D + 31) / 32;
  float acc[PER_LANE];
#pragma unroll
  for (int u = 0; u < PER_LANE; ++u) acc[u] = 0.f;
  const float* po = p.part_o + row * p.nsplit * D;
  // 32 splits at a time: lane j holds split s0 + j's weight; the partial rows of four splits are
  // requested together (no branch between them), so their L2 round trips overlap
  for (int s0 = 0; s0 < p.nsplit; s0 += 32) {
    const int sl = s0 + lane;
    const float ls = sl < p.nsplit ? __ldcg(lse + sl) : -CUDART_INF_F;
    const float wk = (ls == -CUDART_INF_F) ? 0.f : fast_exp2(ls - mmax) * inv;
    const int cnt = min(32, p.nsplit - s0);
#pragma unroll 4
    for (int j = 0; j < cnt; ++j) {
      const float w = __shfl_sync(0xffffffffu, wk, j);
      const float* prow = po + static_cast<long long>(s0 + j) * D;
#pragma unroll
      for (int u = 0; u < PER_LANE; ++u) {
        const int d = lane + 32 * u;
        if (d < D) {
          // an empty split wrote only its log-sum-exp: its O row is unset memory, never used
          const float x = __ldcg(prow + d);
          acc[u] = w != 0.f ? fmaf(w, x, acc[u]) : acc[u];
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < PER_LANE; ++u) {
    const int d = lane + 32 * u;
    if (d < D) p.out[row * D + d] = float_to_bf16_bits(acc[u]);
  }
}

// A split CTA of the partials plan has written its partial rows r0 .. r1-1: it bumps the row
// group's arrival counter (the barrier orders every thread's stores before thread 0's release),
// and the CTA that arrives last merges all the group's partials into the output and resets the
// counter.  No CTA waits for another and no second kernel runs.
template <int D>
__device__ __forceinline__ void split_publish(const SplitAttnParams& p, int group, int b, int kvh,
                                              int r0, int r1, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int* counter = p.counters + group;
    const int prev = atom_add_acq_rel_gpu(counter, 1);
    const int last = prev == p.nsplit - 1;
    if (last) *counter = 0;  // every split has arrived: ready for the next call
    *flag = last;
  }
  __syncthreads();
  if (!*flag) return;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int r = r0 + warp; r < r1; r += kAttnThreads / 32) {
    const int t = r / p.G, h = kvh * p.G + r % p.G;
    merge_split_row<D>(p, (static_cast<long long>(b) * p.T + t) * p.Hq + h, lane);
  }
}

// The 2-stage copy for head size <= 64 and 8-row groups exists to fit 6 CTAs per SM (config 2's
// 768 CTAs in one wave): 160 threads x 64 registers each.
template <int D, int NQT, int KPW, int STAGES, bool FP8 = false>
__global__ void __launch_bounds__(kAttnThreads, (STAGES == 2 && D <= 64 && NQT == 1 && !FP8) ? 6 : 1)
    decode_attn_split_kernel(const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const SplitAttnParams p) {
  using C = SplitAttnConfig<D, NQT, KPW, STAGES, FP8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFFSET);
  uint64_t* empty_bar = full_bar + STAGES;
  float* stat_m = reinterpret_cast<float*>(smem + C::STAT_OFFSET);
  float* stat_l = stat_m + kAttnConsumerWarps * C::kRows;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- which (b, kv head, query block, split) ----
  int x = blockIdx.x;
  const int split = x % p.nsplit;
  x /= p.nsplit;
  const int qb = x % p.nqb;
  x /= p.nqb;
  const int kvh = x % p.Hkv;
  const int b = x / p.Hkv;

  const int rows_total = p.T * p.G;
  const int r0 = qb * C::kRows;
  const int r1 = min(r0 + C::kRows, rows_total);
  const int t_first = r0 / p.G;
  const int t_last = (r1 - 1) / p.G;
  const int L = p.cache_seqlens[b];
  int hi = L + t_last;
  if ((!p.ring && hi >= p.Tmax) || L < 0) {
    if (threadIdx.x == 0) record_error(kErrPositionBeyondCache);
    hi = min(max(hi, 0), p.Tmax - 1);
  }
  const int lo = p.window >= 0 ? max(0, L + t_first - p.window) : 0;
  const int kb = (min(lo, hi) / C::TK) * C::TK;
  const int ntiles = (hi - kb) / C::TK + 1;
  // The host sizes the splits for the longest possible row (tiles_per_split).  On small grids
  // (row_cuts) a row is cut by its own length into nsplit parts of at least
  // min(8, tiles_per_split) tiles, so that the splits of a long row all share its keys while a
  // short row's keys stay in a few CTAs; on large grids the fixed size keeps the CTAs few and
  // the waves balanced.
  const int tps = p.row_cuts ? max((ntiles + p.nsplit - 1) / p.nsplit, min(8, p.tiles_per_split))
                             : p.tiles_per_split;
  const int tile0 = split * tps;
  const int my_tiles = max(0, min(ntiles - tile0, tps));
  // fused append: this CTA's tiles hold the row's new position (the single-token case)
  const int tile_new = (L - kb) / C::TK;
  const bool own_new = !FP8 && p.fuse && p.k_new != nullptr && L >= 0 && tile_new >= tile0 &&
                       tile_new < tile0 + my_tiles;

  if (my_tiles == 0 && !p.cluster) {  // an empty split: its partial carries no weight
    // the workspace and the counters may still be in use by the launch ahead (its last-arrival
    // merges): wait for it before writing either
    pdl_wait();
    if (threadIdx.x < C::kRows) {
      const int r = r0 + threadIdx.x;
      if (r < r1) {
        const int t = r / p.G, h = kvh * p.G + r % p.G;
        p.part_lse[((static_cast<long long>(b) * p.T + t) * p.Hq + h) * p.nsplit + split] =
            -CUDART_INF_F;
      }
    }
    if (p.counters != nullptr)
      split_publish<D>(p, static_cast<int>(blockIdx.x) / p.nsplit, b, kvh, r0, r1,
                       reinterpret_cast<int*>(smem + C::CTL_OFFSET));
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kAttnConsumerWarps);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  // push merge, phase 1 of the cluster barrier: this CTA runs (its receive buffer exists); the
  // matching wait comes before the first remote store, long after every CTA has arrived
  if (C::PUSH && p.cluster) cluster_arrive_relaxed();

  if (warp == kAttnConsumerWarps) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const uint64_t policy = l2_policy_evict_first();
      bool waited = false;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty_bar[s], ((i / STAGES) - 1) & 1)) break;
        const int key0 = kb + (tile0 + i) * C::TK;
        // keys below L are from earlier steps, written at least two launches back (complete: see
        // pdl_launch_dependents in common.cuh); a tile reaching L holds this step's new key,
        // written by the append kernel this launch may have overlapped (PDL) -- or, fused, by
        // this launch itself, whose owner warp overwrites the stale bytes in shared memory
        if (!waited && key0 + C::TK > L) {
          pdl_wait();
          waited = true;
        }
        const int slot0 = p.ring ? key0 % p.Tmax : key0;  // a ring slot: Tmax % TK == 0
        uint8_t* kdst = smem + s * C::STAGE_BYTES;
        if constexpr (FP8) {
          mbar_arrive_expect_tx(&full_bar[s], 2 * C::F8_TILE + C::F8_SCALES);
          tma_load_4d(kdst, &kmap, &full_bar[s], 0, kvh, slot0, b, policy);
          tma_load_4d(kdst + C::F8_TILE, &vmap, &full_bar[s], 0, kvh, slot0, b, policy);
          // the tile's scales; scale_tmax >= Tmax rounded up to TK keeps them in bounds
          const long long so = (static_cast<long long>(b) * p.Hkv + kvh) * p.scale_tmax + slot0;
          bulk_load(kdst + 2 * C::F8_TILE, p.k_scale + so, C::TK * 4, &full_bar[s]);
          bulk_load(kdst + 2 * C::F8_TILE + C::TK * 4, p.v_scale + so, C::TK * 4, &full_bar[s]);
        } else {
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          uint8_t* vdst = kdst + C::TILE_BYTES;
#pragma unroll
          for (int pn = 0; pn < C::NPANEL; ++pn) {
            tma_load_4d(kdst + pn * C::PANEL_BYTES, &kmap, &full_bar[s], pn * C::PANEL, kvh, slot0, b,
                        policy);
            tma_load_4d(vdst + pn * C::PANEL_BYTES, &vmap, &full_bar[s], pn * C::PANEL, kvh, slot0, b,
                        policy);
          }
        }
      }
    }
  }

  // Per-thread softmax state for rows n = j*8 + 2*(lane%4) + e.
  float m_run[NQT][2], l_run[NQT][2];
  float o_acc[NQT][D / 16][4];
  int row_hi[NQT][2], row_lo[NQT][2];

  if (warp < kAttnConsumerWarps) {
    // ---------------- consumer warps ----------------
    pdl_wait();  // q comes from the append kernel ahead of this one (fused: the projection)
    // the kernel after this one may start its prologue and its loads of earlier steps' keys
    pdl_launch_dependents();
    uint16_t* qbuf = reinterpret_cast<uint16_t*>(smem + C::FUSE_OFFSET);  // [kRows][D]
    uint16_t* kvbuf = qbuf + C::kRows * D;                                 // [2][D]
    if (!FP8 && (p.fuse || (D == 128 && p.pair))) {
      if (D == 128 && p.pair && warp == 0) {
        // head pairs: groups of four lanes, one 64-dimension vector each -- the query heads (roped,
        // normed and scaled when fused, else copied) into their half of the row, zeros in the
        // other; then (the CTA with the new position) the pair's two keys and two values
        constexpr int DH = 64, LG = DH / 16, VPW = 32 / LG, HALF = DH / 2;  // (D = 128 only)
        const int nq = r1 - r0;
        const int nvec = nq + (own_new ? 4 : 0);
        const int sub = lane % LG;
        const bool rot_ok = L >= 0 && L < p.rot_len;
        for (int v0 = 0; v0 < nvec; v0 += VPW) {
          const int vi = v0 + lane / LG;
          const bool valid = vi < nvec;
          const bool is_q = vi < nq;
          const int kv = vi - nq;              // 0, 1: the keys of heads 2 kvh, 2 kvh + 1; 2, 3: values
          const bool is_k = !is_q && kv < 2;
          const int half = is_q ? (r0 + vi) & 1 : (kv & 1);
          const uint16_t* src = nullptr;
          if (valid)
            src = is_q ? p.q + b * p.qs[0] + (kvh * p.G + r0 + vi) * p.qs[2]
                       : (is_k ? p.k_new + b * p.kns[0] + (2 * kvh + half) * p.kns[2]
                               : p.v_new + b * p.vns[0] + (2 * kvh + half) * p.vns[2]);
          const bool rotate = valid && p.fuse && (is_q || (is_k && p.rotate_k));
          if (rotate && !rot_ok && sub == 0) record_error(kErrPositionBeyondRotary);
          const uint4 x1v = valid ? *reinterpret_cast<const uint4*>(src + 8 * sub) : make_uint4(0, 0, 0, 0);
          const uint4 x2v = valid ? *reinterpret_cast<const uint4*>(src + HALF + 8 * sub) : make_uint4(0, 0, 0, 0);
          uint4 w1, w2;
          rope_norm_vec<DH>(x1v, x2v, p.rot_cos, p.rot_sin, L, sub, rotate && rot_ok, p.norm_eps, p.qk_scale, w1,
                            w2);
          if (valid) {
            uint16_t* dst = (is_q ? qbuf + vi * D : kvbuf + (is_k ? 0 : D)) + half * DH;
            *reinterpret_cast<uint4*>(dst + 8 * sub) = w1;
            *reinterpret_cast<uint4*>(dst + HALF + 8 * sub) = w2;
            if (is_q) {  // the other head's half of the row
              uint16_t* other = qbuf + vi * D + (1 - half) * DH;
              *reinterpret_cast<uint4*>(other + 8 * sub) = make_uint4(0, 0, 0, 0);
              *reinterpret_cast<uint4*>(other + HALF + 8 * sub) = make_uint4(0, 0, 0, 0);
            } else if (p.ring || L < p.Tmax) {
              const int idx = p.ring ? L % p.Tmax : L;
              uint16_t* cdst = (is_k ? p.kc_out : p.vc_out) +
                               ((static_cast<long long>(b) * p.Tmax + idx) * p.Hkv + kvh) * D + half * DH;
              *reinterpret_cast<uint4*>(cdst + 8 * sub) = w1;
              *reinterpret_cast<uint4*>(cdst + HALF + 8 * sub) = w2;
            }
          }
        }
      } else if (warp == 0) {
        // groups of D/16 lanes, one vector each: the query heads r0 .. r1-1, then (the CTA with
        // the new position) the key and the value
        constexpr int LG = D / 16, VPW = 32 / LG, HALF = D / 2;
        const int nq = r1 - r0;
        const int nvec = nq + (own_new ? 2 : 0);
        const int sub = lane % LG;
        const bool rot_ok = L >= 0 && L < p.rot_len;
        for (int v0 = 0; v0 < nvec; v0 += VPW) {
          const int vi = v0 + lane / LG;
          const bool valid = vi < nvec;
          const bool is_q = vi < nq, is_k = vi == nq;
          const uint16_t* src = nullptr;
          if (valid)
            src = is_q ? p.q + b * p.qs[0] + (kvh * p.G + r0 + vi) * p.qs[2]
                       : (is_k ? p.k_new + b * p.kns[0] + kvh * p.kns[2] : p.v_new + b * p.vns[0] + kvh * p.vns[2]);
          const bool rotate = valid && (is_q || (is_k && p.rotate_k));
          if (rotate && !rot_ok && sub == 0) record_error(kErrPositionBeyondRotary);
          const uint4 x1v = valid ? *reinterpret_cast<const uint4*>(src + 8 * sub) : make_uint4(0, 0, 0, 0);
          const uint4 x2v = valid ? *reinterpret_cast<const uint4*>(src + HALF + 8 * sub) : make_uint4(0, 0, 0, 0);
          uint4 w1, w2;
          rope_norm_vec<D>(x1v, x2v, p.rot_cos, p.rot_sin, L, sub, rotate && rot_ok, p.norm_eps, p.qk_scale, w1,
                           w2);
          if (valid) {
            uint16_t* dst = is_q ? qbuf + vi * D : kvbuf + (is_k ? 0 : D);
            *reinterpret_cast<uint4*>(dst + 8 * sub) = w1;
            *reinterpret_cast<uint4*>(dst + HALF + 8 * sub) = w2;
            if (!is_q && (p.ring || L < p.Tmax)) {
              const int idx = p.ring ? L % p.Tmax : L;
              uint16_t* cdst = (is_k ? p.kc_out : p.vc_out) +
                               ((static_cast<long long>(b) * p.Tmax + idx) * p.Hkv + kvh) * D;
              *reinterpret_cast<uint4*>(cdst + 8 * sub) = w1;
              *reinterpret_cast<uint4*>(cdst + HALF + 8 * sub) = w2;
            }
          }
        }
      }
      named_barrier(2, kAttnConsumerWarps * 32);  // the query rows and the new key are in place
    }
    // Q^T fragments (B operand): row n = j*8 + lane/4, columns d = kk*16 + 2*(lane%4) + {0,1}, +8.
    uint32_t qf[NQT][D / 16][2];
#pragma unroll
    for (int j = 0; j < NQT; ++j) {
      const int r = r0 + j * 8 + (lane >> 2);
      const uint16_t* qrow = nullptr;
      if (r < r1) {
        if (!FP8 && (p.fuse || (D == 128 && p.pair))) {
          qrow = qbuf + (r - r0) * D;
        } else {
          const int t = r / p.G, h = kvh * p.G + r % p.G;
          qrow = p.q + b * p.qs[0] + t * p.qs[1] + h * p.qs[2];
        }
      }
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        // fp8: the key fragments come straight from the e4m3 rows, lane quad t holding head
        // dimensions [t D/4, (t+1) D/4) (four per k-step); the query fragments follow the same
        // order (a permutation of the summed dimension: the same dot product)
        const int d0 = FP8 ? (lane & 3) * (D / 4) + 4 * kk : kk * 16 + 2 * (lane & 3);
        const int d1 = FP8 ? d0 + 2 : d0 + 8;
        qf[j][kk][0] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
        qf[j][kk][1] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d1) : 0u;
        if (FP8) {  // the products run in f16 against the exactly converted e4m3 keys
#pragma unroll
          for (int u = 0; u < 2; ++u)
            qf[j][kk][u] = pack_f16x2(__uint_as_float(qf[j][kk][u] << 16),
                                      __uint_as_float(qf[j][kk][u] & 0xffff0000u));
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int rr = r0 + j * 8 + 2 * (lane & 3) + e;
        m_run[j][e] = -CUDART_INF_F;
        l_run[j][e] = 0.f;
        if (rr < r1) {
          const int qpos = L + rr / p.G;
          row_hi[j][e] = qpos;
          row_lo[j][e] = p.window >= 0 ? qpos - p.window : 0;
        } else {
          row_hi[j][e] = -1;  // padding row: every key masked
          row_lo[j][e] = 0;
        }
      }
#pragma unroll
      for (int db = 0; db < D / 16; ++db)
#pragma unroll
        for (int c = 0; c < 4; ++c) o_acc[j][db][c] = 0.f;
    }

    constexpr int NCH = KPW / 16;  // 16-key chunks per warp per stage
    // fp8: this warp's f16 scratch for its value rows, at rows 0 .. KPW-1
    const uint32_t scr_v = smem_u32(smem + C::SCR_OFFSET + warp * C::SCR_WARP);
    for (int i = 0; i < my_tiles; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(&full_bar[s], (i / STAGES) & 1)) break;
      uint32_t kbase = smem_u32(smem + s * C::STAGE_BYTES);
      uint32_t vbase = kbase + C::TILE_BYTES;
      int row0 = warp * KPW;                  // this warp's first key row in the tile buffers
      int panel_bytes = C::PANEL_BYTES;
      const int tile_key0 = kb + (tile0 + i) * C::TK;
      if constexpr (!FP8) {
        // fused append: the tile arrived with the slot's old bytes at the new position; the warp
        // that owns that row writes the new key and value over it before reading the tile
        const int rr = L - tile_key0;
        if (own_new && rr >= warp * KPW && rr < (warp + 1) * KPW) {
          constexpr int NCHK = D / 8;  // 16-byte chunks per row
          if (lane < 2 * NCHK) {
            const int isv = lane >= NCHK ? 1 : 0;
            const int col = (lane % NCHK) * 8;
            const uint32_t dst = (isv ? vbase : kbase) + (col / C::PANEL) * C::PANEL_BYTES +
                                 swz<C::ROW_BYTES, C::SWZ_MASK>(rr, (col % C::PANEL) / 8);
            sts128(dst, lds128(smem_u32(kvbuf + isv * D + col)));
          }
          fence_proxy_async_shared();  // TMA refills this stage later
          __syncwarp();
        }
      }
      float ks[NCH][2], vs[NCH][2];           // fp8: the scales of this lane's key rows
      uint32_t kw[NCH][2][FP8 ? D / 16 : 1];  // fp8: this lane's e4m3 key words (see below)
      if constexpr (FP8) {
        const uint32_t f8k = kbase, f8v = kbase + C::F8_TILE;
        const float* scl = reinterpret_cast<const float*>(smem + s * C::STAGE_BYTES + 2 * C::F8_TILE);
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int kr = warp * KPW + ch * 16 + (lane >> 2) + hh * 8;
            ks[ch][hh] = scl[kr];
            vs[ch][hh] = scl[C::TK + kr];
          }
        // this lane's e4m3 key bytes, rows g and g + 8 of each 16-key chunk, head dimensions
        // [t D/4, (t+1) D/4): read before the stage is released, converted at the products
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int kr = warp * KPW + ch * 16 + (lane >> 2) + hh * 8;
#pragma unroll
            for (int c = 0; c < D / 64; ++c) {
              const uint4 w = lds128(f8k + swz<C::F8_ROW, C::F8_MASK>(kr, (lane & 3) * (D / 64) + c));
              kw[ch][hh][4 * c + 0] = w.x;
              kw[ch][hh][4 * c + 1] = w.y;
              kw[ch][hh][4 * c + 2] = w.z;
              kw[ch][hh][4 * c + 3] = w.w;
            }
          }
        // e4m3 rows warp*KPW .. +KPW-1 of V -> f16 (exact), 16 bytes of e4m3 a step
        constexpr int CPR = D / 16;  // 16-byte e4m3 chunks per row
#pragma unroll
        for (int idx = lane; idx < KPW * CPR; idx += 32) {
          // D = 128: each quarter-warp takes half of two adjacent rows (chunks 0-3 of one and 4-7
          // of the other), so its eight 16-byte reads and, in each of the two stores, its eight
          // f16 chunks (two panels, swizzled by row) fall on distinct bank groups
          const int u = idx & 15;
          const int r = CPR == 8 ? (idx >> 4) * 2 + ((u >> 2) & 1) : idx / CPR;
          const int c16 = CPR == 8 ? (u & 3) + 4 * (((u >> 2) ^ (u >> 3)) & 1) : idx % CPR;
          const uint32_t soff = swz<C::F8_ROW, C::F8_MASK>(warp * KPW + r, c16);
          const int col = c16 * 16;  // two 8-column f16 chunks, swizzled independently
          const uint32_t pbase = (col / C::PANEL) * C::SCR_PANEL;
          const uint32_t doff0 = pbase + swz<C::ROW_BYTES, C::SWZ_MASK>(r, (col % C::PANEL) / 8);
          const uint32_t doff1 = pbase + swz<C::ROW_BYTES, C::SWZ_MASK>(r, (col % C::PANEL) / 8 + 1);
          const uint4 w = lds128(f8v + soff);
          uint32_t h[8];
          e4m3x4_to_f16x4(w.x, h[0], h[1]);
          e4m3x4_to_f16x4(w.y, h[2], h[3]);
          e4m3x4_to_f16x4(w.z, h[4], h[5]);
          e4m3x4_to_f16x4(w.w, h[6], h[7]);
          sts128(scr_v + doff0, make_uint4(h[0], h[1], h[2], h[3]));
          sts128(scr_v + doff1, make_uint4(h[4], h[5], h[6], h[7]));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);  // keys read, values converted: refill it
        vbase = scr_v;
        row0 = 0;
        panel_bytes = C::SCR_PANEL;
      }

      float sc[NCH][NQT][4];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
        for (int j = 0; j < NQT; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) sc[ch][j][c] = 0.f;
        const int krow = row0 + ch * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          uint32_t a0, a1, a2, a3;
          if constexpr (FP8) {  // bytes 4kk..4kk+3 of rows g and g + 8: (a0, a2) and (a1, a3)
            e4m3x4_to_f16x4(kw[ch][0][kk], a0, a2);
            e4m3x4_to_f16x4(kw[ch][1][kk], a1, a3);
          } else {
            const int col = kk * 16 + (lane >> 4) * 8;  // first column of this lane's 8-wide chunk
            const uint32_t addr = kbase + (col / C::PANEL) * panel_bytes +
                                  swz<C::ROW_BYTES, C::SWZ_MASK>(krow, (col % C::PANEL) / 8);
            ldsm_x4(addr, a0, a1, a2, a3);
          }
#pragma unroll
          for (int j = 0; j < NQT; ++j) {
            if (FP8)
              mma_16816_f16(sc[ch][j], a0, a1, a2, a3, qf[j][kk][0], qf[j][kk][1]);
            else
              mma_16816(sc[ch][j], a0, a1, a2, a3, qf[j][kk][0], qf[j][kk][1]);
          }
        }
        if (FP8) {  // logits of the stored keys times their scales
#pragma unroll
          for (int j = 0; j < NQT; ++j) {
            sc[ch][j][0] *= ks[ch][0];
            sc[ch][j][1] *= ks[ch][0];
            sc[ch][j][2] *= ks[ch][1];
            sc[ch][j][3] *= ks[ch][1];
          }
        }
      }

      // Mask, then the online-softmax update over this warp's NCH*16 keys.
#pragma unroll
      for (int j = 0; j < NQT; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float mx = -CUDART_INF_F;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int key = tile_key0 + warp * KPW + ch * 16 + (lane >> 2) + hh * 8;
              float& v = sc[ch][j][e + 2 * hh];
              if (key > row_hi[j][e] || key < row_lo[j][e]) v = -CUDART_INF_F;
              mx = fmaxf(mx, v);
            }
          }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m_run[j][e], mx);
          float alpha = 1.f;
          float msub = 0.f;
          if (m_new != -CUDART_INF_F) {
            alpha = fast_exp2((m_run[j][e] - m_new) * p.scale_log2);
            msub = m_new * p.scale_log2;
          }
          m_run[j][e] = m_new;
          float lsum = 0.f;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              float& v = sc[ch][j][e + 2 * hh];
              v = fast_exp2(fmaf(v, p.scale_log2, -msub));  // exp2(-inf) = 0 for masked keys
              lsum += v;
            }
          }
          l_run[j][e] = fmaf(l_run[j][e], alpha, lsum);
#pragma unroll
          for (int db = 0; db < D / 16; ++db) {
            o_acc[j][db][e] *= alpha;
            o_acc[j][db][e + 2] *= alpha;
          }
        }
      }

      // O^T += V^T . P^T
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        uint32_t pb[NQT][2];
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          if (FP8) {  // the value scales ride on the probabilities (l sums them unscaled)
            pb[j][0] = movmatrix_trans(pack_f16x2(sc[ch][j][0] * vs[ch][0], sc[ch][j][1] * vs[ch][0]));
            pb[j][1] = movmatrix_trans(pack_f16x2(sc[ch][j][2] * vs[ch][1], sc[ch][j][3] * vs[ch][1]));
          } else {
            pb[j][0] = movmatrix_trans(pack_bf16x2(sc[ch][j][0], sc[ch][j][1]));
            pb[j][1] = movmatrix_trans(pack_bf16x2(sc[ch][j][2], sc[ch][j][3]));
          }
        }
        const int m = lane >> 3;
        const int vrow = row0 + ch * 16 + (lane & 7) + (m >> 1) * 8;
#pragma unroll
        for (int db = 0; db < D / 16; ++db) {
          const int col = db * 16 + (m & 1) * 8;
          const uint32_t addr = vbase + (col / C::PANEL) * panel_bytes +
                                swz<C::ROW_BYTES, C::SWZ_MASK>(vrow, (col % C::PANEL) / 8);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(addr, a0, a1, a2, a3);
#pragma unroll
          for (int j = 0; j < NQT; ++j) {
            if (FP8)
              mma_16816_f16(o_acc[j][db], a0, a1, a2, a3, pb[j][0], pb[j][1]);
            else
              mma_16816(o_acc[j][db], a0, a1, a2, a3, pb[j][0], pb[j][1]);
          }
        }
      }
      __syncwarp();
      if (!FP8 && lane == 0) mbar_arrive(&empty_bar[s]);
    }

    // Full per-row sums of this warp.
#pragma unroll
    for (int j = 0; j < NQT; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = l_run[j][e];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        l_run[j][e] = v;
      }
  }

  __syncthreads();  // the ring is drained: reuse it as the merge buffer

  float* merge = reinterpret_cast<float*>(smem);
  if (warp < kAttnConsumerWarps) {
#pragma unroll
    for (int j = 0; j < NQT; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = j * 8 + 2 * (lane & 3) + e;
        if (lane < 4) {
          stat_m[warp * C::kRows + n] = m_run[j][e];
          stat_l[warp * C::kRows + n] = l_run[j][e];
        }
#pragma unroll
        for (int db = 0; db < D / 16; ++db) {
          const int d = db * 16 + (lane >> 2);
          float* row = merge + (warp * C::kRows + n) * C::OPITCH;
          row[d] = o_acc[j][db][e];
          row[d + 8] = o_acc[j][db][e + 2];
        }
      }
    }
  }
  __syncthreads();
  float* recv_o = reinterpret_cast<float*>(smem + C::RECV_OFFSET);  // push merge: [RECV_ROWS][D]
  float* recv_lse = recv_o + C::RECV_ROWS * D;                       // [RECV_ROWS]
  const int rpo = (C::kRows + p.nsplit - 1) / p.nsplit;  // rows a rank owns (row n: rank n % nsplit)
  if (C::PUSH && p.cluster) cluster_wait();  // phase 1 done: every rank's buffer may be written

  // Every thread derives the weights of the row it combines itself (the row's CTA max, each
  // warp's weight and the total, in the same operations and order for every thread of the row):
  // no serial statistics phase and no barrier before the combine.  The thread that takes a
  // row's first four columns also publishes the row's log2-sum-exp.
  // Four consecutive head dimensions a thread: 16-byte shared-memory reads, and 16-byte stores to
  // the owner rank (a quarter of the cluster-network transactions of scalar stores).
  for (int idx = threadIdx.x; idx < C::kRows * (D / 4); idx += kAttnThreads) {
    const int n = idx / (D / 4);
    const int d = 4 * (idx - n * (D / 4));
    const int r = r0 + n;
    float mmax = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) mmax = fmaxf(mmax, stat_m[w * C::kRows + n]);
    float fw[kAttnConsumerWarps];
    float ltot = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) {
      const float mw = stat_m[w * C::kRows + n];
      fw[w] = (mw == -CUDART_INF_F) ? 0.f : fast_exp2((mw - mmax) * p.scale_log2);
      ltot = fmaf(stat_l[w * C::kRows + n], fw[w], ltot);
    }
    const float inv = ltot > 0.f ? 1.f / ltot : 0.f;
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) fw[w] *= inv;
    if (d == 0 && p.nsplit > 1) {
      const float lse = (ltot > 0.f) ? mmax * p.scale_log2 + __log2f(ltot) : -CUDART_INF_F;
      if (p.cluster) {
        if constexpr (C::PUSH)
          st_dsmem_f32(map_to_rank(recv_lse + split * rpo + n / p.nsplit, static_cast<uint32_t>(n % p.nsplit)), lse);
        else
          reinterpret_cast<float*>(smem + C::CL_OFFSET)[C::kRows * D + n] = lse;
      } else if (r < r1) {
        const int t = r / p.G, h = kvh * p.G + r % p.G;
        p.part_lse[((static_cast<long long>(b) * p.T + t) * p.Hq + h) * p.nsplit + split] = lse;
      }
    }
    if (r >= r1) continue;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) {
      const float4 m4 = *reinterpret_cast<const float4*>(merge + (w * C::kRows + n) * C::OPITCH + d);
      o.x = fmaf(m4.x, fw[w], o.x);
      o.y = fmaf(m4.y, fw[w], o.y);
      o.z = fmaf(m4.z, fw[w], o.z);
      o.w = fmaf(m4.w, fw[w], o.w);
    }
    const int t = r / p.G, h = kvh * p.G + r % p.G;
    const long long row = (static_cast<long long>(b) * p.T + t) * p.Hq + h;
    if (D == 128 && !FP8 && p.pair) {  // half r of row r, to the real 64-dimension head
      if ((d >> 6) == (h & 1))
        *reinterpret_cast<uint2*>(p.out + row * (D / 2) + (d & 63)) =
            make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
    } else if (p.nsplit == 1) {
      *reinterpret_cast<uint2*>(p.out + row * D + d) = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
    } else if (p.cluster) {
      if constexpr (C::PUSH)
        st_dsmem_f4(map_to_rank(recv_o + (split * rpo + n / p.nsplit) * D + d,
                                static_cast<uint32_t>(n % p.nsplit)), o);
      else
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(smem + C::CL_OFFSET) + n * D + d) = o;
    } else {
      *reinterpret_cast<float4*>(p.part_o + (row * p.nsplit + split) * D + d) = o;
    }
  }
  if (!p.cluster) {
    if (p.nsplit > 1 && p.counters != nullptr)
      split_publish<D>(p, static_cast<int>(blockIdx.x) / p.nsplit, b, kvh, r0, r1,
                       reinterpret_cast<int*>(smem + C::CTL_OFFSET));
    return;
  }

  if constexpr (C::PUSH) {
    // ---- push merge: rank q (= split) owns rows n = q, q + nsplit, .. of the row group, whose
    // partials every rank stored into q's receive buffer before the barrier (one barrier in all;
    // no rank reads another's shared memory, so none has to wait for the others to finish) ----
    cluster_sync();  // phase 2: every rank's stores are visible to their owners
    const int ns = p.nsplit;
    const int my_rows = (C::kRows - split + ns - 1) / ns;
    for (int idx = threadIdx.x; idx < my_rows * (D / 4); idx += kAttnThreads) {
      const int j = idx / (D / 4);
      const int d = 4 * (idx - j * (D / 4));  // four consecutive head dimensions a thread
      const int n = split + j * ns;
      const int r = r0 + n;
      float lq[kMaxClusterSplits];
      float mmax = -CUDART_INF_F;
#pragma unroll
      for (int q = 0; q < kMaxClusterSplits; ++q) {
        lq[q] = q < ns ? recv_lse[q * rpo + j] : -CUDART_INF_F;
        mmax = fmaxf(mmax, lq[q]);
      }
      float wsum = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxClusterSplits; ++q) {
        lq[q] = (lq[q] == -CUDART_INF_F) ? 0.f : fast_exp2(lq[q] - mmax);
        wsum += lq[q];
      }
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kMaxClusterSplits; ++q)
        if (q < ns) {
          const float wq = lq[q] * inv;
          const float4 v = *reinterpret_cast<const float4*>(recv_o + (q * rpo + j) * D + d);
          o.x = fmaf(wq, v.x, o.x);
          o.y = fmaf(wq, v.y, o.y);
          o.z = fmaf(wq, v.z, o.z);
          o.w = fmaf(wq, v.w, o.w);
        }
      if (r < r1) {
        const int t = r / p.G, h = kvh * p.G + r % p.G;
        *reinterpret_cast<uint2*>(p.out + ((static_cast<long long>(b) * p.T + t) * p.Hq + h) * D + d) =
            make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
      }
    }
    return;
  }

  // ---- cluster merge: rank q (= split) writes rows n = q, q + nsplit, .. of the row group ----
  float* cpart = reinterpret_cast<float*>(smem + C::CL_OFFSET);
  float* clse = cpart + C::kRows * D;
  float* cw = clse + C::kRows;  // [kRows][kMaxClusterSplits]
  cluster_sync();  // every rank's partial and lse are written
  const int ns = p.nsplit;
  if (threadIdx.x < C::kRows && static_cast<int>(threadIdx.x) % ns == split) {
    const int n = threadIdx.x;
    float l[kMaxClusterSplits];
    float mmax = -CUDART_INF_F;
#pragma unroll
    for (int q = 0; q < kMaxClusterSplits; ++q) {
      l[q] = q < ns ? ld_dsmem_f32(map_to_rank(clse + n, static_cast<uint32_t>(q))) : -CUDART_INF_F;
      mmax = fmaxf(mmax, l[q]);
    }
    float wsum = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxClusterSplits; ++q) {
      l[q] = (l[q] == -CUDART_INF_F) ? 0.f : fast_exp2(l[q] - mmax);
      wsum += l[q];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int q = 0; q < kMaxClusterSplits; ++q) cw[n * kMaxClusterSplits + q] = l[q] * inv;
  }
  __syncthreads();
  const int my_rows = (C::kRows - split + ns - 1) / ns;
  for (int idx = threadIdx.x; idx < my_rows * D; idx += kAttnThreads) {
    const int n = split + (idx / D) * ns;
    const int d = idx % D;
    const int r = r0 + n;
    // every rank's partial is requested before the first is used: the remote loads overlap
    float part_q[kMaxClusterSplits];
#pragma unroll
    for (int q = 0; q < kMaxClusterSplits; ++q)
      if (q < ns) part_q[q] = ld_dsmem_f32(map_to_rank(cpart + n * D + d, static_cast<uint32_t>(q)));
    float o = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxClusterSplits; ++q)
      if (q < ns) o = fmaf(cw[n * kMaxClusterSplits + q], part_q[q], o);
    if (r < r1) {
      const int t = r / p.G, h = kvh * p.G + r % p.G;
      p.out[((static_cast<long long>(b) * p.T + t) * p.Hq + h) * D + d] = float_to_bf16_bits(o);
    }
  }
  cluster_sync();  // no rank exits while another still reads its shared memory
}

// Merges the split partials of every (b, t, h) row after the split kernel: one warp per row (the
// partials plan on large grids, where a merge inside the last CTA of each row group would hold
// SM slots that the remaining waves need).
template <int D>
__global__ void __launch_bounds__(128) decode_attn_split_combine_kernel(const SplitAttnParams p) {
  const long long row = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= static_cast<long long>(p.B) * p.T * p.Hq) return;
  merge_split_row<D>(p, row, threadIdx.x & 31);
}

}  // namespace mcb
