// Piece 3: decode attention over the KV cache -- a persistent flash-decode with GQA grouping, a
// per-row sliding window and per-row (right-ragged) positions.
//
// Semantics (modelcore/kernels/flash_attn.py:246-264 and :348-366): query token t of row b sits
// at q_pos = L_b + t (L_b = cache_seqlens[b]) and sees key c iff c <= q_pos and
// (window < 0 or q_pos - c <= window); softmax scale 1/sqrt(D); q head h reads kv head h / G.
//
// Work decomposition: a flat tile space, balanced on the device.  An *entry* is (row b, query
// block qb): up to ROWS = 8*NQT flattened query rows r = t*G + g per kv head (for decode, T = 1,
// the G grouped q heads), which share every K/V tile of that head, so each K/V byte is fetched
// once for all of them.  An entry's key range -- the union of its rows' visible ranges -- is cut
// into TK-key tiles; all entries' tiles, in entry order, form one sequence of S tiles.  The grid
// is NG groups of Hkv CTAs: CTA c serves kv head c % Hkv over the tiles
// [g*S/NG, (g+1)*S/NG) of group g = c / Hkv.  The Hkv CTAs of a group read the same positions
// of all kv heads together (whole contiguous (position, head, dim) blocks for DRAM), and every
// CTA computes S itself from cache_seqlens (no host sync, so a CUDA graph stays valid as rows
// grow): the work is balanced to within one tile whatever the batch, lengths or windows.  A row
// group (entry, kv head) that a CTA holds entirely is written as bf16 output.  One cut by a group
// boundary leaves a partial (O/l, log2-sum-exp) in each contributing CTA's slot 0 (its first
// entry) or slot 1 (its last); each contributor then bumps the row group's arrival counter, and
// the contributor that arrives last merges all the partials into the output and resets the
// counter to zero -- no CTA ever waits for another, and no second kernel is launched.
//
// Per CTA a producer warp streams the K and V tiles of its whole tile range with TMA (4-D tensor
// maps over the (B, Tmax, Hkv, D) slot, 128-byte swizzled panels of 64 columns, no multicast) into
// a STAGES-deep shared-memory ring, never draining it between row groups; four consumer warps
// each take KPW keys of every tile.  Per consumer warp the contraction runs on the tensor cores
// with keys on the M side (the K tile is the A operand straight from shared memory) and the
// query rows on the N side:
//   S^T(16 keys x 8 rows)  = K(16 x D) . Q^T(D x 8)        mma.m16n8k16, Q^T fragments in registers
//   O^T(D x 8 rows)       += V^T(D x 16 keys) . P^T(16 x 8)  V^T via ldmatrix.trans, P^T from the S^T
//                                                            accumulators via movmatrix.trans
// Online softmax in fp32 per warp; the four warps merge through a separate shared buffer after
// each row group (named barrier over the consumer warps only, so the producer keeps streaming).
#pragma once

#include <math_constants.h>

#include "common.cuh"
#include "kv_append.cuh"  // rope_norm_vec: the fused append's arithmetic

namespace mcb {

struct AttnParams {
  const uint16_t* q;
  long long qs[3];
  const int32_t* cache_seqlens;
  uint16_t* out;
  float* part_o;    // [(cta*2 + slot)*ROWS + n][D]
  float* part_lse;  // [(cta*2 + slot)*ROWS + n]
  int* counters;     // [entry * Hkv + kv head] arrivals; zero on entry, left zero on exit
  int B, T, Hq, Hkv, G, Tmax, window;
  int ring;  // the slot is a ring of Tmax positions (key c at index c % Tmax)
  float scale_log2;  // softmax_scale * log2(e)
  int nqb;           // query blocks per row
  int n_entries;     // B * nqb
  int grid;          // persistent CTAs = ngroups * Hkv
  int ngroups;       // CTA groups; CTA c serves kv head c % Hkv of group c / Hkv
  // fused append (bf16 slot, one new token a row, D = 64 or 128): q is the raw query projection;
  // every CTA ropes, norms and scales the query heads of each row group it serves, and the CTA
  // whose tile range holds a row's new position writes the new key (roped, normed, scaled unless
  // raw) and value into the slot and into its own copy of that tile -- kv_append_rope_vec_kernel's
  // arithmetic, the same bits
  int fuse;
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

constexpr int kAttnConsumerWarps = 4;
constexpr int kAttnThreads = (kAttnConsumerWarps + 1) * 32;

template <int D, int NQT, int KPW, int STAGES>
struct AttnConfig {
  static constexpr int kRows = 8 * NQT;                      // query rows per row group
  static constexpr int TK = KPW * kAttnConsumerWarps;        // keys per tile
  static constexpr int PANEL = D < 64 ? D : 64;              // columns per swizzled panel
  static constexpr int NPANEL = D / PANEL;
  static constexpr int ROW_BYTES = PANEL * 2;                // 32, 64 or 128
  static constexpr int SWZ_MASK = ROW_BYTES == 128 ? 7 : (ROW_BYTES == 64 ? 3 : 1);
  static constexpr int PANEL_BYTES = TK * ROW_BYTES;
  static constexpr int TILE_BYTES = NPANEL * PANEL_BYTES;    // one K (or V) tile
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int OPITCH = D + 4;                       // merge buffer row pitch (floats)
  static constexpr int MERGE_OFFSET = RING_BYTES;
  static constexpr int MERGE_BYTES = 2 * kAttnConsumerWarps * kRows * OPITCH * 4;  // two copies
  static constexpr int BAR_OFFSET = MERGE_OFFSET + MERGE_BYTES;
  static constexpr int STAT_OFFSET = BAR_OFFSET + 2 * STAGES * 8;
  static constexpr int STAT_BYTES = 2 * 2 * kAttnConsumerWarps * kRows * 4;  // (m, l) x two copies
  static constexpr int CTL_OFFSET = STAT_OFFSET + STAT_BYTES;  // abort flag, start state, last flag
  static constexpr int CTL_BYTES = 64;
  // fused append, by segment parity (this row group and the next), bf16: the processed query
  // rows [2][kRows][D], the processed new key and value [2][2][D], and the staged raw inputs
  // [2][STG]: query rows [kRows][D], key and value [2][D], the rotary rows cos | sin [D]
  static constexpr int FUSE_OFFSET = CTL_OFFSET + CTL_BYTES;
  static constexpr int FUSE_Q = kRows * D;          // elements
  static constexpr int FUSE_KV = 2 * D;
  static constexpr int FUSE_STG = (kRows + 3) * D;
  static constexpr int FUSE_BYTES = (D == 64 || D == 128) ? 2 * (FUSE_Q + FUSE_KV + FUSE_STG) * 2 : 0;
  static constexpr int SMEM_BYTES = FUSE_OFFSET + FUSE_BYTES + 1024;  // + alignment slack
  static_assert(D % 16 == 0 && D >= 16 && D <= 256, "head_dim");
  static_assert(KPW % 16 == 0, "keys per warp");
  static_assert(RING_BYTES % 1024 == 0, "ring alignment");
  static_assert(FUSE_OFFSET % 16 == 0, "fused-append buffers: 16-byte vectors");
};

// Byte offset of the 16-byte chunk `chunk` (0 .. ROW_BYTES/16) of key row `key` in a panel,
// after the TMA swizzle (CU_TENSOR_MAP_SWIZZLE_32B/64B/128B): bits [4, 7) of the offset are
// xor-ed with bits [7, 10).
template <int ROW_BYTES, int SWZ_MASK>
__device__ __forceinline__ uint32_t swz(int key, int chunk) {
  const uint32_t off = static_cast<uint32_t>(key * ROW_BYTES + chunk * 16);
  return off ^ (((off >> 7) & SWZ_MASK) << 4);
}

// One (row b, query block qb) entry: its query rows, visible key range and tile count.
struct Entry {
  int b, r0, r1, L, lo, hi, kb, n;
};

template <int ROWS, int TK>
__device__ __forceinline__ Entry make_entry(const AttnParams& p, int e, int L) {
  Entry x;
  x.b = e / p.nqb;
  const int qb = e - x.b * p.nqb;
  x.r0 = qb * ROWS;
  x.r1 = min(x.r0 + ROWS, p.T * p.G);
  const int t_first = x.r0 / p.G;
  const int t_last = (x.r1 - 1) / p.G;
  x.L = L;
  x.hi = p.ring ? max(L + t_last, 0) : min(max(L + t_last, 0), p.Tmax - 1);  // bad L: the scan reports
  x.lo = p.window >= 0 ? max(0, L + t_first - p.window) : 0;
  x.kb = (min(x.lo, x.hi) / TK) * TK;
  x.n = (x.hi - x.kb) / TK + 1;
  return x;
}

__device__ __forceinline__ long long range_begin(long long c, long long total, int grid) {
  return c * total / grid;
}

// The group whose range [range_begin(g), range_begin(g + 1)) holds tile t.
__device__ __forceinline__ int tile_owner(long long t, long long total, int ngroups) {
  return static_cast<int>(((t + 1) * ngroups - 1) / total);
}

// Walk position through the tile space.
struct Walk {
  int e, kvh, local;
  long long t;
  Entry ent;
};

template <int ROWS, int TK>
__device__ __forceinline__ void walk_next_group(const AttnParams& p, Walk& w) {
  w.local = 0;
  if (++w.e < p.n_entries) w.ent = make_entry<ROWS, TK>(p, w.e, p.cache_seqlens[w.e / p.nqb]);
}

// Warp-cooperative start of a CTA: the total tile count S and the entry holding the first tile
// of the CTA's group.  Writes {S, e, kvh, local} to ctl[1..4] (smem).
template <int ROWS, int TK>
__device__ void locate_start(const AttnParams& p, int* ctl) {
  const int lane = threadIdx.x & 31;
  const int grp = blockIdx.x / p.Hkv;
  long long total = 0;
#pragma unroll 4
  for (int base = 0; base < p.n_entries; base += 32) {
    const int e = base + lane;
    if (e < p.n_entries) {
      const int L = p.cache_seqlens[e / p.nqb];
      const Entry x = make_entry<ROWS, TK>(p, e, L);
      if (L < 0 || (!p.ring && L + (x.r1 - 1) / p.G >= p.Tmax)) record_error(kErrPositionBeyondCache);
      total += x.n;
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) total += __shfl_xor_sync(0xffffffffu, total, m);
  const long long begin = range_begin(grp, total, p.ngroups);
  const long long end = range_begin(grp + 1, total, p.ngroups);
  int e_found = -1, local = 0;
  if (begin < end) {
    long long running = 0;
    for (int base = 0; base < p.n_entries; base += 32) {
      const int e = base + lane;
      long long v = 0;
      if (e < p.n_entries) v = make_entry<ROWS, TK>(p, e, p.cache_seqlens[e / p.nqb]).n;
      long long incl = v;
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const long long o = __shfl_up_sync(0xffffffffu, incl, m);
        if (lane >= m) incl += o;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, running + incl > begin);
      if (hit) {
        const int src = __ffs(hit) - 1;
        const long long excl = running + __shfl_sync(0xffffffffu, incl - v, src);
        e_found = base + src;
        local = static_cast<int>(begin - excl);
        break;
      }
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (lane == 0) {
    const int kvh = blockIdx.x % p.Hkv;
    ctl[1] = static_cast<int>(total);
    ctl[2] = e_found;
    ctl[3] = kvh;
    ctl[4] = local;
  }
}

// Q^T fragments (the B operand of S^T = K Q^T) of a row group: row n = j*8 + lane/4, columns
// d = kk*16 + 2*(lane%4) + {0,1} and + 8; zeros for padding rows.
template <int D, int NQT>
__device__ __forceinline__ void load_q_frags(const AttnParams& p, const Entry& ent, int kvh,
                                             uint32_t (&qf)[NQT][D / 16][2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NQT; ++j) {
    const int r = ent.r0 + j * 8 + (lane >> 2);
    const uint16_t* qrow = nullptr;
    if (r < ent.r1) {
      const int t = r / p.G, h = kvh * p.G + r % p.G;
      qrow = p.q + ent.b * p.qs[0] + t * p.qs[1] + h * p.qs[2];
    }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      qf[j][kk][0] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
      qf[j][kk][1] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d0 + 8) : 0u;
    }
  }
}

// The same from a row group's query rows in shared memory ([kRows][D], nvalid of them).
template <int D, int NQT>
__device__ __forceinline__ void load_q_frags_smem(const uint16_t* qsrc, int nvalid,
                                                  uint32_t (&qf)[NQT][D / 16][2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NQT; ++j) {
    const int n = j * 8 + (lane >> 2);
    const uint16_t* qrow = n < nvalid ? qsrc + n * D : nullptr;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      qf[j][kk][0] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
      qf[j][kk][1] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d0 + 8) : 0u;
    }
  }
}

// Fused append, step 1 (one warp; asynchronous): a row group's raw inputs staged into `stg` by
// cp.async -- its query rows (T = 1: row r of the group is q head kvh * G + r), the raw key and
// value (with k_new) and the rotary rows at its position.  Completed by cp_async_wait_all.
template <int D, int ROWS>
__device__ __forceinline__ void fuse_fetch(const AttnParams& p, const Entry& ent, int kvh, uint16_t* stg) {
  constexpr int CH = D / 8;  // 16-byte chunks a vector
  const int lane = threadIdx.x & 31;
  const int nq = ent.r1 - ent.r0;
  const uint32_t sq = smem_u32(stg), skv = smem_u32(stg + ROWS * D), srot = smem_u32(stg + (ROWS + 2) * D);
  for (int c = lane; c < nq * CH; c += 32) {
    const int v = c / CH, ch = c - v * CH;
    cp_async16(sq + (v * D + ch * 8) * 2, p.q + ent.b * p.qs[0] + (kvh * p.G + ent.r0 + v) * p.qs[2] + ch * 8);
  }
  if (p.k_new != nullptr && lane < 2 * CH) {
    const int isv = lane >= CH ? 1 : 0, ch = lane % CH;
    const uint16_t* src = isv ? p.v_new + ent.b * p.vns[0] + kvh * p.vns[2]
                              : p.k_new + ent.b * p.kns[0] + kvh * p.kns[2];
    cp_async16(skv + (isv * D + ch * 8) * 2, src + ch * 8);
  }
  if (ent.L >= 0 && ent.L < p.rot_len && lane < CH) {  // D/2 cosines, then D/2 sines
    const int is_sin = lane >= CH / 2 ? 1 : 0, ch = lane % (CH / 2);
    const uint16_t* tab = is_sin ? p.rot_sin : p.rot_cos;
    cp_async16(srot + (is_sin * (D / 2) + ch * 8) * 2,
               tab + static_cast<long long>(ent.L) * (D / 2) + ch * 8);
  }
  cp_async_commit();
}

// Fused append, step 2 (the same warp, after cp_async_wait_all and __syncwarp): the staged query
// rows roped, normed and scaled into qdst [kRows][D]; with_kv: the new key (roped, normed and
// scaled when p.rotate_k) and the value into kvdst [2][D] and into the slot at the row's position
// -- groups of D/16 lanes one vector each, kv_append_rope_vec_kernel's arithmetic, the same bits.
template <int D, int ROWS>
__device__ __forceinline__ void fuse_finish(const AttnParams& p, const Entry& ent, int kvh, const uint16_t* stg,
                                            bool with_kv, uint16_t* qdst, uint16_t* kvdst) {
  constexpr int LG = D / 16, VPW = 32 / LG, HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LG;
  const int nq = ent.r1 - ent.r0;
  const int nvec = nq + (with_kv ? 2 : 0);
  const int L = ent.L;
  const bool rot_ok = L >= 0 && L < p.rot_len;
  const uint16_t* srot = stg + (ROWS + 2) * D;
  const uint4 cv = rot_ok ? *reinterpret_cast<const uint4*>(srot + 8 * sub) : make_uint4(0, 0, 0, 0);
  const uint4 sv = rot_ok ? *reinterpret_cast<const uint4*>(srot + HALF + 8 * sub) : make_uint4(0, 0, 0, 0);
  for (int v0 = 0; v0 < nvec; v0 += VPW) {
    const int vi = v0 + lane / LG;
    const bool valid = vi < nvec;
    const bool is_q = vi < nq, is_k = vi == nq;
    const uint16_t* src = is_q ? stg + vi * D : stg + (ROWS + (is_k ? 0 : 1)) * D;
    const bool rotate = valid && (is_q || (is_k && p.rotate_k));
    if (rotate && !rot_ok && sub == 0) record_error(kErrPositionBeyondRotary);
    const uint4 x1v = valid ? *reinterpret_cast<const uint4*>(src + 8 * sub) : make_uint4(0, 0, 0, 0);
    const uint4 x2v = valid ? *reinterpret_cast<const uint4*>(src + HALF + 8 * sub) : make_uint4(0, 0, 0, 0);
    uint4 w1, w2;
    rope_norm_vec_tab<D>(x1v, x2v, cv, sv, rotate && rot_ok, p.norm_eps, p.qk_scale, w1, w2);
    if (valid) {
      uint16_t* dst = is_q ? qdst + vi * D : kvdst + (is_k ? 0 : D);
      *reinterpret_cast<uint4*>(dst + 8 * sub) = w1;
      *reinterpret_cast<uint4*>(dst + HALF + 8 * sub) = w2;
      if (!is_q && (p.ring || L < p.Tmax)) {
        const int idx = p.ring ? L % p.Tmax : L;
        uint16_t* cdst = (is_k ? p.kc_out : p.vc_out) +
                         ((static_cast<long long>(ent.b) * p.Tmax + idx) * p.Hkv + kvh) * D;
        *reinterpret_cast<uint4*>(cdst + 8 * sub) = w1;
        *reinterpret_cast<uint4*>(cdst + HALF + 8 * sub) = w2;
      }
    }
  }
}

// Whether a CTA's segment of `seg` tiles from tile `local` of the entry holds the row's new
// position (T = 1: the entry's last tile), and the new key's row in that tile.
template <int TK>
__device__ __forceinline__ bool segment_owns_new(const Entry& ent, int local, int seg, int* row) {
  const int tile_new = ent.L >= 0 ? (ent.L - ent.kb) / TK : -1;
  *row = ent.L - (ent.kb + tile_new * TK);
  return tile_new >= local && tile_new < local + seg;
}

template <int D, int NQT, int KPW, int STAGES>
__global__ void __launch_bounds__(kAttnThreads)
    decode_attn_kernel(const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const AttnParams p) {
  using C = AttnConfig<D, NQT, KPW, STAGES>;
  constexpr int ROWS = C::kRows;
  constexpr int TK = C::TK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* merge = reinterpret_cast<float*>(smem + C::MERGE_OFFSET);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFFSET);
  uint64_t* empty_bar = full_bar + STAGES;
  float* stat_m = reinterpret_cast<float*>(smem + C::STAT_OFFSET);
  int* ctl = reinterpret_cast<int*>(smem + C::CTL_OFFSET);  // [0] abort, [1..4] start, [5..6] last
  volatile int* abort_flag = ctl;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kAttnConsumerWarps);
    }
    ctl[0] = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) locate_start<ROWS, TK>(p, ctl);
  __syncthreads();

  const long long total = ctl[1];
  if (ctl[2] < 0) return;  // no tiles for this CTA
  const int grp = blockIdx.x / p.Hkv;
  const long long t_end = range_begin(grp + 1, total, p.ngroups);
  Walk w;
  w.e = ctl[2];
  w.kvh = ctl[3];
  w.local = ctl[4];
  w.t = range_begin(grp, total, p.ngroups);
  w.ent = make_entry<ROWS, TK>(p, w.e, p.cache_seqlens[w.e / p.nqb]);

  if (warp == kAttnConsumerWarps) {
    // ---------------- producer warp: one lane streams every tile of the CTA's range ----------------
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const uint64_t policy = l2_policy_evict_first();
      uint32_t g = 0;
      while (w.t < t_end) {
        const int seg = static_cast<int>(min(static_cast<long long>(w.ent.n - w.local), t_end - w.t));
        for (int i = 0; i < seg; ++i, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES && !mbar_wait_or_abort(&empty_bar[s], ((g / STAGES) - 1) & 1, abort_flag))
            return;
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          const int key0 = w.ent.kb + (w.local + i) * TK;
          const int slot0 = p.ring ? key0 % p.Tmax : key0;  // a ring slot: Tmax % TK == 0
          uint8_t* kdst = smem + s * C::STAGE_BYTES;
          uint8_t* vdst = kdst + C::TILE_BYTES;
#pragma unroll
          for (int pn = 0; pn < C::NPANEL; ++pn) {
            tma_load_4d(kdst + pn * C::PANEL_BYTES, &kmap, &full_bar[s], pn * C::PANEL, w.kvh, slot0,
                        w.ent.b, policy);
            tma_load_4d(vdst + pn * C::PANEL_BYTES, &vmap, &full_bar[s], pn * C::PANEL, w.kvh, slot0,
                        w.ent.b, policy);
          }
        }
        w.t += seg;
        w.local += seg;
        if (w.local == w.ent.n) walk_next_group<ROWS, TK>(p, w);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  constexpr int NCH = KPW / 16;  // 16-key chunks per warp per tile
  uint32_t g = 0;
  bool first_segment = true;
  int seg_index = 0;
  // fused append, by segment parity: the processed query rows, new key and value, and the raw
  // inputs staged for them
  uint16_t* qbuf = reinterpret_cast<uint16_t*>(smem + C::FUSE_OFFSET);  // [2][FUSE_Q]
  uint16_t* kvbuf = qbuf + 2 * C::FUSE_Q;                               // [2][FUSE_KV]
  uint16_t* stg = kvbuf + 2 * C::FUSE_KV;                               // [2][FUSE_STG]
  const bool fuse = C::FUSE_BYTES > 0 && p.fuse;
  uint32_t qf[NQT][D / 16][2];
  if (fuse) {
    // the first row group's inputs in the open; later groups' are staged a segment ahead
    if (warp == 0) {
      const int seg0 = static_cast<int>(min(static_cast<long long>(w.ent.n - w.local), t_end - w.t));
      int row;
      const bool own0 = p.k_new != nullptr && segment_owns_new<TK>(w.ent, w.local, seg0, &row);
      fuse_fetch<D, ROWS>(p, w.ent, w.kvh, stg);
      cp_async_wait_all();
      __syncwarp();
      fuse_finish<D, ROWS>(p, w.ent, w.kvh, stg, own0, qbuf, kvbuf);
    }
    named_barrier(1, kAttnConsumerWarps * 32);
    load_q_frags_smem<D, NQT>(qbuf, w.ent.r1 - w.ent.r0, qf);
  } else {
    load_q_frags<D, NQT>(p, w.ent, w.kvh, qf);
  }
  while (w.t < t_end) {
    const Entry& ent = w.ent;
    const int seg = static_cast<int>(min(static_cast<long long>(ent.n - w.local), t_end - w.t));
    const bool complete = (w.local == 0 && seg == ent.n);
    const int slot = first_segment ? 0 : 1;
    const int nvalid = ent.r1 - ent.r0;
    const int par = seg_index & 1;
    // fused append: whether this segment's tiles hold the row's new position (its key and value
    // are in kvbuf[par], prepared before the last merge barrier) and the new key's row there;
    // warp 0 stages the next row group's raw inputs now and finishes them after its tiles
    int new_row = 0;
    const bool own_new = fuse && p.k_new != nullptr && segment_owns_new<TK>(ent, w.local, seg, &new_row);
    if (fuse && warp == 0 && w.t + seg < t_end) {
      Walk wq = w;  // the next row group
      wq.local += seg;
      walk_next_group<ROWS, TK>(p, wq);
      fuse_fetch<D, ROWS>(p, wq.ent, wq.kvh, stg + (par ^ 1) * C::FUSE_STG);
    }

    float m_run[NQT][2], l_run[NQT][2];
    float o_acc[NQT][D / 16][4];
    int row_hi[NQT][2], row_lo[NQT][2];
#pragma unroll
    for (int j = 0; j < NQT; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int rr = ent.r0 + j * 8 + 2 * (lane & 3) + e;
        m_run[j][e] = -CUDART_INF_F;
        l_run[j][e] = 0.f;
        if (rr < ent.r1) {
          const int qpos = ent.L + rr / p.G;
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

    for (int i = 0; i < seg; ++i, ++g) {
      const int s = g % STAGES;
      const bool ready = mbar_wait_or_abort(&full_bar[s], (g / STAGES) & 1, abort_flag);
      if (ready) {
        const uint32_t kbase = smem_u32(smem + s * C::STAGE_BYTES);
        const uint32_t vbase = kbase + C::TILE_BYTES;
        const int tile_key0 = ent.kb + (w.local + i) * TK;
        // fused append: the tile arrived with the slot's old bytes at the new position; the warp
        // that owns that row writes the new key and value over it before reading the tile
        if (own_new && tile_key0 <= ent.L && ent.L < tile_key0 + TK && new_row / KPW == warp) {
          constexpr int NCHK = D / 8;  // 16-byte chunks per row
          if (lane < 2 * NCHK) {
            const int isv = lane >= NCHK ? 1 : 0;
            const int col = (lane % NCHK) * 8;
            const uint32_t dst = (isv ? vbase : kbase) + (col / C::PANEL) * C::PANEL_BYTES +
                                 swz<C::ROW_BYTES, C::SWZ_MASK>(new_row, (col % C::PANEL) / 8);
            sts128(dst, lds128(smem_u32(kvbuf + par * C::FUSE_KV + isv * D + col)));
          }
          fence_proxy_async_shared();  // TMA refills this stage later
          __syncwarp();
        }

        float sc[NCH][NQT][4];
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
          for (int j = 0; j < NQT; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) sc[ch][j][c] = 0.f;
          const int krow = warp * KPW + ch * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int col = kk * 16 + (lane >> 4) * 8;
            const uint32_t addr = kbase + (col / C::PANEL) * C::PANEL_BYTES +
                                  swz<C::ROW_BYTES, C::SWZ_MASK>(krow, (col % C::PANEL) / 8);
            uint32_t a0, a1, a2, a3;
            ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
            for (int j = 0; j < NQT; ++j)
              mma_16816(sc[ch][j], a0, a1, a2, a3, qf[j][kk][0], qf[j][kk][1]);
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
            pb[j][0] = movmatrix_trans(pack_bf16x2(sc[ch][j][0], sc[ch][j][1]));
            pb[j][1] = movmatrix_trans(pack_bf16x2(sc[ch][j][2], sc[ch][j][3]));
          }
          const int m = lane >> 3;
          const int vrow = warp * KPW + ch * 16 + (lane & 7) + (m >> 1) * 8;
#pragma unroll
          for (int db = 0; db < D / 16; ++db) {
            const int col = db * 16 + (m & 1) * 8;
            const uint32_t addr = vbase + (col / C::PANEL) * C::PANEL_BYTES +
                                  swz<C::ROW_BYTES, C::SWZ_MASK>(vrow, (col % C::PANEL) / 8);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_trans(addr, a0, a1, a2, a3);
#pragma unroll
            for (int j = 0; j < NQT; ++j)
              mma_16816(o_acc[j][db], a0, a1, a2, a3, pb[j][0], pb[j][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }

    // The next row group's Q fragments load while this one merges (fused: from warp 0's rows,
    // after the merge barrier below).
    Walk wn = w;
    wn.t += seg;
    wn.local += seg;
    if (wn.local == wn.ent.n) walk_next_group<ROWS, TK>(p, wn);
    uint32_t qf_next[NQT][D / 16][2];
    if (!fuse && wn.t < t_end) load_q_frags<D, NQT>(p, wn.ent, wn.kvh, qf_next);
    if (fuse && warp == 0 && wn.t < t_end) {  // the next row group's rows from the staged inputs
      const int seg_n = static_cast<int>(min(static_cast<long long>(wn.ent.n - wn.local), t_end - wn.t));
      int row;
      const bool own_n = p.k_new != nullptr && segment_owns_new<TK>(wn.ent, wn.local, seg_n, &row);
      cp_async_wait_all();
      __syncwarp();
      fuse_finish<D, ROWS>(p, wn.ent, wn.kvh, stg + (par ^ 1) * C::FUSE_STG, own_n,
                           qbuf + (par ^ 1) * C::FUSE_Q, kvbuf + (par ^ 1) * C::FUSE_KV);
    }

    // ---- merge the four warps' partial softmax states of this row group ----
    // The merge buffer, the statistics and the "last contributor" flag alternate between two
    // copies by row-group parity, so one barrier per row group suffices: a warp can only write
    // a copy again after the next row group's barrier, which every warp reaches after its reads.
    float* mbuf = merge + par * (kAttnConsumerWarps * ROWS * C::OPITCH);
    float* st_m = stat_m + par * (2 * kAttnConsumerWarps * ROWS);
    float* st_l = st_m + kAttnConsumerWarps * ROWS;
#pragma unroll
    for (int j = 0; j < NQT; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = l_run[j][e];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        const int n = j * 8 + 2 * (lane & 3) + e;
        if (n >= nvalid) continue;
        if (lane < 4) {
          st_m[warp * ROWS + n] = m_run[j][e];
          st_l[warp * ROWS + n] = v;
        }
        float* row = mbuf + (warp * ROWS + n) * C::OPITCH;
#pragma unroll
        for (int db = 0; db < D / 16; ++db) {
          const int d = db * 16 + (lane >> 2);
          row[d] = o_acc[j][db][e];
          row[d + 8] = o_acc[j][db][e + 2];
        }
      }
    named_barrier(1, kAttnConsumerWarps * 32);
    if (fuse && wn.t < t_end)
      load_q_frags_smem<D, NQT>(qbuf + (par ^ 1) * C::FUSE_Q, wn.ent.r1 - wn.ent.r0, qf_next);

    for (int idx = threadIdx.x; idx < nvalid * D; idx += kAttnConsumerWarps * 32) {
      const int n = idx / D;
      const int d = idx - n * D;
      float mmax = -CUDART_INF_F;
#pragma unroll
      for (int ww = 0; ww < kAttnConsumerWarps; ++ww) mmax = fmaxf(mmax, st_m[ww * ROWS + n]);
      float ltot = 0.f, o = 0.f;
#pragma unroll
      for (int ww = 0; ww < kAttnConsumerWarps; ++ww) {
        const float mw = st_m[ww * ROWS + n];
        const float f = (mw == -CUDART_INF_F) ? 0.f : fast_exp2((mw - mmax) * p.scale_log2);
        ltot = fmaf(st_l[ww * ROWS + n], f, ltot);
        o = fmaf(mbuf[(ww * ROWS + n) * C::OPITCH + d], f, o);
      }
      o = ltot > 0.f ? o / ltot : 0.f;
      if (complete) {
        const int r = ent.r0 + n;
        const int t = r / p.G, h = w.kvh * p.G + r % p.G;
        p.out[((static_cast<long long>(ent.b) * p.T + t) * p.Hq + h) * D + d] = float_to_bf16_bits(o);
      } else {
        const long long prow = (static_cast<long long>(blockIdx.x) * 2 + slot) * ROWS + n;
        p.part_o[prow * D + d] = o;
        if (d == 0) p.part_lse[prow] = ltot > 0.f ? mmax * p.scale_log2 + __log2f(ltot) : -CUDART_INF_F;
      }
    }
    if (!complete) {
      // Publish this partial (the barrier orders every thread's stores before thread 0's release
      // of the arrival counter); the contributor that arrives last merges every partial of the
      // row group, its own included, into the output and resets the counter.
      named_barrier(1, kAttnConsumerWarps * 32);
      const long long start_e = w.t - w.local;  // tile index of the entry's first tile
      const int g_first = tile_owner(start_e, total, p.ngroups);
      const int g_last = tile_owner(start_e + ent.n - 1, total, p.ngroups);
      const bool first_in_slot1 = start_e != range_begin(g_first, total, p.ngroups);
      if (threadIdx.x == 0) {
        int ncontrib = 0;
        for (int gg = g_first; gg <= g_last; ++gg)
          ncontrib += range_begin(gg, total, p.ngroups) < range_begin(gg + 1, total, p.ngroups);
        int* counter = p.counters + static_cast<long long>(w.e) * p.Hkv + w.kvh;
        const int prev = atom_add_acq_rel_gpu(counter, 1);
        const bool last = prev == ncontrib - 1;
        if (last) *counter = 0;  // every contributor has arrived: ready for the next call
        ctl[5 + par] = last;
      }
      named_barrier(1, kAttnConsumerWarps * 32);
      if (ctl[5 + par]) {
        // Warp `warp` merges rows warp, warp + 4, ...: lanes load the contributors'
        // log-sum-exps in parallel (32 at a time), then stream the weighted partial rows.
        constexpr int PER_LANE = (D + 31) / 32;
        const int ncand = g_last - g_first + 1;
        for (int n = warp; n < nvalid; n += kAttnConsumerWarps) {
          auto row_of = [&](int k) {
            const int gg = g_first + k;
            const int sl = (k == 0 && first_in_slot1) ? 1 : 0;
            return (static_cast<long long>(gg * p.Hkv + w.kvh) * 2 + sl) * ROWS + n;
          };
          auto has_tiles = [&](int k) {
            return range_begin(g_first + k, total, p.ngroups) <
                   range_begin(g_first + k + 1, total, p.ngroups);
          };
          float mmax = -CUDART_INF_F;
          for (int k = lane; k < ncand; k += 32)
            if (has_tiles(k)) mmax = fmaxf(mmax, __ldcg(p.part_lse + row_of(k)));
#pragma unroll
          for (int m = 16; m >= 1; m >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, m));
          float acc[PER_LANE];
#pragma unroll
          for (int u = 0; u < PER_LANE; ++u) acc[u] = 0.f;
          float wsum = 0.f;
          for (int k0 = 0; k0 < ncand; k0 += 32) {
            float wk = 0.f;
            if (k0 + lane < ncand && has_tiles(k0 + lane)) {
              const float ls = __ldcg(p.part_lse + row_of(k0 + lane));
              wk = (ls == -CUDART_INF_F) ? 0.f : fast_exp2(ls - mmax);
            }
            float ws = wk;
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, m);
            wsum += ws;
            const int cnt = min(32, ncand - k0);
#pragma unroll 4
            for (int j = 0; j < cnt; ++j) {
              const float wgt = __shfl_sync(0xffffffffu, wk, j);
              if (wgt == 0.f) continue;
              const float* po = p.part_o + row_of(k0 + j) * D;
#pragma unroll
              for (int u = 0; u < PER_LANE; ++u) {
                const int d = lane + 32 * u;
                if (d < D) acc[u] = fmaf(wgt, __ldcg(po + d), acc[u]);
              }
            }
          }
          const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
          const int r = ent.r0 + n;
          const int t = r / p.G, h = w.kvh * p.G + r % p.G;
          uint16_t* dst = p.out + ((static_cast<long long>(ent.b) * p.T + t) * p.Hq + h) * D;
#pragma unroll
          for (int u = 0; u < PER_LANE; ++u) {
            const int d = lane + 32 * u;
            if (d < D) dst[d] = float_to_bf16_bits(acc[u] * inv);
          }
        }
      }
    }
    first_segment = false;
    ++seg_index;
    w = wn;
#pragma unroll
    for (int j = 0; j < NQT; ++j)
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qf[j][kk][0] = qf_next[j][kk][0];
        qf[j][kk][1] = qf_next[j][kk][1];
      }
  }
}

}  // namespace mcb
