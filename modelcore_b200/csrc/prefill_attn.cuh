// Prefill attention through the cache on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// The attention of flash_attn_with_kvcache with T_new > 1 (modelcore/kernels/flash_attn.py:348-366,
// _sdpa_attention :203-244 with _ragged_decode_mask :246-264): query t of row b sits at position
// L_b + t and sees cache keys c <= L_b + t within the window.  The new tokens' K/V are already in
// the cache (the append ran first), so a prompt's prefill is dense causal attention over its own
// keys plus whatever prefix the row already held.
//
// A work item is two 128-query tiles (Q0, Q1: 256 consecutive queries) of one q head of one row;
// its CTA walks 128-key tiles, each K/V tile serving both query tiles.  The grid is persistent
// (one CTA per SM, items strided over the CTAs, longest first), so TMEM allocation, barrier setup
// and the pipeline fill are paid once per CTA and the next item's loads overlap this one's end.
// The QT = 1 copy (head size 64) takes one query tile an item with ten warps (no Q1 softmax
// warps; two softmax warps a row quarter, 64 key columns each) and 256 TMEM columns, two CTAs
// per SM: the two query-tile chains of an SM are then independent -- neither waits for the
// other's extra causal key tile or epilogue, at the price of K/V tiles read once per query tile
// instead of once per pair.  The roles (QT = 2):
//
//   warp 0       TMA producer: per item Q0 and Q1 (double-buffered for D = 64), then K_j and V_j
//                into a two-stage ring that runs on across items
//   warp 1       allocates all 512 TMEM columns; lane 0 issues the MMAs, ping-ponging the tiles:
//                  S0_j = Q0 K_j^T, S1_j = Q1 K_j^T      kind::f16, M=128 N=128 K=D, A and B
//                                                        from shared memory, fp32 into TMEM
//                  O0 += P0_j V_j, O1 += P1_j V_j        M=128 N=D K=128, A = P from TMEM (P is
//                                                        written over S as bf16), B = V MN-major
//                in the order S0_0 S1_0 | PV0_0 S0_1 | PV1_0 S1_1 | PV0_1 S0_2 | ... so the
//                tensor core computes one tile's S while the other tile's softmax runs
//   warps 2-5    softmax of Q0, warps 6-9 softmax of Q1: one thread per query row (TMEM lane =
//                row; warp w reaches lanes 32 (w % 4) .. +31, so each group of four covers all
//                128; QT = 1: warps 2-9, two a row quarter, each on 64 of the tile's key columns
//                and 32 of O's, the partial row maxima and sums exchanged through shared
//                memory): S from TMEM, mask only on tiles that cross the diagonal, the window
//                edge or the end of the rows; online max with a lazy rescale (the running max moves, and
//                O and the row sum are rescaled, only when a row's max grows by more than 2^8);
//                P = exp2(S * scale * log2 e - max) written back into TMEM as bf16; at the end
//                O / sum as bf16 to the output
//
// Tensor-core MMAs issued by one thread execute in order, so S_{j+1} may overwrite the columns
// that held P_j once PV_j was issued before it, and a completed S_{j+1} implies a completed PV_j
// (the softmax warps rescale O only then).
//
// TMEM: S0 columns [0,128), S1 [128,256), O0 [256, 256+D), O1 [256+D, 256+2D) (QT = 1: S0, then
// O0 at 128).  Every wait is
// bounded (2 s); a timeout raises the CTA's abort flag, every later wait returns at once, the MMA
// issuer waits (bounded) for its committed MMAs, and TMEM is freed before the CTA exits.
#pragma once

#include "common.cuh"

namespace mcb {

constexpr int kPfTile = 128;          // queries per query tile and keys per key tile
// QT query tiles an item (2: one CTA per SM, ten warps, all 512 TMEM columns; 1: two CTAs per SM,
// ten warps -- two softmax warps a row quarter -- and 256 TMEM columns each, every query tile an
// independent chain)
// Softmax warps a row quarter, each taking 128 / pf_split of a tile's key columns.  One query tile
// an item (two CTAs an SM, one softmax chain each): two, so that an SM sub-partition holds four
// softmax warps that hide one another's exponential and TMEM-load latency (config 2's 64 x 512
// prefill 118.8 -> 112.6 us).  Pairs: one -- the two query tiles' chains already interleave,
// and 18 warps would cut a thread's registers from 168 to 96 (8k prompt 289 -> 305 us).
template <int QT>
__host__ __device__ constexpr int pf_split() { return QT == 1 ? 2 : 1; }
template <int QT>
__host__ __device__ constexpr int pf_threads() { return (2 + 4 * QT * pf_split<QT>()) * 32; }
template <int QT>
__host__ __device__ constexpr uint32_t pf_tmem_cols() { return 256u * QT; }

// ---------------------------------------------------------------------------------------------
// tcgen05 helpers
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], bf16 in, fp32 accumulate.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]: A is M rows (TMEM lanes) x K bf16, two per column.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar` when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 128 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane i: row lane_base + i),
// waited for inside the same asm so no use of the values can move above the wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%128];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%129];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95}, [%130];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%131];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr + 0u), "r"(taddr + 32u), "r"(taddr + 64u), "r"(taddr + 96u)
      : "memory");
}

// 64 consecutive 32-bit TMEM columns of this warp's 32 lanes, waited for inside the same asm.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr + 0u), "r"(taddr + 32u)
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane i: row lane_base + i),
// waited for inside the same asm so no use of the values can move above the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 0u)
      : "memory");
}

// Stores 32 consecutive 32-bit TMEM columns of this warp's 32 lanes and waits for them.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      :
      : "r"(taddr + 0u), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Stores 16 consecutive 32-bit TMEM columns of this warp's 32 lanes (no wait: the registers are
// read at issue; tmem_st_wait() orders the stores before a fence).
__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      :
      : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Packed fp32 pairs (sm_100): one instruction for two lanes' worth of FMA.
// (d0, d1) = (a0, a1) * b + c with b, c packed pairs (a pair of equal scalars here).
__device__ __forceinline__ void ffma2_bc(float& d0, float& d1, float a0, float a1, uint64_t b,
                                         uint64_t c) {
  asm("{\n\t.reg .b64 ra, rd;\n\tmov.b64 ra, {%2, %3};\n\t"
      "fma.rn.f32x2 rd, ra, %4, %5;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "l"(b), "l"(c));
}
__device__ __forceinline__ uint64_t pair_f32(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two floats to packed bf16x2 (lo in the low half), round-to-nearest-even, one instruction.
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// 2^x on the FMA pipe, for x <= 8 (and 0 below -125): x = n + f with n = round(x) by the
// 1.5 * 2^23 rounding constant, f in [-1/2, 1/2], 2^f by a cubic fitted here (least squares on
// Chebyshev nodes, reweighted toward equal-ripple relative error: 7.5e-5 at most, far below
// bf16's 2^-8), and n added to the exponent field.  One in four of a tile's exponentials takes
// this path so the MUFU unit, which the two query tiles' softmax warps share, is not the limit.
__device__ __forceinline__ float exp2_poly3(float x) {
  const float xc = fmaxf(x, -125.f);
  const float t = xc + 12582912.f;
  const float f = xc - (t - 12582912.f);
  float q = fmaf(0.0551716648f, f, 0.242611125f);
  q = fmaf(q, f, 0.693260968f);
  q = fmaf(q, f, 0.999928057f);
  const int n = __float_as_int(t) - 0x4B400000;
  const float r = __int_as_float(__float_as_int(q) + (n << 23));
  return x < -125.f ? 0.f : r;
}

// Shared-memory matrix descriptor (tcgen05 "version 1"), 128B swizzle.  Addresses and offsets
// are in bytes; the descriptor keeps them >> 4.
//   K-major tile (rows of 64 bf16 = 128 B, 8-row atoms of 1024 B stacked): LBO 16 B (unused),
//   SBO 1024 B.  MN-major tile (64 N-values per 128 B row, one row per K index): LBO = stride
//   between 64-wide N panels, SBO = stride between 8-row K groups (1024 B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3fffu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) |  // version 1
         (2ull << 61);                                                          // SWIZZLE_128B
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, M x N, A K-major, B K-major
// (b_mn_major = 0) or MN-major (1).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

struct PrefillParams {
  uint16_t* out;              // (B, T, Hq, D) bf16 contiguous
  const int* cache_seqlens;   // (B,) positions before the new tokens
  int B, T, Hq, Hkv, G, Tmax, window;
  int n_qgroups;              // ceil(T / (QT * 128)): query-tile groups (pairs, or single tiles) a row
  int n_items;                // n_qgroups * B * Hq work items: one (query-tile group, row, q head) each
  float scale_log2;           // softmax_scale * log2(e)
  int ring;                   // the slot is a ring of Tmax positions (key c at index c % Tmax)
};

template <int D, int QT>
struct PrefillConfig {
  static constexpr int kPanels = D / 64;
  static constexpr int kTileBytes = kPanels * kPfTile * 128;  // one Q / K / V tile
  // Q (the item's QT tiles) is double-buffered where shared memory allows it (D = 64): the next
  // item's queries land while this item's last MMAs still read the current ones
  static constexpr int kQBufs = D <= 64 ? 2 : 1;
  static constexpr int kQOff = 0;                                  // [kQBufs][QT tiles]
  static constexpr int kKOff = kQOff + kQBufs * QT * kTileBytes;   // K ring, 2 stages
  static constexpr int kVOff = kKOff + 2 * kTileBytes;             // V ring, 2 stages
  static constexpr int kBarOff = kVOff + 2 * kTileBytes;
  // the partial row maxima and sums the softmax warps of a row quarter exchange: two slots x QT
  // query tiles x 4 quarters x pf_split warps x 32 rows, fp32
  static constexpr int kXchOff = kBarOff + 256;
  static constexpr int kBytes = kXchOff + (pf_split<QT>() > 1 ? 2 * QT * 4 * pf_split<QT>() * 32 * 4 : 0);
  // TMEM bounds the CTAs an SM holds (QT = 2: all 512 columns; QT = 1: 256, two CTAs): the
  // shared memory keeps a third CTA off the SM (more than a third of its 228 KB for QT = 1,
  // more than half for QT = 2), so no CTA ever waits in tcgen05.alloc for another to finish
  static constexpr int kMinSmem = QT == 2 ? 118784 : 78848;
  static constexpr int kSmem = (kBytes + 1024 > kMinSmem ? kBytes + 1024 : kMinSmem);
  // TMEM columns.  QT = 2: S0, S1, then O0, O1; P is written over S.  QT = 1: S, then P (packed
  // bf16, 64 columns) apart from S, then O -- 256 columns for head size 64 -- so the next S can be
  // computed while the softmax still works on this one.
  static constexpr uint32_t kPCol = QT == 1 ? kPfTile : 0;
  static constexpr uint32_t kOCol = QT == 1 ? kPfTile + kPfTile / 2 : QT * kPfTile;
  static_assert(QT == 2 || D == 64, "one query tile an item: S, P and O in 256 TMEM columns");
};

// The first key tile a query tile needs and how many tiles (from k_first) it spans.
struct QTileRange {
  int qbase, j_begin, j_end;  // key tiles [j_begin, j_end) of the item's walk
};

// Work item i: query-tile group qp -- QT consecutive query tiles -- (longest groups first, so the
// short tail items fill the gaps at the end) of row b, q head h; rng[1] is empty for QT = 1.
struct PfItem {
  int b, h, hk, L, q0, k_first, nkv;
  bool in_range;
  QTileRange rng[2];
};

template <int QT>
__device__ __forceinline__ PfItem prefill_item(const PrefillParams& p, int i) {
  PfItem it;
  const int bh = p.B * p.Hq;
  const int qp = p.n_qgroups - 1 - i / bh;
  it.b = (i % bh) / p.Hq;
  it.h = (i % bh) % p.Hq;
  it.hk = it.h / p.G;
  it.L = p.cache_seqlens[it.b];
  it.q0 = qp * QT * kPfTile;
  const int pos_last = it.L + min(it.q0 + QT * kPfTile, p.T) - 1;
  it.in_range = it.L >= 0 && (p.ring || pos_last < p.Tmax);
  it.k_first = (p.window >= 0 ? max(0, it.L + it.q0 - p.window) : 0) / kPfTile * kPfTile;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qb = it.q0 + t * kPfTile;
    it.rng[t].qbase = qb;
    if (!it.in_range || qb >= p.T || t >= QT) {
      it.rng[t].j_begin = it.rng[t].j_end = 0;
    } else {
      const int first = (p.window >= 0 ? max(0, it.L + qb - p.window) : 0) / kPfTile * kPfTile;
      it.rng[t].j_begin = (first - it.k_first) / kPfTile;
      it.rng[t].j_end = (it.L + min(qb + kPfTile, p.T) - 1 - it.k_first) / kPfTile + 1;
    }
  }
  it.nkv = max(it.rng[0].j_end, it.rng[1].j_end);
  return it;
}

// The item CTA c takes in round r: items are sorted longest first and dealt in serpentine order
// (even rounds left to right, odd rounds right to left), so a CTA that drew a long item in one
// round draws a short one in the next; -1 past the last item.
__device__ __forceinline__ int prefill_round_item(const PrefillParams& p, int r) {
  const int i = r * static_cast<int>(gridDim.x) +
                ((r & 1) ? static_cast<int>(gridDim.x - 1 - blockIdx.x) : static_cast<int>(blockIdx.x));
  return i < p.n_items ? i : -1;
}

// Persistent: CTA c takes one item a round (prefill_round_item); TMEM, the barriers and the tensor maps are
// set up once per CTA, the K/V ring and every barrier phase run on across items, so the next
// item's loads and first MMAs overlap this item's epilogue.  Items with no key tile (nkv == 0)
// are skipped by every role alike.  Per item the MMA issuer commits q_empty (the Q buffer may be
// refilled) and o_done; every softmax thread waits for o_done, reads its O, and arrives on
// epi_done, which the issuer waits for before the next item's o_done -- so no softmax group, not
// even one with no query tile in an item (T <= 128), can find o_done two phases ahead.
// Registers: QT = 2, 168 a thread -- the 10 warps land three to a sub-partition on two of the
// four, whose 16,384 registers each cap a thread at 170 (a higher cap fails to launch); QT = 1,
// 96 -- two CTAs of 10 warps, five a sub-partition; a few bytes spill in both.
template <int D, int QT>
__global__ void __launch_bounds__(pf_threads<QT>(), 3 - QT)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  using Cfg = PrefillConfig<D, QT>;
  constexpr int QB = Cfg::kQBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* q_full = bars + 0;    // [2] per Q buffer
  uint64_t* q_empty = bars + 2;   // [2] per Q buffer
  uint64_t* k_full = bars + 4;    // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* kv_empty = bars + 8;  // [2]
  uint64_t* s_full = bars + 10;   // [2] per query tile
  uint64_t* p_full = bars + 12;   // [2] per query tile, 128 arrivals
  uint64_t* o_done = bars + 14;
  uint64_t* epi_done = bars + 15;  // 128 QT arrivals: every softmax thread, once per item
  uint64_t* drained = bars + 16;
  uint64_t* s_free = bars + 17;    // QT = 1: the softmax has read S (128 arrivals)
  uint64_t* pv_done = bars + 18;   // QT = 1: a P V product has completed (P and O free again)
  constexpr int SPL = pf_split<QT>();
  uint64_t* pair_bars = bars + 19; // [QT][4] when SPL > 1: the SPL softmax warps of a row quarter
  constexpr int kNumBars = 19 + (SPL > 1 ? 4 * QT : 0);
  static_assert((kNumBars + 2) * 8 <= 256, "the barriers, the TMEM slot and the abort flag in 256 bytes");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kNumBars + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bars + i, (i == 12 || i == 13 || i == 17) ? 128 * SPL
                          : i == 15                         ? 128 * QT * SPL
                          : i >= 19                         ? 32 * SPL
                                                            : 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, pf_tmem_cols<QT>());
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t base = smem_u32(smem);

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol = l2_policy_evict_first();
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    int g = 0;                  // K/V tiles issued (ring position)
    int k = 0;                  // items started
    int q_last[2] = {-1, -1};   // per Q buffer: the use (k / QB) of its last load
    bool ok = true;
    for (int r = 0; ok && r * static_cast<int>(gridDim.x) < p.n_items; ++r) {
      const int i = prefill_round_item(p, r);
      if (i < 0) continue;
      const PfItem it = prefill_item<QT>(p, i);
      if (!it.in_range) record_error(kErrPositionBeyondCache);
      if (it.nkv == 0) continue;
      const int qb = k % QB, qn = k / QB;
      if (qn > 0 && !mbar_wait_or_abort(&q_empty[qb], (qn - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&q_full[qb], QT * Cfg::kTileBytes);
#pragma unroll
      for (int t = 0; t < QT; ++t)
#pragma unroll
        for (int pn = 0; pn < Cfg::kPanels; ++pn)
          tma_load_4d(smem + Cfg::kQOff + (qb * QT + t) * Cfg::kTileBytes + pn * kPfTile * 128, &qmap,
                      &q_full[qb], pn * 64, it.h, it.q0 + t * kPfTile, it.b, pol);
      q_last[qb] = qn;
      for (int j = 0; j < it.nkv; ++j, ++g) {
        const int st = g & 1;
        if (g >= 2 && !mbar_wait_or_abort(&kv_empty[st], ((g >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const int k0 = it.k_first + j * kPfTile;
        const int slot0 = p.ring ? k0 % p.Tmax : k0;  // a ring slot: Tmax % 128 == 0
        mbar_arrive_expect_tx(&k_full[st], Cfg::kTileBytes);
#pragma unroll
        for (int pn = 0; pn < Cfg::kPanels; ++pn)
          tma_load_4d(smem + Cfg::kKOff + st * Cfg::kTileBytes + pn * kPfTile * 128, &kmap,
                      &k_full[st], pn * 64, it.hk, slot0, it.b, pol);
        mbar_arrive_expect_tx(&v_full[st], Cfg::kTileBytes);
#pragma unroll
        for (int pn = 0; pn < Cfg::kPanels; ++pn)
          tma_load_4d(smem + Cfg::kVOff + st * Cfg::kTileBytes + pn * kPfTile * 128, &vmap,
                      &v_full[st], pn * 64, it.hk, slot0, it.b, pol);
      }
      ++k;
    }
    // on an abort, wait (bounded) for the copies still in flight before the CTA can exit
    if (*abort_flag) {
      for (int gg = max(0, g - 2); gg < g; ++gg) {
        mbar_wait(&k_full[gg & 1], (gg >> 1) & 1);
        mbar_wait(&v_full[gg & 1], (gg >> 1) & 1);
      }
      for (int qb = 0; qb < QB; ++qb)
        if (q_last[qb] >= 0) mbar_wait(&q_full[qb], q_last[qb] & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, kPfTile, 0);
    constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 1);
    int g = 0;                   // K/V tiles consumed by earlier items
    int k = 0;                   // items done
    int pv_total[2] = {0, 0};    // PV MMAs issued per query tile (p_full phases)
    int s_all = 0;               // QT = 1: S MMAs issued (s_free phases)
    bool ok = true;
    for (int r = 0; ok && r * static_cast<int>(gridDim.x) < p.n_items; ++r) {
      const int i = prefill_round_item(p, r);
      if (i < 0) continue;
      const PfItem it = prefill_item<QT>(p, i);
      if (it.nkv == 0) continue;
      const int qb = k % QB;
      ok = mbar_wait_or_abort(&q_full[qb], (k / QB) & 1, abort_flag);
      int k_waited = -1, v_waited = -1;
      int pv_item[2] = {0, 0};
      // Q is free for the next load once this item's last S MMA has read it
      const int s_total = (it.rng[0].j_end - it.rng[0].j_begin) + (it.rng[1].j_end - it.rng[1].j_begin);
      int s_issued = 0;
      auto active = [&](int t, int j) { return j >= it.rng[t].j_begin && j < it.rng[t].j_end; };
      auto issue_s = [&](int t, int j) -> bool {
        const int gj = g + j;
        if (k_waited < j) {
          if (!mbar_wait_or_abort(&k_full[gj & 1], (gj >> 1) & 1, abort_flag)) return false;
          k_waited = j;
        }
        tc_fence_after();
        const uint32_t q_base = base + Cfg::kQOff + (qb * QT + t) * Cfg::kTileBytes;
        const uint32_t k_base = base + Cfg::kKOff + (gj & 1) * Cfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kPfTile * 128) + (kk & 3) * 32;
          umma_ss(tmem + t * kPfTile, smem_desc_sw128(q_base + off, 16, 1024),
                  smem_desc_sw128(k_base + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        if (++s_issued == s_total) umma_commit(&q_empty[qb]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        const int gj = g + j;
        if (!mbar_wait_or_abort(&p_full[t], pv_total[t] & 1, abort_flag)) return false;
        if (v_waited < j) {
          if (!mbar_wait_or_abort(&v_full[gj & 1], (gj >> 1) & 1, abort_flag)) return false;
          v_waited = j;
        }
        tc_fence_after();
        const uint32_t v_base = base + Cfg::kVOff + (gj & 1) * Cfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kPfTile / 16; ++kk)
          umma_ts(tmem + Cfg::kOCol + t * D, tmem + (QT == 1 ? Cfg::kPCol : t * kPfTile) + kk * 8,
                  smem_desc_sw128(v_base + kk * 16 * 128, kPfTile * 128, 1024), idesc_o,
                  (pv_item[t] > 0 || kk > 0) ? 1u : 0u);
        ++pv_item[t];
        ++pv_total[t];
        return true;
      };
      if constexpr (QT == 1) {
        // S_{j+1} goes in as soon as the softmax has read S_j (s_free: P has columns of its own),
        // so it runs while the softmax exponentiates; P_j V_j follows once P_j is written
        auto issue_s1 = [&](int j) -> bool {
          if (s_all > 0 && !mbar_wait_or_abort(s_free, (s_all - 1) & 1, abort_flag)) return false;
          ++s_all;
          return issue_s(0, j);
        };
        if (ok) ok = issue_s1(0);
        for (int j = 0; ok && j < it.nkv; ++j) {
          if (ok && j + 1 < it.nkv) ok = issue_s1(j + 1);
          if (ok) ok = issue_pv(0, j);
          if (ok) {
            umma_commit(pv_done);
            umma_commit(&kv_empty[(g + j) & 1]);
          }
        }
      } else {
        if (ok && active(0, 0)) ok = issue_s(0, 0);
        if (ok && active(1, 0)) ok = issue_s(1, 0);
        for (int j = 0; ok && j < it.nkv; ++j) {
          if (ok && active(0, j)) ok = issue_pv(0, j);
          if (ok && active(0, j + 1)) ok = issue_s(0, j + 1);
          if (ok && active(1, j)) ok = issue_pv(1, j);
          if (ok) umma_commit(&kv_empty[(g + j) & 1]);
          if (ok && active(1, j + 1)) ok = issue_s(1, j + 1);
        }
      }
      if (ok && k > 0) ok = mbar_wait_or_abort(epi_done, (k - 1) & 1, abort_flag);
      if (ok) umma_commit(o_done);
      g += it.nkv;
      ++k;
    }
    // every MMA this thread issued has completed before TMEM can be freed
    umma_commit(drained);
    mbar_wait(drained, 0);
  } else if (warp >= 2) {
    // ---------------- softmax: 4 SPL warps a query tile ----------------
    // Warp w reaches TMEM lanes 32 (w % 4) .. +31 (its row quarter); the SPL warps of one
    // quarter take consecutive slices of KC key columns of the tile (and DC columns of O) and
    // meet twice an item: the partial row maxima every tile, the partial row sums at the end.
    constexpr int KC = kPfTile / SPL;   // key columns a thread
    constexpr int DC = D / SPL;         // O columns a thread rescales and stores
    const int idx = warp - 2;
    const int t = idx / (4 * SPL);
    const int h = (idx >> 2) % SPL;     // slice of the row quarter
    const int quarter = warp & 3;            // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;     // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + t * kPfTile + h * KC;
    const uint32_t o_addr = tmem + lane_off + Cfg::kOCol + t * D + h * DC;
    // P (packed bf16, KC / 2 columns a slice): its own columns for QT = 1, over S for QT = 2
    const uint32_t p_addr = (QT == 1 ? tmem + lane_off + Cfg::kPCol : tmem + lane_off + t * kPfTile) + h * (KC / 2);
    uint64_t* pair_bar = pair_bars + t * 4 + quarter;
    float* xch = reinterpret_cast<float*>(smem + Cfg::kXchOff);
    int k = 0;       // items done
    int s_cnt = 0;   // S tiles of this query tile consumed (s_full phases)
    int pv_seen = 0; // QT = 1: P V products observed (pv_done phases), one per tile
    int ex = 0;      // exchanges with the other warps of the quarter (pair_bar phases)
    bool ok = true;
    // The other slices' value of this row, combined by `op` in slice order: written to slot
    // ex % 2, arrive, wait (bounded) for the quarter's phase.  A slot is rewritten two exchanges
    // later, after every warp of the quarter has arrived at the exchange between (so has read it).
    // The fences order this warp's TMEM loads before the other slices' P stores over S.
    auto exchange = [&](float v, auto op) -> float {
      if constexpr (SPL == 1) return v;
      float* slot = xch + (((ex & 1) * QT + t) * 4 + quarter) * (SPL * 32);
      slot[h * 32 + lane] = v;
      tc_fence_before();
      mbar_arrive(pair_bar);
      const bool w = __all_sync(0xffffffffu, mbar_wait_or_abort(pair_bar, ex & 1, abort_flag));
      tc_fence_after();
      ++ex;
      if (!w) {
        ok = false;
        return v;
      }
      float acc = slot[lane];
#pragma unroll
      for (int o = 1; o < SPL; ++o) acc = op(acc, slot[o * 32 + lane]);
      return acc;
    };
    for (int r = 0; ok && r * static_cast<int>(gridDim.x) < p.n_items; ++r) {
      const int i = prefill_round_item(p, r);
      if (i < 0) continue;
      const PfItem it = prefill_item<QT>(p, i);
      if (it.nkv == 0) continue;
      // scalars, not it.rng[t]: a runtime index would put the array in local memory
      const int qbase = t ? it.rng[1].qbase : it.rng[0].qbase;
      const int j_begin = t ? it.rng[1].j_begin : it.rng[0].j_begin;
      const int j_end = t ? it.rng[1].j_end : it.rng[0].j_end;
      const int L = it.L;
      const int q = qbase + row;
      const bool valid = q < p.T;
      const int pos = L + q;
      float m_used = -INFINITY, l = 0.f;
      int cnt = 0;
      for (int j = j_begin; j < j_end; ++j, ++cnt, ++s_cnt) {
        // waits are made warp-uniform: the tcgen05.ld/st below are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[t], s_cnt & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kt = it.k_first + j * kPfTile;  // the tile's first key
        const int k0 = kt + h * KC;               // this slice's first key
        uint32_t sr[KC];
        if constexpr (KC == 128) tmem_ld128(s_addr, sr);  // one round trip: the latency dominates
        else tmem_ld64(s_addr, sr);
        if constexpr (QT == 1) {  // S is read: the issuer may compute the next one into it
          tc_fence_before();
          mbar_arrive(s_free);
        }
        // raw scores; the scale is applied inside the exponent's FMA (scale > 0 keeps the max)
        const bool full = kt + kPfTile - 1 <= L + qbase &&
                          (p.window < 0 || L + qbase + kPfTile - 1 - kt <= p.window) &&
                          qbase + kPfTile <= p.T;
        if (!full) {
          // this query row sees the key columns [c_lo, c_hi) of the slice (key <= pos, and
          // pos - key <= window): one unsigned compare a column against the interval's width
          const int c_hi = valid ? min(KC, pos - k0 + 1) : 0;
          const int c_lo = p.window >= 0 ? max(0, pos - p.window - k0) : 0;
          const uint32_t width = c_hi > c_lo ? static_cast<uint32_t>(c_hi - c_lo) : 0u;
#pragma unroll
          for (int c = 0; c < KC; ++c)
            if (static_cast<uint32_t>(c - c_lo) >= width) sr[c] = __float_as_uint(-INFINITY);
        }
        // the slice's row maximum in four independent chains, then the other slices' (max is
        // exact: neither order changes the result)
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < KC / 8; ++c)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            m4[u] = fmax3(m4[u], __uint_as_float(sr[8 * c + 2 * u]), __uint_as_float(sr[8 * c + 2 * u + 1]));
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx = exchange(mx, [](float a, float b) { return fmaxf(a, b); });
        if (!ok) break;
        mx *= p.scale_log2;
        // lazy rescale: move the running max only when it grows by more than 2^8 (every slice of
        // the row takes the same decision: the same max, the same m_used)
        float alpha = 1.f;
        if (mx > m_used + 8.f) {
          alpha = fast_exp2(m_used - mx);  // 0 when m_used is -inf
          m_used = mx;
          l *= alpha;
        }
        if constexpr (QT == 1) {
          // the previous tile's P V has completed before P is rewritten and O rescaled
          if (cnt > 0) {
            if (!__all_sync(0xffffffffu, mbar_wait_or_abort(pv_done, pv_seen & 1, abort_flag))) {
              ok = false;
              break;
            }
            ++pv_seen;
            tc_fence_after();
          }
        }
        const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
        const uint64_t sc2 = pair_f32(p.scale_log2, p.scale_log2), nm2 = pair_f32(neg_m, neg_m);
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int c = 0; c < KC / 32; ++c) {  // 32 keys -> 16 columns of packed bf16 P
#pragma unroll
          for (int u = 0; u < 8; ++u) {  // 4 keys: three exponentials on MUFU, one on the FMA pipe
            const int kx = 32 * c + 4 * u;
            float x0, x1, x2, x3;
            ffma2_bc(x0, x1, __uint_as_float(sr[kx]), __uint_as_float(sr[kx + 1]), sc2, nm2);
            ffma2_bc(x2, x3, __uint_as_float(sr[kx + 2]), __uint_as_float(sr[kx + 3]), sc2, nm2);
            const float e0 = fast_exp2(x0), e1 = fast_exp2(x1), e2 = fast_exp2(x2);
            const float e3 = exp2_poly3(x3);
            sum0 += e0 + e2;
            sum1 += e1 + e3;
            // the packed P words reuse the registers of scores already consumed
            sr[32 * c + 2 * u] = pack_bf16x2_rn(e0, e1);
            sr[32 * c + 2 * u + 1] = pack_bf16x2_rn(e2, e3);
          }
          tmem_st16_nowait(p_addr + 16 * c, *reinterpret_cast<const uint32_t(*)[16]>(&sr[32 * c]));
        }
        const float sum = sum0 + sum1;
        l += sum;  // this slice's part of the row sum
        tmem_st_wait();
        if (cnt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < DC / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(o_addr + c * 32, o);
#pragma unroll
            for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * alpha);
            tmem_st32(o_addr + c * 32, o);
          }
        }
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      // epilogue: O / l -> bf16 -> out[b, q, h, :]; every item's o_done phase is observed (QT = 1:
      // and the pv_done phase of its last P V, so that one phase is observed per tile)
      if constexpr (QT == 1) {
        if (ok && cnt > 0) {
          if (!__all_sync(0xffffffffu, mbar_wait_or_abort(pv_done, pv_seen & 1, abort_flag))) ok = false;
          ++pv_seen;
        }
      }
      if (ok && !__all_sync(0xffffffffu, mbar_wait_or_abort(o_done, k & 1, abort_flag))) ok = false;
      if (ok && cnt > 0) {
        // the row sum: the slices' parts added in slice order
        const float lt = exchange(l, [](float a, float b) { return a + b; });
        tc_fence_after();
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        uint16_t* dst = p.out + ((static_cast<long long>(it.b) * p.T + q) * p.Hq + it.h) * D + h * DC;
#pragma unroll
        for (int c = 0; c < DC / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          if (valid && ok) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * u + 0]) * inv, __uint_as_float(o[8 * u + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + 8 * u) = w;
            }
          }
        }
      }
      // O is read: the issuer may let the next item's o_done phase complete
      tc_fence_before();
      mbar_arrive(epi_done);
      ++k;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, pf_tmem_cols<QT>());
  }
}

}  // namespace mcb
