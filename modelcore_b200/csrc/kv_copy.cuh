// Piece 2: prefill -> broadcast cache copy (KVCache.prefill, modelcore/cache.py:75-90) and the
// one-row copy (KVCache.prefill_row, modelcore/cache.py:92-119).
//
// For every slot the source block positions [0, n_pos) of one row is contiguous
// (n_pos * Hkv * D bf16), and so is each destination row's block.  Each thread loads one 16-byte
// vector of the source once (non-allocating in L1) and streams it to every destination row, so
// HBM sees the source read once and the destinations written once: the copy roofline.
#pragma once

#include "common.cuh"

namespace mcb {

struct CopyParams {
  uint16_t* dst_k;
  uint16_t* dst_v;
  const uint16_t* src_k;
  const uint16_t* src_v;
  int n_slots;
  long long src_slot_stride;   // elements between slots in the source
  long long src_row_offset;    // elements from a slot's start to the source row
  long long dst_slot_stride;   // elements between slots in the destination
  long long dst_row_stride;    // elements between destination rows (dst_tmax * row_elems)
  long long dst_row_begin_offset;
  int dst_row_count;
  long long vecs_per_slot;     // 16-byte vectors per (slot, row) block
  int32_t* dst_seqlens;
  int dst_seqlen_begin;
  int seqlen_value;
};

__device__ __forceinline__ uint4 ld_nc_v4(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_cs_v4(uint4* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// grid.y selects K (0) or V (1); grid.x strides over (slot, vector).
__global__ void __launch_bounds__(256) kv_copy_rows_kernel(const CopyParams p) {
  const bool is_v = blockIdx.y == 1;
  const uint16_t* src = is_v ? p.src_v : p.src_k;
  uint16_t* dst = is_v ? p.dst_v : p.dst_k;
  const long long total = p.vecs_per_slot * p.n_slots;
  if (p.dst_seqlens != nullptr && blockIdx.x == 0 && blockIdx.y == 0) {
    for (int r = threadIdx.x; r < p.dst_row_count; r += blockDim.x)
      p.dst_seqlens[p.dst_seqlen_begin + r] = p.seqlen_value;
  }
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long slot = i / p.vecs_per_slot;
    const long long v = i - slot * p.vecs_per_slot;
    const uint4* s =
        reinterpret_cast<const uint4*>(src + slot * p.src_slot_stride + p.src_row_offset) + v;
    const uint4 val = ld_nc_v4(s);
    uint16_t* dslot = dst + slot * p.dst_slot_stride + p.dst_row_begin_offset;
    for (int r = 0; r < p.dst_row_count; ++r)
      st_cs_v4(reinterpret_cast<uint4*>(dslot + r * p.dst_row_stride) + v, val);
  }
}

// No trigger: the kernel after an advance may read cache_seqlens before its own wait (decode
// attention does), so it must not start until the advance has completed.
__global__ void kv_advance_kernel(int32_t* seqlens, int B, int n) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < B) seqlens[i] += n;
}

}  // namespace mcb
