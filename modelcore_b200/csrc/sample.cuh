// Sampling the next token from fp32 logits: sample_next_token, modelcore/generate.py:19-34.
//
//   top_k in [1, V):                 the k largest logits (torch.topk), divided by the
//                                    temperature, softmax, one multinomial draw
//   otherwise:                       softmax over the whole row (logits / temperature), one draw
//
// logits / T is evaluated as logits * fp32(1 / T), as torch's CUDA division by a Python number
// does; softmax weights are expf(x - max).  The draw is an inverse CDF on a caller-provided
// uniform u in [0, 1): the first candidate whose inclusive cumulative weight exceeds
// u * (total weight).  Candidates are ordered by descending
// logit with ties by ascending index (the top-k path; torch.topk leaves tie order unspecified)
// or by index (the full-row path), so a draw is a deterministic function of (logits, u) that the
// CPU oracle restates; over u it has the reference's distribution.
//
// One 1024-thread CTA per row.  Top-k: a 4-pass radix select (8 bits a pass, MSB first) over the
// order-preserving integer image of the logits finds the k-th largest value tau; the row's
// elements above tau and the first (k - count above) elements equal to tau (by index) are the
// candidates.  Up to kSampleMaxK of them are gathered, bitonic-sorted in shared memory, and
// scanned; more are drawn from without sorting (sample_large_k: a radix descent over integer
// weights).  Each thread owns a contiguous chunk
// of the row, so "first by index" is a prefix count over threads.
#pragma once

#include "common.cuh"

namespace mcb {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;

struct SampleParams {
  const float* logits;
  const float* uniforms;
  int64_t* out;
  long long ls, os;
  int rows, V, top_k;
  float inv_temperature;  // 1 / T rounded to fp32
};

// Order-preserving map float -> uint32 (larger float, larger key; -0 below +0 is harmless here).
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive prefix sum of one value per thread (1024 threads, 32 warps); also returns
// the block total.  `scratch` holds 33 floats / ints.
template <class T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* scratch, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = scratch[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    scratch[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const T before_warp = warp > 0 ? scratch[warp - 1] : T(0);
  *total = scratch[31];
  const T excl = before_warp + x - v;
  __syncthreads();
  return excl;
}

// Inverse of float_key.
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Candidate weights of the large-k draw as fixed-point integers: round(expf(x / T - x0) * 2^40),
// x0 the largest logit / T, so every weight is in [0, 2^40] and a row's total stays below 2^56.
// Integer sums do not depend on their order, so the draw is deterministic however the threads
// accumulate them.
constexpr float kSampleFix = 1099511627776.0f;  // 2^40

__device__ __forceinline__ unsigned long long sample_weight(float v, float inv_t, float x0) {
  return __float2ull_rn(__fmul_rn(expf(__fmul_rn(v, inv_t) - x0), kSampleFix));
}

// top_k > kSampleMaxK (up to V - 1): the candidates are the elements above tau plus the first
// `remaining` elements equal to tau (by index), as in the sorted path, but too many to sort in
// shared memory.  The inverse-CDF draw over them in descending-logit order (ties by index) is
// found without sorting: the target u * total is located by a 4-pass radix descent over the
// candidates' order-preserving keys, MSB first, each pass a 256-bucket histogram of candidate
// weights (walked from the largest bucket down, as the descending order walks them); the last
// pass leaves the drawn key and the target's remainder within the candidates holding that key,
// which share one weight, so the remainder divided by it is the rank of the drawn one among them
// by index.
__device__ __noinline__ void sample_large_k(const SampleParams& p, const float* lg, int row, int beg,
                                            int end, uint32_t tau, int remaining, float u,
                                            float* fscratch, int* iscratch, uint32_t* sel) {
  __shared__ unsigned long long whist[256];
  __shared__ unsigned long long wsum, wrem;
  const int tid = threadIdx.x, lane = tid & 31;
  const float inv_t = p.inv_temperature;
  // x0: the largest logit / T (the first candidate)
  float mx = -INFINITY;
  for (int i = beg; i < end; ++i) mx = fmaxf(mx, lg[i]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) fscratch[tid >> 5] = mx;
  __syncthreads();
  mx = fscratch[0];
  for (int w = 1; w < 32; ++w) mx = fmaxf(mx, fscratch[w]);
  const float x0 = __fmul_rn(mx, inv_t);
  // rank of this thread's first tie with tau among all ties (by index)
  int n_eq = 0;
  for (int i = beg; i < end; ++i) n_eq += float_key(lg[i]) == tau;
  int tot_eq;
  const int off_eq = block_exclusive_scan(n_eq, iscratch, &tot_eq);
  // total candidate weight
  unsigned long long t = 0;
  {
    int e = off_eq;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      const bool cand = k > tau || (k == tau && e < remaining);
      e += k == tau;
      if (cand) t += sample_weight(lg[i], inv_t, x0);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (tid == 0) wsum = 0;
  __syncthreads();
  if (lane == 0) atomicAdd(&wsum, t);
  __syncthreads();
  const unsigned long long total = wsum;
  unsigned long long rem = static_cast<unsigned long long>(static_cast<double>(u) * static_cast<double>(total));
  if (rem >= total) rem = total - 1;
  // radix descent to the drawn key
  uint32_t pre = 0, msk = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (tid < 256) whist[tid] = 0;
    __syncthreads();
    int e = off_eq;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      const bool cand = k > tau || (k == tau && e < remaining);
      e += k == tau;
      if (cand && (k & msk) == pre) atomicAdd(&whist[(k >> shift) & 0xffu], sample_weight(lg[i], inv_t, x0));
    }
    __syncthreads();
    if (tid == 0) {
      unsigned long long acc = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + whist[b] > rem) break;
        acc += whist[b];
      }
      sel[0] = pre | (static_cast<uint32_t>(b) << shift);
      sel[1] = msk | (0xffu << shift);
      wrem = rem - acc;
    }
    __syncthreads();
    pre = sel[0];
    msk = sel[1];
    rem = wrem;
    __syncthreads();
  }
  // the drawn key; its candidates share one weight: the rank among them (by index) follows
  const uint32_t kappa = pre;
  const unsigned long long wk = sample_weight(key_float(kappa), inv_t, x0);
  long long j = wk > 0 ? static_cast<long long>(rem / wk) : 0;
  int n_k = 0;
  {
    int e = off_eq;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      const bool cand = k > tau || (k == tau && e < remaining);
      e += k == tau;
      n_k += cand && k == kappa;
    }
  }
  int tot_k;
  const int off_k = block_exclusive_scan(n_k, iscratch, &tot_k);
  if (j >= tot_k) j = tot_k - 1;
  if (off_k <= j && j < off_k + n_k) {
    int c = off_k, e = off_eq;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      const bool cand = k > tau || (k == tau && e < remaining);
      e += k == tau;
      if (cand && k == kappa) {
        if (c == j) {
          p.out[static_cast<long long>(row) * p.os] = i;
          break;
        }
        ++c;
      }
    }
  }
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleParams p) {
  pdl_wait();  // logits come from the kernel ahead (programmatic dependent launch)
  pdl_launch_dependents();
  __shared__ uint32_t hist[256];
  __shared__ float cand_v[kSampleMaxK];
  __shared__ int cand_i[kSampleMaxK];
  __shared__ float fscratch[33];
  __shared__ int iscratch[33];
  __shared__ uint32_t sel[4];  // prefix, prefix mask, remaining k, chosen index
  const int row = blockIdx.x;
  const float* lg = p.logits + static_cast<long long>(row) * p.ls;
  const int V = p.V;
  const int tid = threadIdx.x;
  const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int beg = min(V, tid * chunk), end = min(V, beg + chunk);
  const float inv_t = p.inv_temperature;  // torch divides by a Python number as x * (1 / T)
  const float u = p.uniforms[row];
  const bool topk = p.top_k >= 1 && p.top_k < V;

  if (!topk) {
    // ---- the whole row: softmax(logits / T) in index order ----
    float mx = -INFINITY;
    for (int i = beg; i < end; ++i) mx = fmaxf(mx, __fmul_rn(lg[i], inv_t));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) fscratch[tid >> 5] = mx;
    __syncthreads();
    mx = fscratch[0];
    for (int w = 1; w < 32; ++w) mx = fmaxf(mx, fscratch[w]);
    __syncthreads();
    float s = 0.f;
    for (int i = beg; i < end; ++i) s += expf(__fmul_rn(lg[i], inv_t) - mx);
    float total;
    const float before = block_exclusive_scan(s, fscratch, &total);
    const float target = u * total;
    if (tid == 0) sel[3] = 0xffffffffu;
    __syncthreads();
    if (before <= target && target < before + s) {
      float c = before;
      int pick = end - 1;
      for (int i = beg; i < end; ++i) {
        c += expf(__fmul_rn(lg[i], inv_t) - mx);
        if (c > target) { pick = i; break; }
      }
      atomicMin(&sel[3], static_cast<uint32_t>(pick));
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t pick = sel[3];
      if (pick == 0xffffffffu) {  // rounding put the target at the very end: last nonzero weight
        pick = V - 1;
        while (pick > 0 && !(expf(__fmul_rn(lg[pick], inv_t) - mx) > 0.f)) --pick;
      }
      p.out[static_cast<long long>(row) * p.os] = pick;
    }
    return;
  }

  // ---- top-k: radix select of the k-th largest key ----
  uint32_t prefix = 0, mask = 0;
  int remaining = p.top_k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0, b = 255;
      for (; b > 0; --b) {
        if (acc + static_cast<int>(hist[b]) >= remaining) break;
        acc += hist[b];
      }
      sel[0] = prefix | (static_cast<uint32_t>(b) << shift);
      sel[1] = mask | (0xffu << shift);
      sel[2] = static_cast<uint32_t>(remaining - acc);
    }
    __syncthreads();
    prefix = sel[0];
    mask = sel[1];
    remaining = static_cast<int>(sel[2]);
    __syncthreads();
  }
  // tau = prefix (all 32 bits); `remaining` elements equal to tau complete the k
  const uint32_t tau = prefix;
  if (p.top_k > kSampleMaxK) {
    sample_large_k(p, lg, row, beg, end, tau, remaining, u, fscratch, iscratch, sel);
    return;
  }
  int n_gt = 0, n_eq = 0;
  for (int i = beg; i < end; ++i) {
    const uint32_t k = float_key(lg[i]);
    n_gt += k > tau;
    n_eq += k == tau;
  }
  int tot_gt, tot_eq;
  const int off_gt = block_exclusive_scan(n_gt, iscratch, &tot_gt);
  const int off_eq = block_exclusive_scan(n_eq, iscratch, &tot_eq);
  {
    int g = off_gt, e = off_eq;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = float_key(lg[i]);
      if (k > tau) {
        cand_v[g] = lg[i];
        cand_i[g] = i;
        ++g;
      } else if (k == tau) {
        if (e < remaining) {
          cand_v[tot_gt + e] = lg[i];
          cand_i[tot_gt + e] = i;
        }
        ++e;
      }
    }
  }
  const int K = p.top_k;  // == tot_gt + remaining
  for (int i = K + tid; i < kSampleMaxK; i += kSampleThreads) {
    cand_v[i] = -INFINITY;
    cand_i[i] = 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort, descending value, ascending index on ties
  for (int size = 2; size <= kSampleMaxK; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = tid, j = i ^ stride;
      if (j > i) {
        const bool desc = (i & size) == 0;
        const float vi = cand_v[i], vj = cand_v[j];
        const int ii = cand_i[i], ij = cand_i[j];
        const bool i_first = vi > vj || (vi == vj && ii < ij);
        if (desc != i_first) {
          cand_v[i] = vj; cand_v[j] = vi;
          cand_i[i] = ij; cand_i[j] = ii;
        }
      }
      __syncthreads();
    }
  }
  // softmax over vals / T and the inverse-CDF draw
  const float x0 = __fmul_rn(cand_v[0], inv_t);
  const float w = tid < K ? expf(__fmul_rn(cand_v[tid], inv_t) - x0) : 0.f;
  float total;
  const float before = block_exclusive_scan(w, fscratch, &total);
  const float target = u * total;
  if (tid == 0) sel[3] = static_cast<uint32_t>(K - 1);
  __syncthreads();
  if (tid < K && before + w > target) atomicMin(&sel[3], static_cast<uint32_t>(tid));
  __syncthreads();
  if (tid == 0) p.out[static_cast<long long>(row) * p.os] = cand_i[sel[3]];
}

}  // namespace mcb
