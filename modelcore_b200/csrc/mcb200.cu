// C-ABI entry points of libmcb200 (declared in include/mcb200.h): host-side validation, launch
// planning, TMA descriptor encoding and the kernel launches for the KV-cache decode path.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <type_traits>

#include "../../include/mcb200.h"
#include "common.cuh"
#include "decode_attn.cuh"
#include "decode_attn_split.cuh"
#include "kv_append.cuh"
#include "kv_copy.cuh"
#include "prefill_attn.cuh"
#include "decode_proj.cuh"
#include "sample.cuh"
#include "step_fused.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
// The attention kernel (template instance) this thread enqueued last: mcb_last_attn_kernel.
thread_local char g_last_attn_kernel[96] = "";

void note_attn_kernel(const char* name, int D, int nqt, int stages, bool fp8) {
  if (nqt > 0)
    snprintf(g_last_attn_kernel, sizeof(g_last_attn_kernel), "mcb::%s<%d,%d,16,%d%s>", name, D, nqt,
             stages, fp8 ? ",true" : "");
  else if (stages > 0)  // the prefill kernel: stages carries its query tiles an item
    snprintf(g_last_attn_kernel, sizeof(g_last_attn_kernel), "mcb::%s<%d,%d>", name, D, stages);
  else
    snprintf(g_last_attn_kernel, sizeof(g_last_attn_kernel), "mcb::%s<%d>", name, D);
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MCB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static std::mutex mu;
  static int cache[64] = {0};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Sets the dynamic shared-memory limit of a kernel once per device.
template <typename K>
cudaError_t ensure_smem(K kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

// Whether clusters of n CTAs of `kernel` (shared-memory limit already raised) can be resident on
// the current device; a size above the portable 8 is allowed on the kernel first.
template <typename K>
bool cluster_fits(K kernel, int smem, int n) {
  if (n > 8 && cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n));
  cfg.blockDim = dim3(mcb::kAttnThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(n);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return clusters > 0;
}

// The combine kernel after a split launch whose partials no CTA merged (counters == null).
template <int D>
int launch_combine(const mcb::SplitAttnParams& prm, cudaStream_t st) {
  if (prm.nsplit <= 1 || prm.cluster || prm.counters != nullptr) return MCB_OK;
  const long long rows = static_cast<long long>(prm.B) * prm.T * prm.Hq;
  mcb::decode_attn_split_combine_kernel<D><<<static_cast<unsigned>((rows + 3) / 4), 128, 0, st>>>(prm);
  g_launches++;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode_attn_split_combine launch");
  return MCB_OK;
}

// Caches a per-device answer (0 = not yet known); `compute` runs once per device.
template <typename F>
int per_device(int (&cache)[64], std::mutex& mu, F compute) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) cache[dev] = compute();
  return cache[dev];
}

// Launches `kernel` with programmatic stream serialization: it may start while the kernel ahead
// in the stream finishes (every kernel of this library calls pdl_wait() before reading anything
// another kernel wrote).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ------------------------------------------------------------------------------------------
// Decode attention planning.  Two kernels share the semantics: the persistent one
// (decode_attn.cuh: a balanced partition of every row's key tiles over a resident grid) and the
// split one (decode_attn_split.cuh: one CTA per row group and key split).  With num_ctas == 0 the
// host picks by how many key tiles a row can hold: up to kSplitMaxTiles the split kernel (short
// rows: the persistent kernel's start-up scan and cross-CTA merges are not amortised), beyond it
// the persistent one.  num_ctas > 0 forces a persistent grid of that size, num_ctas < 0 forces
// the split kernel with -num_ctas key splits per row group.
constexpr int kKPW = 16;             // keys per consumer warp per tile (tile = 64 keys)
constexpr long long kSplitMaxTiles = 33;  // 2048 keys + one tile of alignment slack

enum AttnMode { kModePersistent = 0, kModeSplit = 1, kModePrefill = 2 };

// CTAs per SM of the grid-stride append kernel (256 threads of at most 64 registers each).
constexpr int kAppendVecCtasPerSm = 4;

// With num_ctas == 0, T_new >= kPrefillMinT and head_dim 64 or 128, the tensor-core prefill
// kernel (prefill_attn.cuh) runs instead: 128-query tiles on tcgen05, no workspace.
constexpr int kPrefillMinT = 64;

template <int D, int QT>
struct PrefillVariant {
  using Cfg = mcb::PrefillConfig<D, QT>;
  static constexpr auto kernel = mcb::prefill_attn_kernel<D, QT>;
  static int launch(long long grid, const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                    const mcb::PrefillParams& prm, cudaStream_t st) {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = ensure_smem(kernel, Cfg::kSmem, done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_attn)");
    kernel<<<static_cast<unsigned>(grid), mcb::pf_threads<QT>(), Cfg::kSmem, st>>>(qm, km, vm, prm);
    g_launches++;
    note_attn_kernel("prefill_attn_kernel", D, 0, QT, false);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "prefill_attn launch");
    return MCB_OK;
  }
};

template <int D, int NQT>
struct AttnVariant {
  // Ring depth per head_dim (persistent): 144-256 KB of tiles in flight per SM at this occupancy.
  static constexpr int STAGES = D <= 32 ? 8 : (D == 64 ? 3 : (D == 128 ? 4 : 2));
  using Cfg = mcb::AttnConfig<D, NQT, kKPW, STAGES>;
  static constexpr auto kernel = mcb::decode_attn_kernel<D, NQT, kKPW, STAGES>;
  // Split kernel: 3-4 stages, 2-3 CTAs per SM; and a 2-stage copy with about twice the CTAs
  // per SM, used when it makes the whole grid resident at once while the deep one would need a
  // second, partly empty wave (config 2: 768 CTAs, 3 vs 6 per SM -> 0.85 vs 0.91 of the copy
  // bandwidth at 819 keys a row).
  static constexpr int SPLIT_STAGES = D >= 128 ? 3 : 4;
  using SplitCfg = mcb::SplitAttnConfig<D, NQT, kKPW, SPLIT_STAGES>;
  static constexpr auto split_kernel = mcb::decode_attn_split_kernel<D, NQT, kKPW, SPLIT_STAGES>;
  using SplitCfgLo = mcb::SplitAttnConfig<D, NQT, kKPW, 2>;
  static constexpr auto split_kernel_lo = mcb::decode_attn_split_kernel<D, NQT, kKPW, 2>;

  // Resident split CTAs on the whole device for the deep (lo = false) or 2-stage kernel; also
  // raises the kernel's shared-memory limit.  Cached per device.
  static int split_slots(bool lo, long long* out) {
    static std::atomic<uint64_t> done_hi{0}, done_lo{0};
    static std::mutex mu;
    static long long cache[2][64] = {{0}};
    cudaError_t e = lo ? ensure_smem(split_kernel_lo, SplitCfgLo::SMEM_BYTES, done_lo)
                       : ensure_smem(split_kernel, SplitCfg::SMEM_BYTES, done_hi);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_attn_split)");
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[lo][dev] > 0) {
      *out = cache[lo][dev];
      return MCB_OK;
    }
    int n = 0;
    e = lo ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, split_kernel_lo, mcb::kAttnThreads,
                                                           SplitCfgLo::SMEM_BYTES)
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, split_kernel, mcb::kAttnThreads,
                                                           SplitCfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    const long long slots = static_cast<long long>(n) * device_sm_count();
    if (dev >= 0 && dev < 64) cache[lo][dev] = slots;
    *out = slots;
    return MCB_OK;
  }

  // The most splits merged inside one cluster: kMaxClusterSplits where the device schedules
  // clusters of that size of both split kernels, else the portable 8 (also without a device).
  static int max_cluster() {
    static std::mutex mu;
    static int cache[64] = {0};
    const int n = per_device(cache, mu, [] {
      long long s = 0;
      const bool ok = split_slots(false, &s) == MCB_OK && split_slots(true, &s) == MCB_OK &&
                      cluster_fits(split_kernel, SplitCfg::SMEM_BYTES, mcb::kMaxClusterSplits) &&
                      cluster_fits(split_kernel_lo, SplitCfgLo::SMEM_BYTES, mcb::kMaxClusterSplits);
      return ok ? mcb::kMaxClusterSplits : 8;
    });
    return n > 0 ? n : 8;
  }

  // Raises the persistent kernel's shared-memory limit on the current device (once) and returns
  // how many of its CTAs stay resident per SM.
  static int ctas_per_sm(int* out) {
    static std::atomic<uint64_t> done{0};
    static std::mutex mu;
    static int cache[64] = {0};
    cudaError_t e = ensure_smem(kernel, Cfg::SMEM_BYTES, done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_attn)");
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[dev] > 0) {
      *out = cache[dev];
      return MCB_OK;
    }
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, mcb::kAttnThreads, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (n <= 0) return fail(MCB_ERR_UNSUPPORTED, "decode_attn<%d,%d> cannot be resident on an SM", D, NQT);
    if (dev >= 0 && dev < 64) cache[dev] = n;
    *out = n;
    return MCB_OK;
  }

  static int launch(int grid, const CUtensorMap& km, const CUtensorMap& vm, const mcb::AttnParams& prm,
                    cudaStream_t st) {
    int dummy = 0;
    int rc = ctas_per_sm(&dummy);  // also sets the shared-memory limit
    if (rc != MCB_OK) return rc;
    kernel<<<grid, mcb::kAttnThreads, Cfg::SMEM_BYTES, st>>>(km, vm, prm);
    g_launches++;
    note_attn_kernel("decode_attn_kernel", D, NQT, STAGES, false);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn launch");
    return MCB_OK;
  }

  static int launch_split(long long grid, const CUtensorMap& km, const CUtensorMap& vm,
                          const mcb::SplitAttnParams& prm, cudaStream_t st) {
    long long hi_slots = 0, lo_slots = 0;
    int rc = split_slots(false, &hi_slots);
    if (rc != MCB_OK) return rc;
    rc = split_slots(true, &lo_slots);
    if (rc != MCB_OK) return rc;
    const bool lo = grid > hi_slots && grid <= lo_slots;
    cudaError_t e;
    // programmatic stream serialization: the K/V tiles of earlier steps stream in while the
    // append kernel ahead finishes (the kernel waits for it before q and the new keys)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(mcb::kAttnThreads);
    cfg.dynamicSmemBytes = lo ? SplitCfgLo::SMEM_BYTES : SplitCfg::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
    if (prm.cluster) {
      attrs[1].id = cudaLaunchAttributeClusterDimension;
      attrs[1].val.clusterDim.x = static_cast<unsigned>(prm.nsplit);
      attrs[1].val.clusterDim.y = 1;
      attrs[1].val.clusterDim.z = 1;
      cfg.numAttrs = 2;
    }
    cfg.attrs = attrs;
    e = lo ? cudaLaunchKernelEx(&cfg, split_kernel_lo, km, vm, prm)
           : cudaLaunchKernelEx(&cfg, split_kernel, km, vm, prm);
    g_launches++;
    note_attn_kernel("decode_attn_split_kernel", D, NQT, lo ? 2 : SPLIT_STAGES, false);
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn_split launch");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn_split launch");
    return launch_combine<D>(prm, st);
  }
};

#define MCB_DISPATCH_D(D_, NQT_, CALL)                                   \
  switch (D_) {                                                          \
    case 16: return (NQT_) == 1 ? AttnVariant<16, 1>::CALL : AttnVariant<16, 2>::CALL;   \
    case 32: return (NQT_) == 1 ? AttnVariant<32, 1>::CALL : AttnVariant<32, 2>::CALL;   \
    case 64: return (NQT_) == 1 ? AttnVariant<64, 1>::CALL : AttnVariant<64, 2>::CALL;   \
    case 128: return (NQT_) == 1 ? AttnVariant<128, 1>::CALL : AttnVariant<128, 2>::CALL; \
    case 256: return AttnVariant<256, 1>::CALL;                          \
  }                                                                      \
  return fail(MCB_ERR_UNSUPPORTED, "head_dim %d", D_);

int variant_ctas_per_sm(int D, int nqt, int* out) { MCB_DISPATCH_D(D, nqt, ctas_per_sm(out)) }

int variant_launch(int D, int nqt, int grid, const CUtensorMap& km, const CUtensorMap& vm,
                   const mcb::AttnParams& p, cudaStream_t st) {
  MCB_DISPATCH_D(D, nqt, launch(grid, km, vm, p, st))
}

int variant_launch_split(int D, int nqt, long long grid, const CUtensorMap& km, const CUtensorMap& vm,
                         const mcb::SplitAttnParams& p, cudaStream_t st) {
  MCB_DISPATCH_D(D, nqt, launch_split(grid, km, vm, p, st))
}

// The split kernel over an fp8 (e4m3) cache: half the bytes per tile, so a 4-stage ring holds as
// many keys in flight as 2 bf16 stages (2 CTAs per SM); a 3-stage copy fits 3 per SM.
template <int D, int NQT>
struct SplitF8Variant {
  using Cfg = mcb::SplitAttnConfig<D, NQT, kKPW, 4, true>;
  static constexpr auto kernel = mcb::decode_attn_split_kernel<D, NQT, kKPW, 4, true>;
  using CfgLo = mcb::SplitAttnConfig<D, NQT, kKPW, 3, true>;
  static constexpr auto kernel_lo = mcb::decode_attn_split_kernel<D, NQT, kKPW, 3, true>;

  static int slots(bool lo, long long* out) {
    static std::atomic<uint64_t> done_hi{0}, done_lo{0};
    cudaError_t e = lo ? ensure_smem(kernel_lo, CfgLo::SMEM_BYTES, done_lo)
                       : ensure_smem(kernel, Cfg::SMEM_BYTES, done_hi);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_attn_split fp8)");
    int n = 0;
    e = lo ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel_lo, mcb::kAttnThreads, CfgLo::SMEM_BYTES)
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, mcb::kAttnThreads, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    *out = static_cast<long long>(n) * device_sm_count();
    return MCB_OK;
  }

  static int max_cluster() {
    static std::mutex mu;
    static int cache[64] = {0};
    const int n = per_device(cache, mu, [] {
      long long s = 0;
      const bool ok = slots(false, &s) == MCB_OK && slots(true, &s) == MCB_OK &&
                      cluster_fits(kernel, Cfg::SMEM_BYTES, mcb::kMaxClusterSplits) &&
                      cluster_fits(kernel_lo, CfgLo::SMEM_BYTES, mcb::kMaxClusterSplits);
      return ok ? mcb::kMaxClusterSplits : 8;
    });
    return n > 0 ? n : 8;
  }

  static int launch(long long grid, const CUtensorMap& km, const CUtensorMap& vm, const mcb::SplitAttnParams& prm,
                    cudaStream_t st) {
    long long hi_slots = 0, lo_slots = 0;
    int rc = slots(false, &hi_slots);
    if (rc != MCB_OK) return rc;
    rc = slots(true, &lo_slots);
    if (rc != MCB_OK) return rc;
    // the 3-stage copy (3 CTAs per SM against 2): when it makes the grid resident at once, and on
    // grids of many waves, whose consumer-bound CTAs gain from more warps per SM (config 5 at
    // batch 64 / 256, full rows: 467 -> 430 us, 1,848 -> 1,724 us; batch 8, about 7 CTAs per SM,
    // runs faster with the deeper ring: 78 vs 87 us)
    const bool lo = grid > hi_slots && (grid <= lo_slots || grid >= 8ll * device_sm_count());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(mcb::kAttnThreads);
    cfg.dynamicSmemBytes = lo ? CfgLo::SMEM_BYTES : Cfg::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
    if (prm.cluster) {
      attrs[1].id = cudaLaunchAttributeClusterDimension;
      attrs[1].val.clusterDim.x = static_cast<unsigned>(prm.nsplit);
      attrs[1].val.clusterDim.y = 1;
      attrs[1].val.clusterDim.z = 1;
      cfg.numAttrs = 2;
    }
    cfg.attrs = attrs;
    cudaError_t e = lo ? cudaLaunchKernelEx(&cfg, kernel_lo, km, vm, prm) : cudaLaunchKernelEx(&cfg, kernel, km, vm, prm);
    g_launches++;
    note_attn_kernel("decode_attn_split_kernel", D, NQT, lo ? 3 : 4, true);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn_split (fp8) launch");
    return launch_combine<D>(prm, st);
  }
};

int variant_launch_split_f8(int D, int nqt, long long grid, const CUtensorMap& km, const CUtensorMap& vm,
                            const mcb::SplitAttnParams& p, cudaStream_t st) {
  if (D == 64) return nqt == 1 ? SplitF8Variant<64, 1>::launch(grid, km, vm, p, st)
                               : SplitF8Variant<64, 2>::launch(grid, km, vm, p, st);
  if (D == 128) return nqt == 1 ? SplitF8Variant<128, 1>::launch(grid, km, vm, p, st)
                                : SplitF8Variant<128, 2>::launch(grid, km, vm, p, st);
  return fail(MCB_ERR_UNSUPPORTED, "fp8 cache: head_dim %d (64 or 128)", D);
}

// The most key splits of one row group merged inside a cluster for this kernel family.
int variant_max_cluster(int D, int nqt, bool fp8) {
  if (fp8) {
    if (D == 64) return nqt == 1 ? SplitF8Variant<64, 1>::max_cluster() : SplitF8Variant<64, 2>::max_cluster();
    return nqt == 1 ? SplitF8Variant<128, 1>::max_cluster() : SplitF8Variant<128, 2>::max_cluster();
  }
  MCB_DISPATCH_D(D, nqt, max_cluster())
}

struct AttnPlan {
  int D, nqt, rows, tk, nqb, mode;
  bool cluster = false;  // split plan merged inside a cluster
  int grid;         // persistent CTAs (persistent mode)
  int nsplit, tps;  // key splits per row group and tiles per split (split mode)
  bool small_grid = false;  // split mode: at most about four CTAs per SM
  size_t part_o_bytes, part_lse_bytes, ws_bytes, counter_count;
};

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Validates the shape and plans the launch.  Without a usable device (a CPU-only process asking
// for the workspace size) an automatic persistent grid assumes one CTA per SM of a B200.
int plan_attn(const mcb_attn_args* a, AttnPlan* pl) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_decode_attn: args is NULL");
  if (a->B < 0 || a->T < 0 || a->Hq <= 0 || a->Hkv <= 0 || a->D <= 0 || a->Tmax <= 0)
    return fail(MCB_ERR_INVALID_ARG,
                "mcb_decode_attn: bad sizes B=%d T=%d Hq=%d Hkv=%d D=%d Tmax=%d", a->B, a->T,
                a->Hq, a->Hkv, a->D, a->Tmax);
  if (a->Hq % a->Hkv != 0)
    return fail(MCB_ERR_INVALID_ARG, "mcb_decode_attn: n_head (%d) must be divisible by n_kv_head (%d)",
                a->Hq, a->Hkv);
  if (a->D != 16 && a->D != 32 && a->D != 64 && a->D != 128 && a->D != 256)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: head_dim %d not supported (16/32/64/128/256)",
                a->D);
  if (a->ring && (a->window < 0 || static_cast<long long>(a->window) + a->T > a->Tmax ||
                  a->Tmax % 128 != 0))
    return fail(MCB_ERR_INVALID_ARG,
                "mcb_decode_attn: a ring slot needs window >= 0, window + T <= Tmax and Tmax a "
                "multiple of 128 (window=%d T=%d Tmax=%d)", a->window, a->T, a->Tmax);
  const bool fp8 = a->k_scale != nullptr;
  if (fp8 && (a->v_scale == nullptr || (a->D != 64 && a->D != 128) || a->num_ctas > 0 ||
              a->scale_tmax < a->Tmax || a->scale_tmax % 64 != 0))
    return fail(MCB_ERR_UNSUPPORTED,
                "mcb_decode_attn: an fp8 cache needs k_scale and v_scale, D = 64 or 128, the split "
                "plan (num_ctas <= 0), and scale_tmax >= Tmax, a multiple of 64");
  const int G = a->Hq / a->Hkv;
  pl->D = a->D;
  if (!fp8 && a->num_ctas == 0 && a->T >= kPrefillMinT && (a->D == 64 || a->D == 128)) {
    pl->mode = kModePrefill;
    pl->nqt = pl->rows = pl->nqb = 0;
    pl->tk = mcb::kPfTile;
    pl->grid = pl->nsplit = pl->tps = 0;
    pl->part_o_bytes = pl->part_lse_bytes = pl->ws_bytes = pl->counter_count = 0;
    const long long qtiles = (a->T + mcb::kPfTile - 1) / mcb::kPfTile;
    if (qtiles * a->B * a->Hq > 0x7fffffffll)
      return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: prefill grid too large");
    return MCB_OK;
  }
  const long long rows_total = static_cast<long long>(a->T) * G;
  pl->nqt = (rows_total <= 8 || a->D == 256) ? 1 : 2;
  pl->rows = 8 * pl->nqt;
  pl->tk = kKPW * mcb::kAttnConsumerWarps;
  pl->nqb = rows_total > 0 ? static_cast<int>((rows_total + pl->rows - 1) / pl->rows) : 0;
  const long long cap_keys =
      a->window >= 0 ? std::min<long long>(a->Tmax, static_cast<long long>(a->window) + a->T)
                     : a->Tmax;
  const long long max_tiles = (cap_keys + pl->tk - 1) / pl->tk + 1;
  const long long base = static_cast<long long>(a->B) * a->Hkv * pl->nqb;
  if (base * max_tiles > 0x7fffffffll)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: more than 2^31 key tiles");
  // Long rows of few row groups (config 5 at batch 1 and 8): a fixed split count beats the
  // persistent partition, whose start-up scan and cross-CTA merge are not amortised over so few
  // groups (measured on B200 at 4,096-key windows and 32k-key rows).
  const bool few_long = a->num_ctas == 0 && max_tiles > kSplitMaxTiles && base <= 128;
  pl->mode = (fp8 || a->num_ctas < 0 || few_long || (a->num_ctas == 0 && max_tiles <= kSplitMaxTiles))
                 ? kModeSplit
                 : kModePersistent;
  const size_t rows_out = static_cast<size_t>(a->B) * a->T * a->Hq;
  if (pl->mode == kModeSplit) {
    int nsplit;
    if (a->num_ctas < 0) {
      nsplit = static_cast<int>(std::min<long long>(-static_cast<long long>(a->num_ctas), max_tiles));
    } else if (few_long) {
      // (up to 16 row groups: 16 splits from 4 tiles a split -- batch 1, window 4096 (65 tiles):
      // 8 splits 8.6 us, 16 splits 7.35 us on B200)
      nsplit = base <= 16 ? static_cast<int>(std::max<long long>(2, std::min<long long>(16, max_tiles / 4)))
                          : static_cast<int>(std::max<long long>(2, std::min<long long>(4, max_tiles / 16)));
    } else {
      // A split costs a CTA start, a pipeline fill and a cluster merge, and the CTAs of a grid
      // start and drain together, so an extra split only pays while the row groups alone leave
      // the GPU short of streaming CTAs.  Measured on B200 (head_dim 64 and 128, rows of 256 to
      // 2,000 keys, 8 to 768 row groups): splitting loses once 128 groups (bf16; 384 for fp8,
      // whose CTAs are bound by the e4m3 conversion, not by HBM) fill the machine, rows under 12
      // tiles are never worth cutting, and cluster sizes 3 and 6 schedule badly on full grids --
      // so the split count is a power of two, at most 8, each split at least 2 tiles.
      const long long fill = fp8 ? 384 : 128;
      long long want = base > 0 ? std::min<long long>({8, fill / base, max_tiles / 2}) : 1;
      nsplit = 1;
      if (max_tiles >= 12)
        while (nsplit * 2 <= want) nsplit *= 2;
    }
    // an fp8 cache has no persistent plan and its CTAs are bound by the e4m3 conversion: rows of
    // thousands of keys are cut into CTAs of at most kSplitMaxTiles - 1 tiles, so that uneven
    // row lengths still balance over the waves, and into at least two CTAs per SM (measured on
    // config 5, full context: batch 64 943 -> 611 us, batch 8 167 -> 99 us, batch 1 39 -> 33 us;
    // windows of 4,096 keys run faster uncut)
    if (fp8 && a->num_ctas == 0 && max_tiles > 4 * (kSplitMaxTiles - 1) && base > 0)
      nsplit = static_cast<int>(std::max<long long>(
          {nsplit, (max_tiles + kSplitMaxTiles - 2) / (kSplitMaxTiles - 1),
           std::min<long long>(max_tiles, (2ll * device_sm_count() + base - 1) / base)}));
    pl->tps = static_cast<int>((max_tiles + nsplit - 1) / nsplit);
    pl->nsplit = static_cast<int>((max_tiles + pl->tps - 1) / pl->tps);
    if (base * pl->nsplit > 0x7fffffffll) return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: grid too large");
    pl->grid = 0;
    // up to 8 splits of a row group form a thread-block cluster and merge through distributed
    // shared memory: no partials in global memory.  Up to 16 where the
    // device schedules clusters of 16 and the grid is at most two CTAs per SM (measured on B200:
    // batch 1 at 22k keys, 16 splits, 25.0 -> 21.0 us; on grids of 768 CTAs and more the
    // clusters of 16 schedule worse than partials merged by a combine kernel)
    pl->cluster = pl->nsplit >= 2 &&
                  (pl->nsplit <= 8 || (base * pl->nsplit <= 2ll * device_sm_count() &&
                                       pl->nsplit <= variant_max_cluster(a->D, pl->nqt, fp8)));
    pl->small_grid = base * pl->nsplit <= 4ll * device_sm_count();
    if (pl->nsplit > 1 && !pl->cluster) {
      // partials in the workspace.  On grids of at most about four CTAs per SM the last split of
      // a row group to finish merges them (no second kernel: batch 1, fp8, 37 splits 30.8 ->
      // 26.2 us); on larger grids a combine kernel after the launch does (config 5 fp8, batch 64,
      // full rows, 17 splits: merges inside the grid held SM slots that its later waves needed,
      // 636 -> 694-708 us)
      pl->part_o_bytes = round256(rows_out * pl->nsplit * a->D * 4);
      pl->part_lse_bytes = round256(rows_out * pl->nsplit * 4);
      pl->counter_count = pl->small_grid ? static_cast<size_t>(base) : 0;
    } else {
      pl->part_o_bytes = pl->part_lse_bytes = 0;
      pl->counter_count = 0;
    }
  } else {
    if (a->num_ctas > 0) {
      pl->grid = a->num_ctas;
    } else {
      int per_sm = 1;
      int dev = 0;
      if (cudaGetDevice(&dev) == cudaSuccess) {
        const int rc = variant_ctas_per_sm(a->D, pl->nqt, &per_sm);
        if (rc != MCB_OK) return rc;
      } else {
        cudaGetLastError();
      }
      pl->grid = device_sm_count() * per_sm;
    }
    // whole groups of Hkv CTAs (one per kv head), at least one group
    pl->grid = std::max(a->Hkv, pl->grid / a->Hkv * a->Hkv);
    pl->nsplit = pl->tps = 0;
    const size_t slots = static_cast<size_t>(pl->grid) * 2 * pl->rows;
    pl->part_o_bytes = round256(slots * a->D * 4);
    pl->part_lse_bytes = round256(slots * 4);
    pl->counter_count = static_cast<size_t>(base);
  }
  pl->ws_bytes = pl->part_o_bytes + pl->part_lse_bytes;
  return MCB_OK;
}

int encode_cache_map(CUtensorMap* map, const void* base, int D, int Hkv, int Tmax, int B, int tk) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int panel = D < 64 ? D : 64;
  const CUtensorMapSwizzle swz = panel == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : panel == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hkv),
                        static_cast<cuuint64_t>(Tmax), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(Hkv) * D * 2,
                           static_cast<cuuint64_t>(Tmax) * Hkv * D * 2};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(panel), 1u, static_cast<cuuint32_t>(tk), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return MCB_OK;
}

// An e4m3 cache slot {D, Hkv, Tmax, B} (one byte per element): boxes of tk keys x one head x all D
// bytes, 128-byte (D = 128) or 64-byte (D = 64) swizzled rows.
int encode_cache_map_f8(CUtensorMap* map, const void* base, int D, int Hkv, int Tmax, int B, int tk) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hkv),
                        static_cast<cuuint64_t>(Tmax), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hkv) * D,
                           static_cast<cuuint64_t>(Tmax) * Hkv * D};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(D), 1u, static_cast<cuuint32_t>(tk), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled(fp8 cache) failed (CUresult %d)", (int)r);
  return MCB_OK;
}

int check_attn_pointers(const mcb_attn_args* a, const char* who) {
  if (a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr || a->out == nullptr ||
      a->cache_seqlens == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "%s: NULL pointer argument", who);
  if (a->k_scale != nullptr && (!aligned(a->k_scale, 256) || !aligned(a->v_scale, 256)))
    return fail(MCB_ERR_ALIGNMENT, "%s: fp8 scale arrays must be 256-byte aligned", who);
  if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16) || !aligned(a->q, 16) ||
      !aligned(a->out, 16))
    return fail(MCB_ERR_ALIGNMENT, "%s: q, out and cache pointers must be 16-byte aligned", who);
  for (int i = 0; i < 3; ++i)
    if (a->q_stride[i] < 0 || (a->q_stride[i] % 8) != 0)
      return fail(MCB_ERR_ALIGNMENT, "%s: q strides must be non-negative multiples of 8 elements", who);
  if (a->fuse_append) {
    if ((a->k_new == nullptr) != (a->v_new == nullptr) || a->rot_cos == nullptr || a->rot_sin == nullptr ||
        a->rot_len <= 0)
      return fail(MCB_ERR_INVALID_ARG, "%s: fused append needs rot_cos, rot_sin, rot_len > 0 and both or "
                  "neither of k_new, v_new", who);
    if (!aligned(a->rot_cos, 16) || !aligned(a->rot_sin, 16) ||
        (a->k_new != nullptr && (!aligned(a->k_new, 16) || !aligned(a->v_new, 16))))
      return fail(MCB_ERR_ALIGNMENT, "%s: fused append vectors and tables must be 16-byte aligned", who);
    for (int i = 0; i < 3; ++i)
      if (a->k_new != nullptr && (a->k_new_stride[i] < 0 || a->k_new_stride[i] % 8 || a->v_new_stride[i] < 0 ||
                                  a->v_new_stride[i] % 8))
        return fail(MCB_ERR_ALIGNMENT, "%s: k_new / v_new strides must be non-negative multiples of 8", who);
  }
  return MCB_OK;
}

// Whether the planned call can fuse the append (the split or persistent kernel's bf16 path, one
// new token).
bool plan_fusable(const mcb_attn_args* a, const AttnPlan& pl) {
  return a->T == 1 && a->k_scale == nullptr && (a->D == 64 || a->D == 128) &&
         (pl.mode == kModeSplit || pl.mode == kModePersistent);
}

// The fused-append fields shared by the split and the persistent kernels' parameters.
template <class P>
void fill_fused_append(P& p, const mcb_attn_args* a) {
  p.fuse = a->fuse_append ? 1 : 0;
  p.k_new = static_cast<const uint16_t*>(a->k_new);
  p.v_new = static_cast<const uint16_t*>(a->v_new);
  for (int i = 0; i < 3; ++i) {
    p.kns[i] = a->k_new_stride[i];
    p.vns[i] = a->v_new_stride[i];
  }
  p.kc_out = static_cast<uint16_t*>(const_cast<void*>(a->k_cache));  // written with fuse_append
  p.vc_out = static_cast<uint16_t*>(const_cast<void*>(a->v_cache));
  p.rot_cos = static_cast<const uint16_t*>(a->rot_cos);
  p.rot_sin = static_cast<const uint16_t*>(a->rot_sin);
  p.rot_len = a->rot_len;
  p.rotate_k = a->rotate_k;
  p.norm_eps = a->norm_eps;
  p.qk_scale = a->qk_scale;
}

// q as a 4-D tensor map {D, Hq, T, B} with its own strides; 128-query boxes of 64-column panels.
int encode_q_map(CUtensorMap* map, const mcb_attn_args* a) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a->D), static_cast<cuuint64_t>(a->Hq),
                        static_cast<cuuint64_t>(a->T), static_cast<cuuint64_t>(a->B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a->q_stride[2]) * 2,
                           static_cast<cuuint64_t>(a->q_stride[1]) * 2,
                           static_cast<cuuint64_t>(a->q_stride[0]) * 2};
  cuuint32_t box[4] = {64u, 1u, static_cast<cuuint32_t>(mcb::kPfTile), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a->q), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled(q) failed (CUresult %d)", (int)r);
  return MCB_OK;
}

int run_prefill(const mcb_attn_args* a, cudaStream_t st) {
  CUtensorMap qm, km, vm;
  int rc = encode_q_map(&qm, a);
  if (rc != MCB_OK) return rc;
  rc = encode_cache_map(&km, a->k_cache, a->D, a->Hkv, a->Tmax, a->B, mcb::kPfTile);
  if (rc != MCB_OK) return rc;
  rc = encode_cache_map(&vm, a->v_cache, a->D, a->Hkv, a->Tmax, a->B, mcb::kPfTile);
  if (rc != MCB_OK) return rc;
  mcb::PrefillParams p;
  p.out = static_cast<uint16_t*>(a->out);
  p.cache_seqlens = a->cache_seqlens;
  p.B = a->B;
  p.T = a->T;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.G = a->Hq / a->Hkv;
  p.Tmax = a->Tmax;
  p.window = a->window;
  // head size 64: one query tile an item, two CTAs per SM (independent chains); 128: pairs
  const int qt = a->D == 64 ? 1 : 2;
  p.n_qgroups = (a->T + qt * mcb::kPfTile - 1) / (qt * mcb::kPfTile);
  p.ring = a->ring != 0;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  const long long items = static_cast<long long>(p.n_qgroups) * a->B * a->Hq;
  if (items > INT32_MAX) return fail(MCB_ERR_UNSUPPORTED, "mcb_prefill_attn: %lld work items", items);
  p.n_items = static_cast<int>(items);
  // persistent: QT = 2, one CTA per SM (each holds all of its SM's TMEM); QT = 1, two per SM
  // (256 TMEM columns each); items dealt over them
  const long long grid = std::min<long long>(items, static_cast<long long>(3 - qt) * device_sm_count());
  if (a->D == 64) return PrefillVariant<64, 1>::launch(grid, qm, km, vm, p, st);
  return PrefillVariant<128, 2>::launch(grid, qm, km, vm, p, st);
}

// Encodes the tensor maps, fills the kernel parameters with the workspace `ws` (and, for the
// persistent kernel, the arrival counters) and launches.
// Head pairs: a decode step over kv heads of 64 with one query head each (G = 1) whose split
// plan takes one split a row group runs as kv heads of 128 -- two real heads side by side, the
// same bytes -- with two query rows a group (the split kernel's `pair` mode): half the CTAs, each
// with twice the bytes in flight.  Measured on config 2's attention (a graph of 12 launches):
// 26.0 -> 25.4 us at ragged lengths of 512-1024 keys, 24.7 -> 23.4 us at 768.  `va` and `vpl`
// receive the paired shape and its plan.
bool pair_plan(const mcb_attn_args* a, const AttnPlan& pl, mcb_attn_args* va, AttnPlan* vpl) {
  if (a->T != 1 || a->D != 64 || a->Hq != a->Hkv || a->Hkv % 2 != 0 || a->k_scale != nullptr ||
      a->num_ctas != 0 || pl.mode != kModeSplit || pl.nsplit != 1)
    return false;
  *va = *a;
  va->Hkv = a->Hkv / 2;
  va->D = 128;
  if (plan_attn(va, vpl) != MCB_OK) return false;
  return vpl->mode == kModeSplit && vpl->nsplit == 1 && vpl->nqt == 1;
}

int run_attn(const mcb_attn_args* a0, const AttnPlan& pl0, void* ws, int32_t* counters, cudaStream_t st) {
  if (a0->fuse_append && !plan_fusable(a0, pl0))
    return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: the append fuses only for T = 1, a bf16 slot, D = 64 "
                "or 128 and the split or persistent plan (mcb_decode_attn_fusable)");
  mcb_attn_args va;
  AttnPlan vpl;
  const bool pair = pair_plan(a0, pl0, &va, &vpl);
  const mcb_attn_args* a = pair ? &va : a0;
  const AttnPlan& pl = pair ? vpl : pl0;
  if (pl.mode == kModePrefill) return run_prefill(a, st);
  const bool fp8 = a->k_scale != nullptr;
  CUtensorMap km, vm;
  int rc = fp8 ? encode_cache_map_f8(&km, a->k_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk)
               : encode_cache_map(&km, a->k_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;
  rc = fp8 ? encode_cache_map_f8(&vm, a->v_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk)
           : encode_cache_map(&vm, a->v_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;
  uint8_t* w = static_cast<uint8_t*>(ws);
  if (pl.mode == kModeSplit) {
    mcb::SplitAttnParams p;
    p.q = static_cast<const uint16_t*>(a->q);
    for (int i = 0; i < 3; ++i) p.qs[i] = a->q_stride[i];
    p.cache_seqlens = a->cache_seqlens;
    p.out = static_cast<uint16_t*>(a->out);
    p.part_o = pl.nsplit > 1 && !pl.cluster ? reinterpret_cast<float*>(w) : nullptr;
    p.part_lse = pl.nsplit > 1 && !pl.cluster ? reinterpret_cast<float*>(w + pl.part_o_bytes) : nullptr;
    p.cluster = pl.cluster ? 1 : 0;
    p.counters = pl.counter_count > 0 ? counters : nullptr;
    fill_fused_append(p, a);
    p.ring = a->ring != 0;
    p.B = a->B;
    p.T = a->T;
    p.Hq = a->Hq;
    p.Hkv = a->Hkv;
    p.G = a->Hq / a->Hkv;
    p.Tmax = a->Tmax;
    p.window = a->window;
    p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
    p.nsplit = pl.nsplit;
    p.tiles_per_split = pl.tps;
    // rows cut by their own lengths only on small grids (batch 1, 8,192 keys, 4 splits: 64 ->
    // 20.7 us; on large grids the cuts multiply the CTAs: config 5 fp8 at batch 64, full rows,
    // 17 splits, 636 vs 679 us)
    p.row_cuts = pl.small_grid ? 1 : 0;
    p.nqb = pl.nqb;
    p.k_scale = a->k_scale;
    p.v_scale = a->v_scale;
    p.scale_tmax = a->scale_tmax;
    p.pair = pair ? 1 : 0;
    const long long grid = static_cast<long long>(a->B) * a->Hkv * pl.nqb * pl.nsplit;
    return fp8 ? variant_launch_split_f8(a->D, pl.nqt, grid, km, vm, p, st)
               : variant_launch_split(a->D, pl.nqt, grid, km, vm, p, st);
  }
  mcb::AttnParams p;
  p.q = static_cast<const uint16_t*>(a->q);
  for (int i = 0; i < 3; ++i) p.qs[i] = a->q_stride[i];
  p.cache_seqlens = a->cache_seqlens;
  p.out = static_cast<uint16_t*>(a->out);
  p.part_o = reinterpret_cast<float*>(w);
  p.part_lse = reinterpret_cast<float*>(w + pl.part_o_bytes);
  p.counters = counters;
  p.B = a->B;
  p.T = a->T;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.G = a->Hq / a->Hkv;
  p.Tmax = a->Tmax;
  p.window = a->window;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  p.nqb = pl.nqb;
  p.n_entries = a->B * pl.nqb;
  p.ring = a->ring != 0;
  p.grid = pl.grid;
  p.ngroups = pl.grid / a->Hkv;
  fill_fused_append(p, a);
  return variant_launch(a->D, pl.nqt, pl.grid, km, vm, p, st);
}

}  // namespace

// One warp per row; CPL = 16-byte chunks per lane, the smallest of 1, 2, 4, 8, 16 that covers C.
// A decode step has few rows (one per sequence): one row per 32-thread block spreads them over
// as many SMs as possible (these launches are latency-bound); prefill-sized row counts use
// 4 rows per block.
template <class F>
static void launch_row_norm(int C, int rows, cudaStream_t st, F&& launch) {
  const int chunks = C / 8;
  const int per_block = rows <= 1024 ? 1 : 4;
  const dim3 grid((rows + per_block - 1) / per_block), block(32 * per_block);
  if (chunks <= 32) launch(std::integral_constant<int, 1>{}, grid, block, st);
  else if (chunks <= 64) launch(std::integral_constant<int, 2>{}, grid, block, st);
  else if (chunks <= 128) launch(std::integral_constant<int, 4>{}, grid, block, st);
  else if (chunks <= 256) launch(std::integral_constant<int, 8>{}, grid, block, st);
  else launch(std::integral_constant<int, 16>{}, grid, block, st);
  g_launches++;
}

// ---------------------------------------------------------------------------------------------
// Decode projections (decode_proj.cuh)
int encode_rows_map(CUtensorMap* map, const void* base, long long rows, long long cols,
                    long long stride, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), 1, 1};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(stride) * 2, static_cast<cuuint64_t>(stride) * 2 * rows,
                           static_cast<cuuint64_t>(stride) * 2 * rows};
  cuuint32_t box[4] = {64u, static_cast<cuuint32_t>(box_rows), 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCB_ERR_CUDA, "cuTensorMapEncodeTiled(rows) failed (CUresult %d)", (int)r);
  return MCB_OK;
}

constexpr int kMaxSmemOptin = 232448;

template <int F, bool NORM, bool ADD, bool GATED = false, int RB = mcb::kProjRows>
int launch_proj(const CUtensorMap& wm, const CUtensorMap& xm, const CUtensorMap& dm, const mcb::ProjParams& prm,
                bool pdl, cudaStream_t st) {
  static std::atomic<uint64_t> done{0};
  auto kernel = mcb::proj_kernel<F, NORM, ADD, GATED, RB>;
  cudaError_t e = ensure_smem(kernel, kMaxSmemOptin, done);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(linear)");
  cudaLaunchConfig_t cfg = {};
  constexpr int FO = GATED ? F / 2 : F;  // output features a CTA
  cfg.gridDim = dim3(static_cast<unsigned>((prm.N + FO - 1) / FO), static_cast<unsigned>((prm.R + RB - 1) / RB));
  cfg.blockDim = dim3(mcb::kProjThreads);
  cfg.dynamicSmemBytes = mcb::proj_smem_bytes(F, prm.panels, ADD, RB);
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kernel, wm, xm, dm, prm);
  g_launches++;
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "linear launch");
  return MCB_OK;
}

// Norm out: 64 features a CTA, 16 rows a cluster of N / 64 CTAs (one per 64-column panel of the
// output row); clusters above the portable 8 need the non-portable size, which the host checks
// the device schedules (with this kernel's shared memory) before the first launch.
constexpr int kProjNoutRows = 16;
using ProjNoutKernel = decltype(&mcb::proj_kernel<64, false, false, false, kProjNoutRows, true>);

cudaError_t nout_prepare(ProjNoutKernel kernel, int smem) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

// Whether a norm-out launch with `npanel` CTAs a cluster and `smem` bytes each can be scheduled on
// the current device (cached per device, cluster size and shared-memory size).
bool nout_schedulable(int npanel, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, bool> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(dev, npanel, smem);
  auto itc = cache.find(key);
  if (itc != cache.end()) return itc->second;
  auto kernel = mcb::proj_kernel<64, false, false, false, kProjNoutRows, true>;
  bool ok = nout_prepare(kernel, smem) == cudaSuccess;
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(npanel), 1);
    cfg.blockDim = dim3(mcb::kProjThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(npanel);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    ok = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess && n > 0;
  }
  cudaGetLastError();
  cache[key] = ok;
  return ok;
}

int launch_proj_nout(const CUtensorMap& wm, const CUtensorMap& xm, const mcb::ProjParams& prm, bool pdl,
                     cudaStream_t st) {
  auto kernel = mcb::proj_kernel<64, false, false, false, kProjNoutRows, true>;
  const int smem = mcb::proj_smem_bytes(64, prm.panels, false, kProjNoutRows);
  cudaError_t e = nout_prepare(kernel, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(linear, norm out)");
  cudaLaunchConfig_t cfg = {};
  const int npanel = prm.N / 64;
  cfg.gridDim = dim3(static_cast<unsigned>(npanel), static_cast<unsigned>((prm.R + kProjNoutRows - 1) / kProjNoutRows));
  cfg.blockDim = dim3(mcb::kProjThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = static_cast<unsigned>(npanel);
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kernel, wm, xm, xm, prm);
  g_launches++;
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "linear launch (norm out)");
  return MCB_OK;
}

template <int F>
int launch_proj_f(bool norm, bool add, const CUtensorMap& wm, const CUtensorMap& xm, const CUtensorMap& dm,
                  const mcb::ProjParams& prm, bool pdl, cudaStream_t st) {
  if (add) return launch_proj<F, true, true>(wm, xm, dm, prm, pdl, st);
  if (norm) return launch_proj<F, true, false>(wm, xm, dm, prm, pdl, st);
  return launch_proj<F, false, false>(wm, xm, dm, prm, pdl, st);
}

bool ranges_overlap(const void* a, long long a_stride, int a_cols, const void* b, long long b_stride,
                    int b_cols, int rows) {
  if (a == nullptr || b == nullptr || rows <= 0) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  const uintptr_t a1 = a0 + static_cast<uintptr_t>(((rows - 1) * a_stride + a_cols) * 2);
  const uintptr_t b1 = b0 + static_cast<uintptr_t>(((rows - 1) * b_stride + b_cols) * 2);
  return a0 < b1 && b0 < a1;
}

extern "C" {

int mcb_abi_version(void) { return MCB_ABI_VERSION; }

int mcb_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    const size_t n = std::min(len - 1, g_last_error.size());
    std::memcpy(buf, g_last_error.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(g_last_error.size());
}

uint64_t mcb_launch_count(void) { return g_launches.load(); }

int mcb_last_attn_kernel(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return fail(MCB_ERR_INVALID_ARG, "mcb_last_attn_kernel: empty buffer");
  snprintf(buf, len, "%s", g_last_attn_kernel);
  return MCB_OK;
}

int mcb_kv_append_rope(const mcb_append_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: args is NULL");
  const uint32_t known = MCB_APPEND_ROTATE_Q | MCB_APPEND_ROTATE_K | MCB_APPEND_WRITE_KV;
  if (a->flags & ~known) return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: unknown flags 0x%x", a->flags);
  if (a->flags == 0) return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: no work requested (flags 0)");
  const bool rq = a->flags & MCB_APPEND_ROTATE_Q, rk = a->flags & MCB_APPEND_ROTATE_K,
             wkv = a->flags & MCB_APPEND_WRITE_KV;
  if (rk && !wkv)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: ROTATE_K requires WRITE_KV");
  if (a->B < 0 || a->T < 0 || a->D <= 0 || (a->D & 1) || a->D > 256)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: bad sizes B=%d T=%d D=%d", a->B, a->T, a->D);
  if (a->cache_seqlens == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: cache_seqlens is NULL");
  if (rq && (a->q == nullptr || a->q_out == nullptr || a->Hq <= 0))
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: ROTATE_Q needs q, q_out and Hq > 0");
  if (wkv && (a->k == nullptr || a->v == nullptr || a->k_cache == nullptr ||
              a->v_cache == nullptr || a->Hkv <= 0 || a->Tmax <= 0))
    return fail(MCB_ERR_INVALID_ARG,
                "mcb_kv_append_rope: WRITE_KV needs k, v, k_cache, v_cache, Hkv > 0, Tmax > 0");
  if ((rq || rk) && (a->cos == nullptr || a->sin == nullptr || a->rot_len <= 0))
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: rotation needs the cos/sin tables");
  for (int i = 0; i < 3; ++i)
    if ((rq && a->q_stride[i] < 0) || (wkv && (a->k_stride[i] < 0 || a->v_stride[i] < 0)))
      return fail(MCB_ERR_INVALID_ARG, "mcb_kv_append_rope: negative stride");
  const bool fp8 = a->k_scale != nullptr;
  if (fp8 && (a->v_scale == nullptr || !wkv || a->scale_tmax < a->Tmax || a->scale_tmax % 64 != 0))
    return fail(MCB_ERR_INVALID_ARG,
                "mcb_kv_append_rope: an fp8 cache needs WRITE_KV, k_scale and v_scale, and scale_tmax >= "
                "Tmax, a multiple of 64");
  if (fp8 && a->D != 64 && a->D != 128)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_kv_append_rope: an fp8 cache needs D = 64 or 128 (D=%d)", a->D);

  mcb::AppendParams p;
  p.q = static_cast<const uint16_t*>(a->q);
  p.k = static_cast<const uint16_t*>(a->k);
  p.v = static_cast<const uint16_t*>(a->v);
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = a->q_stride[i];
    p.ks[i] = a->k_stride[i];
    p.vs[i] = a->v_stride[i];
  }
  p.q_out = static_cast<uint16_t*>(a->q_out);
  p.k_cache = static_cast<uint16_t*>(a->k_cache);
  p.v_cache = static_cast<uint16_t*>(a->v_cache);
  p.cache_seqlens = a->cache_seqlens;
  p.cos = static_cast<const uint16_t*>(a->cos);
  p.sin = static_cast<const uint16_t*>(a->sin);
  p.B = a->B;
  p.T = a->T;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.D = a->D;
  p.Tmax = a->Tmax;
  p.rot_len = a->rot_len;
  p.eps = a->eps;
  p.scale = a->scale;
  p.nq = rq ? a->Hq : 0;
  p.nk = wkv ? a->Hkv : 0;
  p.rotate_k = rk;
  p.ring = a->ring != 0;
  p.k_scale = a->k_scale;
  p.v_scale = a->v_scale;
  p.scale_tmax = a->scale_tmax;
  p.total_vectors = static_cast<long long>(a->B) * a->T * (p.nq + 2 * p.nk);
  if (p.total_vectors == 0) return MCB_OK;
  // 16-byte chunks when every row the kernel touches starts on a 16-byte boundary.
  bool vec = (a->D == 16 || a->D == 32 || a->D == 64 || a->D == 128 || a->D == 256);
  auto rows16 = [](const void* ptr, const int64_t* st) {
    return aligned(ptr, 16) && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0;
  };
  if (rq) vec = vec && rows16(a->q, a->q_stride) && aligned(a->q_out, 16);
  if (wkv) vec = vec && rows16(a->k, a->k_stride) && rows16(a->v, a->v_stride) &&
                 aligned(a->k_cache, 16) && aligned(a->v_cache, 16);
  if (rq || rk) vec = vec && aligned(a->cos, 16) && aligned(a->sin, 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp8 && !vec)
    return fail(MCB_ERR_ALIGNMENT, "mcb_kv_append_rope: an fp8 cache needs 16-byte aligned rows");
  if (vec) {
    // a grid-stride kernel: at most kAppendVecCtasPerSm CTAs per SM, each warp looping over
    // batches of vector groups with every load of a batch in flight before its arithmetic
    if (p.total_vectors > 0x7fffffffll)
      return fail(MCB_ERR_UNSUPPORTED, "mcb_kv_append_rope: %lld vectors in one call (at most 2^31 - 1)",
                  p.total_vectors);
    const long long vpw = 32 / (a->D / 16);
    const long long warps = (p.total_vectors + vpw - 1) / vpw;
    const long long wpb = mcb::kAppendVecThreads / 32;
    const long long blocks = std::min<long long>((warps + wpb - 1) / wpb,
                                                 static_cast<long long>(kAppendVecCtasPerSm) * device_sm_count());
    const dim3 grid(static_cast<unsigned>(blocks)), block(mcb::kAppendVecThreads);
    cudaError_t e;
    switch (a->D) {
      case 16: e = launch_pdl(mcb::kv_append_rope_vec_kernel<16, false>, grid, block, 0, st, p); break;
      case 32: e = launch_pdl(mcb::kv_append_rope_vec_kernel<32, false>, grid, block, 0, st, p); break;
      case 64:
        e = fp8 ? launch_pdl(mcb::kv_append_rope_vec_kernel<64, true>, grid, block, 0, st, p)
                : launch_pdl(mcb::kv_append_rope_vec_kernel<64, false>, grid, block, 0, st, p);
        break;
      case 128:
        e = fp8 ? launch_pdl(mcb::kv_append_rope_vec_kernel<128, true>, grid, block, 0, st, p)
                : launch_pdl(mcb::kv_append_rope_vec_kernel<128, false>, grid, block, 0, st, p);
        break;
      default: e = launch_pdl(mcb::kv_append_rope_vec_kernel<256, false>, grid, block, 0, st, p); break;
    }
    g_launches++;
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kv_append_rope launch");
    return MCB_OK;
  }
  const long long blocks = (p.total_vectors + mcb::kAppendWarpsPerBlock - 1) / mcb::kAppendWarpsPerBlock;
  if (blocks > 0x7fffffffll) return fail(MCB_ERR_UNSUPPORTED, "mcb_kv_append_rope: grid too large");
  cudaError_t e = launch_pdl(mcb::kv_append_rope_kernel, dim3(static_cast<unsigned>(blocks)),
                             dim3(mcb::kAppendWarpsPerBlock * 32), 0, st, p);
  g_launches++;
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_append_rope launch");
  return MCB_OK;
}

int mcb_kv_copy_rows(const mcb_copy_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: args is NULL");
  if (a->n_slots < 0 || a->src_batch <= 0 || a->dst_batch <= 0 || a->n_pos < 0 ||
      a->row_elems <= 0 || a->dst_row_count < 0)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: bad sizes");
  if (a->src_row < 0 || a->src_row >= a->src_batch)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: src_row %d out of range for batch %d",
                a->src_row, a->src_batch);
  if (a->dst_row_begin < 0 || a->dst_row_begin + a->dst_row_count > a->dst_batch)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: rows [%d, %d) out of range for batch %d",
                a->dst_row_begin, a->dst_row_begin + a->dst_row_count, a->dst_batch);
  if (a->n_pos > a->src_tmax || a->n_pos > a->dst_tmax)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: %d positions exceed cache length (src %d, dst %d)",
                a->n_pos, a->src_tmax, a->dst_tmax);
  if ((a->row_elems % 8) != 0)
    return fail(MCB_ERR_ALIGNMENT, "mcb_kv_copy_rows: Hkv*D (%d) must be a multiple of 8", a->row_elems);
  const long long nvec_bytes = static_cast<long long>(a->n_pos) * a->row_elems * 2;
  if (a->n_slots > 0 && nvec_bytes > 0) {
    if (!a->dst_k || !a->dst_v || !a->src_k || !a->src_v)
      return fail(MCB_ERR_INVALID_ARG, "mcb_kv_copy_rows: NULL cache pointer");
    if (!aligned(a->dst_k, 16) || !aligned(a->dst_v, 16) || !aligned(a->src_k, 16) ||
        !aligned(a->src_v, 16))
      return fail(MCB_ERR_ALIGNMENT, "mcb_kv_copy_rows: cache pointers must be 16-byte aligned");
  }
  mcb::CopyParams p;
  p.dst_k = static_cast<uint16_t*>(a->dst_k);
  p.dst_v = static_cast<uint16_t*>(a->dst_v);
  p.src_k = static_cast<const uint16_t*>(a->src_k);
  p.src_v = static_cast<const uint16_t*>(a->src_v);
  p.n_slots = a->n_slots;
  const long long src_row_len = static_cast<long long>(a->src_tmax) * a->row_elems;
  const long long dst_row_len = static_cast<long long>(a->dst_tmax) * a->row_elems;
  p.src_slot_stride = src_row_len * a->src_batch;
  p.src_row_offset = src_row_len * a->src_row;
  p.dst_slot_stride = dst_row_len * a->dst_batch;
  p.dst_row_stride = dst_row_len;
  p.dst_row_begin_offset = dst_row_len * a->dst_row_begin;
  p.dst_row_count = a->dst_row_count;
  p.vecs_per_slot = nvec_bytes / 16;
  p.dst_seqlens = a->dst_seqlens;
  p.dst_seqlen_begin = a->dst_row_begin;
  p.seqlen_value = a->n_pos;
  const long long total = p.vecs_per_slot * p.n_slots;
  if (total == 0 && p.dst_seqlens == nullptr) return MCB_OK;
  const long long want = (total + 255) / 256;
  const long long cap = 8ll * device_sm_count();
  const unsigned gx = static_cast<unsigned>(std::max(1ll, std::min(want, cap)));
  mcb::kv_copy_rows_kernel<<<dim3(gx, 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  g_launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_copy_rows launch");
  return MCB_OK;
}

int mcb_add_rms_norm(const mcb_add_norm_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_add_rms_norm: args is NULL");
  if (a->rows < 0 || a->C <= 0 || a->C % 8 != 0 || a->C > 4096)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_add_rms_norm: C=%d must be a positive multiple of 8, at most 4096",
                a->C);
  if (a->x == nullptr || a->h_out == nullptr || (a->delta != nullptr && a->x_out == nullptr))
    return fail(MCB_ERR_INVALID_ARG, "mcb_add_rms_norm: NULL pointer argument");
  const bool ok16 = aligned(a->x, 16) && aligned(a->h_out, 16) && a->x_stride % 8 == 0 &&
                    a->h_stride % 8 == 0 &&
                    (a->delta == nullptr ||
                     (aligned(a->delta, 16) && aligned(a->x_out, 16) && a->delta_stride % 8 == 0 &&
                      a->x_out_stride % 8 == 0));
  if (!ok16) return fail(MCB_ERR_ALIGNMENT, "mcb_add_rms_norm: rows must start on 16-byte boundaries");
  if (a->rows == 0) return MCB_OK;
  mcb::AddNormParams p;
  p.x = static_cast<const uint16_t*>(a->x);
  p.delta = static_cast<const uint16_t*>(a->delta);
  p.x_out = a->delta ? static_cast<uint16_t*>(a->x_out) : nullptr;
  p.h_out = static_cast<uint16_t*>(a->h_out);
  p.xs = a->x_stride;
  p.ds = a->delta_stride;
  p.xos = a->x_out_stride;
  p.hs = a->h_stride;
  p.rows = a->rows;
  p.C = a->C;
  p.eps = a->eps;
  launch_row_norm(a->C, a->rows, static_cast<cudaStream_t>(stream), [&](auto cpl, dim3 g, dim3 b,
                                                                        cudaStream_t st) {
    launch_pdl(mcb::add_rms_norm_kernel<decltype(cpl)::value>, g, b, 0, st, p);
  });
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "add_rms_norm launch");
  return MCB_OK;
}

int mcb_embed_rms_norm(const mcb_embed_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_embed_rms_norm: args is NULL");
  if (a->rows < 0 || a->C <= 0 || a->C % 8 != 0 || a->C > 4096)
    return fail(MCB_ERR_UNSUPPORTED,
                "mcb_embed_rms_norm: C=%d must be a positive multiple of 8, at most 4096", a->C);
  if (a->V <= 0) return fail(MCB_ERR_INVALID_ARG, "mcb_embed_rms_norm: V=%lld", (long long)a->V);
  if (a->ids == nullptr || a->table == nullptr || a->x_out == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_embed_rms_norm: NULL pointer argument");
  if (!aligned(a->table, 16) || !aligned(a->x_out, 16) || a->table_stride % 8 || a->x_stride % 8 ||
      (a->h_out != nullptr && (!aligned(a->h_out, 16) || a->h_stride % 8)))
    return fail(MCB_ERR_ALIGNMENT, "mcb_embed_rms_norm: rows must start on 16-byte boundaries");
  if (a->rows == 0) return MCB_OK;
  mcb::EmbedNormParams p;
  p.ids = a->ids;
  p.table = static_cast<const uint16_t*>(a->table);
  p.x_out = static_cast<uint16_t*>(a->x_out);
  p.h_out = static_cast<uint16_t*>(a->h_out);
  p.ts = a->table_stride;
  p.xs = a->x_stride;
  p.hs = a->h_stride;
  p.V = a->V;
  p.rows = a->rows;
  p.C = a->C;
  p.eps = a->eps;
  launch_row_norm(a->C, a->rows, static_cast<cudaStream_t>(stream), [&](auto cpl, dim3 g, dim3 b,
                                                                        cudaStream_t st) {
    launch_pdl(mcb::embed_rms_norm_kernel<decltype(cpl)::value>, g, b, 0, st, p);
  });
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "embed_rms_norm launch");
  return MCB_OK;
}

int mcb_softcap_argmax(const mcb_softcap_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_softcap_argmax: args is NULL");
  if (a->rows < 0 || a->V <= 0 || a->logits_stride < a->V ||
      (a->out != nullptr && a->out_stride < a->V))
    return fail(MCB_ERR_INVALID_ARG, "mcb_softcap_argmax: rows=%d V=%d logits_stride=%lld", a->rows,
                a->V, (long long)a->logits_stride);
  if (a->logits == nullptr || (a->out == nullptr && a->argmax == nullptr))
    return fail(MCB_ERR_INVALID_ARG, "mcb_softcap_argmax: NULL logits, or neither out nor argmax");
  if (a->rows == 0) return MCB_OK;
  mcb::SoftcapParams p;
  p.logits = static_cast<const uint16_t*>(a->logits);
  p.out = a->out;
  p.argmax = a->argmax;
  p.ls = a->logits_stride;
  p.os = a->out_stride;
  p.as = a->argmax_stride;
  p.rows = a->rows;
  p.V = a->V;
  p.cap = a->softcap;
  p.inv_cap = a->softcap > 0.f ? 1.0f / a->softcap : 0.f;
  p.vec = a->V % 8 == 0 && aligned(a->logits, 16) && a->logits_stride % 8 == 0 &&
          (a->out == nullptr || (aligned(a->out, 16) && a->out_stride % 4 == 0));
  // Split a row over a cluster when the rows alone leave SMs idle: up to 8 CTAs a row, each with
  // at least one chunk (or element) per thread.
  const int units = p.vec ? p.V / 8 : p.V;
  int cs = 1;
  if (a->rows < 2 * device_sm_count()) {
    cs = (units + mcb::kSoftcapThreads - 1) / mcb::kSoftcapThreads;
    cs = cs < 1 ? 1 : (cs > 8 ? 8 : cs);
  }
  if (static_cast<long long>(a->rows) * cs > 0x7fffffffll)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_softcap_argmax: %d rows is too many", a->rows);
  p.cs = cs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->rows * cs));
  cfg.blockDim = dim3(mcb::kSoftcapThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = static_cast<unsigned>(cs);
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = cs > 1 ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, mcb::softcap_argmax_kernel, p);
  g_launches++;
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "softcap_argmax launch");
  return MCB_OK;
}

int mcb_sample(const mcb_sample_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_sample: args is NULL");
  if (a->rows < 0 || a->V <= 0 || a->logits_stride < a->V)
    return fail(MCB_ERR_INVALID_ARG, "mcb_sample: rows=%d V=%d logits_stride=%lld", a->rows, a->V,
                (long long)a->logits_stride);
  if (!(a->temperature > 0.f))
    return fail(MCB_ERR_INVALID_ARG, "mcb_sample: temperature must be > 0 (greedy: top_k = 1)");
  if (a->logits == nullptr || a->uniforms == nullptr || a->out == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_sample: NULL pointer argument");
  if (a->rows == 0) return MCB_OK;
  mcb::SampleParams p;
  p.logits = a->logits;
  p.uniforms = a->uniforms;
  p.out = a->out;
  p.ls = a->logits_stride;
  p.os = a->out_stride;
  p.rows = a->rows;
  p.V = a->V;
  p.top_k = a->top_k;
  p.inv_temperature = 1.0f / a->temperature;
  launch_pdl(mcb::sample_kernel, dim3(a->rows), dim3(mcb::kSampleThreads), 0, static_cast<cudaStream_t>(stream), p);
  g_launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sample launch");
  return MCB_OK;
}

}  // extern "C"

// The checks of mcb_linear and its launch shape, without launching.
struct LinearPlan {
  int F, rb, panels;
  bool norm, gated, add, nout;
};

int plan_linear(const mcb_linear_args* a, LinearPlan* pl) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_linear: args is NULL");
  if (a->R < 0 || a->N <= 0 || a->K <= 0)
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: R=%d N=%d K=%d", a->R, a->N, a->K);
  if (a->flags & ~(MCB_LINEAR_NORM | MCB_LINEAR_GATED | MCB_LINEAR_NORM_OUT))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: flags %d", a->flags);
  const bool norm = (a->flags & MCB_LINEAR_NORM) != 0;
  const bool gated = (a->flags & MCB_LINEAR_GATED) != 0;
  const bool nout = (a->flags & MCB_LINEAR_NORM_OUT) != 0;
  const bool add = a->delta != nullptr;
  if (add && !norm) return fail(MCB_ERR_INVALID_ARG, "mcb_linear: delta needs MCB_LINEAR_NORM");
  if (gated && (norm || add || a->res != nullptr))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: MCB_LINEAR_GATED takes no norm, delta or res");
  if (nout && (norm || gated))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: MCB_LINEAR_NORM_OUT takes no other flag");
  if (gated && a->N % 16 != 0)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: gated N=%d must be a multiple of 16", a->N);
  if (nout && (a->N % 64 != 0 || a->N > 64 * mcb::kMaxClusterSplits))
    return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: MCB_LINEAR_NORM_OUT needs N a multiple of 64, at most %d (N=%d)",
                64 * mcb::kMaxClusterSplits, a->N);
  if (a->R > mcb::kProjRows || a->K % 64 != 0 || (norm && a->K > 32 * 8 * mcb::kProjNormCpl))
    return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: R=%d (at most %d), K=%d (a multiple of 64%s)", a->R,
                mcb::kProjRows, a->K, norm ? ", at most 1024 with the norm" : "");
  if (a->x == nullptr || a->w == nullptr || a->y == nullptr || (add && a->x_out == nullptr) ||
      (nout && a->h_out == nullptr))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: NULL pointer argument");
  if (a->x_stride < a->K || a->w_stride < a->K || a->y_stride < a->N ||
      (a->res != nullptr && a->res_stride < a->N) ||
      (add && (a->delta_stride < a->K || a->x_out_stride < a->K)) || (nout && a->h_out_stride < a->N))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: row strides shorter than the rows");
  if (!aligned(a->x, 16) || !aligned(a->w, 16) || !aligned(a->y, 2) || a->x_stride % 8 || a->w_stride % 8 ||
      (a->res != nullptr && !aligned(a->res, 2)) ||
      (add && (!aligned(a->delta, 16) || !aligned(a->x_out, 16) || a->delta_stride % 8 || a->x_out_stride % 8)))
    return fail(MCB_ERR_ALIGNMENT, "mcb_linear: x, delta, x_out and w rows must start on 16-byte boundaries");
  if (nout && (!aligned(a->y, 16) || a->y_stride % 8 || !aligned(a->h_out, 16) || a->h_out_stride % 8 ||
               (a->res != nullptr && (!aligned(a->res, 16) || a->res_stride % 8))))
    return fail(MCB_ERR_ALIGNMENT, "mcb_linear: with MCB_LINEAR_NORM_OUT the y, res and h_out rows must start "
                "on 16-byte boundaries");
  // every CTA reads all of x (and delta) while others write y and x_out
  if (ranges_overlap(a->y, a->y_stride, a->N, a->x, a->x_stride, a->K, a->R) ||
      ranges_overlap(a->res, a->res_stride, a->N, a->x, a->x_stride, a->K, a->R) ||
      (add && (ranges_overlap(a->x_out, a->x_out_stride, a->K, a->x, a->x_stride, a->K, a->R) ||
               ranges_overlap(a->x_out, a->x_out_stride, a->K, a->delta, a->delta_stride, a->K, a->R) ||
               ranges_overlap(a->y, a->y_stride, a->N, a->delta, a->delta_stride, a->K, a->R) ||
               ranges_overlap(a->y, a->y_stride, a->N, a->x_out, a->x_out_stride, a->K, a->R))))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: y, res and x_out must not overlap x or delta");
  if (nout && (ranges_overlap(a->h_out, a->h_out_stride, a->N, a->x, a->x_stride, a->K, a->R) ||
               ranges_overlap(a->h_out, a->h_out_stride, a->N, a->y, a->y_stride, a->N, a->R) ||
               ranges_overlap(a->h_out, a->h_out_stride, a->N, a->res, a->res_stride, a->N, a->R)))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: h_out must not overlap x, y or res");
  if (a->res != nullptr && a->res != a->y &&
      ranges_overlap(a->y, a->y_stride, a->N, a->res, a->res_stride, a->N, a->R))
    return fail(MCB_ERR_INVALID_ARG, "mcb_linear: res must be y itself or not overlap it");
  pl->panels = a->K / 64;
  pl->norm = norm;
  pl->gated = gated;
  pl->add = add;
  pl->nout = nout;
  if (nout) {
    pl->F = 64;
    pl->rb = kProjNoutRows;
    const int smem = mcb::proj_smem_bytes(64, pl->panels, false, kProjNoutRows);
    if (smem > kMaxSmemOptin)
      return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: K=%d does not fit the shared memory (norm out)", a->K);
    if (!nout_schedulable(a->N / 64, smem))
      return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: the device does not schedule clusters of %d CTAs with %d "
                  "bytes of shared memory (norm out)", a->N / 64, smem);
    return MCB_OK;
  }
  // the narrower feature slice while it keeps the grid within about one CTA per SM (always with
  // delta: its panels leave no room for a wider weight slice)
  // gated: 16 gate and 16 up rows of W a CTA (the epilogue pairs them)
  pl->F = gated ? 32 : (add || (a->N + 15) / 16 <= device_sm_count() + device_sm_count() / 8 ? 16 : 32);
  // a plain product whose 64-row activation block does not fit splits the rows over two CTAs
  pl->rb = (!norm && !gated && mcb::proj_smem_bytes(pl->F, pl->panels, false) > kMaxSmemOptin) ? 32
                                                                                             : mcb::kProjRows;
  if (mcb::proj_smem_bytes(pl->F, pl->panels, add, pl->rb) > kMaxSmemOptin)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_linear: K=%d does not fit the shared memory (%d features a CTA%s)",
                a->K, pl->F, add ? ", with delta" : "");
  return MCB_OK;
}

extern "C" {

int mcb_linear_supported(const mcb_linear_args* a) {
  LinearPlan pl;
  return plan_linear(a, &pl) == MCB_OK ? 1 : 0;
}

int mcb_linear(const mcb_linear_args* a, void* stream) {
  LinearPlan pl;
  const int prc = plan_linear(a, &pl);
  if (prc != MCB_OK) return prc;
  const int F = pl.F, rb = pl.rb, panels = pl.panels;
  const bool norm = pl.norm, gated = pl.gated, add = pl.add, nout = pl.nout;
  if (a->R == 0) return MCB_OK;
  CUtensorMap wm, xm, dm;
  int rc = gated ? encode_rows_map(&wm, a->w, 2ll * a->N, a->K, a->w_stride, F / 2)
                 : encode_rows_map(&wm, a->w, a->N, a->K, a->w_stride, F);
  if (rc != MCB_OK) return rc;
  rc = encode_rows_map(&xm, a->x, a->R, a->K, a->x_stride, rb);
  if (rc != MCB_OK) return rc;
  if (add) {
    rc = encode_rows_map(&dm, a->delta, a->R, a->K, a->delta_stride, mcb::kProjRows);
    if (rc != MCB_OK) return rc;
  } else {
    dm = xm;
  }
  mcb::ProjParams p;
  p.res = static_cast<const uint16_t*>(a->res);
  p.y = static_cast<uint16_t*>(a->y);
  p.x_out = add ? static_cast<uint16_t*>(a->x_out) : nullptr;
  p.h_out = nout ? static_cast<uint16_t*>(a->h_out) : nullptr;
  p.ress = a->res_stride;
  p.ys = a->y_stride;
  p.xos = add ? a->x_out_stride : 0;
  p.hs = nout ? a->h_out_stride : 0;
  p.R = a->R;
  p.N = a->N;
  p.K = a->K;
  p.panels = panels;
  p.vec_out = aligned(a->y, 16) && a->y_stride % 8 == 0 && a->N % 8 == 0 &&
              (a->res == nullptr || (aligned(a->res, 16) && a->res_stride % 8 == 0));
  p.eps = a->eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool pdl = a->pdl != 0;
  if (nout) return launch_proj_nout(wm, xm, p, pdl, st);
  if (gated) return launch_proj<32, false, false, true>(wm, xm, dm, p, pdl, st);
  if (rb == 32)
    return F == 16 ? launch_proj<16, false, false, false, 32>(wm, xm, dm, p, pdl, st)
                   : launch_proj<32, false, false, false, 32>(wm, xm, dm, p, pdl, st);
  return F == 16 ? launch_proj_f<16>(norm, add, wm, xm, dm, p, pdl, st)
                 : launch_proj_f<32>(norm, add, wm, xm, dm, p, pdl, st);
}

int mcb_gated_silu(const mcb_gated_silu_args* a, void* stream) {
  if (a == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_gated_silu: args is NULL");
  if (a->rows < 0 || a->H <= 0 || a->H % 8 != 0)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_gated_silu: H=%d must be a positive multiple of 8", a->H);
  if (a->gate == nullptr || a->up == nullptr || a->out == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_gated_silu: NULL pointer argument");
  if (!aligned(a->gate, 16) || !aligned(a->up, 16) || !aligned(a->out, 16) || a->gate_stride % 8 ||
      a->up_stride % 8 || a->out_stride % 8)
    return fail(MCB_ERR_ALIGNMENT, "mcb_gated_silu: rows must start on 16-byte boundaries");
  if (a->rows == 0) return MCB_OK;
  mcb::GatedActParams p;
  p.gate = static_cast<const uint16_t*>(a->gate);
  p.up = static_cast<const uint16_t*>(a->up);
  p.out = static_cast<uint16_t*>(a->out);
  p.gs = a->gate_stride;
  p.us = a->up_stride;
  p.os = a->out_stride;
  p.rows = a->rows;
  p.H = a->H;
  const long long total = static_cast<long long>(a->rows) * (a->H / 8);
  launch_pdl(mcb::gated_silu_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), p);
  g_launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gated_silu launch");
  return MCB_OK;
}

int mcb_kv_advance(int32_t* cache_seqlens, int32_t B, int32_t n, void* stream) {
  if (cache_seqlens == nullptr || B < 0)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_advance: bad arguments");
  if (B == 0) return MCB_OK;
  launch_pdl(mcb::kv_advance_kernel, dim3((B + 255) / 256), dim3(256), 0, static_cast<cudaStream_t>(stream), cache_seqlens, B, n);
  g_launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_advance launch");
  return MCB_OK;
}

size_t mcb_decode_attn_workspace_size(const mcb_attn_args* a) {
  AttnPlan pl;
  if (plan_attn(a, &pl) != MCB_OK) return 0;
  return pl.ws_bytes;
}

size_t mcb_decode_attn_counter_count(const mcb_attn_args* a) {
  AttnPlan pl;
  if (plan_attn(a, &pl) != MCB_OK) return 0;
  return pl.counter_count;
}

int mcb_decode_attn_fusable(const mcb_attn_args* a) {
  AttnPlan pl;
  if (plan_attn(a, &pl) != MCB_OK) return 0;
  return plan_fusable(a, pl) ? 1 : 0;
}

int mcb_prefill_attn(const mcb_attn_args* a, void* stream) {
  AttnPlan pl;
  int rc = plan_attn(a, &pl);  // shape validation
  if (rc != MCB_OK) return rc;
  if (a->D != 64 && a->D != 128)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_prefill_attn: head_dim %d not supported (64/128)", a->D);
  if ((static_cast<long long>(a->T) + mcb::kPfTile - 1) / mcb::kPfTile * a->B * a->Hq > 0x7fffffffll)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_prefill_attn: grid too large");
  rc = check_attn_pointers(a, "mcb_prefill_attn");
  if (rc != MCB_OK) return rc;
  if (a->B == 0 || a->T == 0) return MCB_OK;
  return run_prefill(a, static_cast<cudaStream_t>(stream));
}

int mcb_decode_attn(const mcb_attn_args* a, void* stream) {
  AttnPlan pl;
  int rc = plan_attn(a, &pl);
  if (rc != MCB_OK) return rc;
  rc = check_attn_pointers(a, "mcb_decode_attn");
  if (rc != MCB_OK) return rc;
  if (pl.ws_bytes > 0 &&
      (a->workspace == nullptr || a->workspace_bytes < pl.ws_bytes || !aligned(a->workspace, 256)))
    return fail(MCB_ERR_WORKSPACE, "mcb_decode_attn: needs %zu bytes of 256-byte aligned workspace, got %zu",
                pl.ws_bytes, a->workspace ? a->workspace_bytes : size_t(0));
  if (pl.counter_count > 0 &&
      (a->counters == nullptr || a->counter_count < pl.counter_count || !aligned(a->counters, 4)))
    return fail(MCB_ERR_WORKSPACE, "mcb_decode_attn: needs %zu zero-initialised int32 counters, got %zu",
                pl.counter_count, a->counters ? a->counter_count : size_t(0));
  if (a->B == 0 || a->T == 0) return MCB_OK;
  return run_attn(a, pl, a->workspace, a->counters, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Allocation-free decode attention (mcb_decode_attn_noalloc): the split partials live in this
// file-scope device array instead of a caller-provided workspace.  In host code the name
// g_noalloc_scratch is only a host-side stand-in; its device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MCB_NOALLOC_SCRATCH_BYTES];

namespace {

int noalloc_scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mcb_decode_attn_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn_noalloc: device ordinal %d >= 64", dev);
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "mcb_decode_attn_noalloc: cudaGetSymbolAddress(scratch)");
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return MCB_OK;
}

}  // namespace

extern "C" {

int mcb_decode_attn_noalloc(const mcb_attn_args* a, void* stream) {
  AttnPlan pl;
  int rc = plan_attn(a, &pl);
  if (rc != MCB_OK) return rc;
  rc = check_attn_pointers(a, "mcb_decode_attn_noalloc");
  if (rc != MCB_OK) return rc;
  const size_t counter_bytes = round256(pl.counter_count * 4);
  if (pl.ws_bytes + counter_bytes > MCB_NOALLOC_SCRATCH_BYTES) {
    if (pl.mode == kModePersistent)
      return fail(MCB_ERR_WORKSPACE,
                  "mcb_decode_attn_noalloc: %d persistent CTAs and %zu row groups need %zu bytes of "
                  "scratch, more than the %u-byte static scratch; pass fewer CTAs (a smaller "
                  "num_ctas > 0) or use mcb_decode_attn with a workspace",
                  pl.grid, pl.counter_count, pl.ws_bytes + counter_bytes, MCB_NOALLOC_SCRATCH_BYTES);
    return fail(MCB_ERR_WORKSPACE,
                "mcb_decode_attn_noalloc: %d key splits of %lld row groups need %zu bytes of scratch, "
                "more than the %u-byte static scratch; pass fewer splits (num_ctas < 0 of a smaller "
                "magnitude) or use mcb_decode_attn with a workspace",
                pl.nsplit, static_cast<long long>(a->B) * a->Hkv * pl.nqb, pl.ws_bytes + counter_bytes, MCB_NOALLOC_SCRATCH_BYTES);
  }
  if (a->B == 0 || a->T == 0) return MCB_OK;
  void* scratch = nullptr;
  rc = noalloc_scratch_ptr(&scratch);
  if (rc != MCB_OK) return rc;
  // The arrival counters (after the partials) must start at zero; the scratch keeps whatever the
  // last call left there.
  int32_t* counters = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + pl.ws_bytes);
  if (counter_bytes > 0) {
    cudaError_t e = cudaMemsetAsync(counters, 0, counter_bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "mcb_decode_attn_noalloc: clearing the counters");
  }
  return run_attn(a, pl, scratch, counters, static_cast<cudaStream_t>(stream));
}

int mcb_device_error(int32_t* code, void* stream) {
  if (code == nullptr) return fail(MCB_ERR_INVALID_ARG, "mcb_device_error: code is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, mcb::g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "mcb_device_error read");
  const int zero = 0;
  e = cudaMemcpyToSymbolAsync(mcb::g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "mcb_device_error clear");
  *code = value;
  return MCB_OK;
}

}  // extern "C"
