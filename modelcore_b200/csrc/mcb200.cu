// C-ABI entry points of libmcb200 (declared in include/mcb200.h): host-side validation, launch
// planning, TMA descriptor encoding and the kernel launches for the KV-cache decode path.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mcb200.h"
#include "common.cuh"
#include "decode_attn.cuh"
#include "kv_append.cuh"
#include "kv_copy.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

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

// ------------------------------------------------------------------------------------------
// Decode attention planning.
struct AttnPlan {
  int D, nqt, tk, rows, nqb, nsplit, tps;
  size_t part_o_bytes, part_lse_bytes, ws_bytes;
};

constexpr int kKPW = 16;

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
  const int G = a->Hq / a->Hkv;
  pl->D = a->D;
  const int rows_total = a->T * G;
  pl->nqt = (rows_total <= 8 || a->D == 256) ? 1 : 2;
  pl->rows = 8 * pl->nqt;
  pl->tk = kKPW * mcb::kAttnConsumerWarps;
  pl->nqb = rows_total > 0 ? (rows_total + pl->rows - 1) / pl->rows : 0;
  const long long cap_keys =
      a->window >= 0 ? std::min<long long>(a->Tmax, static_cast<long long>(a->window) + a->T)
                     : a->Tmax;
  const int max_tiles = static_cast<int>((cap_keys + pl->tk - 1) / pl->tk) + 1;
  long long base = static_cast<long long>(a->B) * a->Hkv * pl->nqb;
  int nsplit;
  if (a->num_splits > 0) {
    nsplit = std::min(a->num_splits, max_tiles);
  } else {
    const long long target = 4ll * device_sm_count();
    nsplit = base > 0 ? static_cast<int>((target + base - 1) / base) : 1;
    nsplit = std::max(1, std::min(nsplit, std::max(1, max_tiles / 4)));
  }
  pl->tps = (max_tiles + nsplit - 1) / nsplit;
  pl->nsplit = (max_tiles + pl->tps - 1) / pl->tps;
  if (base * pl->nsplit > 0x7fffffffll)
    return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: grid too large");
  const size_t rows_out = static_cast<size_t>(a->B) * a->T * a->Hq;
  if (pl->nsplit > 1) {
    pl->part_o_bytes = (rows_out * pl->nsplit * a->D * 4 + 255) & ~size_t(255);
    pl->part_lse_bytes = (rows_out * pl->nsplit * 4 + 255) & ~size_t(255);
  } else {
    pl->part_o_bytes = pl->part_lse_bytes = 0;
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

template <int D, int NQT>
int launch_attn_variant(const AttnPlan& pl, const CUtensorMap& km, const CUtensorMap& vm,
                        const mcb::AttnParams& prm, cudaStream_t st) {
  constexpr int STAGES = D >= 128 ? 3 : 4;
  using Cfg = mcb::AttnConfig<D, NQT, kKPW, STAGES>;
  static std::atomic<uint64_t> done{0};
  auto kern = mcb::decode_attn_kernel<D, NQT, kKPW, STAGES>;
  cudaError_t e = ensure_smem(kern, Cfg::SMEM_BYTES, done);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_attn)");
  const long long grid = static_cast<long long>(prm.B) * prm.Hkv * pl.nqb * pl.nsplit;
  kern<<<static_cast<unsigned>(grid), mcb::kAttnThreads, Cfg::SMEM_BYTES, st>>>(km, vm, prm);
  g_launches++;
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode_attn launch");
  if (pl.nsplit > 1) {
    const long long rows = static_cast<long long>(prm.B) * prm.T * prm.Hq;
    mcb::decode_attn_combine_kernel<D><<<static_cast<unsigned>((rows + 3) / 4), 128, 0, st>>>(prm);
    g_launches++;
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn_combine launch");
  }
  return MCB_OK;
}

}  // namespace

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
  p.total_vectors = static_cast<long long>(a->B) * a->T * (p.nq + 2 * p.nk);
  if (p.total_vectors == 0) return MCB_OK;
  const long long blocks = (p.total_vectors + mcb::kAppendWarpsPerBlock - 1) / mcb::kAppendWarpsPerBlock;
  if (blocks > 0x7fffffffll) return fail(MCB_ERR_UNSUPPORTED, "mcb_kv_append_rope: grid too large");
  mcb::kv_append_rope_kernel<<<static_cast<unsigned>(blocks), mcb::kAppendWarpsPerBlock * 32, 0,
                               static_cast<cudaStream_t>(stream)>>>(p);
  g_launches++;
  cudaError_t e = cudaGetLastError();
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

int mcb_kv_advance(int32_t* cache_seqlens, int32_t B, int32_t n, void* stream) {
  if (cache_seqlens == nullptr || B < 0)
    return fail(MCB_ERR_INVALID_ARG, "mcb_kv_advance: bad arguments");
  if (B == 0) return MCB_OK;
  mcb::kv_advance_kernel<<<(B + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(cache_seqlens, B, n);
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

int mcb_decode_attn(const mcb_attn_args* a, void* stream) {
  AttnPlan pl;
  int rc = plan_attn(a, &pl);
  if (rc != MCB_OK) return rc;
  if (a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr || a->out == nullptr ||
      a->cache_seqlens == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_decode_attn: NULL pointer argument");
  if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16) || !aligned(a->q, 16) ||
      !aligned(a->out, 16))
    return fail(MCB_ERR_ALIGNMENT, "mcb_decode_attn: q, out and cache pointers must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (a->q_stride[i] < 0 || (a->q_stride[i] % 8) != 0)
      return fail(MCB_ERR_ALIGNMENT, "mcb_decode_attn: q strides must be non-negative multiples of 8 elements");
  if (pl.ws_bytes > 0 && (a->workspace == nullptr || a->workspace_bytes < pl.ws_bytes || !aligned(a->workspace, 256)))
    return fail(MCB_ERR_WORKSPACE, "mcb_decode_attn: needs %zu bytes of 256-byte aligned workspace, got %zu",
                pl.ws_bytes, a->workspace ? a->workspace_bytes : size_t(0));
  if (a->B == 0 || a->T == 0) return MCB_OK;

  CUtensorMap km, vm;
  rc = encode_cache_map(&km, a->k_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;
  rc = encode_cache_map(&vm, a->v_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;

  mcb::AttnParams p;
  p.q = static_cast<const uint16_t*>(a->q);
  for (int i = 0; i < 3; ++i) p.qs[i] = a->q_stride[i];
  p.cache_seqlens = a->cache_seqlens;
  p.out = static_cast<uint16_t*>(a->out);
  p.part_o = pl.nsplit > 1 ? static_cast<float*>(a->workspace) : nullptr;
  p.part_lse = pl.nsplit > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(a->workspace) + pl.part_o_bytes)
                             : nullptr;
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
  p.nqb = pl.nqb;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->D) {
    case 16: return pl.nqt == 1 ? launch_attn_variant<16, 1>(pl, km, vm, p, st) : launch_attn_variant<16, 2>(pl, km, vm, p, st);
    case 32: return pl.nqt == 1 ? launch_attn_variant<32, 1>(pl, km, vm, p, st) : launch_attn_variant<32, 2>(pl, km, vm, p, st);
    case 64: return pl.nqt == 1 ? launch_attn_variant<64, 1>(pl, km, vm, p, st) : launch_attn_variant<64, 2>(pl, km, vm, p, st);
    case 128: return pl.nqt == 1 ? launch_attn_variant<128, 1>(pl, km, vm, p, st) : launch_attn_variant<128, 2>(pl, km, vm, p, st);
    case 256: return launch_attn_variant<256, 1>(pl, km, vm, p, st);
  }
  return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn: head_dim %d", a->D);
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
  if (a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr || a->out == nullptr ||
      a->cache_seqlens == nullptr)
    return fail(MCB_ERR_INVALID_ARG, "mcb_decode_attn_noalloc: NULL pointer argument");
  if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16) || !aligned(a->q, 16) ||
      !aligned(a->out, 16))
    return fail(MCB_ERR_ALIGNMENT,
                "mcb_decode_attn_noalloc: q, out and cache pointers must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (a->q_stride[i] < 0 || (a->q_stride[i] % 8) != 0)
      return fail(MCB_ERR_ALIGNMENT,
                  "mcb_decode_attn_noalloc: q strides must be non-negative multiples of 8 elements");
  if (pl.ws_bytes > MCB_NOALLOC_SCRATCH_BYTES)
    return fail(MCB_ERR_WORKSPACE,
                "mcb_decode_attn_noalloc: this shape's %d-way split needs %zu bytes of scratch, more "
                "than the %u-byte static scratch; pass a smaller num_splits or use mcb_decode_attn "
                "with a workspace",
                pl.nsplit, pl.ws_bytes, MCB_NOALLOC_SCRATCH_BYTES);
  if (a->B == 0 || a->T == 0) return MCB_OK;
  void* scratch = nullptr;
  if (pl.ws_bytes > 0) {
    rc = noalloc_scratch_ptr(&scratch);
    if (rc != MCB_OK) return rc;
  }

  CUtensorMap km, vm;
  rc = encode_cache_map(&km, a->k_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;
  rc = encode_cache_map(&vm, a->v_cache, a->D, a->Hkv, a->Tmax, a->B, pl.tk);
  if (rc != MCB_OK) return rc;

  mcb::AttnParams p;
  p.q = static_cast<const uint16_t*>(a->q);
  for (int i = 0; i < 3; ++i) p.qs[i] = a->q_stride[i];
  p.cache_seqlens = a->cache_seqlens;
  p.out = static_cast<uint16_t*>(a->out);
  p.part_o = pl.nsplit > 1 ? static_cast<float*>(scratch) : nullptr;
  p.part_lse = pl.nsplit > 1
                   ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + pl.part_o_bytes)
                   : nullptr;
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
  p.nqb = pl.nqb;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->D) {
    case 16: return pl.nqt == 1 ? launch_attn_variant<16, 1>(pl, km, vm, p, st) : launch_attn_variant<16, 2>(pl, km, vm, p, st);
    case 32: return pl.nqt == 1 ? launch_attn_variant<32, 1>(pl, km, vm, p, st) : launch_attn_variant<32, 2>(pl, km, vm, p, st);
    case 64: return pl.nqt == 1 ? launch_attn_variant<64, 1>(pl, km, vm, p, st) : launch_attn_variant<64, 2>(pl, km, vm, p, st);
    case 128: return pl.nqt == 1 ? launch_attn_variant<128, 1>(pl, km, vm, p, st) : launch_attn_variant<128, 2>(pl, km, vm, p, st);
    case 256: return launch_attn_variant<256, 1>(pl, km, vm, p, st);
  }
  return fail(MCB_ERR_UNSUPPORTED, "mcb_decode_attn_noalloc: head_dim %d", a->D);
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
