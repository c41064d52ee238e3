/*
 * mcb200.h -- C ABI of the B200 (sm_100a) KV-cache decode path for modelcore.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, returns an int status
 * (MCB_OK == 0, a negative mcb_status otherwise) and enqueues its work on the caller's CUDA
 * stream (`stream` is a cudaStream_t passed as void*; NULL means the legacy default stream).
 * Nothing here allocates device memory, synchronises the stream or keeps a pointer past the
 * call, so every launch entry point can be recorded into a CUDA graph.  A failed host-side check
 * returns before anything is enqueued; mcb_last_error() then returns the message (per thread).
 *
 * Tensor conventions (all device pointers, bf16 = IEEE bfloat16 stored as uint16):
 *   cache slot   (B, Tmax, Hkv, D) contiguous bf16 -- one slot of modelcore's
 *                (n_slots, B, Tmax, Hkv, D) KVCache.k_cache / v_cache, modelcore/cache.py:22-23.
 *                Base 16-byte aligned; D a multiple of 16 in [16, 256] for decode attention.
 *   q / k / v    (B, T, H, D) bf16 with arbitrary element strides for (b, t, h) and unit
 *                stride on d (the view c_q(x).view(B, T, H, D) of modelcore/components/attention.py:139-143).
 *   cache_seqlens (B,) int32 -- KVCache.cache_seqlens, modelcore/cache.py:25.  Row b's new
 *                tokens sit at positions [cache_seqlens[b], cache_seqlens[b] + T).
 *
 * The reference interfaces each entry point replaces are cited beside it (paths relative to
 * the modelcore project root).
 */
#ifndef MCB200_H
#define MCB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MCB_ABI_VERSION 9

typedef enum {
  MCB_OK = 0,
  MCB_ERR_INVALID_ARG = -1,   /* a NULL pointer, a negative or inconsistent size         */
  MCB_ERR_UNSUPPORTED = -2,   /* a head_dim / group shape the kernels are not built for  */
  MCB_ERR_ALIGNMENT = -3,     /* a pointer or stride that breaks the 16-byte layout rule */
  MCB_ERR_WORKSPACE = -4,     /* workspace missing or smaller than required              */
  MCB_ERR_CUDA = -5           /* a CUDA runtime / driver call failed                     */
} mcb_status;

/* Bits of mcb_append_args.flags. */
#define MCB_APPEND_ROTATE_Q 1u  /* q_out = 1.2 * rms_norm(rope(q))   (attention.py:147-150, :156-158) */
#define MCB_APPEND_ROTATE_K 2u  /* k' = 1.2 * rms_norm(rope(k)) before it is written             */
#define MCB_APPEND_WRITE_KV 4u  /* write k' (or raw k) and v at rows' positions, flash_attn.py:337-346 */

/* Version of this ABI (MCB_ABI_VERSION of the library that was loaded). */
int mcb_abi_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to len) into buf.
 * Returns the full message length. */
int mcb_last_error(char* buf, size_t len);

/* ---------------------------------------------------------------------------------------------
 * Piece 1: per-step K/V append fused with rotary, QK-norm and the 1.2 scale.
 * Replaces, for one attention layer on the decode path:
 *   RotaryEmbedding._cos_sin / forward / apply_to_q   modelcore/components/rotary.py:43-81
 *   apply_rotary_emb                                  modelcore/components/rope.py:4-12
 *   norm(q), norm(k) (F.rms_norm), q*1.2, k*1.2       modelcore/components/attention.py:147-150
 *   the cache insert in flash_attn_with_kvcache      modelcore/kernels/flash_attn.py:337-346
 * Rounding follows the reference op by op: every rope product and sum is rounded to bf16; the
 * norm accumulates in fp32 and rounds once; the scale multiplies in fp32 and rounds once.
 * Does NOT advance cache_seqlens (Model.forward does that once per forward, model.py:99-100).
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;              /* (B,T,Hq,D)  bf16, read when ROTATE_Q                       */
  const void* k;              /* (B,T,Hkv,D) bf16, read when ROTATE_K or WRITE_KV           */
  const void* v;              /* (B,T,Hkv,D) bf16, read when WRITE_KV                       */
  int64_t q_stride[3];        /* element strides of q for b, t, h                           */
  int64_t k_stride[3];
  int64_t v_stride[3];
  void* q_out;                /* (B,T,Hq,D) bf16 contiguous, written when ROTATE_Q          */
  void* k_cache;              /* cache slot (B,Tmax,Hkv,D), written when WRITE_KV           */
  void* v_cache;
  const int32_t* cache_seqlens; /* (B,) positions before this step                          */
  const void* cos;            /* (rot_len, D/2) bf16 rotary table rows, rope.py:15-27       */
  const void* sin;
  int32_t B, T, Hq, Hkv, D, Tmax, rot_len;
  float eps;                  /* rms_norm epsilon as fp32 (torch: fp32 machine eps when None) */
  float scale;                /* 1.2f in modelcore                                          */
  uint32_t flags;             /* MCB_APPEND_* bits                                          */
  int32_t ring;               /* 0: position p at index p; 1: the slot is a ring of Tmax
                                 positions, position p at index p % Tmax                    */
  /* fp8 cache (k_scale != NULL): k_cache / v_cache hold float8 e4m3 bytes, one per element, and
     each (row, position, kv head) vector its scale at k_scale / v_scale[(b * Hkv + h) *
     scale_tmax + index] (fp32, scale_tmax >= Tmax and a multiple of 64): the vector of bf16
     values x a bf16 cache would hold is stored as e4m3(x * (448 / amax)) rounded to nearest
     even and saturated, with scale amax / 448 (amax = max |x|; 0 stores zeros and scale 0).
     Needs D = 64 or 128 and 16-byte aligned rows. */
  float* k_scale;
  float* v_scale;
  int32_t scale_tmax;
} mcb_append_args;

int mcb_kv_append_rope(const mcb_append_args* args, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Piece 2: prefill -> broadcast cache copy, and the single-row copy.
 * Replaces KVCache.prefill   (modelcore/cache.py:75-90: k/v slice copy + cache_seqlens.fill_)
 *          KVCache.prefill_row (modelcore/cache.py:92-119: row copy + cache_seqlens[row] = P)
 * Copies positions [0, n_pos) of source row src_row in every slot into destination rows
 * [dst_row_begin, dst_row_begin + dst_row_count); the source is read once and written to every
 * destination row.  When dst_seqlens is not NULL, dst_seqlens[row] = n_pos for those rows in
 * the same launch.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  void* dst_k;  void* dst_v;           /* (n_slots, dst_batch, dst_tmax, Hkv, D) bf16          */
  const void* src_k; const void* src_v;/* (n_slots, src_batch, src_tmax, Hkv, D) bf16          */
  int32_t n_slots;
  int32_t src_batch, src_row, src_tmax;
  int32_t dst_batch, dst_row_begin, dst_row_count, dst_tmax;
  int32_t n_pos;                       /* positions copied                                     */
  int32_t row_elems;                   /* Hkv * D                                              */
  int32_t* dst_seqlens;                /* optional (dst_batch,) int32                          */
} mcb_copy_args;

int mcb_kv_copy_rows(const mcb_copy_args* args, void* stream);

/* cache_seqlens[b] += n for every row.  Replaces KVCache.advance's device half,
 * modelcore/cache.py:71 (the host mirror, :72-73, stays with the caller). */
int mcb_kv_advance(int32_t* cache_seqlens, int32_t B, int32_t n, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Piece 3: decode attention over the cache (flash-decode on the tensor cores).
 * Replaces the attention half of flash_attn_with_kvcache's SDPA path,
 * modelcore/kernels/flash_attn.py:348-366 with _sdpa_attention (:203-244) and
 * _ragged_decode_mask (:246-264):
 *   out[b,t,h] = softmax_c(q[b,t,h] . K[b,c,h/G] * softmax_scale) . V[b,c,h/G]
 * over keys c with c <= L_b + t and (window < 0 or L_b + t - c <= window), L_b = cache_seqlens[b]
 * and G = Hq / Hkv (SDPA's enable_gqa mapping q head h -> kv head h / G).  The new tokens'
 * keys/values must already be in the cache (mcb_kv_append_rope with WRITE_KV).
 * A row group (one row's G grouped q heads of one kv head) shares every K/V tile, streamed by
 * TMA through a shared-memory ring.  Two launch plans, same results up to fp32 summation order:
 *  - persistent: all row groups' key tiles form one sequence that a resident grid divides
 *    evenly on the device, from cache_seqlens (no host knowledge of the lengths); row groups
 *    cut between CTAs are merged by the last CTA to finish them.  Chosen for rows that can hold
 *    more than 2048 keys (min(Tmax, window + T)) when there are more than 128 row groups.
 *  - split: one CTA per row group and key split.  Up to 8 splits of a row group form a
 *    thread-block cluster and merge through distributed shared memory; more splits write
 *    partials that a second kernel merges.  Chosen for shorter rows, where the persistent plan's
 *    fixed costs do not pay off, and for long rows of at most 128 row groups (2-16 splits).
 *  - prefill (num_ctas == 0, T >= 64, D 64 or 128): 128-query x 128-key tiles on the tcgen05
 *    tensor cores with TMEM accumulators (mcb_prefill_attn below); no workspace or counters.
 * The split plan is launched with programmatic stream serialization and reads cache_seqlens and
 * the keys and values below each row's cache_seqlens before it waits for the kernel ahead of it in
 * the stream: that one kernel must not write them (every kernel before it has completed when
 * this one starts, since the library's kernels let their successor start only after their own
 * wait).  The new tokens' positions are read after the wait.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;              /* (B,T,Hq,D) bf16                                            */
  int64_t q_stride[3];        /* element strides of q for b, t, h                           */
  const void* k_cache;        /* cache slot (B,Tmax,Hkv,D) bf16                             */
  const void* v_cache;
  const int32_t* cache_seqlens;
  void* out;                  /* (B,T,Hq,D) bf16 contiguous                                 */
  int32_t B, T, Hq, Hkv, D, Tmax;
  int32_t window;             /* left window; < 0 = full context                            */
  float softmax_scale;        /* 1/sqrt(D) in modelcore (SDPA default)                      */
  int32_t num_ctas;           /* 0: choose the plan; > 0: persistent grid of that many CTAs
                                 (rounded down to whole groups of Hkv); < 0: split plan with
                                 -num_ctas key splits per row group                         */
  void* workspace;            /* partials: mcb_decode_attn_workspace_size() bytes, no
                                 initialisation needed                                      */
  size_t workspace_bytes;
  int32_t* counters;          /* mcb_decode_attn_counter_count() int32 arrival counters, one
                                 per row group: zero before the first call, and every
                                 completed call leaves the ones it used at zero again, so one
                                 array serves every call of a stream (of any shape that fits)*/
  size_t counter_count;
  int32_t ring;               /* 1: the slot is a ring of Tmax positions (p at p % Tmax);
                                 needs window >= 0, window + T <= Tmax and Tmax a multiple of
                                 128, so every visible key is resident and no key tile wraps */
  /* fp8 cache (k_scale != NULL): e4m3 k_cache / v_cache with per-vector scales as written by
     mcb_kv_append_rope (layout (B, Hkv, scale_tmax) fp32, zero where never written); keys are
     read as e4m3 * scale.  The split plan only (D = 64 or 128). */
  const float* k_scale;
  const float* v_scale;
  int32_t scale_tmax;
  /* fused append (fuse_append = 1; T = 1, a bf16 slot, D = 64 or 128, and the split or the
     persistent plan -- mcb_decode_attn_fusable): q is the RAW query projection (B, 1, Hq, D);
     the kernel does what
     mcb_kv_append_rope does for this step (rope at position cache_seqlens[b] from rot_cos /
     rot_sin, rms_norm with norm_eps, x qk_scale, bit for bit) on the query and, with k_new /
     v_new, on the new key, writes the key and value into k_cache / v_cache at that position,
     and attends over the slot including them -- one launch instead of two.  k_new = v_new = NULL:
     a layer that reads another layer's slot (only q is rotated).  cache_seqlens is not advanced. */
  int32_t fuse_append;
  const void* k_new;          /* (B, 1, Hkv, D) bf16 at k_new_stride (elements)               */
  const void* v_new;
  int64_t k_new_stride[3];
  int64_t v_new_stride[3];
  const void* rot_cos;        /* (rot_len, D/2) bf16 rotary tables, 16-byte aligned           */
  const void* rot_sin;
  int32_t rot_len;
  int32_t rotate_k;           /* 1: the key is roped, normed and scaled like q; 0: raw insert */
  float norm_eps;
  float qk_scale;
} mcb_attn_args;

/* Bytes of workspace mcb_decode_attn needs for its partial results (0: none): persistent plan,
 * two slots per CTA, ctas * 2 * rows * (D + 1) * 4; split plan with s > 8 splits,
 * B * T * Hq * s * (D + 1) * 4 (2 to 8 splits merge in a cluster and need none); in two 256-byte-rounded parts (rows = 8 or 16).  It does not
 * depend on the row lengths.  Calls that can overlap on the GPU need separate workspaces and
 * counter arrays. */
size_t mcb_decode_attn_workspace_size(const mcb_attn_args* args);

/* int32 arrival counters mcb_decode_attn needs: one per row group,
 * B * ceil(T * Hq / Hkv / rows) * Hkv, for the persistent plan; 0 for the split plan. */
size_t mcb_decode_attn_counter_count(const mcb_attn_args* args);

/* 1 when mcb_decode_attn can run this call with fuse_append = 1 (one new token a row, a bf16
 * slot, D = 64 or 128, and the split or the persistent plan -- not the prefill plan, which
 * num_ctas = 0 picks for T >= 64), else 0 -- the caller then runs mcb_kv_append_rope and
 * mcb_decode_attn.  Decided on the host from
 * the shapes alone (no device read).  Not in the reference, whose append and attention are two
 * calls (kernels/flash_attn.py:306-366). */
int mcb_decode_attn_fusable(const mcb_attn_args* args);

int mcb_decode_attn(const mcb_attn_args* args, void* stream);

/* The prefill plan on its own, for any T >= 1: the attention of flash_attn_with_kvcache with
 * T_new new tokens per row (modelcore/kernels/flash_attn.py:348-366 through _sdpa_attention,
 * :203-244, whose dense causal mask :214-215 is the ragged mask with every L_b = 0).  One CTA
 * per (row, q head, 128-query tile): S = Q K^T and O += P V as tcgen05.mma into TMEM, online
 * softmax in fp32 between them, K/V tiles of 128 keys by TMA.  head_dim 64 or 128; q strides
 * multiples of 8 elements; num_ctas, workspace and counters are ignored. */
int mcb_prefill_attn(const mcb_attn_args* args, void* stream);

/* mcb_decode_attn for callers that cannot allocate device memory.  No counterpart in the
 * reference: modelcore allocates through torch and has no such caller.
 *
 * Some hosts hand this library only the tensors they already own -- a serving engine that has
 * carved all of HBM into its own pools up front, or a foreign-language binding with no device
 * allocator at hand -- and cannot produce the workspace mcb_decode_attn asks for; a cudaMalloc
 * of their own inside a decode step would also synchronise the device.  This entry point keeps
 * the partials and arrival counters in a static device array compiled into the library instead:
 * MCB_NOALLOC_SCRATCH_BYTES (8 MiB) per GPU, held by every GPU that loads the library until the
 * process exits.  args->workspace, workspace_bytes, counters and counter_count are ignored; a
 * call whose partials and counters need more than that (workspace_size + 4 * counter_count,
 * rounded to 256 bytes, > the limit) is rejected with MCB_ERR_WORKSPACE before anything is
 * enqueued -- lower num_ctas, or use mcb_decode_attn.
 * Nothing is allocated: no cudaMalloc, no cudaFree, no allocating library call.
 *
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current, which may load the library's kernels); make that first call before any
 * stream capture on the device.  The address is kept per device ordinal for the life of the
 * process and belongs to the device's primary context: after cudaDeviceReset on that device, or
 * with a non-primary driver context current on it, the kept address is stale, so a process that
 * resets a device or runs its own driver contexts must not call this entry point on that device
 * afterwards.  Every call on a device shares the one array, so calls whose
 * kernels can overlap on the GPU (other streams, other host threads) race on it: serialise them
 * on one stream.  Of the array only the arrival counters must start at zero, and each call
 * clears the ones it uses first (cudaMemsetAsync on the caller's stream, no allocation); every
 * partial a call reads is written earlier in the same call. */
#define MCB_NOALLOC_SCRATCH_BYTES (8u << 20)
int mcb_decode_attn_noalloc(const mcb_attn_args* args, void* stream);

/* ---------------------------------------------------------------------------------------------
 * The decode step either side of attention (one launch each, any number of rows):
 *
 * mcb_add_rms_norm: x_out = x + delta; h_out = rms_norm(x_out) (delta NULL: h_out = rms_norm(x)).
 * Replaces the residual add of Block.forward followed by the next norm() call,
 * modelcore/components/block.py:57-59 with RMSNorm.forward, modelcore/components/norm.py:43-44.
 * The add rounds once to bf16; the norm accumulates in fp32 and rounds once (eps as for
 * mcb_append_args).  x_out may alias x.  C a multiple of 8, at most 4096; rows 16-byte aligned.
 *
 * mcb_gated_silu: out = silu(gate) * up, silu in fp32 rounded to bf16, product rounded to bf16.
 * Replaces GatedMLP.forward's act(gate_proj(x)) * up_proj(x) for activation "silu",
 * modelcore/components/mlp.py:89-90.  H a multiple of 8; rows 16-byte aligned.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* x;              /* (rows, C) bf16 residual stream                             */
  const void* delta;          /* (rows, C) bf16 to add, or NULL                             */
  void* x_out;                /* (rows, C) bf16 x + delta (NULL when delta is NULL)         */
  void* h_out;                /* (rows, C) bf16 rms_norm(x + delta)                         */
  int64_t x_stride, delta_stride, x_out_stride, h_stride;  /* row strides, elements          */
  int32_t rows, C;
  float eps;
} mcb_add_norm_args;

int mcb_add_rms_norm(const mcb_add_norm_args* args, void* stream);

typedef struct {
  const void* gate;           /* (rows, H) bf16                                             */
  const void* up;             /* (rows, H) bf16                                             */
  void* out;                  /* (rows, H) bf16                                             */
  int64_t gate_stride, up_stride, out_stride;  /* row strides, elements                     */
  int32_t rows, H;
} mcb_gated_silu_args;

int mcb_gated_silu(const mcb_gated_silu_args* args, void* stream);

/* mcb_embed_rms_norm: x_out = rms_norm(table[ids[r]]); h_out = rms_norm(x_out) (h_out optional).
 * Replaces TokenEmbedding.forward without smear (wte lookup + norm,
 * modelcore/components/embedding.py:71-75) followed by the first Block's norm (block.py:57).
 * An id outside [0, V) sets device error 4 and writes zeros (torch raises a device assert).
 * Same C and alignment rules as mcb_add_rms_norm; ids is int64. */
typedef struct {
  const int64_t* ids;         /* (rows,) token ids                                          */
  const void* table;          /* (V, C) bf16 embedding table                                */
  void* x_out;                /* (rows, C) bf16                                             */
  void* h_out;                /* (rows, C) bf16, or NULL                                    */
  int64_t table_stride, x_stride, h_stride;  /* row strides, elements                       */
  int64_t V;
  int32_t rows, C;
  float eps;
} mcb_embed_args;

int mcb_embed_rms_norm(const mcb_embed_args* args, void* stream);

/* mcb_softcap_argmax: out[r, j] = cap * tanh(float(logits[r, j]) * (1 / cap)) for j < V (cap <= 0:
 * no cap; the reciprocal rounded to fp32, as torch's CUDA division by a Python number computes it), argmax[r] = the first index of the row's maximum (NaN counts as the maximum).  Replaces
 * LMHead.forward's crop, .float() and softcap (modelcore/components/unembedding.py:52-56) and the
 * greedy branch of sample_next_token (modelcore/generate.py:23-24).  out or argmax may be NULL.
 * logits rows may be padded (logits_stride >= V).  argmax_stride lets the ids feed a (B, 1)
 * token column directly. */
typedef struct {
  const void* logits;         /* (rows, >= V) bf16                                          */
  float* out;                 /* (rows, V) fp32, or NULL                                    */
  int64_t* argmax;            /* (rows,) int64 at argmax_stride, or NULL                    */
  int64_t logits_stride, out_stride, argmax_stride;
  int32_t rows, V;
  float softcap;
} mcb_softcap_args;

int mcb_softcap_argmax(const mcb_softcap_args* args, void* stream);

/* mcb_sample: one token per row from fp32 logits, sample_next_token (modelcore/generate.py:19-34)
 * for temperature > 0: with 1 <= top_k < V the top_k largest logits (ties by ascending index),
 * divided by the temperature, softmax, one draw; otherwise softmax over the whole row, one draw.
 * Above 1024 candidates the weights are fixed-point (2^-40 of the largest), which moves the
 * distribution by at most k * 2^-41 of the total.  The draw is the inverse CDF at u = uniforms[r] in [0, 1) (candidates in
 * descending-logit order, or index order for the whole row), so it is a deterministic function of
 * (logits, u) with the reference's distribution over u.  temperature == 0 is the greedy pick:
 * call with top_k = 1 (any temperature > 0) or use mcb_softcap_argmax. */
typedef struct {
  const float* logits;        /* (rows, >= V) fp32                                          */
  const float* uniforms;      /* (rows,) in [0, 1)                                          */
  int64_t* out;               /* (rows,) int64 at out_stride                                */
  int64_t logits_stride, out_stride;
  int32_t rows, V, top_k;
  float temperature;          /* > 0                                                        */
} mcb_sample_args;

int mcb_sample(const mcb_sample_args* args, void* stream);

/* mcb_linear: Y = X W^T (F.linear without bias, modelcore/components/linear.py:14) for the
 * decode step's few rows, with the Block's elementwise ops around the projection fused in:
 *   flags & MCB_LINEAR_NORM   Y = rms_norm(X, eps) W^T, the norm without weight
 *                             (modelcore/components/norm.py:43-44) -- the bits of
 *                             mcb_add_rms_norm's h; K <= 1024;
 *   ... and delta != NULL     X' = bf16(X + delta) is written to x_out first and normed
 *                             (the residual add of the previous block's MLP; K <= 768);
 *   res != NULL               Y = bf16(res + bf16(X W^T)): the residual add after c_proj
 *                             (modelcore/components/block.py:58); res may be Y (in place).
 *   flags & MCB_LINEAR_GATED  W is the packed [Wg; Wu] of 2N rows and Y (R, N) =
 *                             bf16(bf16(silu(bf16(X Wg^T))) * bf16(X Wu^T)): GatedMLP's gate|up
 *                             projection with act(gate) * up for act "silu"
 *                             (modelcore/components/mlp.py:89-90) -- the bits of mcb_gated_silu
 *                             over the plain projection; no norm, delta or res; N % 16 == 0.
 *   flags & MCB_LINEAR_NORM_OUT  also h_out = rms_norm(Y, eps) (R, N): c_proj's residual add
 *                             and the Block's next norm (modelcore/components/block.py:58-59)
 *                             in one launch -- the bits of mcb_linear then mcb_add_rms_norm
 *                             over Y.  The CTAs of one output row form a thread-block cluster of
 *                             N / 64 (64 features each), whose per-row sums of squares meet in
 *                             distributed shared memory; N a multiple of 64, at most 1024; y,
 *                             res and h_out rows 16-byte aligned; no other flag.  Not in the
 *                             reference, whose residual add and norm are separate torch ops.
 * X, delta, x_out (R, K), W (N, K) as nn.Linear stores it, Y and res (R, N), bf16, fp32
 * accumulation.  R <= 64, K a multiple of 64, x / delta / x_out / w rows 16-byte aligned; Y, res
 * and x_out must not overlap X or delta.  Every CTA takes 16 or 32 output features and all of K:
 * its W slice and the activation panels arrive by TMA, warp-level tensor-core MMAs (mma.sync)
 * split K over the CTA's warps.  With pdl != 0 the kernel is launched with programmatic stream
 * serialization: the W slice is requested while the previous kernel in the stream finishes; the
 * activations are read only after that kernel completed. */
#define MCB_LINEAR_NORM 1
#define MCB_LINEAR_GATED 2
#define MCB_LINEAR_NORM_OUT 4

typedef struct {
  const void* x;              /* (R, K) bf16                                                */
  const void* w;              /* (N, K) bf16                                                */
  void* y;                    /* (R, N) bf16                                                */
  const void* res;            /* (R, N) bf16 residual, or NULL                              */
  const void* delta;          /* (R, K) bf16 added to x before the norm, or NULL            */
  void* x_out;                /* (R, K) bf16: x + delta (with delta)                        */
  int64_t x_stride, w_stride, y_stride, res_stride, delta_stride, x_out_stride;  /* elements */
  int32_t R, N, K;
  int32_t flags;              /* MCB_LINEAR_NORM, MCB_LINEAR_GATED or MCB_LINEAR_NORM_OUT   */
  float eps;                  /* the norm's eps                                             */
  int32_t pdl;
  void* h_out;                /* (R, N) bf16: rms_norm(Y) (MCB_LINEAR_NORM_OUT), or NULL    */
  int64_t h_out_stride;       /* elements                                                   */
} mcb_linear_args;

int mcb_linear(const mcb_linear_args* args, void* stream);

/* 1 when mcb_linear would run this call on the current device (the same host-side checks,
 * including whether the device schedules MCB_LINEAR_NORM_OUT's clusters), else 0 with
 * mcb_last_error saying why.  Nothing is launched or read from the device. */
int mcb_linear_supported(const mcb_linear_args* args);

/* ---------------------------------------------------------------------------------------------
 * Device-side status.  Kernels never trap: an out-of-range position (a cache or rotary table
 * overflow) or a timed-out pipeline wait sets a device error word and skips the access.
 * mcb_device_error synchronises `stream`, returns the word in *code and clears it.
 * Codes: 0 none, 1 position beyond Tmax, 2 position beyond the rotary table, 3 pipeline wait
 * timed out, 4 token id outside the embedding table.
 * ------------------------------------------------------------------------------------------- */
int mcb_device_error(int32_t* code, void* stream);

/* Kernels this library has enqueued in this process (host-side count, for launch accounting). */
uint64_t mcb_launch_count(void);

/* The template instance of the attention kernel the calling thread enqueued last (e.g.
 * "mcb::decode_attn_split_kernel<64,1,16,2>"; empty before the first), as the profiler names
 * it: lets a benchmark report the kernel its timing is about.  No counterpart in the reference
 * (modelcore has no native kernels).  Returns MCB_OK, or MCB_ERR_INVALID_ARG for an empty buffer. */
int mcb_last_attn_kernel(char* buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* MCB200_H */
