/*
 * kvq.h — C ABI of libkvq, the B200 (sm_100a) quantized-KV attention library.
 *
 * A drop-in for mlx-bun's quantized-KV cache + SDPA hot path.  Every entry
 * point takes plain integers, f32 scalars and pointers (no doubles by value,
 * no C++ types), returns int32 status (0 = KVQ_OK) and leaves a message for
 * kvq_last_error() on failure — the same convention as the mlx-c calls the
 * reference binds through bun:ffi (src/mlx/ffi.ts:1-11, :270-293, :338-348).
 * CUDA streams are passed as void* (cudaStream_t); NULL is the legacy
 * default stream.  All device work is stream-ordered; no call synchronizes
 * the host except where stated.
 *
 * Tensor layout (kept identical to MLX's affine quantized triple,
 * src/mlx/ops.ts:607-611):
 *   packed [B, H, rows, D*bits/32] uint32 — element e of a row in word
 *          e/(32/bits) at bit bits*(e%(32/bits)), LSB first;
 *   scales [B, H, rows, D/group_size] in the cache dtype (fp16 / bf16);
 *   biases [B, H, rows, D/group_size] in the cache dtype.
 * A kvq_qtensor names one such triple by three base pointers and row strides.
 *
 * Threading: a kvq_cache is not thread-safe; callers serialize access (the
 * reference serializes generation the same way, src/model/gemma4-base.ts:43-46).
 */
#ifndef KVQ_H
#define KVQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* mlx_dtype enum values (src/mlx/ffi.ts:297-300). */
#define KVQ_DTYPE_FLOAT16 9
#define KVQ_DTYPE_BFLOAT16 12

/* Status codes. */
#define KVQ_OK 0
#define KVQ_ERR_ARG 1         /* invalid argument / unsupported shape */
#define KVQ_ERR_CUDA 2        /* a CUDA runtime call failed */
#define KVQ_ERR_OOM 3         /* device allocation failed */
#define KVQ_ERR_STATE 4       /* cache state does not allow the operation */
#define KVQ_ERR_WORKSPACE 5   /* caller workspace too small */

/* Mask modes for kvq_sdpa_prefill / kvq_debug_scores. */
#define KVQ_MASK_NONE 0    /* attend every key ("" mode) */
#define KVQ_MASK_CAUSAL 1  /* bottom-right aligned causal; window > 0 adds a sliding window */

typedef struct kvq_cache kvq_cache;

/* Cache description.  Replaces the constructor arguments of
 * QuantizedKVCache(groupSize, bits) (src/model/gemma4-base.ts:419-431) and
 * RotatingQuantizedKVCache(maxSize, groupSize, bits) (:932-951) plus the
 * shape/dtype the reference takes from the first update. */
typedef struct kvq_desc {
  int32_t batch;        /* B */
  int32_t kv_heads;     /* H (kv heads) */
  int32_t head_dim;     /* D, same for K and V; multiple of group_size */
  int32_t bits;         /* 4 or 8 */
  int32_t group_size;   /* 32, 64 or 128 */
  int32_t dtype;        /* KVQ_DTYPE_FLOAT16 or KVQ_DTYPE_BFLOAT16 */
  int32_t max_size;     /* 0: growing QuantizedKVCache; > 0: rotating window of max_size rows */
  int32_t reserve_rows; /* physical rows per head allocated up front (0: as the reference grows) */
  int32_t device;       /* CUDA device ordinal the cache lives on */
} kvq_desc;

/* One quantized tensor [batch, heads, len, D] (a QuantizedTensor view,
 * src/mlx/ops.ts:607-611).  Strides are in rows; row r of component c starts
 * at c + r * (row size of c).  Row sizes: packed D*bits/32 uint32, scales and
 * biases D/group_size dtype elements. */
typedef struct kvq_qtensor {
  void* packed;
  void* scales;
  void* biases;
  int64_t batch_stride; /* rows between consecutive batch entries */
  int64_t head_stride;  /* rows between consecutive heads */
  int32_t batch;
  int32_t heads;
  int32_t len;          /* rows visible to attention */
  int32_t head_dim;
  int32_t bits;
  int32_t group_size;
  int32_t dtype;
} kvq_qtensor;

/* Message of the last failed call on this thread ("" if none). */
const char* kvq_last_error(void);
/* Library ABI version (major*10000 + minor*100 + patch). */
int32_t kvq_version(void);

/* ---- cache lifecycle ---------------------------------------------------- */

/* Create an empty cache (no device memory until the first append, unless
 * reserve_rows > 0).  Replaces `new QuantizedKVCache` / `new
 * RotatingQuantizedKVCache` (src/model/gemma4-base.ts:431, :951). */
int32_t kvq_cache_create(const kvq_desc* desc, kvq_cache** out);

/* Free the cache and its device memory (QuantizedKVCache.dispose, :593-597).
 * Synchronizes the cache's device. */
int32_t kvq_cache_free(kvq_cache* cache);

/* Quantize-on-append: S new K/V rows per (batch, head), written at the
 * position the reference's state machine picks, including growth in
 * 256-row steps (QuantizedKVCache.updateAndFetchQuantized, :452-507) and,
 * for rotating caches, the in-place ring write with wraparound for S == 1
 * (#updateInPlace, :1026-1086) or the temporal re-layout + trim + concat for
 * S > 1 (#updateConcat, :1003-1024).
 * k, v: device pointers to dtype values of logical shape [B, H, S, D] with
 * element strides k_strides[4] / v_strides[4] for (b, h, s, d); the d stride
 * must be 1 (so both [B,H,S,D] and [B,S,H,D] inputs work without a copy).
 * Host-side offset / ring index follow the reference exactly. */
int32_t kvq_append(kvq_cache* cache, const void* k, const void* v, int32_t S,
                   const int64_t* k_strides, const int64_t* v_strides, void* stream);

/* ---- fused K/V projection + norms + RoPE + quantize-on-append ----------- */

/* One MLX affine-quantized linear layer (QuantizedLinear, src/model/
 * gemma4-base.ts:76-158; the weight triple of mlx quantize): packed codes
 * [out_features, in_features * bits / 32] (16-byte aligned rows, LSB-first),
 * scales and biases [out_features, in_features / group_size] in the
 * activation dtype (biases NULL: none).  bits 4 or 8, group_size 32, 64 or
 * 128. */
typedef struct kvq_qlinear {
  const uint32_t* packed;
  const void* scales;
  const void* biases;
  int32_t bits, group_size;
  int32_t in_features, out_features;
} kvq_qlinear;

/* The K/V side of one attention layer ahead of its cache, and optionally its
 * query side (q_proj below) (Attention.forward, src/model/gemma4.ts:234-268):
 *   k = k_proj(x); v = v_from_k ? k : v_proj(x)   (attention_k_eq_v)
 *   k = rope(k_norm(k), offset); v = v_norm(v)
 * with out_features = kv_heads * head_dim.  k_norm / v_norm: apply RMSNorm
 * (mlx fast::rms_norm: x * 1/sqrt(mean(x^2) + eps), rounded to the dtype,
 * then times the weight, rounded; weight NULL: no multiply).  RoPE (mlx
 * fast::rope): the first rope_dims elements of each K row rotate in pairs
 * (i, i + rope_dims/2), or (2i, 2i + 1) with rope_traditional, by theta =
 * rope_scale * position * inv_freq_i, inv_freq_i = rope_base^(-2i/rope_dims),
 * or 1 / rope_freqs[i] when rope_freqs (device f32 [rope_dims / 2]) is given
 * (ProportionalRoPE's freqs, :131-165, whose infinite entries leave their
 * pair unrotated; the llama3 / yarn / longrope tables of
 * src/model/universal/rope.ts); the rest of the row passes through;
 * rope_dims 0: no RoPE.  rope_pre_scale (yarn's mscale, longrope's su
 * scale; UniversalRope.apply, rope.ts:51-75) multiplies the first rope_dims
 * elements of K, after its norm and before RoPE, by the scale rounded to
 * the dtype, rounding the product.  Position of token l = the cache offset
 * before the append + l. */
typedef struct kvq_kv_projection {
  kvq_qlinear k_proj;
  kvq_qlinear v_proj;          /* ignored when v_from_k */
  int32_t v_from_k;
  int32_t k_norm, v_norm;
  const void* k_norm_weight;   /* device [head_dim] dtype, nullable */
  const void* v_norm_weight;
  float norm_eps;
  int32_t rope_dims;
  int32_t rope_traditional;
  float rope_base, rope_scale;
  float rope_pre_scale;        /* 0 or 1: none */
  const float* rope_freqs;
  /* The query side (qProj, qNorm, Q's RoPE; gemma4.ts:224-226 and the
   * rope of q before attention): q_proj.packed NULL for none.  q_heads
   * query heads of head_dim, out_features = q_heads * head_dim; the same
   * RoPE as K. */
  kvq_qlinear q_proj;
  int32_t q_heads;
  int32_t q_norm;
  const void* q_norm_weight;   /* device [head_dim] dtype, nullable */
} kvq_kv_projection;

/* kvq_append of the projected, normed and roped K/V rows of x (device [B,
 * L, in_features] in the cache's dtype, B = the cache's batch): the K and V
 * projections run from the quantized weights, the norms, RoPE and the
 * quantize-on-append run in the same pass, and the rows land where
 * kvq_append would put them (same growth / ring state machine).  Replaces
 * kProj/vProj + kNorm/vNorm + rope + transposes + updateAndFetchQuantized
 * (src/model/gemma4.ts:234-268), and with a query projection also qProj +
 * qNorm + transpose + rope of q (:224-226, generated/gemma4-12b.ts:52-54,
 * :73-74): q_out (device [B, q_heads, L, head_dim] dtype, required then)
 * receives the query rows attention takes.  k_out / v_out (nullable,
 * device [B, kv_heads, L, head_dim] dtype) receive the K / V rows before
 * quantisation.
 * workspace NULL: the library-managed scratch; else at least
 * kvq_append_projected_workspace bytes.  The layer's parameters (the
 * weight triples, norm weights, rope_freqs) are read-only here and may be
 * read before the call's kernels wait for the kernel launched just before
 * them on the stream (programmatic dependent launch): that kernel must not
 * write them.  x, the cache and k_out / v_out are ordered normally. */
int32_t kvq_append_projected(kvq_cache* cache, const void* x, int32_t L,
                             const kvq_kv_projection* proj, void* q_out, void* k_out,
                             void* v_out, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes kvq_append_projected needs for L tokens. */
int32_t kvq_append_projected_workspace(const kvq_cache* cache, int32_t L,
                                       const kvq_kv_projection* proj, size_t* bytes);

/* Active quantized views after the last append (the [0:offset] slices of
 * updateAndFetchQuantized, :499-506, or #activeSlices, :1097-1104). */
int32_t kvq_cache_fetch(const kvq_cache* cache, kvq_qtensor* keys, kvq_qtensor* values);

/* Host state: offset (tokens seen), ring index (rotating caches; equals the
 * offset-derived write index the reference keeps in `ringIdx`), buffer length
 * in rows (the reference's keys.packed.shape[2]) and physical capacity. */
int32_t kvq_cache_state(const kvq_cache* cache, int64_t* offset, int64_t* ring_idx,
                        int64_t* seq_len, int64_t* capacity);

/* Drop the last n tokens (QuantizedKVCache.trim :589-591; rotating trim
 * :1137-1163 with the speculative-decode `bypass` form). */
int32_t kvq_cache_trim(kvq_cache* cache, int32_t n, int32_t bypass);

/* Mask for an N-token step given the cache state (makeMask, :509-519 and
 * :1113-1122), as a (mode, window) pair for kvq_sdpa_prefill.  window_size
 * <= 0 means "no window" (the reference's null). */
int32_t kvq_cache_make_mask(const kvq_cache* cache, int32_t N, int32_t window_size,
                            int32_t* mask_mode, int32_t* mask_window);

/* ---- batched serving: per-sequence positions on the device -------------- */

/* Ragged append for a batch whose sequences sit at different lengths (the
 * quantized-KV unlock of mlx-bun's batch scheduler, which is bf16-only,
 * src/serve/generation-gateway.ts:83-84, :156; and the dynamic-offset
 * writes of the compiled-decode adapters, src/model/compiled-decode.ts:99-190
 * with slice_update_dynamic, src/mlx/ops.ts:513-525).  Batch entry b
 * quantizes its first counts[b] rows of k / v ([B, H, S, D], strides as
 * kvq_append; counts NULL: all S) into rows [seq_lens[b], seq_lens[b] +
 * counts[b]) of its own (b, h) rows, then seq_lens[b] += counts[b].
 * seq_lens and counts are DEVICE int32[B]: positions are read and advanced
 * on the GPU, so a CUDA graph of append + decode appends at the next row on
 * every replay.  Growing caches only, created with reserve_rows > 0 (the
 * capacity); an entry whose rows would pass it is skipped (its length stays)
 * and the cache's error flag is raised — see kvq_cache_check.  The host
 * offset is not used or changed: do not mix with kvq_append on one cache.
 * Decode over it with kvq_cache_fetch_all views and the same seq_lens. */
int32_t kvq_append_ragged(kvq_cache* cache, const void* k, const void* v, int32_t S,
                          const int64_t* k_strides, const int64_t* v_strides, int32_t* seq_lens,
                          const int32_t* counts, void* stream);

/* Views of the cache's whole physical capacity (len = capacity rows), for
 * kvq_sdpa_decode with per-sequence seq_lens after ragged appends. */
int32_t kvq_cache_fetch_all(const kvq_cache* cache, kvq_qtensor* keys, kvq_qtensor* values);

/* Synchronize `stream`, report (then clear) the cache's error flag: a
 * ragged append skipped an entry that would have passed the capacity. */
int32_t kvq_cache_check(kvq_cache* cache, void* stream);

/* ---- conversion and persistence ----------------------------------------- */

/* Quantized cache from a dense fp16 / bf16 K/V buffer with its state
 * (KVCache.toQuantized, src/model/gemma4-base.ts:395-404, and
 * RotatingKVCache.toQuantized, :892-902 — the per-layer step of
 * maybeQuantizeKv, src/generate.ts:101-129).  Every one of the `rows` rows
 * per (batch, head) is quantized as laid out: the padding of a growing
 * buffer and the ring order of a rotating one are kept, and offset and
 * ring_idx are adopted (ring_idx is ignored for growing caches), so the
 * cache continues exactly where the dense one stood.  k, v: device [B, H,
 * rows, D] with element strides (d stride 1).  desc->max_size picks growing
 * (0) or rotating.  Stream-ordered; the dense buffers may be released once
 * the stream has passed this call. */
int32_t kvq_cache_from_dense(const kvq_desc* desc, const void* k, const void* v, int32_t rows,
                             const int64_t* k_strides, const int64_t* v_strides, int64_t offset,
                             int64_t ring_idx, void* stream, kvq_cache** out);

/* Copy rows [0, rows) of every (batch, head) of the six components to host
 * memory, contiguous [B, H, rows, *] each, in the order K packed, K scales,
 * K biases, V packed, V scales, V biases — the tensors of a saved cache
 * (saveKvCache, src/kv-store.ts:54-123, which keeps the live [0:offset]
 * rows of a growing cache and the whole buffer of a ring).  Synchronizes
 * `stream`. */
int32_t kvq_cache_export(const kvq_cache* cache, int64_t rows, void* const* host, void* stream);

/* A cache holding `rows` rows per (batch, head) read from six host buffers
 * laid out as kvq_cache_export writes them, with the given offset and ring
 * index (loadKvCache + restoreState, src/kv-store.ts:147-175,
 * src/model/gemma4-base.ts:385-391, :880-886).  Synchronizes `stream`. */
int32_t kvq_cache_import(const kvq_desc* desc, const void* const* host, int32_t rows,
                         int64_t offset, int64_t ring_idx, void* stream, kvq_cache** out);

/* ---- quantize ------------------------------------------------------------ */

/* Affine group quantize of `rows` contiguous rows of D dtype values into
 * contiguous packed / scales / biases (mlx_quantize as called by
 * ops.quantize, src/mlx/ops.ts:615-637; also the bulk step of
 * KVCache.toQuantized, src/model/gemma4-base.ts:395-404). */
int32_t kvq_quantize(const void* x, int64_t rows, int32_t head_dim, int32_t group_size,
                     int32_t bits, int32_t dtype, void* packed, void* scales, void* biases,
                     void* stream);

/* ---- attention ---------------------------------------------------------- */

/* Workspace bytes kvq_sdpa_decode / kvq_sdpa_decode_partial need for these
 * shapes.  Replaces nothing in the reference (MLX allocates internally).
 *
 * Library-managed workspace (workspace == NULL in the attention calls): one
 * buffer per device.  The first call that needs more than it holds
 * allocates a larger one (cudaMalloc, at least twice the old size), zeroes
 * it and synchronizes the calling stream; that call must not be made while
 * a stream capture is open.  The replaced buffer is not freed, so work
 * queued earlier and graphs captured earlier keep valid memory. */
int32_t kvq_sdpa_decode_workspace(const kvq_qtensor* keys, int32_t q_heads, size_t* bytes);

/* L = 1 attention over a quantized K/V pair (quantizedSdpa's decode cases:
 * fusedDecodeSdpa, src/model/fused-decode-kernel.ts:274-312, and
 * quantizedSdpaUnfused with mask "", src/model/gemma4-base.ts:1273-1342).
 * q:   device [B, q_heads, 1, D] dtype, contiguous; query head h uses kv head
 *      h / (q_heads / kv_heads).
 * out: device [B, q_heads, 1, D] dtype.
 * scale is applied as q * dtype(scale) rounded to dtype, like mulScalar.
 * seq_lens: NULL, or a DEVICE int32[B] of per-sequence key counts
 *      (<= keys->len) for ragged batches.
 * workspace: NULL (library-managed, cached per device) or a device buffer of
 *      at least kvq_sdpa_decode_workspace() bytes whose first 256 KiB are
 *      zero before its first use (split tickets live there; every call
 *      leaves them zero again).  Calls sharing one workspace must not
 *      overlap on the GPU. */
int32_t kvq_sdpa_decode(const kvq_qtensor* keys, const kvq_qtensor* values, const void* q,
                        int32_t q_heads, float scale, const int32_t* seq_lens, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Same attention, but instead of the normalized output it writes the
 * log-sum-exp partials of this key range for a context split across GPUs:
 * m[B*q_heads] (max logit), l[B*q_heads] (sum of exp(s - m)), and
 * o[B*q_heads, D] (sum of exp(s - m) * v, f32, unnormalized).  No
 * reference counterpart (the reference is single-device). */
int32_t kvq_sdpa_decode_partial(const kvq_qtensor* keys, const kvq_qtensor* values,
                                const void* q, int32_t q_heads, float scale,
                                const int32_t* seq_lens, float* m, float* l, float* o,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Merge `parts` partial sets into out[rows][D] in dtype, in fixed part
 * order (deterministic, like the reference's merge kernel,
 * src/model/fused-decode-kernel.ts:205-222).  Part p's values are
 * m[p*part_stride + r], l[p*part_stride + r] and
 * o[p*part_stride + r*head_dim + d] (part_stride in floats), so the three
 * arrays may live inside one packed buffer per part, as gathered from all
 * ranks of a context split. */
int32_t kvq_sdpa_merge(const float* m, const float* l, const float* o, int32_t parts,
                       int64_t part_stride, int32_t rows, int32_t head_dim, int32_t dtype,
                       void* out, void* stream);

/* L > 1 attention of L new query rows per head over the cache (chunked
 * prefill; quantizedSdpaTiled, src/model/gemma4-base.ts:1356-1521, and the
 * unfused window-mask case).  q: device [B, q_heads, L, D]; out likewise.
 * Query row i sits at key position keys->len - L + i (bottom-right aligned);
 * mask_mode KVQ_MASK_CAUSAL keeps keys j <= that position, and window > 0
 * additionally keeps only j > position - window (createCausalMask,
 * :1595-1614).  Workspace as for kvq_sdpa_decode (may be NULL).  For
 * 8-bit codes, D 128, group 64 without seq_lens, the tensor-core kernel
 * spreads the key tiles evenly over one CTA per SM and merges the units cut
 * between CTAs; that needs 262,400 + SMs * 135,168 bytes (20.3 MB on 148
 * SMs).  A smaller caller buffer runs one CTA per (query block, kv head,
 * batch entry) instead, with the same results within rounding. */
int32_t kvq_sdpa_prefill(const kvq_qtensor* keys, const kvq_qtensor* values, const void* q,
                         int32_t q_heads, int32_t L, float scale, int32_t mask_mode,
                         int32_t window, void* out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Debug: the scaled, masked logits [B, q_heads, L, keys->len] as f32, each
 * rounded to dtype as the reference's quantized_matmul output is
 * (src/model/gemma4-base.ts:1307-1330); masked entries are -inf.  Not a hot
 * path. */
int32_t kvq_debug_scores(const kvq_qtensor* keys, const void* q, int32_t q_heads, int32_t L,
                         float scale, int32_t mask_mode, int32_t window, float* scores,
                         void* stream);

/* Scratch held by kvq_sdpa_decode_noalloc: the 256 KiB flag-and-ticket
 * prefix of the decode workspace plus 2 MiB of split partials. */
#define KVQ_NOALLOC_SCRATCH_BYTES (256u * 1024u + 256u + 2u * 1024u * 1024u)

/* kvq_sdpa_decode for callers that cannot have device memory allocated on
 * their behalf: serving processes that give all free device memory to their
 * own pool at start-up, and latency-bound decode loops that must never meet
 * the implicit device synchronization of a cudaMalloc.  No counterpart in
 * the reference (MLX allocates internally).  Same arguments and results as
 * kvq_sdpa_decode without the workspace: the kernel's scratch is a fixed
 * KVQ_NOALLOC_SCRATCH_BYTES array inside the library that every GPU loading
 * libkvq keeps until exit.  The first call on a device looks up that
 * array's device address (make it before any stream capture).  Each call
 * clears the scratch's split tickets with a stream-ordered memset; all
 * calls share the array, so calls that overlap on the GPU race — issue them
 * on one stream.  The error flag at the array's start is left as it is, so
 * a timed-out wait stays visible until kvq_check_device(NULL, ...) reports
 * it.  When the full launch's split partials would not fit, the decode runs
 * on fewer CTAs (or without a key split) so that they do; shapes whose
 * partials do not fit even then return KVQ_ERR_WORKSPACE with the sizes in
 * kvq_last_error(). */
int32_t kvq_sdpa_decode_noalloc(const kvq_qtensor* keys, const kvq_qtensor* values,
                                const void* q, int32_t q_heads, float scale,
                                const int32_t* seq_lens, void* out, void* stream);

/* ---- context split across the GPUs of one node (peer memory) ----------- */

/* Exchange of context-split partials among the nranks ranks (one process
 * per GPU) of one node, over peer memory: no NCCL call on the data path.
 * No reference counterpart (the reference is single-device).
 * Each rank allocates an exchange buffer on its current device (flags, a
 * device-resident step epoch and 2 x nranks slots of rows * (head_dim + 2)
 * floats) and writes its CUDA IPC handle (64 bytes) to handle_out.
 * Synchronizes the device. */
typedef struct kvq_peer_group kvq_peer_group;
int32_t kvq_peer_group_create(int32_t rank, int32_t nranks, int32_t rows, int32_t head_dim,
                              void* handle_out, kvq_peer_group** out);

/* Map the other ranks' exchange buffers: handles holds all nranks handles
 * (64 bytes each) in rank order, as gathered from every rank. */
int32_t kvq_peer_group_connect(kvq_peer_group* group, const void* handles);

/* One exchange + merge step, stream-ordered: this rank's packed partial
 * (device [m rows | l rows | o rows*head_dim] f32, the layout
 * kvq_sdpa_decode_partial writes when its three outputs are carved out of
 * one buffer) is stored into every rank's buffer, and once all nranks
 * partials of the step have arrived (bounded wait, 2 s) they are merged in
 * rank order into out[rows][head_dim] in dtype — identical on every rank.
 * Every rank must make the same sequence of calls; the step counter lives on
 * the device, so the call may be recorded in a CUDA graph and replayed. */
int32_t kvq_peer_exchange_merge(kvq_peer_group* group, const float* packed, int32_t dtype,
                                void* out, void* stream);

/* Synchronize `stream` and report (then clear) the group's error flag,
 * raised when a rank's partials did not arrive within the wait limit. */
int32_t kvq_peer_group_check(kvq_peer_group* group, void* stream);

/* Unmap the peers' buffers and free this rank's (synchronizes the device).
 * Call only after every rank has finished its last exchange step. */
int32_t kvq_peer_group_free(kvq_peer_group* group);

/* Synchronize `stream` and report (then clear) the device error flag that a
 * kernel raises when a bounded wait on its own TMA copies times out.
 * workspace: the caller workspace used by the calls, or NULL for the
 * current device's library-managed workspaces (the live one and any it
 * replaced) and its kvq_sdpa_decode_noalloc scratch. */
int32_t kvq_check_device(void* workspace, void* stream);

/* Test hook: raise the error flag(s) kvq_check_device(workspace, ...) would
 * read, stream-ordered, so a test can see a raised flag reported without
 * making a kernel time out.  Not a hot path; no reference counterpart. */
int32_t kvq_debug_raise_flag(void* workspace, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVQ_H */
