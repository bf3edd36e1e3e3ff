/*
 * krill_kv.h — C ABI of the B200 int8 KV-cache hot path.
 *
 * This is the drop-in boundary for Krill's KrillCache / KrillEngine cache
 * path (srvsngh99/Krill, Swift + MLX). Each entry point names the reference
 * interface it replaces (file:line within the reference project). A Swift
 * module map over this header lets the engine call it in place of
 * QuantizedKVCache / RotatingKVCache / PrefixCache and the batched
 * stack/scatter helpers.
 *
 * Model of the cache:
 *   pool      One device-resident block pool per (device, layer group). It owns
 *             all KV memory: 256-token blocks, each holding every layer and
 *             KV head of the group (int8 codes + fp16 scale/zero per group of
 *             `group_size` elements).
 *   sequence  One request's per-layer caches (the reference's
 *             `[QuantizedKVCache]` for one row): a block table plus a length
 *             per layer. Blocks are ref-counted and shared copy-on-write
 *             between sequences and prefix-cache entries.
 *   prefix    A prefix cache bound to one pool; entries keep block references
 *             instead of tensor copies.
 *
 * Conventions:
 *   - Every function returns krill_status_t (KRILL_OK = 0). On error,
 *     krill_last_error_string() gives a thread-local message. Nothing aborts.
 *   - Device pointers are plain `void*`; `stream` is a `cudaStream_t` passed as
 *     `void*` (NULL = legacy default stream). Buffers passed in and out are
 *     caller-owned; the pool owns only its blocks and its scratch.
 *   - Calls on one pool must be externally serialised (one host thread at a
 *     time); the prefix cache is internally locked.
 *   - Tensors are dense, row-major, in the reference's layouts:
 *       new K/V   [layer_count][n_seqs][num_kv_heads][n_new][head_dim]
 *       q / out   [layer_count][n_seqs][num_q_heads][head_dim]
 *       snapshot  codes [num_kv_heads][S][head_dim] u8,
 *                 scales/zeros [num_kv_heads][S][head_dim/group_size] f16
 */
#ifndef KRILL_KV_H_
#define KRILL_KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t krill_status_t;
enum {
  KRILL_OK = 0,
  KRILL_ERR_INVALID = 1,   /* bad argument, handle, shape or state        */
  KRILL_ERR_OOM = 2,       /* block pool exhausted or allocation failed   */
  KRILL_ERR_CUDA = 3,      /* a CUDA runtime call failed                  */
  KRILL_ERR_PEER = 4,      /* peer access / peer copy unavailable          */
  KRILL_ERR_TIMEOUT = 5,   /* a device-side bounded wait gave up          */
  KRILL_ERR_NOT_FOUND = 6, /* lookup miss (not an error for lookups)      */
  KRILL_ERR_NO_DEVICE = 7  /* compute call on a host-only pool            */
};

enum {
  KRILL_DTYPE_F16 = 0,
  KRILL_DTYPE_BF16 = 1,
  KRILL_DTYPE_F32 = 2,
  KRILL_DTYPE_U8 = 3
};

/* Quantizer arithmetic. F32 follows MLX's promotion of an f16/bf16 array
 * against a Float32 scalar array (QuantizedKVCache.swift:185-192): scale and
 * quotient in float32. F16 keeps them in the input dtype. */
enum { KRILL_QUANT_F32 = 0, KRILL_QUANT_INPUT_DTYPE = 1 };

/* Decode-attention implementation, a performance knob (all give the same
 * results within the attention tolerance):
 *   TENSOR_CORE       per-sequence decode on mma.sync m16n8k16 over the
 *                     dequantized tiles; the shared-prefix (cascade) part on
 *                     tcgen05 with tensor-memory accumulators (head_dim <= 128),
 *                     one CTA per item (M = 128 per instruction)
 *   CUDA_CORE         per-sequence decode on FMA, no cascade
 *   TENSOR_CORE_SYNC  as TENSOR_CORE with the cascade part on mma.sync
 *   TENSOR_CORE_PAIR  as TENSOR_CORE with the tcgen05 cascade on pairs of
 *                     CTAs (cta_group::2, M = 256 per instruction) where its
 *                     items have more than 128 query rows */
enum {
  KRILL_ATTN_TENSOR_CORE = 0,
  KRILL_ATTN_CUDA_CORE = 1,
  KRILL_ATTN_TENSOR_CORE_SYNC = 2,
  KRILL_ATTN_TENSOR_CORE_PAIR = 3
};

/* Storage format of a pool: int8 codes with fp16 scale/zero per group (the
 * reference's QuantizedKVCache), or raw bf16 K/V (the unquantized KVCache of
 * Sources/KrillCache/KVCache.swift:94, kept for comparison; head_dim 64 or 128,
 * bf16 k/v/q, no quantized snapshots or cascade). */
enum { KRILL_KV_INT8 = 0, KRILL_KV_BF16 = 1 };

typedef struct krill_pool_s* krill_pool_t;
typedef uint64_t krill_seq_t;               /* generation << 32 | slot */
typedef struct krill_prefix_s* krill_prefix_t;
typedef struct krill_prefix_entry_s* krill_prefix_entry_t;

typedef struct {
  int32_t num_layers;     /* layers in this layer group                          */
  int32_t num_kv_heads;   /* Hkv                                                 */
  int32_t num_q_heads;    /* Hq (multiple of Hkv; Hq/Hkv <= 8)                    */
  int32_t head_dim;       /* D: 64, 128 or 256                                   */
  int32_t group_size;     /* quantization group: 64 or head_dim                  */
  int32_t window;         /* 0 = full history (QuantizedKVCache); > 1 = sliding
                             window of that many tokens (RotatingKVCache)        */
  int32_t max_append;     /* largest n_new per append on a windowed pool (sizes
                             the ring: window - 1 + max_append tokens); 0 -> 256  */
  int32_t quant_variant;  /* KRILL_QUANT_*                                       */
  int32_t attn_impl;      /* KRILL_ATTN_*                                        */
  int32_t split_tokens;   /* decode split-K piece in tokens (multiple of 64).
                             0 = adaptive: pieces and head groups follow the
                             batch shape (results depend on shapes, never on
                             other sequences' contents). > 0 = fixed pieces and
                             whole-layer head groups: a sequence's output is
                             then bit-identical whatever else is batched.      */
  int32_t cascade_min_tokens; /* shared-prefix (cascade) attention: sequences of
                             one call whose block tables begin with the same
                             blocks (forks of one prefix entry) attend at least
                             this many common tokens together, read and
                             dequantized once. 0 -> 256; < 0 -> off. Applies
                             to full-history pools with a tensor-core
                             implementation and split_tokens = 0.           */
  int32_t kv_format;      /* KRILL_KV_INT8 (default) or KRILL_KV_BF16           */
  int64_t num_blocks;     /* pool capacity in 256-token blocks                  */
  int32_t wait_timeout_us; /* bound of every device-side wait in this pool's
                             kernels (a stage copy, a stage release), in
                             microseconds (counted in 1.024 us units of the
                             GPU timer); 0 -> 100000 (about 0.1 s). A wait that
                             runs out sets KRILL_DEVICE_ERR_TIMEOUT in the
                             device error flag and the kernel runs to its end
                             instead of hanging; that launch's outputs are
                             then not valid.                                */
} krill_pool_cfg;

/* ---- errors ------------------------------------------------------------- */
const char* krill_last_error_string(void);
const char* krill_version(void);

/* ---- pool ----------------------------------------------------------------
 * Replaces makeQuantizedKVCaches(numLayers:) (QuantizedKVCache.swift:208-210)
 * and makeKVCaches(spec:numLayers:) for `.rotating(window:)` layers
 * (KVCache.swift:198-209). device < 0 creates a host-only dry-run pool: block
 * accounting, copy-on-write decisions, lengths, planning and the prefix cache
 * run exactly as on a device pool, while no device memory exists and no
 * kernel or copy is issued (append / attention / restore update only the
 * bookkeeping; snapshots, stacking and peer fetch return KRILL_ERR_NO_DEVICE). */
krill_status_t krill_pool_create(const krill_pool_cfg* cfg, int32_t device, krill_pool_t* out);
krill_status_t krill_pool_destroy(krill_pool_t pool);
krill_status_t krill_pool_block_bytes(krill_pool_t pool, int64_t* bytes);
krill_status_t krill_pool_free_blocks(krill_pool_t pool, int64_t* n);
krill_status_t krill_pool_block_refcount(krill_pool_t pool, int32_t block, int32_t* refcount);
/* Device error flag set by a kernel whose bounded wait gave up (and cleared
 * by reading it): a bit mask of KRILL_DEVICE_ERR_*. Reading it synchronises
 * with the pool's device. */
#define KRILL_DEVICE_ERR_TIMEOUT 1
krill_status_t krill_pool_device_error(krill_pool_t pool, int32_t* flag);
/* Testing only (no reference counterpart): while enabled, an otherwise idle
 * warp of CTA 0 of each decode-attention launch on this pool waits for a
 * shared-memory word that nothing sets, so that its bounded wait runs out
 * (KRILL_DEVICE_ERR_TIMEOUT; that launch's outputs are not valid). Nothing
 * faults or hangs. Synchronises with the device. For tests of the failure
 * path; never enabled otherwise. */
krill_status_t krill_pool_test_stall(krill_pool_t pool, int32_t enable);

/* Measurement hook (no reference counterpart): while enabled, every attention
 * and append kernel the pool launches is bracketed by a CUDA event pair on its
 * launching stream. krill_pool_kernel_times() waits for the recorded events,
 * returns the accumulated device milliseconds and launch counts since the
 * last call, and resets them. Any output pointer may be NULL. */
krill_status_t krill_pool_set_profiling(krill_pool_t pool, int32_t enable);
krill_status_t krill_pool_kernel_times(krill_pool_t pool, double* attn_ms, int32_t* attn_launches,
                                       double* append_ms, int32_t* append_launches);
/* Measurement hook (no reference counterpart): device kernels this pool
 * launched (append, attention with its cascade and combine passes, gathers,
 * scatters) since the previous call; resets the count. */
krill_status_t krill_pool_kernel_count(krill_pool_t pool, int64_t* kernels);

/* Introspection (no reference counterpart): the decomposition chosen by the
 * last krill_decode_attention on this pool — sequence piece length in 64-token
 * sub-blocks, kv heads per work item, number of items and of persistent CTAs. */
krill_status_t krill_pool_last_plan(krill_pool_t pool, int32_t* piece_subblocks,
                                    int32_t* heads_per_item, int64_t* items, int32_t* ctas);
/* Introspection (no reference counterpart): the kernel instances the last
 * krill_decode_attention (or verify / prefill / step) on this pool launched,
 * in order, joined by '+', e.g. "attn_tc_kernel<128,2,8,1,13,0>+
 * attn_combine_kernel<128>" (template arguments: head_dim, groups per head,
 * consumer warps, warps per head, pipeline stages, pool format). Written into
 * buf (NUL-terminated, truncated to cap bytes). */
krill_status_t krill_pool_last_kernels(krill_pool_t pool, char* buf, int32_t cap);
/* Introspection (no reference counterpart): the shared-prefix part of the last
 * krill_decode_attention — number of sequence groups attended together, their
 * cascade work items, partial-record slots per member and persistent CTAs
 * (0 everywhere when no group qualified). */
krill_status_t krill_pool_last_cascade(krill_pool_t pool, int32_t* groups, int64_t* shared_items,
                                       int32_t* prefix_slots, int32_t* ctas);

/* ---- sequences (one request's per-layer caches) -------------------------- */
/* New empty sequence: every layer at length 0 (QuantizedKVCache.init). */
krill_status_t krill_seq_create(krill_pool_t pool, krill_seq_t* out);
/* Drop the sequence and its block references. */
krill_status_t krill_seq_release(krill_pool_t pool, krill_seq_t seq);
/* reset(): all layers back to empty (QuantizedKVCache.swift:92-99). */
krill_status_t krill_seq_reset(krill_pool_t pool, krill_seq_t seq);
/* sequenceLength of one layer (QuantizedKVCache.swift:28-30; for a windowed
 * pool the total tokens seen, RotatingKVCache.swift:60). */
krill_status_t krill_seq_length(krill_pool_t pool, krill_seq_t seq, int32_t layer, int64_t* len);
/* Rows physically retained for a layer (RotatingKVCache.retainedLength,
 * RotatingKVCache.swift:63; equals the length on a full-history pool). */
krill_status_t krill_seq_retained(krill_pool_t pool, krill_seq_t seq, int32_t layer, int64_t* n);
/* memorySizeBytes (QuantizedKVCache.swift:33-42), generalised to groups. */
krill_status_t krill_seq_memory_bytes(krill_pool_t pool, krill_seq_t seq, int32_t layer, int64_t* bytes);
/* truncate(to:) on every layer (QuantizedKVCache.swift:135-145; on a windowed
 * pool RotatingKVCache.truncate, RotatingKVCache.swift:134-142, which fails
 * with KRILL_ERR_INVALID where canTruncate is false). n >= length is a no-op. */
krill_status_t krill_seq_truncate(krill_pool_t pool, krill_seq_t seq, int64_t n);
/* canTruncate(to:) (RotatingKVCache.swift:128-130; KVCache.swift:218). */
krill_status_t krill_seq_can_truncate(krill_pool_t pool, krill_seq_t seq, int64_t n, int32_t* ok);
/* Number of blocks in the sequence's table and their ids (for tests/tools). */
krill_status_t krill_seq_blocks(krill_pool_t pool, krill_seq_t seq, int32_t* ids, int32_t cap, int32_t* n);

/* ---- hot path ------------------------------------------------------------ */
/* Quantize n_new tokens of K and V per (token, head, group) and append them at
 * each layer's current length, in place (no concatenation copy). Replaces the
 * quantize + concatenate half of QuantizedKVCache.update
 * (QuantizedKVCache.swift:49-69) and quantizePerHead (:181-197).
 * k_new/v_new: [layer_count][n_seqs][Hkv][n_new][D], dtype F16 or BF16. */
krill_status_t krill_append_quantize(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                     int32_t layer_begin, int32_t layer_count, int32_t n_new,
                                     const void* k_new, const void* v_new, int32_t dtype,
                                     void* stream);
/* Fused RoPE + quantize + append (no reference counterpart as one call; it
 * fuses MLXFast.RoPE(dimensions: head_dim, traditional: false) applied to the
 * new K at each token's position, Gemma4Model.swift:502-509 and the per-row
 * offsets of Attention.swift:13-20, with the update above). Token t of a
 * sequence whose layer holds `len` tokens sits at position len + t; element
 * d < head_dim/2 becomes x[d]*cos[p][d] - x[d+h]*sin[p][d] and element d + h
 * becomes x[d]*sin[p][d] + x[d+h]*cos[p][d] (h = head_dim/2), each product
 * and sum rounded to f32 and the result rounded to `dtype` before it is
 * quantized. rope_cos / rope_sin: device f32 tables [rope_rows][head_dim/2]
 * owned by the caller (angle(p, d) = p * base^(-2d/head_dim)); positions must
 * stay below rope_rows. V is appended unrotated. int8 pools only. */
krill_status_t krill_append_quantize_rope(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                          int32_t layer_begin, int32_t layer_count, int32_t n_new,
                                          const void* k_new, const void* v_new, int32_t dtype,
                                          const float* rope_cos, const float* rope_sin,
                                          int64_t rope_rows, void* stream);

/* Decode attention for one query token per (layer, sequence), reading the
 * int8 cache directly: dequantization (with the reference's fp16 rounding) is
 * fused into q·Kᵀ, online softmax and ·V. Replaces the dequantize half of
 * QuantizedKVCache.update (:71-74) plus MLXFast.scaledDotProductAttention with
 * GQA (Gemma4Model.swift:516, Attention.swift:95). Each sequence attends its
 * current length (its window on a windowed pool), so no pad mask is needed.
 * q: [layer_count][n_seqs][Hq][D] F16 or BF16; out: same shape, F16, BF16 or
 * F32. scale: 1/sqrt(D) for Llama (Attention.swift:44), 1.0 for Gemma 4. */
krill_status_t krill_decode_attention(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, const void* q,
                                      int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                      void* stream);
/* Multi-query verify attention for speculative decoding: the batched verify
 * forward with buildBatchedVerifyMask (BatchedDecode.swift:299-312). The last
 * n_query tokens of each sequence (appended beforehand, e.g. by
 * krill_append_quantize with n_new = n_query) are the queries; query j attends
 * the cache up to and including its own token and none of the later drafts, so
 * the result equals n_query sequential single-token decode steps.
 * q / out: [layer_count][n_seqs][n_query][Hq][D]. Full-history pools only.
 * Few queries run as one decode unit per query; many (n_query x GQA group >=
 * 64, head_dim <= 128, tensor-core implementation) run as causal tcgen05
 * items that read each sequence's K/V once per block of 256 query rows. */
krill_status_t krill_verify_attention(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, int32_t n_query,
                                      const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                                      float scale, void* stream);
/* Chunked-prefill attention over the int8 cache (chunkedTextPrefill,
 * InferenceEngine.swift:3122-3147: each chunk's K/V goes into the cache, then
 * the chunk's queries attend the whole cache causally). The same operation as
 * krill_verify_attention with n_query = the chunk length: append the chunk
 * first, then call this. */
krill_status_t krill_prefill_attention(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                       int32_t layer_begin, int32_t layer_count, int32_t n_query,
                                       const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                                       float scale, void* stream);

/* Allocation-free decode attention. No counterpart in the reference: it
 * exists for callers that cannot have the library allocate memory while they
 * decode — an engine that has reserved all device memory for its own
 * allocator, a serving loop that must not take the driver's allocation locks
 * mid-step, a host that accounts for every device byte. Same arguments,
 * layouts and results (within the attention tolerance) as
 * krill_decode_attention, which grows its staging and split scratch with
 * cudaMalloc / cudaMallocHost; this variant calls no allocating routine on
 * success and instead uses a fixed scratch array of
 * KRILL_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU that
 * loads the library holds until the process exits, plus a fixed host buffer.
 *   - Limit: a call whose metadata plus split partials exceed the scratch
 *     (roughly: many sequences longer than 4096 tokens at once) is rejected
 *     with KRILL_ERR_INVALID and a message giving the bytes it would need.
 *   - The scratch is reserved on a device when the first pool on it is
 *     created (krill_pool_create looks up its device address with the device
 *     current, which under lazy module loading is when the driver loads it),
 *     not during a decode call.
 *   - A call on a stream that is being captured is rejected with
 *     KRILL_ERR_INVALID: the metadata is copied from a host buffer that the
 *     next call overwrites.
 *   - All calls share the one scratch. Every call writes the metadata and
 *     partial results it reads; the arrival counters that merge split
 *     sequences carry a per-call tag, so values left by an earlier call count
 *     as zero (nothing has to be cleared between calls). Calls serialise on the host,
 *     and calls whose GPU work overlaps (different streams, no ordering
 *     between them) race on the scratch: order them on one stream or
 *     synchronise between them. */
#define KRILL_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
krill_status_t krill_decode_attention_noalloc(krill_pool_t pool, int32_t n_seqs,
                                              const krill_seq_t* seqs, int32_t layer_begin,
                                              int32_t layer_count, const void* q, int32_t q_dtype,
                                              void* out, int32_t out_dtype, float scale,
                                              void* stream);

/* One decode step: krill_append_quantize (n_new = 1) then
 * krill_decode_attention over the same layers. */
krill_status_t krill_decode_step(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                 int32_t layer_begin, int32_t layer_count, const void* k_new,
                                 const void* v_new, int32_t kv_dtype, const void* q,
                                 int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                 void* stream);

/* One decode step from HOST buffers (same layouts as krill_decode_step):
 * k_new/v_new [layer_count][n_seqs][Hkv][1][D], q and out
 * [layer_count][n_seqs][Hq][D]. The reference's cache calls take arrays in
 * the unified memory of the Apple device (QuantizedKVCache.update,
 * QuantizedKVCache.swift:118-142, then SDPA, Gemma4Model.swift:508,516); on a
 * discrete GPU this call is that step with the transfers included. The layers
 * are processed in chunks of layer_chunk (0 = all layers in one chunk):
 * chunk c's inputs are copied in on a second stream while chunk c-1 computes,
 * and its output is copied back on a third while chunk c+1 computes. The call
 * returns once the work is enqueued on `stream`; `out` is complete when
 * `stream` has finished. Page-locked host buffers (cudaHostAlloc or
 * cudaHostRegister) let the copies overlap; pageable ones work, without the
 * overlap. A page-locked q is not copied: the attention kernels read it in
 * place through its device mapping, so its transfer overlaps the cache reads
 * (q must then stay unchanged until `stream` has finished). On an error after
 * the first chunk, the layers of the chunks already enqueued have been
 * appended. */
krill_status_t krill_decode_step_host(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, const void* k_new,
                                      const void* v_new, int32_t kv_dtype, const void* q,
                                      int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                      int32_t layer_chunk, void* stream);

/* ---- snapshots / restore -------------------------------------------------- */
/* quantizedSnapshot() for one layer (QuantizedKVCache.swift:106-115): the raw
 * codes and fp16 scales/zeros of the retained rows, in the QuantizedKVSnapshot
 * layout (QuantizedKVCache.swift:150-157). Any output pointer may be NULL. */
krill_status_t krill_seq_snapshot_quantized(krill_pool_t pool, krill_seq_t seq, int32_t layer,
                                            void* keys, void* values, void* key_scales,
                                            void* key_zeros, void* value_scales,
                                            void* value_zeros, void* stream);
/* snapshot() / the tensors update() returns (QuantizedKVCache.swift:82-89,
 * :72-74): the retained rows dequantized to fp16, bit-exact with the
 * reference's dequantize (:200-204). Output [Hkv][S][D] f16 each. */
krill_status_t krill_seq_snapshot_dequantized(krill_pool_t pool, krill_seq_t seq, int32_t layer,
                                              void* keys, void* values, void* stream);
/* restoreQuantized(_:) for one layer (QuantizedKVCache.swift:122-129): copy
 * (never alias) `rows` rows in the snapshot layout into the sequence; the
 * layer's length becomes total_seen (= rows on a full-history pool; on a
 * windowed pool the rows are the tail ending at total_seen - 1, as
 * RotatingKVCache.restore, RotatingKVCache.swift:148-163). */
krill_status_t krill_seq_restore_quantized(krill_pool_t pool, krill_seq_t seq, int32_t layer,
                                           int64_t rows, int64_t total_seen, const void* keys,
                                           const void* values, const void* key_scales,
                                           const void* key_zeros, const void* value_scales,
                                           const void* value_zeros, void* stream);

/* ---- continuous-batch glue ------------------------------------------------ */
/* stackCachesLeftPaddedQuantized for one layer (BatchedDecode.swift:96-151):
 * rows right-aligned at s_max = max length, left pad = code 0, scale 0,
 * zero 0. Outputs [n_seqs][Hkv][s_max][D] u8 and [n_seqs][Hkv][s_max][D/G] f16. */
krill_status_t krill_stack_left_padded(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                       int32_t layer, int64_t s_max, void* keys, void* values,
                                       void* key_scales, void* key_zeros, void* value_scales,
                                       void* value_zeros, void* stream);
/* ContinuousBatcher.scatterBack int8 branch (ContinuousBatcher.swift:763-773):
 * row i's columns [s_max - base_len[i], s_max + steps) of a stacked layer are
 * restored into sequence i (its new length for that layer). */
krill_status_t krill_scatter_back(krill_pool_t pool, int32_t n_seqs, const krill_seq_t* seqs,
                                  int32_t layer, const int64_t* base_lens, int64_t s_max,
                                  int64_t steps, const void* keys, const void* values,
                                  const void* key_scales, const void* key_zeros,
                                  const void* value_scales, const void* value_zeros,
                                  void* stream);
/* buildBatchedDecodeMask (BatchedDecode.swift:277-287), host memory:
 * out [n][total_len] float, -10000 on each row's left pad, 0 elsewhere. */
krill_status_t krill_build_decode_mask(const int64_t* lengths, int32_t n, int64_t s_max,
                                       int64_t total_len, float* out);

/* ---- prefix cache ---------------------------------------------------------
 * PrefixCache (PrefixCache.swift:15-114) bound to one pool. Entries hold
 * block references (zero-copy store); a hit is consumed by forking a new
 * sequence that shares the entry's blocks copy-on-write. */
krill_status_t krill_prefix_create(krill_pool_t pool, int32_t max_memory_entries,
                                   int32_t min_prefix_length, krill_prefix_t* out);
krill_status_t krill_prefix_destroy(krill_prefix_t pc);
/* storeQuantized(tokens:modelId:snapshots:mediaHash:) (PrefixCache.swift:369-400):
 * the first n_tokens positions of `seq` become an entry keyed by
 * FNV-1a(v3, int8, modelId, mediaHash, tokens) (:513-532); LRU-evicts at
 * max_memory_entries (:540-551). n_tokens < min_prefix_length is a no-op. */
krill_status_t krill_prefix_store(krill_prefix_t pc, krill_seq_t seq, const int64_t* tokens,
                                  int64_t n_tokens, const char* model_id, const char* media_hash);
/* lookupQuantized (PrefixCache.swift:161-170 via scan :273-308): exact-key
 * scan from the full length down in steps of max(1, min/2). On a hit *entry
 * holds a reference (release it) and *prefix_length is the matched length;
 * a miss returns KRILL_ERR_NOT_FOUND with *entry = NULL. */
krill_status_t krill_prefix_lookup(krill_prefix_t pc, const int64_t* tokens, int64_t n_tokens,
                                   const char* model_id, const char* media_hash,
                                   krill_prefix_entry_t* entry, int64_t* prefix_length);
/* lookupLongestPrefixQuantized (PrefixCache.swift:235-263): the in-memory
 * entry with the longest common prefix >= min_prefix_length. */
krill_status_t krill_prefix_lookup_longest(krill_prefix_t pc, const int64_t* tokens,
                                           int64_t n_tokens, const char* model_id,
                                           const char* media_hash, krill_prefix_entry_t* entry,
                                           int64_t* prefix_length);
/* Stored token count of an entry (PrefixCacheHit.storedLength, :443-448). */
krill_status_t krill_prefix_entry_length(krill_prefix_entry_t entry, int64_t* stored_length);
krill_status_t krill_prefix_entry_release(krill_prefix_t pc, krill_prefix_entry_t entry);
/* Restore-and-truncate of a hit (InferenceEngine.swift:1305-1320, 1378-1417):
 * a new sequence sharing the entry's blocks for positions [0, keep); no KV is
 * copied and no prefill runs. keep <= stored length. */
krill_status_t krill_seq_fork_prefix(krill_prefix_t pc, krill_prefix_entry_t entry, int64_t keep,
                                     krill_seq_t* out);
/* clear() (PrefixCache.swift:403-414) and memoryCount (:417-420). */
/* clear(): drops the memory entries and, with the disk tier on, its files
 * (PrefixCache.swift:403-415). */
krill_status_t krill_prefix_clear(krill_prefix_t pc);
/* Disk tier (PrefixCache.swift:496-501, 553-695), off by default. budget_bytes
 * 0 disables it, < 0 is unbounded, > 0 evicts least-recently-used files (by
 * modification time) down to 90 % of the budget after a write. Each stored
 * entry is written behind the caller, by a worker thread, as
 * `<cache_dir>/<key %016llx>.q8.safetensors` with the reference's tensors
 * layer_{i}_qk / _qv (U8 [1, Hkv, S, D]) and _ks / _kz / _vs / _vz
 * (F16 [1, Hkv, S, D/G]). krill_prefix_lookup probes memory, then disk, at
 * every scan length; a disk hit is read into new pool blocks and joins the
 * memory tier without tokens (longest-prefix matching skips it). Device int8
 * pools with full history only. */
krill_status_t krill_prefix_set_disk(krill_prefix_t pc, const char* cache_dir, int64_t budget_bytes);
/* waitForDiskWrites(): blocks until every queued write finished. */
krill_status_t krill_prefix_wait_disk(krill_prefix_t pc);
/* diskCount: number of entry files in the cache directory. */
krill_status_t krill_prefix_disk_count(krill_prefix_t pc, int32_t* count);
krill_status_t krill_prefix_memory_count(krill_prefix_t pc, int32_t* count);
/* FNV-1a cache key (PrefixCache.swift:513-532) for tools and tests. */
uint64_t krill_prefix_key(const int64_t* tokens, int64_t n_tokens, const char* model_id,
                          const char* media_hash, int32_t dtype_tag);

/* ---- multi-GPU ------------------------------------------------------------
 * Copy a prefix entry owned by another GPU's pool into dst's pool over NVLink
 * (cudaMemcpyPeerAsync, copy engine) and register it in dst's prefix cache.
 * Pools must have identical geometry. No reference counterpart (the reference
 * is single-device); the entry is afterwards ref-counted locally. */
krill_status_t krill_prefix_peer_fetch(krill_prefix_t dst, krill_prefix_t src,
                                       krill_prefix_entry_t src_entry, void* stream,
                                       krill_prefix_entry_t* dst_entry);

/* Cross-process form of the same fetch, for one process per GPU (no
 * reference counterpart). The owner publishes its pool's IPC handle
 * (krill_pool_ipc_handle, 64 bytes) and an entry descriptor
 * (krill_prefix_entry_describe: geometry, key, length, block ids, per-layer
 * lengths, model id, media hash, tokens; call with buf = NULL for the size);
 * the caller moves both to the other process. krill_prefix_import maps the
 * owner's pool once per process (cudaIpcOpenMemHandle), copies the entry's
 * blocks over NVLink into new local blocks on `stream` and registers the entry
 * in dst, returning a held reference. The owner must keep the entry alive
 * until the copy on `stream` has finished. */
krill_status_t krill_pool_ipc_handle(krill_pool_t pool, void* handle);
krill_status_t krill_prefix_entry_describe(krill_prefix_t pc, krill_prefix_entry_t entry, void* buf,
                                           int64_t cap, int64_t* size);
krill_status_t krill_prefix_import(krill_prefix_t dst, const void* pool_handle, const void* desc,
                                   int64_t desc_size, void* stream, krill_prefix_entry_t* dst_entry);

#ifdef __cplusplus
}
#endif
#endif /* KRILL_KV_H_ */
