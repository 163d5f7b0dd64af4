/*
 * cacheflow_b200.h -- C ABI of the B200 (sm_100a) KV-cache kernel layer.
 *
 * Every entry point is a drop-in for one operator of CacheFlow's CUDA layer
 * (the headers under src/cacheflow/cuda/ in the CacheFlow sources); the comment above each
 * declaration names the reference interface it replaces (file:line).
 *
 * Conventions shared by all entry points:
 *   - All tensor pointers are DEVICE pointers unless a comment says otherwise;
 *     the caller owns every buffer and no entry point allocates device memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call is asynchronous on that stream and re-entrant.
 *   - Host-visible arguments are validated before any launch; a bad argument
 *     returns CF_ERR_INVALID_ARGUMENT and launches nothing.  Values that only
 *     the device can see (block ids, slots, context lengths) are range-checked
 *     inside the kernels: a bad value is skipped and recorded in a per-device
 *     error word that cf_get_device_errors() reads.  No kernel traps.
 *   - Cache layout (both K and V):  [num_blocks, num_kv_heads, block_size,
 *     head_dim], contiguous, element type `dtype` (CacheFlow's layout,
 *     paged_attention.cuh:27-28).
 */
#ifndef CACHEFLOW_B200_H_
#define CACHEFLOW_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CF_API __attribute__((visibility("default")))
#else
#define CF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CF_ABI_VERSION 1

typedef enum cf_status {
  CF_OK = 0,
  CF_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad shape     */
  CF_ERR_UNSUPPORTED = 2,      /* no kernel for this head_dim/block_size/dtype */
  CF_ERR_WORKSPACE = 3,        /* caller-provided scratch is too small       */
  CF_ERR_CUDA = 4,             /* a CUDA runtime call failed; see cf_last_cuda_error() */
  CF_ERR_PLAN = 5              /* a block-move plan would race (overlapping src/dst) */
} cf_status;

typedef enum cf_dtype {
  CF_F32 = 0,  /* float  (the reference's only type) */
  CF_F16 = 1,  /* IEEE half                          */
  CF_BF16 = 2, /* bfloat16                           */
  CF_FP8_E4M3 = 3 /* 8-bit float e4m3 (OCP FP8, finite-only, max 448): KV caches
                   * only, value = stored * per-cache scale; the block
                   * operators move it as bytes */
} cf_dtype;

/* Bits of the per-device error word (cf_get_device_errors). */
#define CF_DEVERR_BLOCK_ID 0x1u    /* block-table / pair entry outside [0, num_blocks) */
#define CF_DEVERR_SLOT 0x2u        /* slot_mapping entry outside the pool              */
#define CF_DEVERR_CONTEXT_LEN 0x4u /* context length < 0 or > max_blocks_per_seq*bs   */
#define CF_DEVERR_TIMEOUT 0x8u     /* a bounded pipeline wait gave up (kernel returned) */

/* Parameters of one paged decode-attention call.  Same fields and meaning as
 * cacheflow::cuda::PagedAttentionParams (paged_attention.cuh:25-40) plus
 * `num_blocks` (pool size, used to range-check block ids; 0 = unchecked) and
 * `dtype` (type of query, caches and output). */
typedef struct cf_paged_attention_params {
  const void* query;            /* [num_seqs, num_heads, head_dim]            */
  const void* key_cache;        /* [num_blocks, num_kv_heads, block_size, head_dim] */
  const void* value_cache;      /* same layout as key_cache                   */
  void* output;                 /* [num_seqs, num_heads, head_dim]            */
  const int32_t* block_tables;  /* [num_seqs, max_blocks_per_seq]            */
  const int32_t* context_lens;  /* [num_seqs]                                 */
  float scale;                  /* softmax scale, usually 1/sqrt(head_dim)    */
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;         /* num_heads % num_kv_heads == 0 (GQA/MQA)    */
  int32_t head_dim;             /* 64, 128 or 256                             */
  int32_t block_size;           /* tokens per KV block: 16                    */
  int32_t max_context_len;      /* host-side upper bound of context_lens      */
  int32_t max_blocks_per_seq;   /* row stride of block_tables                 */
  int64_t num_blocks;           /* pool size; 0 = do not range-check ids      */
  int32_t dtype;                /* cf_dtype                                   */
} cf_paged_attention_params;

/* Decode attention, one query token per sequence.
 * Replaces cacheflow::cuda::launch_paged_attention_v1 (paged_attention.cuh:44-46).
 * `workspace` is optional: with NULL the whole context of a (sequence, KV head)
 * is handled by one CTA; with at least cf_paged_attention_v1_workspace_size()
 * bytes the context is split across CTAs and merged by a second kernel. */
CF_API cf_status cf_paged_attention_v1(const cf_paged_attention_params* params,
                                void* workspace, size_t workspace_bytes,
                                void* stream);

/* Bytes of workspace the split path of cf_paged_attention_v1 uses for these
 * params, or for the same sizes with any shorter max_context_len (a host
 * sizes the workspace once for its longest context); depends only on
 * host-side fields; 0 means it never splits. */
CF_API size_t cf_paged_attention_v1_workspace_size(const cf_paged_attention_params* params);

/* Partitioned decode attention: partitions of 512 tokens, then an exp-sum/max
 * reduce kernel.  Replaces cacheflow::cuda::launch_paged_attention_v2
 * (paged_attention.cuh:48-54).  exp_sums/max_logits are
 * [num_seqs, num_heads, num_partitions] and tmp_output is
 * [num_seqs, num_heads, num_partitions, head_dim], all float32.  They are
 * overwritten (no pre-zeroing needed) and hold, per partition: the max logit,
 * the sum of exp(logit - max) and the partition's normalised output.
 * num_partitions must be >= ceil(max_context_len / 512). */
CF_API cf_status cf_paged_attention_v2(const cf_paged_attention_params* params,
                                float* exp_sums, float* max_logits,
                                float* tmp_output, int32_t num_partitions,
                                void* stream);

/* Fused decode step: appends every row's newest token to the cache and
 * attends, in one launch.  Equal to cf_reshape_and_cache(key, value,
 * key_cache, value_cache, slot_mapping, num_tokens = num_seqs, ...) followed by
 * cf_paged_attention_v1 (same workspace rules) on `params`, for batches in
 * which row s's new token sits at position context_lens[s] - 1 (it is already
 * counted in context_lens, as in CacheFlow's prepare_kv_cache_inputs,
 * batch_decode.cpp:103-114).  Replaces the pair
 * cacheflow::cuda::launch_reshape_and_cache (kv_cache_kernels.cuh:17-27) +
 * launch_paged_attention_v1 (paged_attention.cuh:44-46) that
 * BatchDecodeEngine issues per step.
 *   key, value    [num_seqs, num_kv_heads, head_dim] of params->dtype, 16-byte
 *                 aligned: the new token of each row.
 *   slot_mapping  [num_seqs] or NULL.  NULL: the slot is the one the block
 *                 table gives position context_lens[s] - 1.  An entry < 0:
 *                 row s appends nothing.  An entry >= 0 must equal that slot;
 *                 otherwise CF_DEVERR_SLOT is recorded and the row appends
 *                 nothing.
 * params->key_cache / value_cache are WRITTEN (the appended rows), so
 * params->num_blocks must be the pool size (> 0).  No row may
 * read a slot that another row appends in the same call (a sequence appends
 * into its own last block; copy-on-write forks run before, as in CacheFlow's
 * scheduler).  Rows with context 0 append nothing. */
CF_API cf_status cf_paged_attention_append_v1(const cf_paged_attention_params* params,
                                              const void* key, const void* value,
                                              const int32_t* slot_mapping, void* workspace,
                                              size_t workspace_bytes, void* stream);

/* The same fused step on the partitioned path: cf_reshape_and_cache followed
 * by cf_paged_attention_v2 (same scratch rules).  Replaces
 * launch_reshape_and_cache + launch_paged_attention_v2 (paged_attention.cuh:48-54). */
CF_API cf_status cf_paged_attention_append_v2(const cf_paged_attention_params* params,
                                              const void* key, const void* value,
                                              const int32_t* slot_mapping, float* exp_sums,
                                              float* max_logits, float* tmp_output,
                                              int32_t num_partitions, void* stream);

/* Decode attention over fp8 (e4m3) KV caches: the stored values times the
 * per-cache scales are K and V (K = k_scale * stored, V = v_scale * stored).
 * params->dtype is the type of the query and the output (CF_F16 or CF_BF16);
 * head_dim 128 or 256.  Same workspace rules and results as
 * cf_paged_attention_v1 over the dequantized caches, within the 16-bit
 * attention tolerance.  Halves the KV bytes of a 16-bit cache.  No reference
 * counterpart (CacheFlow's caches are fp32); fill such caches with
 * cf_reshape_and_cache_fp8; cf_copy_blocks / cf_compact_kv_cache /
 * cf_memset_blocks / cf_swap_blocks take them with dtype CF_FP8_E4M3. */
CF_API cf_status cf_paged_attention_fp8_v1(const cf_paged_attention_params* params,
                                           float k_scale, float v_scale, void* workspace,
                                           size_t workspace_bytes, void* stream);

/* Partitioned form of cf_paged_attention_fp8_v1 (scratch as cf_paged_attention_v2). */
CF_API cf_status cf_paged_attention_fp8_v2(const cf_paged_attention_params* params,
                                           float k_scale, float v_scale, float* exp_sums,
                                           float* max_logits, float* tmp_output,
                                           int32_t num_partitions, void* stream);

/* Fused decode step over fp8 caches: cf_reshape_and_cache_fp8(key, value, ...,
 * slot_mapping, num_tokens = num_seqs, k_scale, v_scale) followed by
 * cf_paged_attention_fp8_v1, in one launch.  Same rules as
 * cf_paged_attention_append_v1 (row s appends at position context_lens[s] - 1;
 * key / value [num_seqs, num_kv_heads, head_dim] of params->dtype, 16-byte
 * aligned) and the same stored bytes as cf_reshape_and_cache_fp8. */
CF_API cf_status cf_paged_attention_fp8_append_v1(const cf_paged_attention_params* params,
                                                  float k_scale, float v_scale, const void* key,
                                                  const void* value, const int32_t* slot_mapping,
                                                  void* workspace, size_t workspace_bytes,
                                                  void* stream);

/* Partitioned form of cf_paged_attention_fp8_append_v1 (scratch as
 * cf_paged_attention_v2). */
CF_API cf_status cf_paged_attention_fp8_append_v2(const cf_paged_attention_params* params,
                                                  float k_scale, float v_scale, const void* key,
                                                  const void* value, const int32_t* slot_mapping,
                                                  float* exp_sums, float* max_logits,
                                                  float* tmp_output, int32_t num_partitions,
                                                  void* stream);

/* cf_reshape_and_cache into fp8 (e4m3) caches: key/value rows of `dtype`
 * (CF_F32, CF_F16 or CF_BF16) are stored as e4m3(x / scale) -- x / scale
 * rounded to f32, then to the nearest e4m3 (ties to even), saturating at
 * +-448.  head_dim a multiple of 16; all four pointers 16-byte aligned. */
CF_API cf_status cf_reshape_and_cache_fp8(const void* key, const void* value, void* key_cache,
                                          void* value_cache, const int32_t* slot_mapping,
                                          int32_t num_tokens, int32_t num_kv_heads,
                                          int32_t head_dim, int32_t block_size,
                                          int64_t num_blocks, int32_t dtype, float k_scale,
                                          float v_scale, void* stream);

/* Device-side batch preparation.  Builds, on the device, what CacheFlow's
 * BatchDecodeEngine::prepare_kv_cache_inputs (batch_decode.cpp:92-131) builds
 * on the host each step, from every row's block ids in one contiguous list:
 * row s owns block_ids[block_offsets[s] .. block_offsets[s + 1]).
 *   block_tables [num_seqs, max_blocks_per_seq]: the row's ids, then 0
 *   context_lens [num_seqs]: positions[s] + 1 (0 for a negative position)
 *   slot_mapping [num_seqs]: the slot of position positions[s], or -1 when the
 *                row has no block for it (the reference leaves it unset)
 * block_offsets is int64 [num_seqs + 1].  A row with more than
 * max_blocks_per_seq ids keeps the first ones and records
 * CF_DEVERR_CONTEXT_LEN. */
CF_API cf_status cf_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                        const int32_t* block_ids, int32_t num_seqs,
                                        int32_t max_blocks_per_seq, int32_t block_size,
                                        int32_t* block_tables, int32_t* context_lens,
                                        int32_t* slot_mapping, void* stream);

/* Parameters of one chunked-prefill attention call.  Chunk c owns query
 * tokens [query_start[c], query_start[c+1]) (its chunk length n_c) and a
 * sequence whose first context_lens[c] tokens are in the cache, the chunk's
 * own K/V rows included (write them with cf_reshape_and_cache first).  Query
 * token i of the chunk sits at position context_lens[c] - n_c + i and attends
 * to positions 0..that position (causal). */
typedef struct cf_prefill_params {
  const void* query;            /* [total query tokens, num_heads, head_dim]  */
  const void* key_cache;        /* [num_blocks, num_kv_heads, block_size, head_dim] */
  const void* value_cache;
  void* output;                 /* [total query tokens, num_heads, head_dim]  */
  const int32_t* block_tables;  /* [num_chunks, max_blocks_per_seq]          */
  const int32_t* context_lens;  /* [num_chunks]                               */
  const int32_t* query_start;   /* [num_chunks + 1], query_start[0] = 0       */
  float scale;
  int32_t num_chunks;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;             /* 64 or 128                                  */
  int32_t block_size;           /* 16                                         */
  int32_t max_query_len;        /* host-side upper bound of the chunk lengths */
  int32_t max_blocks_per_seq;
  int64_t num_blocks;           /* pool size (> 0)                            */
  int32_t dtype;                /* CF_F16 or CF_BF16                          */
} cf_prefill_params;

/* Chunked-prefill attention over the paged cache: for every chunk, all its
 * query tokens x the query heads of one KV head share one stream of the
 * context through shared memory, on tensor cores.  Equal, within the 16-bit
 * attention tolerance, to one cf_paged_attention_v1 row per query token with
 * context length = its position + 1 (what CacheFlow would have to do: it has
 * no multi-query operator; its forward pass is the abstract ForwardFn of
 * batch_decode.h:34-42). */
CF_API cf_status cf_paged_prefill_attention(const cf_prefill_params* params, void* stream);

/* Size of the library's built-in scratch for
 * cf_paged_attention_v2_static_scratch: 16 MiB of device memory on every GPU
 * where the entry point has been called, held until the process exits.  With
 * CUDA's lazy module loading (the default) the array is placed in device
 * memory by the first call on a device, not when the library loads. */
#define CF_STATIC_SCRATCH_BYTES (16u << 20)

/* The same computation as cf_paged_attention_v2 for callers that cannot
 * allocate device memory: hosts whose own pool already owns all of the GPU's
 * memory, hosts that must not call cudaMalloc/cudaFree on the decode path
 * because those calls can synchronise the device, and foreign-function hosts
 * that hold raw device pointers but no allocator.  The caller passes only the
 * inputs and the output (params); the partition scratch lives in a fixed
 * array inside the library, so this call allocates nothing.
 *
 * Limit: num_seqs * num_heads * ceil(max_context_len / 512) * (head_dim + 2)
 * floats (plus alignment) must fit in CF_STATIC_SCRATCH_BYTES; a larger call
 * returns CF_ERR_WORKSPACE and launches nothing.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current, which can also place the
 * array in device memory: make that first call before any stream capture
 * starts and before the host's own pool takes the device's free memory.  A
 * failed lookup returns its error and is retried by the next call.  All calls share the one array, which
 * keeps the last call's contents (nothing in it needs to start at zero):
 * calls whose kernels overlap on the GPU -- on different streams, or from
 * different threads -- race on it and must be serialised by the caller.
 * This entry point has no counterpart in CacheFlow. */
CF_API cf_status cf_paged_attention_v2_static_scratch(const cf_paged_attention_params* params,
                                                      void* stream);

/* Scatter new K/V rows into their cache slots:
 *   cache[slot / block_size, h, slot % block_size, :] = kv[t, h, :]
 * with slot = slot_mapping[t].  A negative slot skips the token (padding).
 * Replaces cacheflow::cuda::launch_reshape_and_cache (kv_cache_kernels.cuh:17-27). */
CF_API cf_status cf_reshape_and_cache(const void* key, const void* value,
                               void* key_cache, void* value_cache,
                               const int32_t* slot_mapping, int32_t num_tokens,
                               int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, int64_t num_blocks,
                               int32_t dtype, void* stream);

/* Copy whole K and V blocks within one cache (copy-on-write forks):
 * for each pair i, block block_mapping[2i+1] := block block_mapping[2i].
 * Pairs run concurrently: a destination must not be another pair's source.
 * Replaces cacheflow::cuda::launch_copy_blocks (kv_cache_kernels.cuh:29-37). */
CF_API cf_status cf_copy_blocks(void* key_cache, void* value_cache,
                         const int64_t* block_mapping, int32_t num_pairs,
                         int32_t num_kv_heads, int32_t head_dim,
                         int32_t block_size, int64_t num_blocks, int32_t dtype,
                         void* stream);

/* Copy blocks of `block_size_bytes` between two caches, one of which may be
 * pinned host memory (device <-> host swap): for each pair i, block
 * block_mapping[2i+1] of dst_cache := block block_mapping[2i] of src_cache.
 * block_mapping is device-readable (device or pinned host).  Runs on the SMs
 * through the host link, like the reference.
 * Replaces cacheflow::cuda::launch_swap_blocks (kv_cache_kernels.cuh:39-45). */
CF_API cf_status cf_swap_blocks(const void* src_cache, void* dst_cache,
                         const int64_t* block_mapping, int32_t num_pairs,
                         int64_t block_size_bytes, void* stream);

/* Same copy as cf_swap_blocks, with block_mapping in HOST memory, the pairs
 * applied in order: pairs whose source and destination ids both advance by
 * one are merged into one cudaMemcpyAsync (within one pool only while the
 * merged run reads no block it writes), so the copy engines move them (no SM
 * time).  Use a side stream so the swap overlaps attention. */
CF_API cf_status cf_swap_blocks_dma(const void* src_cache, void* dst_cache,
                             const int64_t* host_block_mapping,
                             int32_t num_pairs, int64_t block_size_bytes,
                             void* stream);

/* Executes one scheduling step's block operations -- CacheFlow's
 * SchedulerOutput::block_swaps_out, block_swaps_in and block_copies
 * (scheduler.h:22-29, produced at scheduler.cpp:223,252) -- on `stream`, in
 * that order and for both K and V: swap-outs (GPU block -> CPU block),
 * swap-ins (CPU block -> GPU block), then copy-on-write copies (GPU -> GPU).
 * Each list is HOST int64 [n, 2] of (src, dst) block ids; every id is checked
 * against its pool before anything is enqueued (CF_ERR_INVALID_ARGUMENT).
 * Within one list the pairs apply in order.  A list of scattered ids runs on
 * the SM copy kernel (K and V in one launch per 4000 pairs, the pairs passed
 * in the kernel parameters, so the host lists may be freed on return and
 * nothing is allocated); a list of long runs of consecutive ids (16 or more
 * per run on average), a list whose destinations repeat or feed another
 * pair, or a CPU pool the device cannot address (pageable memory) runs on the
 * copy engines instead, one cudaMemcpyAsync per run.  CPU pools should be
 * pinned: pageable ones make the copies synchronous. */
CF_API cf_status cf_execute_block_ops(void* gpu_key_cache, void* gpu_value_cache,
                                      void* cpu_key_cache, void* cpu_value_cache,
                                      int64_t block_size_bytes, int64_t num_gpu_blocks,
                                      int64_t num_cpu_blocks, const int64_t* swaps_out,
                                      int32_t num_swaps_out, const int64_t* swaps_in,
                                      int32_t num_swaps_in, const int64_t* copies,
                                      int32_t num_copies, void* stream);

/* In-place defragmentation: for each i, K and V block dst_ids[i] := block
 * src_ids[i] (src == dst is skipped).  All moves run concurrently, so the
 * plan must not overlap: no destination may also be a source, and no
 * destination may repeat (cf_compaction_plan builds such plans and
 * cf_check_compaction_plan verifies one on the host).
 * Replaces cacheflow::cuda::launch_compact_kv_cache (kv_cache_kernels.cuh:47-56). */
CF_API cf_status cf_compact_kv_cache(void* key_cache, void* value_cache,
                              const int32_t* src_block_ids,
                              const int32_t* dst_block_ids, int32_t num_moves,
                              int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, int64_t num_blocks,
                              int32_t dtype, void* stream);

/* Zero the listed blocks of one cache (blocks of block_size_bytes bytes).
 * Replaces cacheflow::cuda::launch_memset_blocks (memory_utils.cuh:28-33). */
CF_API cf_status cf_memset_blocks(void* cache, const int32_t* block_ids,
                           int32_t num_listed, int64_t block_size_bytes,
                           int64_t num_blocks, void* stream);

/* HOST-side planner for compaction.  `used` has num_blocks bytes (non-zero =
 * block holds live data).  Emits moves that pack the live blocks into
 * [0, num_used): every live block at or above num_used moves into a free slot
 * below it, so sources and destinations never overlap.  `src_out`/`dst_out`
 * need room for num_blocks entries; *num_moves receives the count.
 * Pure host code; counterpart of the planning CacheFlow leaves to
 * BlockManager::compute_fragmentation (block_manager.cpp:177-222). */
CF_API cf_status cf_compaction_plan(const uint8_t* used, int64_t num_blocks,
                             int32_t* src_out, int32_t* dst_out,
                             int32_t* num_moves);

/* HOST-side check that a compaction / copy plan is race-free: ids in range,
 * destinations unique, and no destination also used as a source.
 * Returns CF_OK, CF_ERR_INVALID_ARGUMENT (out of range) or CF_ERR_PLAN. */
CF_API cf_status cf_check_compaction_plan(const int32_t* src_ids, const int32_t* dst_ids,
                                   int32_t num_moves, int64_t num_blocks);

/* Reads (and optionally clears) the OR of all device error bits recorded by
 * kernels on `device` since the last clear.  Synchronises that device. */
CF_API cf_status cf_get_device_errors(int32_t device, uint32_t* flags, int32_t clear);

/* TEST HOOK, not for production use.  Every decode-attention launch after
 * this call (cf_paged_attention_* of every form, process-wide) gives up a
 * pipeline wait after wait_limit_ns nanoseconds instead of 2 s (0 restores
 * 2 s), and with unarm_first_stage = 1 leaves the first shared-memory stage
 * of every warp unarmed: no copy is issued for it and nothing arrives on its
 * barrier, so that wait can only run out.  The kernel then records
 * CF_DEVERR_TIMEOUT, writes no output and returns: the path a copy that never
 * completes would take, exercised with no copy in flight.  (0, 0) restores
 * normal operation.  No counterpart in CacheFlow. */
CF_API cf_status cf_testing_set_pipeline_faults(int64_t wait_limit_ns, int32_t unarm_first_stage);

/* The last cudaError_t seen by any entry point on this thread. */
CF_API int32_t cf_last_cuda_error(void);

CF_API const char* cf_status_string(cf_status status);

/* CF_ABI_VERSION of the loaded library. */
CF_API int32_t cf_abi_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CACHEFLOW_B200_H_ */
