/*
 * cf_oracle.h -- CPU restatement of CacheFlow's KV-cache kernel path.
 *
 * TEST INFRASTRUCTURE ONLY.  This code is the oracle: tests, the smoke test
 * and the CPU-baseline leg of bench.py call it to produce expected results.
 * The product (libcacheflow_b200.so) never links, loads or calls it.
 *
 * Each function restates one operator of CacheFlow's CUDA layer
 * (src/cacheflow/cuda/) on host memory, citing the reference lines it
 * follows.  Element types use the C-ABI codes: 0 = f32, 1 = f16, 2 = bf16,
 * 3 = e4m3 (caches only).
 * Attention accumulates in double and computes the normalised softmax the
 * reference intends; the cache operators are byte copies.
 */
#ifndef CF_ORACLE_H_
#define CF_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

double cfo_load(const void* base, int64_t index, int32_t dtype);

/* out[s, h, d] (double) = softmax_t(scale * q.k_t) . v_t, t < context_lens[s]. */
void cfo_paged_attention(const void* query, const void* key_cache, const void* value_cache,
                         double* out, const int32_t* block_tables, const int32_t* context_lens,
                         float scale, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t block_size, int32_t max_blocks_per_seq,
                         int32_t dtype, int32_t num_threads);

/* Partition statistics of v2: for partition p of `partition_size` tokens,
 * max_logits[s,h,p] = max scaled logit, exp_sums = sum exp(logit - max),
 * tmp_out[s,h,p,:] = sum exp(logit - max) v / exp_sum.  Partitions past the
 * end of a sequence are left untouched. */
void cfo_paged_attention_partitions(const void* query, const void* key_cache,
                                    const void* value_cache, const int32_t* block_tables,
                                    const int32_t* context_lens, float scale, int32_t num_seqs,
                                    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t block_size, int32_t max_blocks_per_seq, int32_t dtype,
                                    int32_t partition_size, int32_t num_partitions,
                                    double* max_logits, double* exp_sums, double* tmp_out);

/* v2 reduce: out = sum_p w_p tmp_p / sum_p w_p, w_p = exp_sum_p exp(max_p - max). */
void cfo_paged_attention_reduce(const double* max_logits, const double* exp_sums,
                                const double* tmp_out, const int32_t* context_lens,
                                int32_t num_seqs, int32_t num_heads, int32_t head_dim,
                                int32_t partition_size, int32_t num_partitions, double* out);

void cfo_reshape_and_cache(const void* key, const void* value, void* key_cache,
                           void* value_cache, const int32_t* slot_mapping, int32_t num_tokens,
                           int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                           int32_t elem_bytes);

void cfo_copy_blocks(void* key_cache, void* value_cache, const int64_t* block_mapping,
                     int32_t num_pairs, int64_t block_bytes);

void cfo_swap_blocks(const void* src_cache, void* dst_cache, const int64_t* block_mapping,
                     int32_t num_pairs, int64_t block_bytes);

void cfo_compact_kv_cache(void* key_cache, void* value_cache, const int32_t* src_ids,
                          const int32_t* dst_ids, int32_t num_moves, int64_t block_bytes);

void cfo_memset_blocks(void* cache, const int32_t* block_ids, int32_t num_listed,
                       int64_t block_bytes);

/* fp8 (e4m3) caches: K = k_scale * stored, V = v_scale * stored, the query
 * of element type `dtype`; otherwise as cfo_paged_attention. */
void cfo_paged_attention_fp8(const void* query, const void* key_cache, const void* value_cache,
                             double* out, const int32_t* block_tables, const int32_t* context_lens,
                             float scale, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t block_size, int32_t max_blocks_per_seq,
                             int32_t dtype, float k_scale, float v_scale, int32_t num_threads);

/* Round to e4m3 (OCP "E4M3FN"): nearest, ties to even, saturating at 448;
 * NaN -> 0x7f. */
uint8_t cfo_e4m3_from_float(float x);

/* reshape_and_cache into e4m3 caches: cache = e4m3(float(x) / scale). */
void cfo_reshape_and_cache_fp8(const void* key, const void* value, uint8_t* key_cache,
                               uint8_t* value_cache, const int32_t* slot_mapping,
                               int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, int32_t dtype, float k_scale, float v_scale);

/* Decode-batch preparation of BatchDecodeEngine::prepare_kv_cache_inputs
 * (batch_decode.cpp:92-131), rows given as CSR block lists: row s at
 * positions[s] owns block_ids[block_offsets[s] .. block_offsets[s+1]).
 * Writes block_tables [num_seqs, max_blocks_per_seq] (ids, then 0),
 * context_lens = position + 1 (0 for a negative position) and slot_mapping
 * (-1 where the reference leaves the slot unset); rows longer than
 * max_blocks_per_seq are cut.  Returns the number of cut rows. */
int32_t cfo_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                const int32_t* block_ids, int32_t num_seqs,
                                int32_t max_blocks_per_seq, int32_t block_size,
                                int32_t* block_tables, int32_t* context_lens,
                                int32_t* slot_mapping);

#ifdef __cplusplus
}
#endif

#endif /* CF_ORACLE_H_ */
