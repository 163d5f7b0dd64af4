// ref_cuda_shim.cu -- extern "C" entry points over CacheFlow's OWN CUDA
// kernels, compiled from the reference sources into oracle/_ref/ (see
// oracle/Makefile).  TEST INFRASTRUCTURE ONLY: GPU parity tests use it to run
// the reference kernels on the same device buffers as ours, and
// tests/golden/make_golden.py uses it to record golden vectors.
//
// Only inputs the reference handles correctly are passed through it:
// the four data-movement kernels (fp32), and V1 attention with
// head_dim 128 or 64, block 16 and every context <= 128 tokens (above that
// the reference's 128-float shared array overflows, paged_attention.cu:64).
#include <cuda_runtime.h>

#include <cstdint>

#include "cacheflow/cuda/kv_cache_kernels.cuh"
#include "cacheflow/cuda/memory_utils.cuh"
#include "cacheflow/cuda/paged_attention.cuh"

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API int ref_paged_attention_v1(const float* q, const float* k, const float* v, float* out,
                                   const int32_t* block_tables, const int32_t* context_lens,
                                   float scale, int32_t num_seqs, int32_t num_heads,
                                   int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                   int32_t max_context_len, int32_t max_blocks_per_seq) {
  if (max_context_len > 128 || block_size != 16 || (head_dim != 128 && head_dim != 64)) return 1;
  cacheflow::cuda::PagedAttentionParams p{};
  p.query = q;
  p.key_cache = k;
  p.value_cache = v;
  p.output = out;
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.scale = scale;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.max_context_len = max_context_len;
  p.max_blocks_per_seq = max_blocks_per_seq;
  cacheflow::cuda::launch_paged_attention_v1(p, nullptr);
  return (int)cudaDeviceSynchronize();
}

REF_API int ref_reshape_and_cache(const float* key, const float* value, float* key_cache,
                                  float* value_cache, const int32_t* slot_mapping,
                                  int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t block_size) {
  cacheflow::cuda::launch_reshape_and_cache(key, value, key_cache, value_cache, slot_mapping,
                                            num_tokens, num_kv_heads, head_dim, block_size,
                                            nullptr);
  return (int)cudaDeviceSynchronize();
}

REF_API int ref_copy_blocks(float* key_cache, float* value_cache, const int64_t* block_mapping,
                            int32_t num_pairs, int32_t num_kv_heads, int32_t head_dim,
                            int32_t block_size) {
  cacheflow::cuda::launch_copy_blocks(key_cache, value_cache, block_mapping, num_pairs,
                                      num_kv_heads, head_dim, block_size, nullptr);
  return (int)cudaDeviceSynchronize();
}

REF_API int ref_swap_blocks(float* src, float* dst, const int64_t* block_mapping,
                            int32_t num_pairs, int32_t block_size_bytes) {
  cacheflow::cuda::launch_swap_blocks(src, dst, block_mapping, num_pairs, block_size_bytes,
                                      nullptr);
  return (int)cudaDeviceSynchronize();
}

REF_API int ref_compact_kv_cache(float* key_cache, float* value_cache, const int32_t* src_ids,
                                 const int32_t* dst_ids, int32_t num_moves, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t block_size) {
  cacheflow::cuda::launch_compact_kv_cache(key_cache, value_cache, src_ids, dst_ids, num_moves,
                                           num_kv_heads, head_dim, block_size, nullptr);
  return (int)cudaDeviceSynchronize();
}

REF_API int ref_memset_blocks(float* cache, const int32_t* block_ids, int32_t num_listed,
                              int32_t block_size_bytes) {
  cacheflow::cuda::launch_memset_blocks(cache, block_ids, num_listed, block_size_bytes, nullptr);
  return (int)cudaDeviceSynchronize();
}
