// ref_api_driver.cpp -- CacheFlow's own CUDA-layer call shape, compiled
// against CacheFlow's UNCHANGED headers (src/cacheflow/cuda/paged_attention.cuh,
// kv_cache_kernels.cuh, memory_utils.cuh) and linked against
// libcacheflow_b200.so, so every cacheflow::cuda::launch_* call below resolves
// to this library's exported C++ entry points.  TEST INFRASTRUCTURE ONLY
// (built into oracle/_ref/ by oracle/Makefile): the GPU tests call these
// extern "C" wrappers through ctypes and compare the results with CacheFlow's
// own kernels (ref_cuda_shim.cu) and with the oracle.
//
// Each wrapper returns cacheflow::cuda::last_status(), this library's status
// of the call (not part of CacheFlow's headers, declared here).
#include <cuda_runtime.h>

#include <cstdint>

#include "cacheflow/cuda/kv_cache_kernels.cuh"
#include "cacheflow/cuda/memory_utils.cuh"
#include "cacheflow/cuda/paged_attention.cuh"

namespace cacheflow {
namespace cuda {
int last_status();  // libcacheflow_b200 addition: cf_status of the last call on this thread
}  // namespace cuda
}  // namespace cacheflow

#define API extern "C" __attribute__((visibility("default")))

namespace {
cacheflow::cuda::PagedAttentionParams params(const float* q, const float* k, const float* v, float* out,
                                             const int32_t* bt, const int32_t* cl, float scale,
                                             int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                             int32_t head_dim, int32_t block_size, int32_t max_context_len,
                                             int32_t max_blocks_per_seq) {
  cacheflow::cuda::PagedAttentionParams p{};
  p.query = q;
  p.key_cache = k;
  p.value_cache = v;
  p.output = out;
  p.block_tables = bt;
  p.context_lens = cl;
  p.scale = scale;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.max_context_len = max_context_len;
  p.max_blocks_per_seq = max_blocks_per_seq;
  return p;
}
}  // namespace

API int api_paged_attention_v1(const float* q, const float* k, const float* v, float* out, const int32_t* bt,
                               const int32_t* cl, float scale, int32_t num_seqs, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int32_t max_context_len, int32_t max_blocks_per_seq, void* stream) {
  cacheflow::cuda::launch_paged_attention_v1(
      params(q, k, v, out, bt, cl, scale, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
             max_context_len, max_blocks_per_seq),
      (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_paged_attention_v2(const float* q, const float* k, const float* v, float* out, const int32_t* bt,
                               const int32_t* cl, float scale, int32_t num_seqs, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int32_t max_context_len, int32_t max_blocks_per_seq, float* exp_sums,
                               float* max_logits, float* tmp_output, int32_t num_partitions, void* stream) {
  cacheflow::cuda::launch_paged_attention_v2(
      params(q, k, v, out, bt, cl, scale, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
             max_context_len, max_blocks_per_seq),
      exp_sums, max_logits, tmp_output, num_partitions, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_reshape_and_cache(const float* key, const float* value, float* key_cache, float* value_cache,
                              const int32_t* slot_mapping, int32_t num_tokens, int32_t num_kv_heads,
                              int32_t head_dim, int32_t block_size, void* stream) {
  cacheflow::cuda::launch_reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, num_tokens,
                                            num_kv_heads, head_dim, block_size, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_copy_blocks(float* key_cache, float* value_cache, const int64_t* block_mapping, int32_t num_pairs,
                        int32_t num_kv_heads, int32_t head_dim, int32_t block_size, void* stream) {
  cacheflow::cuda::launch_copy_blocks(key_cache, value_cache, block_mapping, num_pairs, num_kv_heads, head_dim,
                                      block_size, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_swap_blocks(float* src_cache, float* dst_cache, const int64_t* block_mapping, int32_t num_pairs,
                        int32_t block_size_bytes, void* stream) {
  cacheflow::cuda::launch_swap_blocks(src_cache, dst_cache, block_mapping, num_pairs, block_size_bytes,
                                      (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_compact_kv_cache(float* key_cache, float* value_cache, const int32_t* src_ids, const int32_t* dst_ids,
                             int32_t num_moves, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             void* stream) {
  cacheflow::cuda::launch_compact_kv_cache(key_cache, value_cache, src_ids, dst_ids, num_moves, num_kv_heads,
                                           head_dim, block_size, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_memset_blocks(float* cache, const int32_t* block_ids, int32_t num_listed, int32_t block_size_bytes,
                          void* stream) {
  cacheflow::cuda::launch_memset_blocks(cache, block_ids, num_listed, block_size_bytes, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API int api_async_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  cacheflow::cuda::async_memcpy_d2d(dst, src, bytes, (cudaStream_t)stream);
  return cacheflow::cuda::last_status();
}

API void api_synchronize_device() { cacheflow::cuda::synchronize_device(); }

API int api_last_status() { return cacheflow::cuda::last_status(); }
