// cacheflow_b200_compat.hpp -- the C++ entry points of CacheFlow's CUDA layer,
// exported by libcacheflow_b200.so with the reference's exact signatures, so
// CacheFlow's host code (BatchDecodeEngine and friends) links against this
// library instead of compiling src/cacheflow/cuda/*.cu.
//
// The declarations must match the reference's headers symbol for symbol:
//   src/cacheflow/cuda/paged_attention.cuh:25-54
//   src/cacheflow/cuda/kv_cache_kernels.cuh:17-56
//   src/cacheflow/cuda/memory_utils.cuh:17-36
// The reference headers themselves can be used unchanged instead of this one.
//
// Behaviour differences from the reference (all in the caller's favour):
//   - every shape the reference silently skipped either runs or logs once to
//     stderr; the status of the last call is in cacheflow::cuda::last_status();
//   - paged attention is normalised softmax attention for every context length;
//   - launch_paged_attention_v2 overwrites its scratch (no pre-zeroing).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define CF_COMPAT_API __attribute__((visibility("default")))
#else
#define CF_COMPAT_API
#endif

namespace cacheflow {
namespace cuda {

struct PagedAttentionParams {
  const float* query;          // [num_seqs, num_heads, head_dim]
  const float* key_cache;      // [num_blocks, num_kv_heads, block_size, head_dim]
  const float* value_cache;    // [num_blocks, num_kv_heads, block_size, head_dim]
  float* output;               // [num_seqs, num_heads, head_dim]
  const int32_t* block_tables; // [num_seqs, max_blocks_per_seq]
  const int32_t* context_lens; // [num_seqs]
  float scale;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t block_size;
  int32_t max_context_len;
  int32_t max_blocks_per_seq;
};

CF_COMPAT_API void launch_paged_attention_v1(const PagedAttentionParams& params,
                               cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_paged_attention_v2(const PagedAttentionParams& params,
                               float* exp_sums, float* max_logits,
                               float* tmp_output, int32_t num_partitions,
                               cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_reshape_and_cache(const float* key, const float* value,
                              float* key_cache, float* value_cache,
                              const int32_t* slot_mapping, int32_t num_tokens,
                              int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_copy_blocks(float* key_cache, float* value_cache,
                        const int64_t* block_mapping, int32_t num_pairs,
                        int32_t num_kv_heads, int32_t head_dim,
                        int32_t block_size, cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_swap_blocks(float* src_cache, float* dst_cache,
                        const int64_t* block_mapping, int32_t num_pairs,
                        int32_t block_size_bytes, cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_compact_kv_cache(float* key_cache, float* value_cache,
                             const int32_t* src_block_ids,
                             const int32_t* dst_block_ids, int32_t num_blocks,
                             int32_t num_kv_heads, int32_t head_dim,
                             int32_t block_size, cudaStream_t stream = nullptr);

CF_COMPAT_API size_t get_gpu_free_memory();
CF_COMPAT_API size_t get_gpu_total_memory();
CF_COMPAT_API float get_gpu_memory_utilization();

CF_COMPAT_API void async_memcpy_h2d(void* dst, const void* src, size_t bytes,
                      cudaStream_t stream = nullptr);
CF_COMPAT_API void async_memcpy_d2h(void* dst, const void* src, size_t bytes,
                      cudaStream_t stream = nullptr);
CF_COMPAT_API void async_memcpy_d2d(void* dst, const void* src, size_t bytes,
                      cudaStream_t stream = nullptr);

CF_COMPAT_API void launch_memset_blocks(float* cache, const int32_t* block_ids,
                          int32_t num_blocks, int32_t block_size_bytes,
                          cudaStream_t stream = nullptr);

CF_COMPAT_API void synchronize_stream(cudaStream_t stream);
CF_COMPAT_API void synchronize_device();

// Not in the reference: status (cf_status value) of the last compat call on
// this thread, for callers that want to check the void entry points.
CF_COMPAT_API int last_status();

}  // namespace cuda
}  // namespace cacheflow
