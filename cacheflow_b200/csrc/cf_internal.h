// cf_internal.h -- host-side declarations shared by the library's translation
// units (launchers, per-TU device error words, status helpers).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cacheflow_b200.h"

namespace cfb {

// Records the CUDA error (thread-local) and maps it to a status.
cf_status cuda_status(cudaError_t err);

// Checks the launch that was just issued.
inline cf_status check_launch() { return cuda_status(cudaGetLastError()); }

inline int dtype_bytes(int32_t dtype) {
  return dtype == CF_F32 ? 4 : (dtype == CF_F16 || dtype == CF_BF16) ? 2 : dtype == CF_FP8_E4M3 ? 1 : 0;
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---- paged attention (paged_attention.cu) ---------------------------------
struct AttnLaunch {
  const cf_paged_attention_params* p;
  int32_t part_tokens;  // tokens per partition; <= 0: one partition per sequence
  int32_t num_parts;    // partition stride of the scratch arrays
  float* part_max;      // [num_seqs, num_heads, num_parts] or null (unsplit)
  float* part_sum;
  float* part_out;      // [num_seqs, num_heads, num_parts, head_dim]
  cudaStream_t stream;
  // Fused append of each row's newest token (null new_k: attention only).
  const void* new_k = nullptr;  // [num_seqs, num_kv_heads, head_dim]
  const void* new_v = nullptr;
  const int32_t* slot_mapping = nullptr;  // [num_seqs] or null
  // Element type of the caches when it differs from p->dtype (CF_FP8_E4M3),
  // else -1; an fp8 cache holds K / k_scale and V / v_scale.
  int32_t cache_dtype = -1;
  float k_scale = 1.f;
  float v_scale = 1.f;
};
cf_status launch_paged_attention(const AttnLaunch& l);
bool attention_supported(int32_t head_dim, int32_t block_size, int32_t dtype);
// fp8 (e4m3) caches with f16 / bf16 queries.
bool attention_fp8_supported(int32_t head_dim, int32_t block_size, int32_t dtype);
// K or V cache as a 2-D tensor map [rows, D] of 16-bit (or fp8) elements,
// boxes of 16 rows x 128 bytes (64 or 128 elements) with the 128-byte
// swizzle; false if it cannot be encoded.
bool kv_tensor_map(CUtensorMap* map, const void* base, int64_t rows, int D, int32_t dtype);
cf_status attention_read_errors(uint32_t* bits, bool clear);

// ---- chunked-prefill attention (prefill_attention.cu) ------------------------
bool prefill_supported(int32_t head_dim, int32_t block_size, int32_t dtype, int32_t group);
cf_status launch_paged_prefill(const cf_prefill_params& p, cudaStream_t stream);
cf_status prefill_read_errors(uint32_t* bits, bool clear);

// ---- KV-cache data movement (cache_ops.cu) ---------------------------------
cf_status launch_reshape_and_cache(const void* key, const void* value, void* key_cache,
                                   void* value_cache, const int32_t* slot_mapping,
                                   int32_t num_tokens, int32_t num_kv_heads, int64_t row_bytes,
                                   int32_t block_size, int64_t num_blocks, cudaStream_t stream);
cf_status launch_copy_pairs64(void* key_cache, void* value_cache, const int64_t* mapping,
                              int32_t num_pairs, int64_t block_bytes, int64_t num_blocks,
                              cudaStream_t stream);
cf_status launch_swap_pairs64(const void* src_cache, void* dst_cache, const int64_t* mapping,
                              int32_t num_pairs, int64_t block_bytes, cudaStream_t stream);
cf_status launch_move_blocks32(void* key_cache, void* value_cache, const int32_t* src_ids,
                               const int32_t* dst_ids, int32_t num_moves, int64_t block_bytes,
                               int64_t num_blocks, cudaStream_t stream);
// K and V blocks copied for a HOST list of int64 (src, dst) pairs (ids below
// 2^31), the list passed by value in the kernel parameters (no device copy of
// it); one launch per 4000 pairs.  Pairs of one launch run concurrently.
cf_status launch_host_pairs(const void* src_k, void* dst_k, const void* src_v, void* dst_v,
                            const int64_t* host_pairs, int32_t num_pairs, int64_t block_bytes,
                            int64_t num_src_blocks, int64_t num_dst_blocks, cudaStream_t stream);
cf_status launch_memset_blocks(void* cache, const int32_t* ids, int32_t num_listed,
                               int64_t block_bytes, int64_t num_blocks, cudaStream_t stream);
cf_status launch_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                     const int32_t* block_ids, int32_t num_seqs,
                                     int32_t max_blocks_per_seq, int32_t block_size,
                                     int32_t* block_tables, int32_t* context_lens,
                                     int32_t* slot_mapping, cudaStream_t stream);
// Quantizing scatter into fp8 (e4m3) caches: cache = e4m3(kv / scale).
cf_status launch_reshape_and_cache_fp8(const void* key, const void* value, void* key_cache,
                                       void* value_cache, const int32_t* slot_mapping,
                                       int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                       int32_t block_size, int64_t num_blocks, int32_t dtype,
                                       float k_scale, float v_scale, cudaStream_t stream);
cf_status cache_ops_read_errors(uint32_t* bits, bool clear);

}  // namespace cfb
