// capi.cu -- the library's C ABI (include/cacheflow_b200.h) and the C++
// entry points with CacheFlow's exact signatures
// (include/cacheflow_b200_compat.hpp).  Host code only: argument checks,
// dispatch to the launchers, status / error-word plumbing, the copy-engine
// swap path and the host-side compaction planner.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "../../include/cacheflow_b200.h"
#include "../../include/cacheflow_b200_compat.hpp"
#include "cf_internal.h"

namespace cfb {

namespace {
thread_local int32_t t_last_cuda_error = 0;
}

cf_status cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return CF_OK;
  t_last_cuda_error = (int32_t)err;
  return CF_ERR_CUDA;
}

namespace {

constexpr int32_t kV2PartitionTokens = 512;  // CacheFlow's PARTITION_SIZE (paged_attention.cu:368)

// Tokens per partition of the split path of cf_paged_attention_v1 (policy
// below).  Shorter partitions do not pay: below ~512 tokens the extra reduce
// launch costs more than the added parallelism (the fp32 8-sequence batch
// steps in 34 us at 128- or 256-token partitions against 29 us unsplit).
// 0 disables splitting; CF_V1_SPLIT_TOKENS (a multiple of 16; 0 = never)
// overrides the choice.
int32_t v1_split_tokens(const cf_paged_attention_params* p, bool fp8_cache) {
  static const int32_t forced = [] {
    if (const char* e = std::getenv("CF_V1_SPLIT_TOKENS")) {
      long x = std::strtol(e, nullptr, 10);
      if (x >= 0 && x % 16 == 0 && x <= (1 << 24)) return (int32_t)x;
    }
    return (int32_t)-1;
  }();
  if (forced >= 0) return forced;
  // Partitions of 2048 tokens, 4096 past 8192 tokens (2048 again for an fp8
  // cache), and 8192 when such a batch also has 4096 or more (row, KV head)
  // pairs; halved down to 512 while that is needed for about four CTAs per
  // SM.  Longer partitions mean fewer CTAs (each with its own set-up and
  // merge) and fewer partial results to write and merge; shorter ones a
  // shorter tail.  Measured (attention launch, 8 KV heads, at 8192 / 4096 /
  // 2048): bf16, 1024 rows of 512-32K tokens 9.71 / 9.78 / 9.99 ms; 128 such
  // rows 1.362 / 1.356 / 1.366 ms; 16 rows of 16K-128K tokens 0.619 / 0.589
  // / 0.594 ms; fp8, 1024 rows of 512-32K tokens 5.43 / 5.54 / 5.82 ms; 16
  // rows of 16K-128K tokens 0.349 / 0.332 / 0.322 ms; 64 bf16 rows of
  // 128-4096 tokens (32 KV heads) 0.336 / 0.339 / 0.340 ms at 2048 / 1024 /
  // unsplit.
  constexpr int64_t kTargetCtas = 4 * 148;
  const int64_t pairs = (int64_t)p->num_seqs * p->num_kv_heads;
  int32_t split = p->max_context_len > 8192 ? (pairs >= 4096 ? 8192 : (fp8_cache ? 2048 : 4096)) : 2048;
  while (split > 512 && pairs * ((p->max_context_len + split - 1) / split) < kTargetCtas) split /= 2;
  return split;
}

// Address under which the current device can dereference `p`, or nullptr if
// it cannot (pageable host memory without pageable-memory access).
const void* device_view(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      return p;
    case cudaMemoryTypeHost:
      return a.devicePointer;
    default: {
      int dev = 0, pageable = 0;
      if (cudaGetDevice(&dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&pageable, cudaDevAttrPageableMemoryAccess, dev) != cudaSuccess)
        return nullptr;
      return pageable ? p : nullptr;
    }
  }
}

// Shape checks; with check_pointers, also the operands (a size query passes
// shapes only).
cf_status check_attention_params(const cf_paged_attention_params* p, bool check_pointers = true) {
  if (p == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_seqs < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_heads % p->num_kv_heads != 0) return CF_ERR_INVALID_ARGUMENT;
  if (dtype_bytes(p->dtype) == 0) return CF_ERR_INVALID_ARGUMENT;
  if (p->max_context_len < 0 || p->max_blocks_per_seq < 0 || p->num_blocks < 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (p->block_size <= 0 || p->head_dim <= 0) return CF_ERR_INVALID_ARGUMENT;
  if (!cfb::attention_supported(p->head_dim, p->block_size, p->dtype)) return CF_ERR_UNSUPPORTED;
  if (p->num_seqs == 0) return CF_OK;
  if (p->num_seqs > 65535 || p->num_heads > 65535) return CF_ERR_UNSUPPORTED;  // grid z / y
  if (p->max_blocks_per_seq < 1) return CF_ERR_INVALID_ARGUMENT;
  if ((int64_t)p->max_context_len > (int64_t)p->max_blocks_per_seq * p->block_size)
    return CF_ERR_INVALID_ARGUMENT;
  if (!check_pointers) return CF_OK;
  if (!p->query || !p->key_cache || !p->value_cache || !p->output || !p->block_tables ||
      !p->context_lens)
    return CF_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->query) || !aligned16(p->key_cache) || !aligned16(p->value_cache) ||
      !aligned16(p->output))
    return CF_ERR_INVALID_ARGUMENT;
  return CF_OK;
}

size_t v1_split_bytes(const cf_paged_attention_params* p, bool fp8_cache, int32_t* parts_out);

// Launch extras beyond the attention params: the fused append's rows and an
// fp8 cache's element type and scales.
struct Extras {
  const void* key = nullptr;
  const void* value = nullptr;
  const int32_t* slots = nullptr;
  int32_t cache_dtype = -1;
  float k_scale = 1.f;
  float v_scale = 1.f;
};

void apply(AttnLaunch& l, const Extras& x) {
  l.new_k = x.key;
  l.new_v = x.value;
  l.slot_mapping = x.slots;
  l.cache_dtype = x.cache_dtype;
  l.k_scale = x.k_scale;
  l.v_scale = x.v_scale;
}

// cf_paged_attention_v1 and its append / fp8 forms.
cf_status run_v1(const cf_paged_attention_params* p, void* workspace, size_t workspace_bytes,
                 void* stream, const Extras& x) {
  cf_status st = check_attention_params(p);
  if (st != CF_OK || p->num_seqs == 0) return st;
  AttnLaunch l{p, 0, 1, nullptr, nullptr, nullptr, (cudaStream_t)stream};
  apply(l, x);
  int32_t parts = 0;
  const bool fp8_cache = x.cache_dtype == CF_FP8_E4M3;
  const size_t need = v1_split_bytes(p, fp8_cache, &parts);
  if (need > 0 && workspace != nullptr && workspace_bytes >= need) {
    if (!aligned16(workspace)) return CF_ERR_INVALID_ARGUMENT;
    const int64_t rows = (int64_t)p->num_seqs * p->num_heads * parts;
    const int64_t r4 = (rows * 4 + 255) / 256 * 256;
    uint8_t* w = static_cast<uint8_t*>(workspace);
    l.part_tokens = v1_split_tokens(p, fp8_cache);
    l.num_parts = parts;
    l.part_max = reinterpret_cast<float*>(w);
    l.part_sum = reinterpret_cast<float*>(w + r4);
    l.part_out = reinterpret_cast<float*>(w + 2 * r4);
  }
  return launch_paged_attention(l);
}

// cf_paged_attention_v2 and its append / fp8 forms.
cf_status run_v2(const cf_paged_attention_params* p, float* exp_sums, float* max_logits,
                 float* tmp_output, int32_t num_partitions, void* stream, const Extras& x) {
  cf_status st = check_attention_params(p);
  if (st != CF_OK || p->num_seqs == 0) return st;
  if (!exp_sums || !max_logits || !tmp_output || num_partitions < 1)
    return CF_ERR_INVALID_ARGUMENT;
  const int64_t need = ((int64_t)p->max_context_len + kV2PartitionTokens - 1) / kV2PartitionTokens;
  if (need > num_partitions) return CF_ERR_WORKSPACE;
  AttnLaunch l{p, kV2PartitionTokens, num_partitions, max_logits, exp_sums, tmp_output,
               (cudaStream_t)stream};
  apply(l, x);
  return launch_paged_attention(l);
}

// Shape and scale checks of the fp8-cache entry points (params->dtype is the
// query / output type).
cf_status check_fp8(const cf_paged_attention_params* p, float k_scale, float v_scale) {
  if (p == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return CF_ERR_INVALID_ARGUMENT;
  if (p->dtype != CF_F16 && p->dtype != CF_BF16) return CF_ERR_UNSUPPORTED;
  if (!attention_fp8_supported(p->head_dim, p->block_size, p->dtype)) return CF_ERR_UNSUPPORTED;
  return CF_OK;
}

Extras fp8_extras(float k_scale, float v_scale) {
  Extras x;
  x.cache_dtype = CF_FP8_E4M3;
  x.k_scale = k_scale;
  x.v_scale = v_scale;
  return x;
}

size_t v1_split_bytes(const cf_paged_attention_params* p, bool fp8_cache, int32_t* parts_out) {
  const int32_t split = v1_split_tokens(p, fp8_cache);
  if (split <= 0 || p->num_seqs <= 0 || p->max_context_len <= split) return 0;
  const int64_t parts = (p->max_context_len + split - 1) / split;
  if (parts_out) *parts_out = (int32_t)parts;
  const int64_t rows = (int64_t)p->num_seqs * p->num_heads * parts;
  // max + sum + output, each region rounded to 256 bytes.
  auto round = [](int64_t b) { return (b + 255) / 256 * 256; };
  return (size_t)(2 * round(rows * 4) + round(rows * p->head_dim * 4));
}

}  // namespace
}  // namespace cfb

using namespace cfb;

extern "C" {

int32_t cf_abi_version(void) { return CF_ABI_VERSION; }

int32_t cf_last_cuda_error(void) { return t_last_cuda_error; }

const char* cf_status_string(cf_status status) {
  switch (status) {
    case CF_OK: return "ok";
    case CF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CF_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case CF_ERR_WORKSPACE: return "workspace too small";
    case CF_ERR_CUDA: return "CUDA runtime error";
    case CF_ERR_PLAN: return "block-move plan would race";
  }
  return "unknown status";
}

size_t cf_paged_attention_v1_workspace_size(const cf_paged_attention_params* p) {
  if (check_attention_params(p, /*check_pointers=*/false) != CF_OK) return 0;
  // Enough for every call with these sizes and any shorter max_context_len
  // (a host sizes the workspace once, for its longest context): the split
  // grows with the context, so a shorter context can need more partitions.
  // The params do not say whether the cache is fp8, so both policies count.
  cf_paged_attention_params q = *p;
  size_t bytes = 0;
  for (int64_t c = 512;; c += 512) {
    q.max_context_len = (int32_t)(c < p->max_context_len ? c : p->max_context_len);
    for (bool fp8_cache : {false, true}) {
      const size_t b = v1_split_bytes(&q, fp8_cache, nullptr);
      bytes = b > bytes ? b : bytes;
    }
    if (c >= p->max_context_len) break;
  }
  return bytes;
}

cf_status cf_paged_attention_v1(const cf_paged_attention_params* p, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return run_v1(p, workspace, workspace_bytes, stream, Extras{});
}

cf_status cf_paged_attention_v2(const cf_paged_attention_params* p, float* exp_sums,
                                float* max_logits, float* tmp_output, int32_t num_partitions,
                                void* stream) {
  return run_v2(p, exp_sums, max_logits, tmp_output, num_partitions, stream, Extras{});
}

cf_status cf_paged_attention_append_v1(const cf_paged_attention_params* p, const void* key,
                                       const void* value, const int32_t* slot_mapping,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  // The append writes the caches: block ids must be range-checked (num_blocks > 0).
  if (!key || !value || !aligned16(key) || !aligned16(value)) return CF_ERR_INVALID_ARGUMENT;
  if (p && p->num_seqs > 0 && p->num_blocks <= 0) return CF_ERR_INVALID_ARGUMENT;
  Extras x;
  x.key = key;
  x.value = value;
  x.slots = slot_mapping;
  return run_v1(p, workspace, workspace_bytes, stream, x);
}

cf_status cf_paged_attention_append_v2(const cf_paged_attention_params* p, const void* key,
                                       const void* value, const int32_t* slot_mapping,
                                       float* exp_sums, float* max_logits, float* tmp_output,
                                       int32_t num_partitions, void* stream) {
  if (!key || !value || !aligned16(key) || !aligned16(value)) return CF_ERR_INVALID_ARGUMENT;
  if (p && p->num_seqs > 0 && p->num_blocks <= 0) return CF_ERR_INVALID_ARGUMENT;
  Extras x;
  x.key = key;
  x.value = value;
  x.slots = slot_mapping;
  return run_v2(p, exp_sums, max_logits, tmp_output, num_partitions, stream, x);
}

cf_status cf_paged_attention_fp8_v1(const cf_paged_attention_params* p, float k_scale,
                                    float v_scale, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  const cf_status st = check_fp8(p, k_scale, v_scale);
  if (st != CF_OK) return st;
  return run_v1(p, workspace, workspace_bytes, stream, fp8_extras(k_scale, v_scale));
}

cf_status cf_paged_attention_fp8_v2(const cf_paged_attention_params* p, float k_scale,
                                    float v_scale, float* exp_sums, float* max_logits,
                                    float* tmp_output, int32_t num_partitions, void* stream) {
  const cf_status st = check_fp8(p, k_scale, v_scale);
  if (st != CF_OK) return st;
  return run_v2(p, exp_sums, max_logits, tmp_output, num_partitions, stream,
                fp8_extras(k_scale, v_scale));
}

cf_status cf_paged_attention_fp8_append_v1(const cf_paged_attention_params* p, float k_scale,
                                           float v_scale, const void* key, const void* value,
                                           const int32_t* slot_mapping, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  const cf_status st = check_fp8(p, k_scale, v_scale);
  if (st != CF_OK) return st;
  if (!key || !value || !aligned16(key) || !aligned16(value)) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_seqs > 0 && p->num_blocks <= 0) return CF_ERR_INVALID_ARGUMENT;
  Extras x = fp8_extras(k_scale, v_scale);
  x.key = key;
  x.value = value;
  x.slots = slot_mapping;
  return run_v1(p, workspace, workspace_bytes, stream, x);
}

cf_status cf_paged_attention_fp8_append_v2(const cf_paged_attention_params* p, float k_scale,
                                           float v_scale, const void* key, const void* value,
                                           const int32_t* slot_mapping, float* exp_sums,
                                           float* max_logits, float* tmp_output,
                                           int32_t num_partitions, void* stream) {
  const cf_status st = check_fp8(p, k_scale, v_scale);
  if (st != CF_OK) return st;
  if (!key || !value || !aligned16(key) || !aligned16(value)) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_seqs > 0 && p->num_blocks <= 0) return CF_ERR_INVALID_ARGUMENT;
  Extras x = fp8_extras(k_scale, v_scale);
  x.key = key;
  x.value = value;
  x.slots = slot_mapping;
  return run_v2(p, exp_sums, max_logits, tmp_output, num_partitions, stream, x);
}

cf_status cf_reshape_and_cache_fp8(const void* key, const void* value, void* key_cache,
                                   void* value_cache, const int32_t* slot_mapping,
                                   int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                   int32_t block_size, int64_t num_blocks, int32_t dtype,
                                   float k_scale, float v_scale, void* stream) {
  if ((dtype != CF_F32 && dtype != CF_F16 && dtype != CF_BF16) || num_tokens < 0 ||
      num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks < 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return CF_ERR_INVALID_ARGUMENT;
  if (head_dim % 16 != 0) return CF_ERR_UNSUPPORTED;
  if (num_tokens == 0) return CF_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping) return CF_ERR_INVALID_ARGUMENT;
  if (!aligned16(key) || !aligned16(value) || !aligned16(key_cache) || !aligned16(value_cache))
    return CF_ERR_INVALID_ARGUMENT;
  const int64_t nb = num_blocks > 0 ? num_blocks : INT64_MAX / ((int64_t)block_size * 2);
  return launch_reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping,
                                      num_tokens, num_kv_heads, head_dim, block_size, nb, dtype,
                                      k_scale, v_scale, (cudaStream_t)stream);
}

cf_status cf_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                 const int32_t* block_ids, int32_t num_seqs,
                                 int32_t max_blocks_per_seq, int32_t block_size,
                                 int32_t* block_tables, int32_t* context_lens,
                                 int32_t* slot_mapping, void* stream) {
  if (num_seqs < 0 || max_blocks_per_seq < 1 || block_size <= 0) return CF_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0) return CF_OK;
  if (num_seqs > 65535) return CF_ERR_UNSUPPORTED;
  if (!positions || !block_offsets || !block_ids || !block_tables || !context_lens ||
      !slot_mapping)
    return CF_ERR_INVALID_ARGUMENT;
  return launch_build_decode_inputs(positions, block_offsets, block_ids, num_seqs,
                                    max_blocks_per_seq, block_size, block_tables, context_lens,
                                    slot_mapping, (cudaStream_t)stream);
}

cf_status cf_paged_prefill_attention(const cf_prefill_params* p, void* stream) {
  if (p == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_chunks < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 ||
      p->num_heads % p->num_kv_heads != 0 || p->max_query_len < 0 || p->max_blocks_per_seq < 0 ||
      p->num_blocks < 0 || p->head_dim <= 0 || p->block_size <= 0 || dtype_bytes(p->dtype) == 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (!prefill_supported(p->head_dim, p->block_size, p->dtype, p->num_heads / p->num_kv_heads))
    return CF_ERR_UNSUPPORTED;
  if (p->num_chunks == 0 || p->max_query_len == 0) return CF_OK;
  if (p->num_chunks > 65535 || p->num_kv_heads > 65535) return CF_ERR_UNSUPPORTED;
  if (p->num_blocks == 0 || p->max_blocks_per_seq < 1) return CF_ERR_INVALID_ARGUMENT;
  if (p->num_blocks * (int64_t)p->num_kv_heads * p->block_size > INT32_MAX) return CF_ERR_UNSUPPORTED;
  if (!p->query || !p->key_cache || !p->value_cache || !p->output || !p->block_tables ||
      !p->context_lens || !p->query_start)
    return CF_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->query) || !aligned16(p->key_cache) || !aligned16(p->value_cache) ||
      !aligned16(p->output))
    return CF_ERR_INVALID_ARGUMENT;
  return launch_paged_prefill(*p, (cudaStream_t)stream);
}

cf_status cf_reshape_and_cache(const void* key, const void* value, void* key_cache,
                               void* value_cache, const int32_t* slot_mapping, int32_t num_tokens,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, int32_t dtype, void* stream) {
  const int eb = dtype_bytes(dtype);
  if (eb == 0 || num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks < 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return CF_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping) return CF_ERR_INVALID_ARGUMENT;
  const int64_t nb = num_blocks > 0 ? num_blocks : INT64_MAX / ((int64_t)block_size * 2);
  return launch_reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, num_tokens,
                                  num_kv_heads, (int64_t)head_dim * eb, block_size, nb,
                                  (cudaStream_t)stream);
}

cf_status cf_copy_blocks(void* key_cache, void* value_cache, const int64_t* block_mapping,
                         int32_t num_pairs, int32_t num_kv_heads, int32_t head_dim,
                         int32_t block_size, int64_t num_blocks, int32_t dtype, void* stream) {
  const int eb = dtype_bytes(dtype);
  if (eb == 0 || num_pairs < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks < 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (num_pairs == 0) return CF_OK;
  if (!key_cache || !value_cache || !block_mapping) return CF_ERR_INVALID_ARGUMENT;
  const int64_t bb = (int64_t)num_kv_heads * block_size * head_dim * eb;
  const int64_t nb = num_blocks > 0 ? num_blocks : INT64_MAX / bb;
  return launch_copy_pairs64(key_cache, value_cache, block_mapping, num_pairs, bb, nb,
                             (cudaStream_t)stream);
}

cf_status cf_swap_blocks(const void* src_cache, void* dst_cache, const int64_t* block_mapping,
                         int32_t num_pairs, int64_t block_size_bytes, void* stream) {
  if (num_pairs < 0 || block_size_bytes <= 0) return CF_ERR_INVALID_ARGUMENT;
  if (num_pairs == 0) return CF_OK;
  if (!src_cache || !dst_cache || !block_mapping) return CF_ERR_INVALID_ARGUMENT;
  // The kernel dereferences all three pointers on the device: pageable host
  // memory (CacheFlow's CPU pool is aligned_alloc, memory_pool.cpp:36) is
  // refused here instead of faulting the GPU.
  const void* dsrc = device_view(src_cache);
  void* ddst = const_cast<void*>(device_view(dst_cache));
  const int64_t* dmap = static_cast<const int64_t*>(device_view(block_mapping));
  if (!dsrc || !ddst || !dmap) return CF_ERR_INVALID_ARGUMENT;
  return launch_swap_pairs64(dsrc, ddst, dmap, num_pairs, block_size_bytes, (cudaStream_t)stream);
}

cf_status cf_swap_blocks_dma(const void* src_cache, void* dst_cache,
                             const int64_t* host_block_mapping, int32_t num_pairs,
                             int64_t block_size_bytes, void* stream) {
  if (num_pairs < 0 || block_size_bytes <= 0) return CF_ERR_INVALID_ARGUMENT;
  if (num_pairs == 0) return CF_OK;
  if (!src_cache || !dst_cache || !host_block_mapping) return CF_ERR_INVALID_ARGUMENT;
  for (int32_t i = 0; i < num_pairs; ++i)
    if (host_block_mapping[2 * i] < 0 || host_block_mapping[2 * i + 1] < 0)
      return CF_ERR_INVALID_ARGUMENT;
  const uint8_t* src = static_cast<const uint8_t*>(src_cache);
  uint8_t* dst = static_cast<uint8_t*>(dst_cache);
  // Within one pool a merged run must not read a block it also writes: the
  // pairs apply in order, so (1->2, 2->3) copies block 1 into both, which one
  // overlapping copy of blocks 1..2 onto 2..3 would not do.
  const bool same_pool = src_cache == dst_cache;
  int32_t i = 0;
  while (i < num_pairs) {
    const int64_t s0 = host_block_mapping[2 * i], d0 = host_block_mapping[2 * i + 1];
    const int64_t max_run = same_pool ? (s0 == d0 ? 1 : (s0 < d0 ? d0 - s0 : s0 - d0)) : INT64_MAX;
    int32_t run = 1;
    while (i + run < num_pairs && run < max_run && host_block_mapping[2 * (i + run)] == s0 + run &&
           host_block_mapping[2 * (i + run) + 1] == d0 + run)
      ++run;
    cudaError_t e = cudaMemcpyAsync(dst + d0 * block_size_bytes, src + s0 * block_size_bytes,
                                    (size_t)run * block_size_bytes, cudaMemcpyDefault,
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_status(e);
    i += run;
  }
  return CF_OK;
}

cf_status cf_execute_block_ops(void* gpu_key_cache, void* gpu_value_cache, void* cpu_key_cache,
                               void* cpu_value_cache, int64_t block_size_bytes,
                               int64_t num_gpu_blocks, int64_t num_cpu_blocks,
                               const int64_t* swaps_out, int32_t num_swaps_out,
                               const int64_t* swaps_in, int32_t num_swaps_in,
                               const int64_t* copies, int32_t num_copies, void* stream) {
  if (block_size_bytes <= 0 || num_gpu_blocks < 0 || num_cpu_blocks < 0 || num_swaps_out < 0 ||
      num_swaps_in < 0 || num_copies < 0)
    return CF_ERR_INVALID_ARGUMENT;
  // Every id is checked on the host before anything is enqueued.
  auto ok = [](const int64_t* pairs, int32_t n, int64_t src_lim, int64_t dst_lim) {
    if (n > 0 && pairs == nullptr) return false;
    for (int32_t i = 0; i < n; ++i)
      if (pairs[2 * i] < 0 || pairs[2 * i] >= src_lim || pairs[2 * i + 1] < 0 || pairs[2 * i + 1] >= dst_lim)
        return false;
    return true;
  };
  if (!ok(swaps_out, num_swaps_out, num_gpu_blocks, num_cpu_blocks) ||
      !ok(swaps_in, num_swaps_in, num_cpu_blocks, num_gpu_blocks) ||
      !ok(copies, num_copies, num_gpu_blocks, num_gpu_blocks))
    return CF_ERR_INVALID_ARGUMENT;
  if ((num_swaps_out + num_swaps_in + num_copies) > 0 && (!gpu_key_cache || !gpu_value_cache))
    return CF_ERR_INVALID_ARGUMENT;
  if ((num_swaps_out + num_swaps_in) > 0 && (!cpu_key_cache || !cpu_value_cache))
    return CF_ERR_INVALID_ARGUMENT;
  // Swap-outs free GPU blocks that swap-ins and copies may then reuse: the
  // three lists run in that order on the stream.  Each list goes either to
  // the SM copy kernel (both caches in one launch per 4000 pairs, the list
  // passed in the kernel parameters) or to the copy engines (one
  // cudaMemcpyAsync per contiguous run):
  //  * copy engines when the list is made of long runs (at least
  //    kDmaMinRun consecutive ids per run on average), where one DMA moves
  //    many blocks at the host link's full rate;
  //  * copy engines when a CPU pool is not addressable from the device
  //    (pageable memory), since the kernel cannot read it;
  //  * copy engines when a pair's destination is another pair's source or
  //    destination in the same list: the kernel runs the pairs of a launch
  //    concurrently, the copy engines apply them in order.
  //  Otherwise (scattered ids, the scheduler's usual lists,
  //  scheduler.cpp:220-224,249-254) the SM kernel, which keeps many blocks in
  //  flight at once.
  constexpr int64_t kDmaMinRun = 16;
  const bool cpu_mapped = (num_swaps_out + num_swaps_in) == 0 ||
                          (device_view(cpu_key_cache) != nullptr && device_view(cpu_value_cache) != nullptr);
  auto use_kernel = [&](const int64_t* pairs, int32_t n, bool crosses_host) {
    if (crosses_host && !cpu_mapped) return false;
    int64_t runs = 0;
    for (int32_t i = 0; i < n; ++i)
      if (i == 0 || pairs[2 * i] != pairs[2 * i - 2] + 1 || pairs[2 * i + 1] != pairs[2 * i - 1] + 1) ++runs;
    if ((int64_t)n >= kDmaMinRun * runs) return false;
    std::unordered_set<int64_t> dsts;
    dsts.reserve((size_t)n * 2);
    for (int32_t i = 0; i < n; ++i) {
      if (pairs[2 * i] > INT32_MAX || pairs[2 * i + 1] > INT32_MAX) return false;
      if (!dsts.insert(pairs[2 * i + 1]).second) return false;  // written twice
    }
    if (!crosses_host)
      for (int32_t i = 0; i < n; ++i)
        if (dsts.count(pairs[2 * i])) return false;  // read after another pair writes it
    return true;
  };
  const struct {
    void* src_k;
    void* src_v;
    void* dst_k;
    void* dst_v;
    const int64_t* pairs;
    int32_t n;
    int64_t num_src, num_dst;
    bool crosses_host;
  } steps[3] = {
      {gpu_key_cache, gpu_value_cache, cpu_key_cache, cpu_value_cache, swaps_out, num_swaps_out,
       num_gpu_blocks, num_cpu_blocks, true},
      {cpu_key_cache, cpu_value_cache, gpu_key_cache, gpu_value_cache, swaps_in, num_swaps_in,
       num_cpu_blocks, num_gpu_blocks, true},
      {gpu_key_cache, gpu_value_cache, gpu_key_cache, gpu_value_cache, copies, num_copies,
       num_gpu_blocks, num_gpu_blocks, false}};
  for (const auto& st : steps) {
    if (st.n == 0) continue;
    cf_status r;
    if (use_kernel(st.pairs, st.n, st.crosses_host)) {
      const void* sk = st.crosses_host ? device_view(st.src_k) : st.src_k;
      const void* sv = st.crosses_host ? device_view(st.src_v) : st.src_v;
      void* dk = const_cast<void*>(st.crosses_host ? device_view(st.dst_k) : st.dst_k);
      void* dv = const_cast<void*>(st.crosses_host ? device_view(st.dst_v) : st.dst_v);
      r = launch_host_pairs(sk, dk, sv, dv, st.pairs, st.n, block_size_bytes, st.num_src, st.num_dst,
                            (cudaStream_t)stream);
    } else {
      r = cf_swap_blocks_dma(st.src_k, st.dst_k, st.pairs, st.n, block_size_bytes, stream);
      if (r == CF_OK) r = cf_swap_blocks_dma(st.src_v, st.dst_v, st.pairs, st.n, block_size_bytes, stream);
    }
    if (r != CF_OK) return r;
  }
  return CF_OK;
}

cf_status cf_compact_kv_cache(void* key_cache, void* value_cache, const int32_t* src_block_ids,
                              const int32_t* dst_block_ids, int32_t num_moves,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              int64_t num_blocks, int32_t dtype, void* stream) {
  const int eb = dtype_bytes(dtype);
  if (eb == 0 || num_moves < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks < 0)
    return CF_ERR_INVALID_ARGUMENT;
  if (num_moves == 0) return CF_OK;
  if (!key_cache || !value_cache || !src_block_ids || !dst_block_ids)
    return CF_ERR_INVALID_ARGUMENT;
  const int64_t bb = (int64_t)num_kv_heads * block_size * head_dim * eb;
  const int64_t nb = num_blocks > 0 ? num_blocks : INT64_MAX / bb;
  return launch_move_blocks32(key_cache, value_cache, src_block_ids, dst_block_ids, num_moves,
                              bb, nb, (cudaStream_t)stream);
}

cf_status cf_memset_blocks(void* cache, const int32_t* block_ids, int32_t num_listed,
                           int64_t block_size_bytes, int64_t num_blocks, void* stream) {
  if (num_listed < 0 || block_size_bytes <= 0 || num_blocks < 0) return CF_ERR_INVALID_ARGUMENT;
  if (num_listed == 0) return CF_OK;
  if (!cache || !block_ids) return CF_ERR_INVALID_ARGUMENT;
  const int64_t nb = num_blocks > 0 ? num_blocks : INT64_MAX / block_size_bytes;
  return launch_memset_blocks(cache, block_ids, num_listed, block_size_bytes, nb,
                              (cudaStream_t)stream);
}

cf_status cf_compaction_plan(const uint8_t* used, int64_t num_blocks, int32_t* src_out,
                             int32_t* dst_out, int32_t* num_moves) {
  if (!used || !src_out || !dst_out || !num_moves || num_blocks < 0 || num_blocks > INT32_MAX)
    return CF_ERR_INVALID_ARGUMENT;
  int64_t live = 0;
  for (int64_t b = 0; b < num_blocks; ++b) live += used[b] ? 1 : 0;
  // Holes below `live` receive the live blocks found at or above `live`,
  // both walked in increasing id order.
  int64_t hole = 0, n = 0;
  for (int64_t b = live; b < num_blocks; ++b) {
    if (!used[b]) continue;
    while (hole < live && used[hole]) ++hole;
    src_out[n] = (int32_t)b;
    dst_out[n] = (int32_t)hole;
    ++n;
    ++hole;
  }
  *num_moves = (int32_t)n;
  return CF_OK;
}

cf_status cf_check_compaction_plan(const int32_t* src_ids, const int32_t* dst_ids,
                                   int32_t num_moves, int64_t num_blocks) {
  if (num_moves < 0 || num_blocks < 0 || num_blocks > INT32_MAX) return CF_ERR_INVALID_ARGUMENT;
  if (num_moves == 0) return CF_OK;
  if (!src_ids || !dst_ids) return CF_ERR_INVALID_ARGUMENT;
  std::vector<uint8_t> role((size_t)num_blocks, 0);  // bit0: source, bit1: destination
  for (int32_t i = 0; i < num_moves; ++i) {
    const int32_t s = src_ids[i], d = dst_ids[i];
    if (s < 0 || s >= num_blocks || d < 0 || d >= num_blocks) return CF_ERR_INVALID_ARGUMENT;
    if (s == d) continue;  // skipped by the kernel
    if (role[(size_t)d] & 2) return CF_ERR_PLAN;
    role[(size_t)d] |= 2;
    role[(size_t)s] |= 1;
  }
  for (int64_t b = 0; b < num_blocks; ++b)
    if (role[(size_t)b] == 3) return CF_ERR_PLAN;
  return CF_OK;
}

cf_status cf_get_device_errors(int32_t device, uint32_t* flags, int32_t clear) {
  if (!flags) return CF_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cf_status st = cuda_status(cudaGetDevice(&prev));
  if (st != CF_OK) return st;
  if ((st = cuda_status(cudaSetDevice(device))) != CF_OK) return st;
  uint32_t bits = 0;
  st = cuda_status(cudaDeviceSynchronize());
  if (st == CF_OK) st = attention_read_errors(&bits, clear != 0);
  if (st == CF_OK) st = cache_ops_read_errors(&bits, clear != 0);
  if (st == CF_OK) st = prefill_read_errors(&bits, clear != 0);
  cudaSetDevice(prev);
  *flags = bits;
  return st;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// CacheFlow's C++ entry points (fp32), same signatures as the reference.
// ---------------------------------------------------------------------------
namespace cacheflow {
namespace cuda {

namespace {
thread_local int t_last_status = CF_OK;

void note(cf_status st, const char* what) {
  t_last_status = st;
  if (st != CF_OK) {
    static std::once_flag once;
    std::call_once(once, [&] {
      std::fprintf(stderr, "cacheflow_b200: %s failed: %s\n", what, cf_status_string(st));
    });
  }
}

cf_paged_attention_params to_c(const PagedAttentionParams& p) {
  cf_paged_attention_params c;
  c.query = p.query;
  c.key_cache = p.key_cache;
  c.value_cache = p.value_cache;
  c.output = p.output;
  c.block_tables = p.block_tables;
  c.context_lens = p.context_lens;
  c.scale = p.scale;
  c.num_seqs = p.num_seqs;
  c.num_heads = p.num_heads;
  c.num_kv_heads = p.num_kv_heads;
  c.head_dim = p.head_dim;
  c.block_size = p.block_size;
  c.max_context_len = p.max_context_len;
  c.max_blocks_per_seq = p.max_blocks_per_seq;
  c.num_blocks = 0;
  c.dtype = CF_F32;
  return c;
}
}  // namespace

int last_status() { return t_last_status; }

void launch_paged_attention_v1(const PagedAttentionParams& params, cudaStream_t stream) {
  cf_paged_attention_params c = to_c(params);
  note(cf_paged_attention_v1(&c, nullptr, 0, stream), "launch_paged_attention_v1");
}

void launch_paged_attention_v2(const PagedAttentionParams& params, float* exp_sums,
                               float* max_logits, float* tmp_output, int32_t num_partitions,
                               cudaStream_t stream) {
  cf_paged_attention_params c = to_c(params);
  note(cf_paged_attention_v2(&c, exp_sums, max_logits, tmp_output, num_partitions, stream),
       "launch_paged_attention_v2");
}

void launch_reshape_and_cache(const float* key, const float* value, float* key_cache,
                              float* value_cache, const int32_t* slot_mapping, int32_t num_tokens,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              cudaStream_t stream) {
  note(cf_reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, num_tokens,
                            num_kv_heads, head_dim, block_size, 0, CF_F32, stream),
       "launch_reshape_and_cache");
}

void launch_copy_blocks(float* key_cache, float* value_cache, const int64_t* block_mapping,
                        int32_t num_pairs, int32_t num_kv_heads, int32_t head_dim,
                        int32_t block_size, cudaStream_t stream) {
  note(cf_copy_blocks(key_cache, value_cache, block_mapping, num_pairs, num_kv_heads, head_dim,
                      block_size, 0, CF_F32, stream),
       "launch_copy_blocks");
}

void launch_swap_blocks(float* src_cache, float* dst_cache, const int64_t* block_mapping,
                        int32_t num_pairs, int32_t block_size_bytes, cudaStream_t stream) {
  note(cf_swap_blocks(src_cache, dst_cache, block_mapping, num_pairs, block_size_bytes, stream),
       "launch_swap_blocks");
}

void launch_compact_kv_cache(float* key_cache, float* value_cache, const int32_t* src_block_ids,
                             const int32_t* dst_block_ids, int32_t num_blocks,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             cudaStream_t stream) {
  note(cf_compact_kv_cache(key_cache, value_cache, src_block_ids, dst_block_ids, num_blocks,
                           num_kv_heads, head_dim, block_size, 0, CF_F32, stream),
       "launch_compact_kv_cache");
}

size_t get_gpu_free_memory() {
  size_t f = 0, t = 0;
  cudaMemGetInfo(&f, &t);
  return f;
}

size_t get_gpu_total_memory() {
  size_t f = 0, t = 0;
  cudaMemGetInfo(&f, &t);
  return t;
}

float get_gpu_memory_utilization() {
  size_t f = 0, t = 0;
  if (cudaMemGetInfo(&f, &t) != cudaSuccess || t == 0) return 0.f;
  return 1.0f - (float)f / (float)t;
}

void async_memcpy_h2d(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  note(cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream)),
       "async_memcpy_h2d");
}

void async_memcpy_d2h(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  note(cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream)),
       "async_memcpy_d2h");
}

void async_memcpy_d2d(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  note(cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream)),
       "async_memcpy_d2d");
}

void launch_memset_blocks(float* cache, const int32_t* block_ids, int32_t num_blocks,
                          int32_t block_size_bytes, cudaStream_t stream) {
  note(cf_memset_blocks(cache, block_ids, num_blocks, block_size_bytes, 0, stream),
       "launch_memset_blocks");
}

void synchronize_stream(cudaStream_t stream) { cudaStreamSynchronize(stream); }

void synchronize_device() { cudaDeviceSynchronize(); }

}  // namespace cuda
}  // namespace cacheflow
