// cache_ops.cu -- KV-cache data movement for sm_100a: reshape_and_cache (and
// its fp8-quantizing form), block-pair copies (copy_blocks, swap_blocks,
// compact_kv_cache), memset_blocks, and the device-side decode-input builder.
//
// All of these are pure byte movement and HBM-bound (or host-link-bound for
// swaps), so the kernels move 16-byte vectors with 64-bit offsets, spread
// every block over many CTAs, and range-check each device-side index
// (skip + record in the error word, never trap).
//
// Reference semantics followed (CacheFlow src/cacheflow/cuda/):
//   reshape_and_cache_kernel  kv_cache_kernels.cu:17-44  (slot math :34-40)
//   copy_blocks_kernel        kv_cache_kernels.cu:63-84  (pair layout :71-73)
//   swap_blocks_kernel        kv_cache_kernels.cu:105-131 (launcher :121-131)
//   compact_kv_cache_kernel   kv_cache_kernels.cu:140-183 (src == dst skipped :152)
//   memset_blocks_kernel      memory_utils.cu:46-69
#include "cf_device.cuh"
#include "cf_internal.h"

namespace cfb {

__device__ uint32_t g_cache_errors;

__device__ __forceinline__ void cache_error(uint32_t bits) { atomicOr(&g_cache_errors, bits); }

// ---------------------------------------------------------------------------
// reshape_and_cache: one thread per 16-byte vector of a (token, kv head) row;
// K and V share the slot lookup.  Rows are written whole and contiguous.
// ---------------------------------------------------------------------------
template <typename V>
__global__ void __launch_bounds__(256)
    reshape_and_cache_kernel(const V* __restrict__ key, const V* __restrict__ value,
                             V* __restrict__ key_cache, V* __restrict__ value_cache,
                             const int32_t* __restrict__ slot_mapping, int64_t num_rows,
                             int32_t num_kv_heads, int32_t vecs_per_row, int32_t block_size,
                             int64_t num_slots) {
  const int64_t total = num_rows * vecs_per_row;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = g / vecs_per_row;
    const int32_t v = (int32_t)(g - row * vecs_per_row);
    const int64_t tok = row / num_kv_heads;
    const int32_t head = (int32_t)(row - tok * num_kv_heads);
    const int64_t slot = slot_mapping[tok];
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {
      if (v == 0) cache_error(CF_DEVERR_SLOT);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    const int64_t dst_row = (blk * num_kv_heads + head) * block_size + off;
    key_cache[dst_row * vecs_per_row + v] = key[g];
    value_cache[dst_row * vecs_per_row + v] = value[g];
  }
}

// ---------------------------------------------------------------------------
// reshape_and_cache into fp8 (e4m3) caches: the same scatter, quantizing on
// the way -- cache = e4m3(x / scale), x / scale correctly rounded in f32,
// then rounded to nearest even with saturation to +-448.  One thread per 16
// elements (16 output bytes) of a (token, kv head) row.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256)
    reshape_and_cache_fp8_kernel(const T* __restrict__ key, const T* __restrict__ value,
                                 uint8_t* __restrict__ key_cache, uint8_t* __restrict__ value_cache,
                                 const int32_t* __restrict__ slot_mapping, int64_t num_rows,
                                 int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                 int64_t num_slots, float k_scale, float v_scale) {
  const int32_t vpr = head_dim / 16;
  const int64_t total = num_rows * vpr;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = g / vpr;
    const int32_t v = (int32_t)(g - row * vpr);
    const int64_t tok = row / num_kv_heads;
    const int32_t head = (int32_t)(row - tok * num_kv_heads);
    const int64_t slot = slot_mapping[tok];
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {
      if (v == 0) cache_error(CF_DEVERR_SLOT);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    const int64_t dst = ((blk * num_kv_heads + head) * block_size + off) * head_dim + v * 16;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const float sc = kv ? v_scale : k_scale;
      float f[16];
      load_widen<T, 16>((kv ? value : key) + row * head_dim + v * 16, f);
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = f2_to_e4m3x2(__fdiv_rn(f[4 * i], sc), __fdiv_rn(f[4 * i + 1], sc));
        const uint32_t hi = f2_to_e4m3x2(__fdiv_rn(f[4 * i + 2], sc), __fdiv_rn(f[4 * i + 3], sc));
        w[i] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>((kv ? value_cache : key_cache) + dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Block-pair copy.  Up to two (src base, dst base) streams share one list of
// (src id, dst id) pairs: copy_blocks uses (K,K) and (V,V) within one pool,
// swap_blocks uses one (src pool, dst pool) stream, compact uses (K,K),(V,V)
// with separate id arrays.  grid = (chunks per block, pairs).
// ---------------------------------------------------------------------------
struct PairStreams {
  const uint8_t* src[2];
  uint8_t* dst[2];
  int32_t count;
};

template <typename IdT>
struct PairIds {
  const IdT* src;  // src id of pair i at src[i * stride]
  const IdT* dst;
  int32_t stride;
};

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;  // 16-byte vectors per thread per stream

// A list of up to kParamPairs (src id, dst id) pairs passed by value in the
// kernel's parameters (CUDA 12.1+ allows 32,764 bytes of parameters on
// sm_70 and later): the host's list needs no device copy, no staging buffer
// and no allocation, and may be freed as soon as the launch returns.
constexpr int kParamPairs = 4000;
struct ParamPairs {
  int32_t id[2 * kParamPairs];  // pair i: id[2i] = src, id[2i + 1] = dst
};

template <typename IdT>
__device__ __forceinline__ int64_t pair_src(const PairIds<IdT>& ids, int64_t i) {
  return (int64_t)ids.src[i * ids.stride];
}
template <typename IdT>
__device__ __forceinline__ int64_t pair_dst(const PairIds<IdT>& ids, int64_t i) {
  return (int64_t)ids.dst[i * ids.stride];
}
__device__ __forceinline__ int64_t pair_src(const ParamPairs& ids, int64_t i) { return ids.id[2 * i]; }
__device__ __forceinline__ int64_t pair_dst(const ParamPairs& ids, int64_t i) { return ids.id[2 * i + 1]; }

template <typename V, typename Ids, bool kSkipSame>
__global__ void __launch_bounds__(kCopyThreads)
    pair_copy_kernel(PairStreams st, Ids ids, int32_t num_pairs, int64_t vecs_per_block,
                     int64_t num_src_blocks, int64_t num_dst_blocks) {
  for (int64_t pair = blockIdx.y; pair < num_pairs; pair += gridDim.y) {
    const int64_t s = pair_src(ids, pair);
    const int64_t d = pair_dst(ids, pair);
    if (s < 0 || s >= num_src_blocks || d < 0 || d >= num_dst_blocks) {
      if (blockIdx.x == 0 && threadIdx.x == 0) cache_error(CF_DEVERR_BLOCK_ID);
      continue;
    }
    if (kSkipSame && s == d) continue;
    const int64_t base = (int64_t)blockIdx.x * kCopyThreads * kCopyUnroll + threadIdx.x;
    for (int k = 0; k < st.count; ++k) {
      const V* src = reinterpret_cast<const V*>(st.src[k]) + s * vecs_per_block;
      V* dst = reinterpret_cast<V*>(st.dst[k]) + d * vecs_per_block;
      V tmp[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + (int64_t)u * kCopyThreads;
        if (i < vecs_per_block) tmp[u] = src[i];
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + (int64_t)u * kCopyThreads;
        if (i < vecs_per_block) dst[i] = tmp[u];
      }
    }
  }
}

template <typename V>
__global__ void __launch_bounds__(kCopyThreads)
    memset_blocks_kernel(uint8_t* cache, const int32_t* __restrict__ ids, int32_t num_listed,
                         int64_t vecs_per_block, int64_t num_blocks) {
  for (int64_t i = blockIdx.y; i < num_listed; i += gridDim.y) {
    const int64_t b = ids[i];
    if (b < 0 || b >= num_blocks) {
      if (blockIdx.x == 0 && threadIdx.x == 0) cache_error(CF_DEVERR_BLOCK_ID);
      continue;
    }
    V* dst = reinterpret_cast<V*>(cache) + b * vecs_per_block;
    const int64_t base = (int64_t)blockIdx.x * kCopyThreads * kCopyUnroll + threadIdx.x;
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t j = base + (int64_t)u * kCopyThreads;
      if (j < vecs_per_block) dst[j] = V{};
    }
  }
}

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
namespace {

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Widest vector (16, 4 or 1 bytes) that every pointer and the block size allow.
int vector_bytes(std::initializer_list<const void*> ptrs, int64_t bytes) {
  int w = 16;
  for (const void* p : ptrs) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    while (w > 1 && (a % w) != 0) w /= 4;
  }
  while (w > 1 && (bytes % w) != 0) w /= 4;
  return w < 4 ? 1 : w;
}

template <typename Ids, bool kSkipSame>
cf_status launch_pairs(const PairStreams& st, const Ids& ids, int32_t num_pairs,
                       int64_t block_bytes, int64_t num_src, int64_t num_dst,
                       cudaStream_t stream) {
  if (num_pairs == 0) return CF_OK;
  const int w = vector_bytes({st.src[0], st.dst[0], st.count > 1 ? st.src[1] : nullptr,
                              st.count > 1 ? st.dst[1] : nullptr},
                             block_bytes);
  const int64_t vecs = block_bytes / w;
  const int64_t per_cta = (int64_t)kCopyThreads * kCopyUnroll;
  const int64_t chunks = (vecs + per_cta - 1) / per_cta;
  if (chunks > 0x7fffffff) return CF_ERR_UNSUPPORTED;
  dim3 grid((unsigned)chunks, (unsigned)(num_pairs < 65535 ? num_pairs : 65535));
  if (w == 16)
    pair_copy_kernel<uint4, Ids, kSkipSame>
        <<<grid, kCopyThreads, 0, stream>>>(st, ids, num_pairs, vecs, num_src, num_dst);
  else if (w == 4)
    pair_copy_kernel<uint32_t, Ids, kSkipSame>
        <<<grid, kCopyThreads, 0, stream>>>(st, ids, num_pairs, vecs, num_src, num_dst);
  else
    pair_copy_kernel<uint8_t, Ids, kSkipSame>
        <<<grid, kCopyThreads, 0, stream>>>(st, ids, num_pairs, vecs, num_src, num_dst);
  return check_launch();
}

}  // namespace

cf_status launch_reshape_and_cache(const void* key, const void* value, void* key_cache,
                                   void* value_cache, const int32_t* slot_mapping,
                                   int32_t num_tokens, int32_t num_kv_heads, int64_t row_bytes,
                                   int32_t block_size, int64_t num_blocks, cudaStream_t stream) {
  if (num_tokens == 0) return CF_OK;
  const int w = vector_bytes({key, value, key_cache, value_cache}, row_bytes);
  const int64_t rows = (int64_t)num_tokens * num_kv_heads;
  const int64_t vpr = row_bytes / w;
  const int64_t total = rows * vpr;
  const int64_t want = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  const int64_t slots = num_blocks * block_size;
  if (w == 16)
    reshape_and_cache_kernel<uint4><<<grid, 256, 0, stream>>>(
        (const uint4*)key, (const uint4*)value, (uint4*)key_cache, (uint4*)value_cache,
        slot_mapping, rows, num_kv_heads, (int32_t)vpr, block_size, slots);
  else if (w == 4)
    reshape_and_cache_kernel<uint32_t><<<grid, 256, 0, stream>>>(
        (const uint32_t*)key, (const uint32_t*)value, (uint32_t*)key_cache,
        (uint32_t*)value_cache, slot_mapping, rows, num_kv_heads, (int32_t)vpr, block_size,
        slots);
  else
    reshape_and_cache_kernel<uint8_t><<<grid, 256, 0, stream>>>(
        (const uint8_t*)key, (const uint8_t*)value, (uint8_t*)key_cache, (uint8_t*)value_cache,
        slot_mapping, rows, num_kv_heads, (int32_t)vpr, block_size, slots);
  return check_launch();
}

cf_status launch_copy_pairs64(void* key_cache, void* value_cache, const int64_t* mapping,
                              int32_t num_pairs, int64_t block_bytes, int64_t num_blocks,
                              cudaStream_t stream) {
  PairStreams st{{(const uint8_t*)key_cache, (const uint8_t*)value_cache},
                 {(uint8_t*)key_cache, (uint8_t*)value_cache},
                 2};
  PairIds<int64_t> ids{mapping, mapping + 1, 2};
  return launch_pairs<PairIds<int64_t>, false>(st, ids, num_pairs, block_bytes, num_blocks, num_blocks,
                                      stream);
}

cf_status launch_swap_pairs64(const void* src_cache, void* dst_cache, const int64_t* mapping,
                              int32_t num_pairs, int64_t block_bytes, cudaStream_t stream) {
  PairStreams st{{(const uint8_t*)src_cache, nullptr}, {(uint8_t*)dst_cache, nullptr}, 1};
  PairIds<int64_t> ids{mapping, mapping + 1, 2};
  // Pool sizes are unknown to the reference interface: ids are checked >= 0 only.
  const int64_t unchecked = INT64_MAX / (block_bytes > 0 ? block_bytes : 1);
  return launch_pairs<PairIds<int64_t>, false>(st, ids, num_pairs, block_bytes, unchecked, unchecked,
                                      stream);
}

cf_status launch_move_blocks32(void* key_cache, void* value_cache, const int32_t* src_ids,
                               const int32_t* dst_ids, int32_t num_moves, int64_t block_bytes,
                               int64_t num_blocks, cudaStream_t stream) {
  PairStreams st{{(const uint8_t*)key_cache, (const uint8_t*)value_cache},
                 {(uint8_t*)key_cache, (uint8_t*)value_cache},
                 2};
  PairIds<int32_t> ids{src_ids, dst_ids, 1};
  return launch_pairs<PairIds<int32_t>, true>(st, ids, num_moves, block_bytes, num_blocks, num_blocks,
                                     stream);
}

cf_status launch_host_pairs(const void* src_k, void* dst_k, const void* src_v, void* dst_v,
                            const int64_t* host_pairs, int32_t num_pairs, int64_t block_bytes,
                            int64_t num_src_blocks, int64_t num_dst_blocks, cudaStream_t stream) {
  PairStreams st{{(const uint8_t*)src_k, (const uint8_t*)src_v}, {(uint8_t*)dst_k, (uint8_t*)dst_v}, 2};
  ParamPairs pl;
  for (int32_t first = 0; first < num_pairs; first += kParamPairs) {
    const int32_t n = num_pairs - first < kParamPairs ? num_pairs - first : kParamPairs;
    for (int32_t i = 0; i < n; ++i) {
      const int64_t s = host_pairs[2 * (int64_t)(first + i)], d = host_pairs[2 * (int64_t)(first + i) + 1];
      if (s < 0 || s > INT32_MAX || d < 0 || d > INT32_MAX) return CF_ERR_INVALID_ARGUMENT;
      pl.id[2 * i] = (int32_t)s;
      pl.id[2 * i + 1] = (int32_t)d;
    }
    const cf_status r = launch_pairs<ParamPairs, false>(st, pl, n, block_bytes, num_src_blocks,
                                                        num_dst_blocks, stream);
    if (r != CF_OK) return r;
  }
  return CF_OK;
}

cf_status launch_reshape_and_cache_fp8(const void* key, const void* value, void* key_cache,
                                       void* value_cache, const int32_t* slot_mapping,
                                       int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                       int32_t block_size, int64_t num_blocks, int32_t dtype,
                                       float k_scale, float v_scale, cudaStream_t stream) {
  if (num_tokens == 0) return CF_OK;
  const int64_t rows = (int64_t)num_tokens * num_kv_heads;
  const int64_t total = rows * (head_dim / 16);
  const int64_t want = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  const int64_t slots = num_blocks * block_size;
  uint8_t* kc = static_cast<uint8_t*>(key_cache);
  uint8_t* vc = static_cast<uint8_t*>(value_cache);
  switch (dtype) {
    case CF_F32:
      reshape_and_cache_fp8_kernel<float><<<grid, 256, 0, stream>>>(
          (const float*)key, (const float*)value, kc, vc, slot_mapping, rows, num_kv_heads, head_dim,
          block_size, slots, k_scale, v_scale);
      break;
    case CF_F16:
      reshape_and_cache_fp8_kernel<__half><<<grid, 256, 0, stream>>>(
          (const __half*)key, (const __half*)value, kc, vc, slot_mapping, rows, num_kv_heads, head_dim,
          block_size, slots, k_scale, v_scale);
      break;
    default:
      reshape_and_cache_fp8_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, kc, vc, slot_mapping, rows,
          num_kv_heads, head_dim, block_size, slots, k_scale, v_scale);
      break;
  }
  return check_launch();
}

cf_status launch_memset_blocks(void* cache, const int32_t* ids, int32_t num_listed,
                               int64_t block_bytes, int64_t num_blocks, cudaStream_t stream) {
  if (num_listed == 0) return CF_OK;
  const int w = vector_bytes({cache}, block_bytes);
  const int64_t vecs = block_bytes / w;
  const int64_t per_cta = (int64_t)kCopyThreads * kCopyUnroll;
  const int64_t chunks = (vecs + per_cta - 1) / per_cta;
  if (chunks > 0x7fffffff) return CF_ERR_UNSUPPORTED;
  dim3 grid((unsigned)chunks, (unsigned)(num_listed < 65535 ? num_listed : 65535));
  if (w == 16)
    memset_blocks_kernel<uint4>
        <<<grid, kCopyThreads, 0, stream>>>((uint8_t*)cache, ids, num_listed, vecs, num_blocks);
  else if (w == 4)
    memset_blocks_kernel<uint32_t>
        <<<grid, kCopyThreads, 0, stream>>>((uint8_t*)cache, ids, num_listed, vecs, num_blocks);
  else
    memset_blocks_kernel<uint8_t>
        <<<grid, kCopyThreads, 0, stream>>>((uint8_t*)cache, ids, num_listed, vecs, num_blocks);
  return check_launch();
}

// ---------------------------------------------------------------------------
// Device-side decode-batch preparation: what the host loop of
// BatchDecodeEngine::prepare_kv_cache_inputs (batch_decode.cpp:92-131) builds,
// from one contiguous list of every row's block ids (CSR: row s owns
// block_ids[block_offsets[s] .. block_offsets[s+1])):
//   block_tables[s, b] = row s's b-th block id, 0 past its blocks (:98, :104-105)
//   context_lens[s]    = positions[s] + 1                           (:103)
//   slot_mapping[s]    = id of block positions[s] / bs * bs + positions[s] % bs
//                        when the row has that block (:107-114), else -1
//                        (the reference leaves it unset; -1 is the padding
//                        slot that reshape_and_cache skips).
// A negative position gives an empty row (context 0, slot -1).  A row with
// more blocks than max_blocks_per_seq keeps the first max_blocks_per_seq
// and records CF_DEVERR_CONTEXT_LEN; a slot past INT32_MAX records
// CF_DEVERR_SLOT.  Grid (ceil(max_blocks_per_seq / 256), rows): one thread per
// table entry, coalesced.
// ---------------------------------------------------------------------------
constexpr int kBuildThreads = 256;

__global__ void __launch_bounds__(kBuildThreads)
    build_decode_inputs_kernel(const int32_t* __restrict__ positions,
                               const int64_t* __restrict__ block_offsets,
                               const int32_t* __restrict__ block_ids, int32_t max_blocks,
                               int32_t block_size, int32_t* __restrict__ block_tables,
                               int32_t* __restrict__ context_lens,
                               int32_t* __restrict__ slot_mapping) {
  const int s = blockIdx.y;
  const int64_t o0 = block_offsets[s];
  const int64_t n = block_offsets[s + 1] - o0;
  const int64_t lim = n < 0 ? 0 : (n < max_blocks ? n : max_blocks);
  const int b = blockIdx.x * kBuildThreads + threadIdx.x;
  if (b < max_blocks) block_tables[(size_t)s * max_blocks + b] = b < lim ? block_ids[o0 + b] : 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (n < 0 || n > max_blocks) cache_error(CF_DEVERR_CONTEXT_LEN);
    const int32_t pos = positions[s];
    int32_t slot = -1;
    if (pos >= 0 && pos < INT32_MAX) {
      context_lens[s] = pos + 1;
      const int64_t bi = pos / block_size;
      if (bi < lim) {
        const int64_t v = (int64_t)block_ids[o0 + bi] * block_size + pos % block_size;
        if (v >= 0 && v <= INT32_MAX)
          slot = (int32_t)v;
        else
          cache_error(CF_DEVERR_SLOT);
      }
    } else {
      context_lens[s] = 0;
    }
    slot_mapping[s] = slot;
  }
}

cf_status launch_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                     const int32_t* block_ids, int32_t num_seqs,
                                     int32_t max_blocks_per_seq, int32_t block_size,
                                     int32_t* block_tables, int32_t* context_lens,
                                     int32_t* slot_mapping, cudaStream_t stream) {
  dim3 grid((unsigned)((max_blocks_per_seq + kBuildThreads - 1) / kBuildThreads), (unsigned)num_seqs);
  build_decode_inputs_kernel<<<grid, kBuildThreads, 0, stream>>>(
      positions, block_offsets, block_ids, max_blocks_per_seq, block_size, block_tables,
      context_lens, slot_mapping);
  return check_launch();
}

cf_status cache_ops_read_errors(uint32_t* bits, bool clear) {
  uint32_t v = 0;
  cf_status s = cuda_status(cudaMemcpyFromSymbol(&v, g_cache_errors, sizeof(v)));
  if (s != CF_OK) return s;
  *bits |= v;
  if (clear) {
    const uint32_t zero = 0;
    s = cuda_status(cudaMemcpyToSymbol(g_cache_errors, &zero, sizeof(zero)));
  }
  return s;
}

}  // namespace cfb
