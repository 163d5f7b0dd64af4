// prefill_attention.cu -- chunked-prefill (multi-query) paged attention for
// sm_100a: every query token of a chunk attends causally to its sequence's
// paged context, which already holds the chunk's own K/V rows.
//
// CacheFlow has no such operator (its forward pass is an abstract ForwardFn,
// src/cacheflow/decode/batch_decode.h:34-42, and its kernels take one query
// per sequence); a chunk of T tokens there is T decode rows with causal
// context lengths, each re-reading the whole context.  Here one CTA takes a
// tile of query tokens x the query heads of one KV head and streams the
// context once for all of them:
//
//   * 4 consumer warps own 16 query rows each (row = token * G + head within
//     the GQA group G), Q held as mma.sync A fragments for the whole tile;
//   * a producer warp streams 64-token stages (4 KV blocks of K and V) with
//     2-D tensor-map TMA into a 3-stage ring of 128-byte-swizzled tiles, full
//     and empty mbarriers between them;
//   * per stage: S = Q K^T (m16n8k16, fp32 accumulate), causal + context mask,
//     online softmax per row, O += P V with P split into a 16-bit head and
//     remainder (two MMAs) so the weights keep ~16 more bits;
//   * rows past the context or of an out-of-pool block are zeroed in the V
//     fragments (registers), never read as garbage.
#include <cmath>
#include <cstring>
#include <mutex>

#include "cf_device.cuh"
#include "cf_internal.h"

namespace cfb {

__device__ uint32_t g_prefill_errors;

__device__ __forceinline__ void prefill_error(uint32_t bits) { atomicOr(&g_prefill_errors, bits); }

namespace {

constexpr int kPBlock = 16;        // tokens per KV block
constexpr int kStageBlocks = 4;    // KV blocks per pipeline stage (64 keys)
constexpr int kStages = 3;         // ring depth
constexpr int kConsumerWarps = 4;  // 16 query rows each
constexpr int kRows = 16 * kConsumerWarps;
constexpr float kPLog2e = 1.4426950408889634f;

struct PrefillArgs {
  const void* q;
  void* out;
  const int32_t* block_tables;
  const int32_t* context_lens;
  const int32_t* query_start;
  float scale_log2;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t group;
  int32_t max_blocks_per_seq;
  int32_t tokens_per_tile;  // kRows / group
  int64_t num_blocks;
};

template <int D>
struct PrefillLayout {
  static constexpr int kTile = kPBlock * D * 2;  // one 16-token K or V tile
  static constexpr int kStage = kStageBlocks * 2 * kTile;
  static constexpr int kBarOffset = kStages * kStage;
  static constexpr int kMaskOffset = kBarOffset + 2 * kStages * 8;
  static constexpr int kBytes = kMaskOffset + kStages * 4;
  static constexpr int kAlloc = kBytes + 1024;
};

// Zero the 16-bit halves of a V fragment whose key is not readable.
__device__ __forceinline__ uint32_t keep_halves(uint32_t v, bool lo_ok, bool hi_ok) {
  return v & ((lo_ok ? 0x0000ffffu : 0u) | (hi_ok ? 0xffff0000u : 0u));
}

}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__((kConsumerWarps + 1) * 32)
    paged_prefill_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tmk,
                         const __grid_constant__ CUtensorMap tmv) {
  using L = PrefillLayout<D>;
  constexpr int TILE = L::kTile;
  constexpr int kKC = D / 16;
  constexpr int kND = D / 8;
  constexpr int kBoxBytes = kPBlock * 128;

  const int tile = blockIdx.x;
  const int kvh = blockIdx.y;
  const int chunk = blockIdx.z;
  const int q0 = a.query_start[chunk];
  const int qlen = a.query_start[chunk + 1] - q0;
  const int tok0 = tile * a.tokens_per_tile;
  if (qlen <= 0 || tok0 >= qlen) return;
  const int cap = a.max_blocks_per_seq * kPBlock;
  int ctx = a.context_lens[chunk];
  if (ctx < qlen || ctx > cap) {
    if (threadIdx.x == 0 && tile == 0 && kvh == 0) prefill_error(CF_DEVERR_CONTEXT_LEN);
    if (qlen > cap) return;
    ctx = ctx < qlen ? qlen : cap;
  }
  const int ntok = min(a.tokens_per_tile, qlen - tok0);
  const int pos0 = ctx - qlen + tok0;  // position of the tile's first query token
  const int nblk = (pos0 + ntok - 1) / kPBlock + 1;  // blocks the last row reads
  const int nstages = (nblk + kStageBlocks - 1) / kStageBlocks;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kStages;
  int* vmask = reinterpret_cast<int*>(smem + L::kMaskOffset);  // valid-block bits per stage
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int32_t* table = a.block_tables + (size_t)chunk * a.max_blocks_per_seq;

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    int ids = 0;
    int issued = 0;
    for (int st = 0; st < nstages; ++st) {
      const int slot = st % kStages;
      if (st >= kStages) {
        bool ready = true;
        if (lane == 0) ready = mbar_wait_bounded(smem_addr(&empty[slot]), (uint32_t)((st / kStages) - 1) & 1u);
        ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        if (!ready) {
          if (lane == 0) prefill_error(CF_DEVERR_TIMEOUT);
          break;
        }
      }
      const int b0 = st * kStageBlocks;
      if ((b0 & 31) == 0) ids = (b0 + lane < nblk) ? table[b0 + lane] : 0;
      int phys[kStageBlocks];
#pragma unroll
      for (int k = 0; k < kStageBlocks; ++k) phys[k] = __shfl_sync(0xffffffffu, ids, (b0 + k) & 31);
      if (lane == 0) {
        int mask = 0, nvalid = 0;
#pragma unroll
        for (int k = 0; k < kStageBlocks; ++k) {
          if (b0 + k >= nblk) continue;
          if (phys[k] < 0 || (int64_t)phys[k] >= a.num_blocks) {
            prefill_error(CF_DEVERR_BLOCK_ID);
            continue;
          }
          mask |= 1 << k;
          ++nvalid;
        }
        vmask[slot] = mask;
        const uint32_t bar = smem_addr(&full[slot]);
        uint8_t* stage = smem + (size_t)slot * L::kStage;
        fence_proxy_async_smem();
        if (nvalid == 0) {
          mbar_arrive(bar);
        } else {
          mbar_arrive_expect_tx(bar, (uint32_t)(nvalid * 2 * TILE));
#pragma unroll
          for (int k = 0; k < kStageBlocks; ++k) {
            if (!(mask & (1 << k))) continue;
            const int32_t row = (int32_t)(((int64_t)phys[k] * a.num_kv_heads + kvh) * kPBlock);
#pragma unroll
            for (int b = 0; b < D / 64; ++b) {
              tma_load_2d(smem_addr(stage + k * TILE + b * kBoxBytes), &tmk, b * 64, row, bar);
              tma_load_2d(smem_addr(stage + (kStageBlocks + k) * TILE + b * kBoxBytes), &tmv, b * 64, row,
                          bar);
            }
          }
        }
      }
      __syncwarp();
      issued = st + 1;
    }
    // No copy may land after the CTA exits: wait (bounded) for the last stages.
    if (lane == 0) {
      const int first = issued > kStages ? issued - kStages : 0;
      for (int st = first; st < issued; ++st)
        mbar_wait_bounded(smem_addr(&full[st % kStages]), (uint32_t)(st / kStages) & 1u);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int G = a.group;
  const int g4 = lane >> 2, tq = lane & 3;
  const int mi = lane >> 3, ri = lane & 7;
  // The two rows of this lane: r = 16*warp + g4 (+8); row -> (token, head).
  int qpos[2];
  bool active[2];
  const T* qrow[2];
  size_t orow[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int r = 16 * warp + g4 + 8 * j;
    const int t = r / G, h = r - t * G;
    active[j] = (t < ntok) && (r < a.tokens_per_tile * G);
    qpos[j] = active[j] ? pos0 + t : -1;
    const size_t tok = (size_t)q0 + tok0 + (active[j] ? t : 0);
    const size_t hq = (size_t)kvh * G + h;
    orow[j] = (tok * a.num_heads + hq) * D;
    qrow[j] = reinterpret_cast<const T*>(a.q) + orow[j];
  }
  uint32_t qa[kKC][4];
#pragma unroll
  for (int kc = 0; kc < kKC; ++kc) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qrow[j] + kc * 16 + 2 * tq);
      qa[kc][j] = active[j] ? q32[0] : 0u;      // (row, k lo)
      qa[kc][2 + j] = active[j] ? q32[4] : 0u;  // (row, k hi)
    }
  }
  float o[kND][4];
#pragma unroll
  for (int n = 0; n < kND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY};
  float l[2] = {0.f, 0.f};

  bool ok = true;
  for (int st = 0; st < nstages; ++st) {
    const int slot = st % kStages;
    const bool ready = mbar_wait_bounded(smem_addr(&full[slot]), (uint32_t)(st / kStages) & 1u);
    if (!__all_sync(0xffffffffu, ready)) {
      if (lane == 0) prefill_error(CF_DEVERR_TIMEOUT);
      ok = false;
      break;
    }
    const int mask = vmask[slot];
    const uint8_t* stage = smem + (size_t)slot * L::kStage;
    const uint32_t kbase = smem_addr(stage);
    const uint32_t vbase = smem_addr(stage + kStageBlocks * TILE);
    const int key0 = st * kStageBlocks * kPBlock;

    float s[2 * kStageBlocks][4];
#pragma unroll
    for (int n = 0; n < 2 * kStageBlocks; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    {
      const int r = (mi >> 1) * 8 + ri;
#pragma unroll
      for (int kc = 0; kc < kKC; ++kc) {
        const int box = kc >> 2;
        const int c = ((kc & 3) << 1) + (mi & 1);
        const uint32_t off = box * kBoxBytes + r * 128 + ((c ^ (r & 7)) << 4);
#pragma unroll
        for (int kb = 0; kb < kStageBlocks; ++kb) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kbase + kb * TILE + off, b0, b1, b2, b3);
          mma_16816<T>(s[2 * kb], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b0, b1);
          mma_16816<T>(s[2 * kb + 1], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b2, b3);
        }
      }
    }
    // causal / context / valid-block mask, then online softmax per row
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2 * kStageBlocks; ++n) {
      const bool blk_ok = (mask >> (n >> 1)) & 1;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = e >> 1;
        const int key = key0 + n * 8 + 2 * tq + (e & 1);
        const float x = s[n][e] * a.scale_log2;
        s[n][e] = (blk_ok && key <= qpos[j]) ? x : -INFINITY;
        mx[j] = fmaxf(mx[j], s[n][e]);
      }
    }
    float alpha[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      mx[j] = fmaxf(mx[j], shfl_xor(mx[j], 1));
      mx[j] = fmaxf(mx[j], shfl_xor(mx[j], 2));
      const float mn = fmaxf(m[j], mx[j]);
      const float mu = (mn == -INFINITY) ? 0.f : mn;
      alpha[j] = exp2f(m[j] - mu);
      m[j] = mn;
      float ps = 0.f;
#pragma unroll
      for (int n = 0; n < 2 * kStageBlocks; ++n) {
        s[n][2 * j] = exp2f(s[n][2 * j] - mu);
        s[n][2 * j + 1] = exp2f(s[n][2 * j + 1] - mu);
        ps += s[n][2 * j] + s[n][2 * j + 1];
      }
      l[j] = l[j] * alpha[j] + ps;
    }
#pragma unroll
    for (int n = 0; n < kND; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // P V per 16-key block: A fragment straight from the S fragments.
    const int rv = (mi & 1) * 8 + ri;
#pragma unroll
    for (int kb = 0; kb < kStageBlocks; ++kb) {
      uint32_t ph[4], pl[4];
      split2<T>(s[2 * kb][0], s[2 * kb][1], ph[0], pl[0]);
      split2<T>(s[2 * kb][2], s[2 * kb][3], ph[1], pl[1]);
      split2<T>(s[2 * kb + 1][0], s[2 * kb + 1][1], ph[2], pl[2]);
      split2<T>(s[2 * kb + 1][2], s[2 * kb + 1][3], ph[3], pl[3]);
      const int blk = st * kStageBlocks + kb;
      const bool blk_ok = (mask >> kb) & 1;
      // Keys this lane's V halves hold: 2tq, 2tq+1 (first 8) and 8+2tq, 9+2tq.
      const bool check = !blk_ok || blk >= nblk - 1;
      const int kbase_key = blk * kPBlock;
      const bool k0 = blk_ok && kbase_key + 2 * tq < ctx;
      const bool k1 = blk_ok && kbase_key + 2 * tq + 1 < ctx;
      const bool k2 = blk_ok && kbase_key + 8 + 2 * tq < ctx;
      const bool k3 = blk_ok && kbase_key + 9 + 2 * tq < ctx;
#pragma unroll
      for (int cp = 0; cp < kND / 2; ++cp) {
        const int c = 2 * cp + (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldmatrix_x4_trans(vbase + kb * TILE + (c >> 3) * kBoxBytes + rv * 128 + (((c & 7) ^ (rv & 7)) << 4),
                          v0, v1, v2, v3);
        if (check) {
          v0 = keep_halves(v0, k0, k1);
          v1 = keep_halves(v1, k2, k3);
          v2 = keep_halves(v2, k0, k1);
          v3 = keep_halves(v3, k2, k3);
        }
        mma_16816<T>(o[2 * cp], ph[0], ph[1], ph[2], ph[3], v0, v1);
        mma_16816<T>(o[2 * cp], pl[0], pl[1], pl[2], pl[3], v0, v1);
        mma_16816<T>(o[2 * cp + 1], ph[0], ph[1], ph[2], ph[3], v2, v3);
        mma_16816<T>(o[2 * cp + 1], pl[0], pl[1], pl[2], pl[3], v2, v3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));
  }
  if (!ok) return;

#pragma unroll
  for (int j = 0; j < 2; ++j) {
    l[j] += shfl_xor(l[j], 1);
    l[j] += shfl_xor(l[j], 2);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (!active[j]) continue;
    const float inv = l[j] > 0.f ? 1.f / l[j] : 0.f;
    T* out = reinterpret_cast<T*>(a.out) + orow[j];
#pragma unroll
    for (int n = 0; n < kND; ++n) {
      const uint32_t packed = pack2<T>(o[n][2 * j] * inv, o[n][2 * j + 1] * inv);
      *reinterpret_cast<uint32_t*>(out + n * 8 + 2 * tq) = packed;
    }
  }
}

namespace {

template <typename T, int D>
cf_status launch_prefill_typed(const cf_prefill_params& p, cudaStream_t stream) {
  using L = PrefillLayout<D>;
  static std::once_flag flags[64];
  static cudaError_t errs[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  auto kern = paged_prefill_kernel<T, D>;
  if (dev < 0 || dev >= 64) return CF_ERR_UNSUPPORTED;
  std::call_once(flags[dev], [&] {
    errs[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  });
  if (errs[dev] != cudaSuccess) return cuda_status(errs[dev]);

  const int64_t rows = p.num_blocks * (int64_t)p.num_kv_heads * kPBlock;
  CUtensorMap tmk, tmv;
  if (!kv_tensor_map(&tmk, p.key_cache, rows, D, p.dtype) ||
      !kv_tensor_map(&tmv, p.value_cache, rows, D, p.dtype))
    return CF_ERR_INVALID_ARGUMENT;
  PrefillArgs a;
  a.q = p.query;
  a.out = p.output;
  a.block_tables = p.block_tables;
  a.context_lens = p.context_lens;
  a.query_start = p.query_start;
  a.scale_log2 = p.scale * kPLog2e;
  a.num_heads = p.num_heads;
  a.num_kv_heads = p.num_kv_heads;
  a.group = p.num_heads / p.num_kv_heads;
  a.max_blocks_per_seq = p.max_blocks_per_seq;
  a.tokens_per_tile = kRows / a.group;
  a.num_blocks = p.num_blocks;
  const int tiles = (p.max_query_len + a.tokens_per_tile - 1) / a.tokens_per_tile;
  dim3 grid((unsigned)tiles, (unsigned)p.num_kv_heads, (unsigned)p.num_chunks);
  paged_prefill_kernel<T, D><<<grid, (kConsumerWarps + 1) * 32, L::kAlloc, stream>>>(a, tmk, tmv);
  return check_launch();
}

}  // namespace

bool prefill_supported(int32_t head_dim, int32_t block_size, int32_t dtype, int32_t group) {
  return block_size == kPBlock && (dtype == CF_F16 || dtype == CF_BF16) &&
         (head_dim == 64 || head_dim == 128) && group >= 1 && group <= kRows;
}

cf_status launch_paged_prefill(const cf_prefill_params& p, cudaStream_t stream) {
  if (p.num_chunks == 0 || p.max_query_len == 0) return CF_OK;
  if (p.dtype == CF_BF16) {
    if (p.head_dim == 128) return launch_prefill_typed<__nv_bfloat16, 128>(p, stream);
    return launch_prefill_typed<__nv_bfloat16, 64>(p, stream);
  }
  if (p.head_dim == 128) return launch_prefill_typed<__half, 128>(p, stream);
  return launch_prefill_typed<__half, 64>(p, stream);
}

cf_status prefill_read_errors(uint32_t* bits, bool clear) {
  uint32_t v = 0;
  cf_status s = cuda_status(cudaMemcpyFromSymbol(&v, g_prefill_errors, sizeof(v)));
  if (s != CF_OK) return s;
  *bits |= v;
  if (clear) {
    const uint32_t zero = 0;
    s = cuda_status(cudaMemcpyToSymbol(g_prefill_errors, &zero, sizeof(zero)));
  }
  return s;
}

}  // namespace cfb
