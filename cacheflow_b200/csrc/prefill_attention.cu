// prefill_attention.cu -- chunked-prefill (multi-query) paged attention for
// sm_100a: every query token of a chunk attends causally to its sequence's
// paged context, which already holds the chunk's own K/V rows.
//
// CacheFlow has no such operator (its forward pass is an abstract ForwardFn,
// src/cacheflow/decode/batch_decode.h:34-42, and its kernels take one query
// per sequence); a chunk of T tokens there is T decode rows with causal
// context lengths, each re-reading the whole context.  Here one CTA takes a
// tile of query tokens x the query heads of one KV head and streams the
// context once for all of them.  Two kernels:
//
//   paged_prefill_tc_kernel (default): tcgen05 tensor cores with tensor-memory
//   accumulators, two 128-row tiles per CTA; described above the kernel.
//
//   paged_prefill_kernel (CF_PREFILL_CONSUMER=mma): mma.sync, 64 rows per CTA:
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
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

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

// ---------------------------------------------------------------------------
// The same operator on 5th-generation tensor cores (tcgen05).  One CTA owns
// two tiles of 128 query rows (A: rows 0-127, B: rows 128-255; each the M of
// its MMAs) that share every K/V stage, and 10 warps:
//   warps 0-3  softmax + epilogue of tile A, warps 4-7 of tile B: thread =
//              row = tensor-memory lane (warp w reads lanes 32 (w % 4) ..);
//   warp 8     TMA producer (64-key stages of K and V, 5-stage ring);
//   warp 9     tensor-memory owner and MMA issuer (one thread).
// Tensor memory (512 columns), per tile: S double-buffered at [0, 64) and
// [64, 128), O at [128, 128 + D); tile B at +256.
// Per stage and tile: S = Q K^T (M 128, N 64, K = D; Q and K K-major in
// 128-byte-swizzled shared memory); the tile's softmax warps read S, mask,
// update the running max / sum and write P over the S buffer it came from
// (16-bit head in its first 32 columns, remainder in the next 32: K-major A
// operands in tensor memory); then O += P_hi V + P_lo V with A read from
// tensor memory and V an MN-major B operand in shared memory.
// The MMA warp alternates the tiles -- PV_A(s), QK_A(s+2), PV_B(s),
// QK_B(s+2): each tile's QK runs two stages ahead on its two S buffers, so
// its softmax finds the next S ready -- and every K/V byte brought in feeds
// 256 query rows.  O is
// rescaled (tcgen05.ld / st) only when a row's max grows by more than 2^8:
// until then P may exceed 1 by at most 2^8, which f32 accumulation absorbs.
// K and V tiles are placed box-major ([64-column box][4 blocks][16 rows]
// [128 B]) so one descriptor spans the 64 keys of a stage with an 8-row
// stride of 1024 bytes.  Completion: tcgen05.commit -> mbarriers; every wait
// is bounded.
// ---------------------------------------------------------------------------
namespace {

constexpr int kTcRows = 128;                 // rows of one tile (the MMA M)
constexpr int kTcTiles = 2;
constexpr int kTcCtaRows = kTcTiles * kTcRows;
constexpr int kTcSoftmaxWarps = kTcTiles * 4;
constexpr int kTcThreads = (kTcSoftmaxWarps + 2) * 32;
constexpr int kTcProducerWarp = kTcSoftmaxWarps;
constexpr int kTcMmaWarp = kTcSoftmaxWarps + 1;
constexpr int kTcStages = 5;
constexpr int kTcStageKeys = kStageBlocks * kPBlock;  // 64
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcTileCols = 256;  // tensor-memory columns of one tile
constexpr uint32_t kTcSCols = 64;      // one S buffer (later P head + remainder)
constexpr uint32_t kTcOCol = 128;      // O after the two S buffers
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct TcLayout {
  static constexpr int kBoxes = D / 64;
  static constexpr int kQBox = kTcRows * 128;         // 16 KB: 128 rows x 128 B
  static constexpr int kQBytes = kBoxes * kQBox;      // one tile's Q
  static constexpr int kKVBox = kTcStageKeys * 128;   // 8 KB: 64 keys x 128 B
  static constexpr int kKBytes = kBoxes * kKVBox;
  static constexpr int kStage = 2 * kKBytes;          // K, then V
  static constexpr int kRingOff = kTcTiles * kQBytes;
  static constexpr int kBarOff = kRingOff + kTcStages * kStage;
  // kv_full, kv_empty per stage; s_full and p_full per tile and S buffer;
  // o_done per tile; fin
  static constexpr int kNumBars = 2 * kTcStages + 5 * kTcTiles + 1;
  static constexpr int kMaskOff = kBarOff + kNumBars * 8;
  static constexpr int kTmemOff = kMaskOff + kTcStages * 4;
  static constexpr int kBytes = kTmemOff + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 227 * 1024, "shared memory of one CTA");
};

}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  using L = TcLayout<D>;
  constexpr uint32_t kAB = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescQK = tc_idesc_f16(kAB, 0, kTcRows, kTcStageKeys);
  constexpr uint32_t kIdescPV = tc_idesc_f16(kAB, 1, kTcRows, D);
  // P as a 16-bit head plus remainder (bf16), or a single f16 (f16 inputs)
  constexpr bool kSplitP = !std::is_same<T, __half>::value;
  constexpr int kBoxBytes = kPBlock * 128;  // one block's 16 rows of one box

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
  const int pos0 = ctx - qlen + tok0;
  const int nblk = (pos0 + ntok - 1) / kPBlock + 1;
  const int nstages = (nblk + kStageBlocks - 1) / kStageBlocks;
  const int G = a.group;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kTcStages;
  uint64_t* s_full = bars + 2 * kTcStages;  // per tile and S buffer: [2 x + buf]
  uint64_t* p_full = s_full + 2 * kTcTiles; // per tile and S buffer: [2 x + buf]
  uint64_t* o_done = p_full + 2 * kTcTiles; // per tile
  uint64_t* fin = o_done + kTcTiles;
  int* vmask = reinterpret_cast<int*>(smem + L::kMaskOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemOff);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(smem_addr(&kv_full[s]), 1);
      mbar_init(smem_addr(&kv_empty[s]), 1);
    }
    for (int x = 0; x < kTcTiles; ++x) {
      mbar_init(smem_addr(&s_full[2 * x]), 1);
      mbar_init(smem_addr(&s_full[2 * x + 1]), 1);
      mbar_init(smem_addr(&p_full[2 * x]), 4 * 32);
      mbar_init(smem_addr(&p_full[2 * x + 1]), 4 * 32);
      mbar_init(smem_addr(&o_done[x]), 1);
    }
    mbar_init(smem_addr(fin), 1);
    fence_mbar_init();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }
  // Q tiles -> shared memory, K-major with the 128-byte swizzle: row r of a
  // tile, 16-byte chunk c of its D elements at box c/8, line r, chunk
  // (c%8)^(r%8).  CTA row R = token R / G, head R % G.
  {
    constexpr int kChunks = D / 8;
    for (int i = threadIdx.x; i < kTcCtaRows * kChunks; i += kTcThreads) {
      const int R = i / kChunks, c = i - (i / kChunks) * kChunks;
      const int t = R / G, h = R - t * G;
      const bool act = (t < ntok) && (R < a.tokens_per_tile * G);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (act)
        v = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.q) +
                                            (((size_t)q0 + tok0 + t) * a.num_heads + (size_t)kvh * G + h) * D +
                                            c * 8);
      const int x = R / kTcRows, r = R - x * kTcRows;
      *reinterpret_cast<uint4*>(smem + x * L::kQBytes + (c >> 3) * L::kQBox + r * 128 +
                                (((c & 7) ^ (r & 7)) << 4)) = v;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int32_t* table = a.block_tables + (size_t)chunk * a.max_blocks_per_seq;

  if (warp == kTcProducerWarp) {
    // ---------------- TMA producer ----------------
    int ids = 0, issued = 0;
    for (int st = 0; st < nstages; ++st) {
      const int slot = st % kTcStages;
      if (st >= kTcStages) {
        bool ready = true;
        if (lane == 0)
          ready = mbar_wait_bounded(smem_addr(&kv_empty[slot]), (uint32_t)((st / kTcStages) - 1) & 1u);
        if (__shfl_sync(0xffffffffu, ready ? 1 : 0, 0) == 0) {
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
        const uint32_t bar = smem_addr(&kv_full[slot]);
        uint8_t* stage = smem + L::kRingOff + (size_t)slot * L::kStage;
        fence_proxy_async_smem();
        if (nvalid == 0) {
          mbar_arrive(bar);
        } else {
          mbar_arrive_expect_tx(bar, (uint32_t)(nvalid * 2 * kPBlock * D * 2));
#pragma unroll
          for (int k = 0; k < kStageBlocks; ++k) {
            if (!(mask & (1 << k))) continue;
            const int32_t row = (int32_t)(((int64_t)phys[k] * a.num_kv_heads + kvh) * kPBlock);
#pragma unroll
            for (int b = 0; b < L::kBoxes; ++b) {
              tma_load_2d(smem_addr(stage + b * L::kKVBox + k * kBoxBytes), &tmk, b * 64, row, bar);
              tma_load_2d(smem_addr(stage + L::kKBytes + b * L::kKVBox + k * kBoxBytes), &tmv, b * 64, row,
                          bar);
            }
          }
        }
      }
      __syncwarp();
      issued = st + 1;
    }
    if (lane == 0) {
      const int first = issued > kTcStages ? issued - kTcStages : 0;
      for (int st = first; st < issued; ++st)
        mbar_wait_bounded(smem_addr(&kv_full[st % kTcStages]), (uint32_t)(st / kTcStages) & 1u);
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      // Shared-memory descriptors: built once from the base addresses; an
      // operand at byte offset o further on is the base descriptor + o / 16
      // (the 14-bit address field holds any shared-memory address / 16, so
      // the addition never carries out of it).
      const uint64_t q_desc = smem_desc_sw128(smem_addr(smem), 16, 1024);
      const uint64_t k_desc = smem_desc_sw128(smem_addr(smem + L::kRingOff), 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(smem_addr(smem + L::kRingOff + L::kKBytes), L::kKVBox, 1024);
      auto issue_qk = [&](int st, int x) {
        const uint64_t qd = q_desc + (uint64_t)((x * L::kQBytes) >> 4);
        const uint64_t kd = k_desc + (uint64_t)(((st % kTcStages) * L::kStage) >> 4);
        const uint32_t d = tmem + x * kTcTileCols + (st & 1) * kTcSCols;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = qd + (uint64_t)(((kk >> 2) * L::kQBox + (kk & 3) * 32) >> 4);
          const uint64_t bd = kd + (uint64_t)(((kk >> 2) * L::kKVBox + (kk & 3) * 32) >> 4);
          tc_mma_f16(d, ad, bd, kIdescQK, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_addr(&s_full[2 * x + (st & 1)]));
      };
      auto issue_pv = [&](int st, int x) {
        const uint64_t vd = v_desc + (uint64_t)(((st % kTcStages) * L::kStage) >> 4);
        const uint32_t pt = tmem + x * kTcTileCols + (st & 1) * kTcSCols;  // P of this stage
        const uint32_t d = tmem + x * kTcTileCols + kTcOCol;
#pragma unroll
        for (int j = 0; j < kStageBlocks; ++j) {
#pragma unroll
          for (int hl = 0; hl < (kSplitP ? 2 : 1); ++hl) {
            const uint64_t bd = vd + (uint64_t)((j * kBoxBytes) >> 4);
            tc_mma_f16_ts(d, pt + hl * (kTcSCols / 2) + j * 8, bd, kIdescPV, (st > 0 || j > 0 || hl > 0) ? 1u : 0u);
          }
        }
        tc_commit(smem_addr(&o_done[x]));
      };
      // S is double-buffered per tile, so a tile's QK runs two stages ahead:
      // QK(st + 2) follows PV(st) (it overwrites the buffer P(st) was read
      // from, in issue order) and is done long before the tile's softmax
      // finishes stage st + 1, which therefore never waits for the tensor
      // pipe's round trip.
      auto wait_kv = [&](int st) {
        const bool r = mbar_wait_bounded(smem_addr(&kv_full[st % kTcStages]), (uint32_t)(st / kTcStages) & 1u);
        tc_fence_after();
        return r;
      };
      for (int st = 0; ok && st < 2 && st < nstages; ++st) {
        if (!wait_kv(st)) {
          ok = false;
          break;
        }
        issue_qk(st, 0);
        issue_qk(st, 1);
      }
      for (int st = 0; ok && st < nstages; ++st) {
        const bool ahead = st + 2 < nstages;
        for (int x = 0; x < kTcTiles; ++x) {
          // P of this tile written (and its S read): PV, then the S two
          // stages on.
          // P of stage st arrives on the tile's barrier of S buffer st & 1,
          // whose k-th completion (k = st / 2) is stage st: the softmax can
          // be at most one stage ahead of this wait (its stage st + 2 needs
          // QK(st + 2), issued after this PV), so the parity is unambiguous.
          if (!mbar_wait_bounded(smem_addr(&p_full[2 * x + (st & 1)]), (uint32_t)(st >> 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(st, x);
          // after the last tile's PV this stage's K/V may be refilled
          if (x == kTcTiles - 1) tc_commit(smem_addr(&kv_empty[st % kTcStages]));
          if (ahead) {
            if (x == 0 && !wait_kv(st + 2)) {
              ok = false;
              break;
            }
            issue_qk(st + 2, x);
          }
        }
      }
      if (!ok) prefill_error(CF_DEVERR_TIMEOUT);
      // Every MMA issued above has finished before tensor memory is released.
      tc_commit(smem_addr(fin));
      mbar_wait_bounded(smem_addr(fin), 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax warps of tile x: thread = row ----------------
    const int x = warp >> 2, quad = warp & 3;
    const int r = 32 * quad + lane;  // row within the tile = tensor-memory lane
    const int R = x * kTcRows + r;   // row within the CTA
    const int t = R / G, h = R - t * G;
    const bool act = (t < ntok) && (R < a.tokens_per_tile * G);
    const int qpos = act ? pos0 + t : -1;
    const uint32_t trow = tmem + ((uint32_t)(32 * quad) << 16) + x * kTcTileCols;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int st = 0; st < nstages; ++st) {
      const int slot = st % kTcStages;
      const bool r1 = mbar_wait_bounded(smem_addr(&s_full[2 * x + (st & 1)]), (uint32_t)(st >> 1) & 1u);
      const bool r2 = mbar_wait_bounded(smem_addr(&kv_full[slot]), (uint32_t)(st / kTcStages) & 1u);
      if (!__all_sync(0xffffffffu, r1 && r2)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTcStageKeys];
      {
        float(&s0)[32] = *reinterpret_cast<float(*)[32]>(&s[0]);
        float(&s1)[32] = *reinterpret_cast<float(*)[32]>(&s[32]);
        tmem_ld32(trow + (st & 1) * kTcSCols, s0);
        tmem_ld32(trow + (st & 1) * kTcSCols + 32, s1);
        tmem_wait_ld();
      }
      const int mask = vmask[slot];
      const int key0 = st * kTcStageKeys;
      // Stages wholly below every row's diagonal, with all blocks valid, need
      // no mask: the max is taken on the raw scores and the scale is folded
      // into the exponent (one FFMA per score).
      const bool unmasked = __all_sync(0xffffffffu, mask == 15 && key0 + kTcStageKeys - 1 <= qpos);
      // Row max and row sum over 8 independent partials (no 64-long
      // dependency chain).
      float part[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) part[i] = -INFINITY;
      if (unmasked) {
#pragma unroll
        for (int j = 0; j < kTcStageKeys; ++j) part[j & 7] = fmaxf(part[j & 7], s[j]);
      } else {
#pragma unroll
        for (int j = 0; j < kTcStageKeys; ++j) {
          const bool valid = ((mask >> (j >> 4)) & 1) && (key0 + j <= qpos);
          s[j] = valid ? s[j] * a.scale_log2 : -INFINITY;
          part[j & 7] = fmaxf(part[j & 7], s[j]);
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3])),
                       fmaxf(fmaxf(part[4], part[5]), fmaxf(part[6], part[7])));
      if (unmasked) mx *= a.scale_log2;
      float alpha = 1.f;
      if (mx != -INFINITY && (m_run == -INFINITY || mx > m_run + kRescaleLog2)) {
        alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - mx);
        m_run = mx;
      }
      const float mu = (m_run == -INFINITY) ? 0.f : m_run;
#pragma unroll
      for (int i = 0; i < 8; ++i) part[i] = 0.f;
      if (unmasked) {
#pragma unroll
        for (int j = 0; j < kTcStageKeys; ++j) {
          s[j] = ex2_approx(fmaf(s[j], a.scale_log2, -mu));
          part[j & 7] += s[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < kTcStageKeys; ++j) {
          s[j] = ex2_approx(s[j] - mu);
          part[j & 7] += s[j];
        }
      }
      const float ps = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
      l_run = l_run * alpha + ps;
      if (st > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // A row of this warp rescales O: the tile's previous PV, which
        // writes O, must be done.  Only then: the buffer this stage's P
        // overwrites was last read by PV(st - 2), which finished before
        // QK(st) wrote S(st) (the tensor pipe runs a thread's MMAs in
        // order).  Skipped waits leave the parity unambiguous: PV(st) needs
        // this stage's P, so o_done has completed st - 1 or st phases here.
        const bool r3 = mbar_wait_bounded(smem_addr(&o_done[x]), (uint32_t)(st - 1) & 1u);
        if (!__all_sync(0xffffffffu, r3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tmem_ld32(trow + kTcOCol + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(trow + kTcOCol + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P (16-bit head and remainder) over this stage's S buffer: keys
      // 2c, 2c+1 in column c (head) and column 32 + c (remainder).  An f16 P
      // (P <= 2^8, 11 significant bits) needs no remainder.
      if constexpr (kSplitP) {
        uint32_t hi[kTcStageKeys / 2], lo[kTcStageKeys / 2];
#pragma unroll
        for (int c = 0; c < kTcStageKeys / 2; ++c) split2<T>(s[2 * c], s[2 * c + 1], hi[c], lo[c]);
        tmem_st32(trow + (st & 1) * kTcSCols, reinterpret_cast<float(&)[32]>(hi));
        tmem_st32(trow + (st & 1) * kTcSCols + 32, reinterpret_cast<float(&)[32]>(lo));
        tmem_wait_st();
      } else {
        uint32_t hi[kTcStageKeys / 2];
#pragma unroll
        for (int c = 0; c < kTcStageKeys / 2; ++c) hi[c] = pack2<T>(s[2 * c], s[2 * c + 1]);
        tmem_st32(trow + (st & 1) * kTcSCols, reinterpret_cast<float(&)[32]>(hi));
        tmem_wait_st();
      }
      // V rows the MMA must not multiply (not loaded this stage, past the
      // context, or of a rejected block) are cleared by tile A's warps before
      // they release tile A's P (tile B's PV follows tile A's): 0 * NaN would
      // not be 0.
      if (x == 0) {
        const int keys_loaded = min(kTcStageKeys, nblk * kPBlock - key0);
        const int keys_ctx = min(kTcStageKeys, ctx - key0);
        const int keep = min(keys_loaded, keys_ctx);
        const int full_mask = (1 << min(kStageBlocks, nblk - st * kStageBlocks)) - 1;
        if (keep < kTcStageKeys || mask != full_mask) {
          uint8_t* vst = smem + L::kRingOff + (size_t)slot * L::kStage + L::kKBytes;
          for (int i = threadIdx.x; i < kTcStageKeys * L::kBoxes * 8; i += 4 * 32) {
            const int key = i / (L::kBoxes * 8);
            const int rem = i - key * (L::kBoxes * 8);
            const int b = rem >> 3, c = rem & 7;
            const bool bad = key >= keep || !((mask >> (key >> 4)) & 1);
            if (bad)
              *reinterpret_cast<uint4*>(vst + b * L::kKVBox + key * 128 + (c << 4)) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();  // the PV MMAs read these rows through the async proxy
        }
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&p_full[2 * x + (st & 1)]));
    }
    if (ok) {
      // The last PV done: `fin` completes once, after every MMA of the CTA
      // (o_done could be one or two phases short here, which its parity
      // cannot tell apart).
      const bool r4 = mbar_wait_bounded(smem_addr(fin), 0u);
      if (__all_sync(0xffffffffu, r4)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* out = reinterpret_cast<T*>(a.out) +
                 (((size_t)q0 + tok0 + (act ? t : 0)) * a.num_heads + (size_t)kvh * G + h) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(trow + kTcOCol + c * 32, o);
          tmem_wait_ld();
          if (act) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = pack2<T>(o[2 * i] * inv, o[2 * i + 1] * inv);
            uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
            dst[3] = make_uint4(w[12], w[13], w[14], w[15]);
          }
        }
      } else {
        ok = false;
      }
    }
    if (!ok && lane == 0) prefill_error(CF_DEVERR_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

namespace {

PrefillArgs make_args(const cf_prefill_params& p, int rows_per_cta) {
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
  a.tokens_per_tile = rows_per_cta / a.group;
  a.num_blocks = p.num_blocks;
  return a;
}

// Opts a kernel into its dynamic shared memory once per device.
template <typename Kernel>
cf_status ensure_prefill_smem(Kernel kern, int bytes, std::once_flag* flags, cudaError_t* errs) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return CF_ERR_UNSUPPORTED;
  std::call_once(flags[dev], [&] {
    errs[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return errs[dev] == cudaSuccess ? CF_OK : cuda_status(errs[dev]);
}

template <typename T, int D>
cf_status launch_prefill_typed(const cf_prefill_params& p, bool tcgen05, cudaStream_t stream) {
  const int64_t rows = p.num_blocks * (int64_t)p.num_kv_heads * kPBlock;
  CUtensorMap tmk, tmv;
  if (!kv_tensor_map(&tmk, p.key_cache, rows, D, p.dtype) ||
      !kv_tensor_map(&tmv, p.value_cache, rows, D, p.dtype))
    return CF_ERR_INVALID_ARGUMENT;
  if (tcgen05) {
    static std::once_flag flags[64];
    static cudaError_t errs[64];
    cf_status s = ensure_prefill_smem(paged_prefill_tc_kernel<T, D>, TcLayout<D>::kAlloc, flags, errs);
    if (s != CF_OK) return s;
    const PrefillArgs a = make_args(p, kTcCtaRows);
    const int tiles = (p.max_query_len + a.tokens_per_tile - 1) / a.tokens_per_tile;
    dim3 grid((unsigned)tiles, (unsigned)p.num_kv_heads, (unsigned)p.num_chunks);
    paged_prefill_tc_kernel<T, D><<<grid, kTcThreads, TcLayout<D>::kAlloc, stream>>>(a, tmk, tmv);
    return check_launch();
  }
  static std::once_flag flags[64];
  static cudaError_t errs[64];
  cf_status s = ensure_prefill_smem(paged_prefill_kernel<T, D>, PrefillLayout<D>::kAlloc, flags, errs);
  if (s != CF_OK) return s;
  const PrefillArgs a = make_args(p, kRows);
  const int tiles = (p.max_query_len + a.tokens_per_tile - 1) / a.tokens_per_tile;
  dim3 grid((unsigned)tiles, (unsigned)p.num_kv_heads, (unsigned)p.num_chunks);
  paged_prefill_kernel<T, D><<<grid, (kConsumerWarps + 1) * 32, PrefillLayout<D>::kAlloc, stream>>>(a, tmk, tmv);
  return check_launch();
}

// The tcgen05 kernel by default; CF_PREFILL_CONSUMER=mma selects the
// mma.sync kernel (=tc the tcgen05 one).
bool use_tcgen05() {
  if (const char* e = std::getenv("CF_PREFILL_CONSUMER")) {
    if (std::strcmp(e, "tc") == 0) return true;
    if (std::strcmp(e, "mma") == 0) return false;
  }
  return true;
}

}  // namespace

bool prefill_supported(int32_t head_dim, int32_t block_size, int32_t dtype, int32_t group) {
  return block_size == kPBlock && (dtype == CF_F16 || dtype == CF_BF16) &&
         (head_dim == 64 || head_dim == 128) && group >= 1 && group <= kRows;
}

cf_status launch_paged_prefill(const cf_prefill_params& p, cudaStream_t stream) {
  if (p.num_chunks == 0 || p.max_query_len == 0) return CF_OK;
  const bool tc = use_tcgen05();
  if (p.dtype == CF_BF16) {
    if (p.head_dim == 128) return launch_prefill_typed<__nv_bfloat16, 128>(p, tc, stream);
    return launch_prefill_typed<__nv_bfloat16, 64>(p, tc, stream);
  }
  if (p.head_dim == 128) return launch_prefill_typed<__half, 128>(p, tc, stream);
  return launch_prefill_typed<__half, 64>(p, tc, stream);
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
