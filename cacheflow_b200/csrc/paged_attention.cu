// paged_attention.cu -- ragged-batch paged decode attention for sm_100a.
//
// Semantics (one query token per sequence), following CacheFlow
// src/cacheflow/cuda/paged_attention.cu:
//   kv head of query head h      = h / (num_heads / num_kv_heads)      (:58)
//   logical block b of sequence s = block_tables[s * max_blocks_per_seq + b] (:78-79)
//   K row of token t              = key_cache[((phys * Hkv + kvh) * 16 + t % 16) * D]  (:85-87)
//   V row                         = value_cache[same index]                          (:151-153)
//   out[s, h, :] = softmax_t(scale * q . k_t) . V  over t < context_lens[s]
// computed as the normalised softmax the reference intends (its V1 overflows
// a 128-entry shared array past 128 tokens and its V2 leaves the result
// unnormalised; neither is reproduced).
//
// Design:
//   * One CTA per (partition, kv head [x head chunk], sequence).  All query
//     heads of a GQA group are handled by the CTA that streams their KV head,
//     so every KV byte is read from HBM once per KV head.
//   * Each of the NW warps streams its own share of the partition's 16-token
//     blocks through a private S-stage ring in shared memory.  Lane 0 of the
//     warp issues the async copies of a block's K and V tiles (4 KB each for
//     bf16/fp16 at D=128): 1-D bulk copies (cp.async.bulk) for the FMA
//     consumer, 2-D tensor-map boxes with the 128-byte swizzle for the
//     tensor-core consumers; completion is tracked by one mbarrier per stage,
//     and the warp computes on stage i while stages i+1..i+S-1 are in flight.
//     Block-table entries are fetched 32 at a time by the warp and broadcast
//     with shuffles.
//   * Consumers (per warp, online softmax in the log2 domain): FMA -- QK dot
//     products by 8-lane groups with xor-shuffle reductions, PV with each lane
//     owning D/32 output columns; MMA -- mma.sync for 16-bit caches with up to
//     8 query heads as the rows; MmaConsumerFp8 -- the same for e4m3 caches,
//     converted to f16 in registers.
//   * Optional fused append: the newest token of each row is patched into its
//     tile and written to the cache by the same launch.
//   * Warps are merged through shared memory at the end of the partition.
//     A sequence that fits one partition writes its output directly;
//     otherwise the partition writes (max logit, exp-sum, normalised partial
//     output) and the reduce kernel merges partitions with the log-sum-exp
//     weights  w_p = exp_sum_p * exp(max_p - max).
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "cf_device.cuh"
#include "cf_internal.h"

namespace cfb {

__device__ uint32_t g_attn_errors;

__device__ __forceinline__ void attn_error(uint32_t bits) { atomicOr(&g_attn_errors, bits); }

constexpr int kBlockTokens = 16;  // KV block size (tokens); CacheFlow's KV_BLOCK_SIZE
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnArgs {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  void* out;
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* part_max;  // [S, H, P]  natural-log units; null when unsplit
  float* part_sum;  // [S, H, P]
  float* part_out;  // [S, H, P, D]
  float scale_log2;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t group;        // num_heads / num_kv_heads
  int32_t head_chunks;  // ceil(group / HG)
  int32_t max_blocks_per_seq;
  int32_t part_blocks;  // KV blocks per partition
  int32_t num_parts;    // partition stride of the scratch
  int64_t num_blocks;   // pool size (checked range of physical ids)
  // Fused append (null new_k: none).  Row s's newest token -- position
  // context_lens[s] - 1 -- takes its K/V from new_k/new_v[s, kvh, :] and is
  // written to the cache at that position's slot.
  const void* new_k;            // [S, Hkv, D]
  const void* new_v;
  const int32_t* slot_mapping;  // [S] or null (slot from the block table)
  void* k_cache_w;              // the caches, written by the append
  void* v_cache_w;
  float v_scale;                // fp8 caches: V = stored * v_scale (else 1)
  float k_scale;                // fp8 caches: K = stored * k_scale (appends store K / k_scale)
  // Pipeline waits give up after this long (kWaitLimitNs unless a test
  // shortened it with cf_testing_set_pipeline_faults).
  uint64_t wait_limit_ns;
  // Test hook: nonzero leaves the first stage of every warp unarmed (no copy
  // issued, no arrive), so its wait can only run out.
  int32_t unarm_first_stage;
};

// ---------------------------------------------------------------------------
// FMA consumer: QK by 8-lane groups (each lane reads D*sizeof(T)/128 16-byte
// chunks of a K row: the 8 lanes of a group cover 128 contiguous bytes, so
// shared-memory reads are conflict-free without swizzling), PV with lane l
// owning columns [l*D/32, (l+1)*D/32).
// ---------------------------------------------------------------------------
template <typename T, typename TC, int D, int HG, int R>
struct FmaConsumer {
  static constexpr int kVec = 16 / (int)sizeof(TC);          // cache elements per 16 B
  static constexpr int kChunks = D * (int)sizeof(TC) / 128;  // 16 B chunks per lane (QK)
  static constexpr int kEpl = D / 32;                        // columns per lane (PV)
  static_assert(kChunks >= 1, "head_dim too small for this element type");

  float q[HG][kChunks * kVec];
  float o[HG][kEpl];
  float m[HG];
  float l[HG];

  __device__ __forceinline__ void init(const T* qrow, int nheads, float scale_log2, int lane) {
    const int i = lane & 7;
#pragma unroll
    for (int h = 0; h < HG; ++h) {
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        if (h < nheads) {
          load_widen<T, kVec>(qrow + (size_t)h * D + (i + 8 * k) * kVec, &q[h][k * kVec]);
#pragma unroll
          for (int e = 0; e < kVec; ++e) q[h][k * kVec + e] *= scale_log2;
        } else {
#pragma unroll
          for (int e = 0; e < kVec; ++e) q[h][k * kVec + e] = 0.f;
        }
      }
#pragma unroll
      for (int e = 0; e < kEpl; ++e) o[h][e] = 0.f;
      m[h] = -INFINITY;
      l[h] = 0.f;
    }
  }

  __device__ __forceinline__ void pv_token(const TC* vrow, const float* pt_h, int t) {
    float vf[kEpl];
    load_widen<TC, kEpl>(vrow + t * D, vf);
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      const float pt = pt_h[h * R + t];
#pragma unroll
      for (int e = 0; e < kEpl; ++e) o[h][e] = fmaf(pt, vf[e], o[h][e]);
    }
  }

  // One tile of R tokens (a 16-token block, or half of one); `ntok` valid
  // tokens (1..R).  `pbuf` is this warp's HG*R-float scratch.
  __device__ __forceinline__ void block(const uint8_t* kraw, const uint8_t* vraw, int ntok,
                                        float* pbuf, int lane) {
    constexpr int kPasses = R / 4;  // 4 tokens per pass (one per 8-lane group)
    const TC* kt = reinterpret_cast<const TC*>(kraw);
    const TC* vt = reinterpret_cast<const TC*>(vraw);
    const int j = lane >> 3;
    const int i = lane & 7;
    float s[kPasses][HG];
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int tok = p * 4 + j;
      const TC* row = kt + tok * D;
      float acc[HG];
#pragma unroll
      for (int h = 0; h < HG; ++h) acc[h] = 0.f;
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        float kf[kVec];
        load_widen<TC, kVec>(row + (i + 8 * k) * kVec, kf);
#pragma unroll
        for (int h = 0; h < HG; ++h)
#pragma unroll
          for (int e = 0; e < kVec; ++e) acc[h] = fmaf(q[h][k * kVec + e], kf[e], acc[h]);
      }
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float a = acc[h];
        a += shfl_xor(a, 1);
        a += shfl_xor(a, 2);
        a += shfl_xor(a, 4);
        s[p][h] = (tok < ntok) ? a : -INFINITY;
      }
    }
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      float bm = s[0][h];
#pragma unroll
      for (int p = 1; p < kPasses; ++p) bm = fmaxf(bm, s[p][h]);
      bm = fmaxf(bm, shfl_xor(bm, 8));
      bm = fmaxf(bm, shfl_xor(bm, 16));
      const float mn = fmaxf(m[h], bm);
      const float mu = (mn == -INFINITY) ? 0.f : mn;
      const float alpha = exp2f(m[h] - mu);
      m[h] = mn;
      float ps = 0.f;
#pragma unroll
      for (int p = 0; p < kPasses; ++p) {
        s[p][h] = exp2f(s[p][h] - mu);
        ps += s[p][h];
      }
      ps += shfl_xor(ps, 8);
      ps += shfl_xor(ps, 16);
      l[h] = l[h] * alpha + ps;
#pragma unroll
      for (int e = 0; e < kEpl; ++e) o[h][e] *= alpha;
      if (i == 0) {
#pragma unroll
        for (int p = 0; p < kPasses; ++p) pbuf[h * R + p * 4 + j] = s[p][h];
      }
    }
    __syncwarp();
    const TC* vrow = vt + lane * kEpl;
    if (ntok == R) {
#pragma unroll
      for (int t = 0; t < R; ++t) pv_token(vrow, pbuf, t);
    } else {
#pragma unroll 1
      for (int t = 0; t < ntok; ++t) pv_token(vrow, pbuf, t);
    }
  }

  // Per-warp result into the merge area: o[h][d] (unnormalised), m, l.
  __device__ __forceinline__ void store(float* mo, float* mm, float* ml, int lane) {
#pragma unroll
    for (int h = 0; h < HG; ++h) {
#pragma unroll
      for (int e = 0; e < kEpl; ++e) mo[h * D + lane * kEpl + e] = o[h][e];
      if (lane == 0) {
        mm[h] = m[h];
        ml[h] = l[h];
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Tensor-core consumer for GQA groups (16-bit caches, up to 8 query heads per
// KV head).  Per 16-token block and warp:
//   S[16 x 16] = Q[16 x D] . K^T   rows 0..7 = the group's query heads (rows
//                                  8..15 of Q are zero), 2 n-tiles of 8 tokens
//   O[16 x D] += P[16 x 16] . V    rows 0..7 carry P rounded to 16 bits, rows
//                                  8..15 the rounding remainder of the same P,
//                                  so O = O[g] + O[g+8] keeps ~16 more bits of
//                                  the softmax weights at no extra MMA cost.
// K and V tiles arrive through 2-D TMA boxes of 16 rows x 128 bytes with the
// 128-byte swizzle (16-byte chunk c of row r stored at chunk c ^ (r % 8)), so
// every ldmatrix phase hits 8 distinct bank groups.  The C fragment of the two
// S n-tiles is exactly the A fragment of P, so P never leaves registers.
// ---------------------------------------------------------------------------
template <typename T, int D>
struct MmaConsumer {
  static constexpr int kKC = D / 16;  // k-chunks of QK
  static constexpr int kND = D / 8;   // n-tiles of PV (8 columns each)
  static constexpr int kBoxBytes = kBlockTokens * 128;

  uint32_t qa[kKC][2];  // A fragment of Q: (row g, k lo) and (row g, k hi)
  float o[kND][4];      // C fragments of O: rows g (16-bit P) and g+8 (remainder)
  float m;              // running max of head g (log2 units), uniform in a quad
  float l;              // this lane's share of the running exp-sum of head g
  float scale_log2;

  __device__ __forceinline__ void init(const T* qrow, int nheads, float sl2, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int kc = 0; kc < kKC; ++kc) {
      if (g < nheads) {
        const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qrow + (size_t)g * D + kc * 16 + 2 * t);
        qa[kc][0] = q32[0];
        qa[kc][1] = q32[4];  // +8 elements
      } else {
        qa[kc][0] = qa[kc][1] = 0u;
      }
    }
#pragma unroll
    for (int n = 0; n < kND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    m = -INFINITY;
    l = 0.f;
    scale_log2 = sl2;
  }

  __device__ __forceinline__ void block(const uint8_t* kt, const uint8_t* vt, int ntok, float*,
                                        int lane) {
    const int t = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const uint32_t kbase = smem_addr(kt), vbase = smem_addr(vt);
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      // ldmatrix.x4 lane address: matrix mi = (token half, chunk parity).
      const int r = (mi >> 1) * 8 + ri;
      const uint32_t rowa = kbase + r * 128;
#pragma unroll
      for (int kc = 0; kc < kKC; ++kc) {
        const int box = kc >> 2;
        const int c = ((kc & 3) << 1) + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(rowa + box * kBoxBytes + ((c ^ (r & 7)) << 4), b0, b1, b2, b3);
        mma_16816<T>(s[0], qa[kc][0], 0u, qa[kc][1], 0u, b0, b1);
        mma_16816<T>(s[1], qa[kc][0], 0u, qa[kc][1], 0u, b2, b3);
      }
    }
    // Online softmax over this block's 16 tokens (4 per lane).
    float bm = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int tok = nt * 8 + 2 * t + j;
        const float x = s[nt][j] * scale_log2;
        s[nt][j] = tok < ntok ? x : -INFINITY;
        bm = fmaxf(bm, s[nt][j]);
      }
    bm = fmaxf(bm, shfl_xor(bm, 1));
    bm = fmaxf(bm, shfl_xor(bm, 2));
    const float mn = fmaxf(m, bm);
    const float mu = (mn == -INFINITY) ? 0.f : mn;
    const float alpha = exp2f(m - mu);
    m = mn;
    float ps = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        s[nt][j] = exp2f(s[nt][j] - mu);
        ps += s[nt][j];
      }
    l = l * alpha + ps;
#pragma unroll
    for (int n = 0; n < kND; ++n) {
      o[n][0] *= alpha;
      o[n][1] *= alpha;
      o[n][2] *= alpha;
      o[n][3] *= alpha;
    }
    uint32_t pa[4];
    split2<T>(s[0][0], s[0][1], pa[0], pa[1]);
    split2<T>(s[1][0], s[1][1], pa[2], pa[3]);

    if (ntok < kBlockTokens) {
      // Rows past the context hold whatever the pool holds (possibly NaN);
      // their weight is 0, but 0 * NaN is not, so clear them before PV.
      constexpr int kChunksPerRow = D * (int)sizeof(T) / 16;
      const int n = (kBlockTokens - ntok) * kChunksPerRow;
      for (int i = lane; i < n; i += 32) {
        const int r = ntok + i / kChunksPerRow;
        const int c = i % kChunksPerRow;  // position inside the row is irrelevant
        *reinterpret_cast<uint4*>(const_cast<uint8_t*>(vt) + (c >> 3) * kBoxBytes + r * 128 +
                                  ((c & 7) << 4)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();  // the next TMA write of this tile follows these stores
      __syncwarp();
    }
    {
      // ldmatrix.x4.trans: matrix mi = (token half, chunk of the pair).
      const int r = (mi & 1) * 8 + ri;
      const uint32_t rowa = vbase + r * 128;
#pragma unroll
      for (int cp = 0; cp < kND / 2; ++cp) {
        const int c = 2 * cp + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(rowa + (c >> 3) * kBoxBytes + (((c & 7) ^ (r & 7)) << 4), b0, b1, b2, b3);
        mma_16816<T>(o[2 * cp], pa[0], pa[1], pa[2], pa[3], b0, b1);
        mma_16816<T>(o[2 * cp + 1], pa[0], pa[1], pa[2], pa[3], b2, b3);
      }
    }
  }

  __device__ __forceinline__ void store(float* mo, float* mm, float* ml, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int n = 0; n < kND; ++n) {
      mo[g * D + n * 8 + 2 * t] = o[n][0] + o[n][2];
      mo[g * D + n * 8 + 2 * t + 1] = o[n][1] + o[n][3];
    }
    float lt = l;
    lt += shfl_xor(lt, 1);
    lt += shfl_xor(lt, 2);
    if (t == 0) {
      mm[g] = m;
      ml[g] = lt;
    }
  }
};

// ---------------------------------------------------------------------------
// Tensor-core consumer for fp8 (e4m3) caches with f16 / bf16 queries.  The
// MMAs run in f16 (e4m3 -> f16 is exact; queries are rounded to f16, exact
// for bf16 values of magnitude 2^-14 .. 65504).  Tiles arrive as for the
// 16-bit consumer: 16 rows x 128-byte boxes (128 e4m3 per box row) with the
// 128-byte swizzle.  No transposing load exists for bytes, so both products
// reorder a contracted or output dimension instead:
//   S = Q.K^T: ldmatrix (b16 view) hands thread (g, t) bytes 4t..4t+3 of a
//     16-byte chunk of token row g; the low two feed k-slots 2t, 2t+1 and the
//     high two k-slots 2t+8, 2t+9.  Q's A fragment is loaded with the same
//     order (elements 4t..4t+3 of the chunk), so the dot product is unchanged.
//   O += P.V: ldmatrix.trans (b16 view) hands thread (g, t) the byte pairs
//     (2g, 2g+1) of tokens 2t and 2t+1; a byte permute pairs the even column
//     of both tokens and the odd column of both tokens, giving the B
//     fragments of two n-tiles: one over the chunk's even columns, one over
//     its odd columns.  store() writes each accumulator column back to its
//     true position.
// P is split into an f16 head and remainder (rows g / g+8) as in the 16-bit
// consumer.  The per-cache scales are applied outside: k_scale is folded into
// the logit scale, v_scale into the final output.
// ---------------------------------------------------------------------------
template <typename T, int D>
struct MmaConsumerFp8 {
  static_assert(D % 128 == 0, "fp8 tiles are whole 128-byte boxes");
  static constexpr int kKC = D / 16;   // k-steps of QK = 16-byte chunks of a row
  static constexpr int kND = D / 8;    // n-tiles of PV (each chunk: even and odd columns)
  static constexpr int kBoxBytes = kBlockTokens * 128;

  uint32_t qa[kKC][2];
  float o[kND][4];
  float m;
  float l;
  float scale_log2;

  __device__ __forceinline__ void init(const T* qrow, int nheads, float sl2, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int kc = 0; kc < kKC; ++kc) {
      if (g < nheads) {
        float f[4];
        load_widen<T, 4>(qrow + (size_t)g * D + kc * 16 + 4 * t, f);
        qa[kc][0] = pack2<__half>(f[0], f[1]);
        qa[kc][1] = pack2<__half>(f[2], f[3]);
      } else {
        qa[kc][0] = qa[kc][1] = 0u;
      }
    }
#pragma unroll
    for (int n = 0; n < kND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    m = -INFINITY;
    l = 0.f;
    scale_log2 = sl2;
  }

  __device__ __forceinline__ void block(const uint8_t* kt, const uint8_t* vt, int ntok, float*,
                                        int lane) {
    const int t = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const uint32_t kbase = smem_addr(kt), vbase = smem_addr(vt);
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      // matrix mi: tokens (mi >> 1) * 8 .., chunk kc + (mi & 1)
      const int r = (mi >> 1) * 8 + ri;
      const uint32_t rowa = kbase + r * 128;
#pragma unroll
      for (int kc = 0; kc < kKC; kc += 2) {
        const int c = kc + (mi & 1);
        uint32_t x[4], b[4][2];
        ldmatrix_x4(rowa + (c >> 3) * kBoxBytes + (((c & 7) ^ (r & 7)) << 4), x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) e4m3x4_to_h2x2(x[i], b[i][0], b[i][1]);
        mma_16816<__half>(s[0], qa[kc][0], 0u, qa[kc][1], 0u, b[0][0], b[0][1]);
        mma_16816<__half>(s[1], qa[kc][0], 0u, qa[kc][1], 0u, b[2][0], b[2][1]);
        mma_16816<__half>(s[0], qa[kc + 1][0], 0u, qa[kc + 1][1], 0u, b[1][0], b[1][1]);
        mma_16816<__half>(s[1], qa[kc + 1][0], 0u, qa[kc + 1][1], 0u, b[3][0], b[3][1]);
      }
    }
    float bm = -INFINITY;
    if (ntok == kBlockTokens) {  // every block but a sequence's last
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          s[nt][j] *= scale_log2;
          bm = fmaxf(bm, s[nt][j]);
        }
    } else {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int tok = nt * 8 + 2 * t + j;
          const float x = s[nt][j] * scale_log2;
          s[nt][j] = tok < ntok ? x : -INFINITY;
          bm = fmaxf(bm, s[nt][j]);
        }
    }
    bm = fmaxf(bm, shfl_xor(bm, 1));
    bm = fmaxf(bm, shfl_xor(bm, 2));
    const float mn = fmaxf(m, bm);
    const float mu = (mn == -INFINITY) ? 0.f : mn;
    const float alpha = ex2_approx(m - mu);
    m = mn;
    float ps = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        s[nt][j] = ex2_approx(s[nt][j] - mu);
        ps += s[nt][j];
      }
    l = l * alpha + ps;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {  // the running max moved for some row
#pragma unroll
      for (int n = 0; n < kND; ++n) {
        o[n][0] *= alpha;
        o[n][1] *= alpha;
        o[n][2] *= alpha;
        o[n][3] *= alpha;
      }
    }
    uint32_t pa[4];
    split2<__half>(s[0][0], s[0][1], pa[0], pa[1]);
    split2<__half>(s[1][0], s[1][1], pa[2], pa[3]);

    if (ntok < kBlockTokens) {
      // Rows past the context may hold NaN patterns; 0 * NaN is not 0.
      constexpr int kChunksPerRow = D / 16;
      const int n = (kBlockTokens - ntok) * kChunksPerRow;
      for (int i = lane; i < n; i += 32) {
        const int r = ntok + i / kChunksPerRow;
        const int c = i % kChunksPerRow;
        *reinterpret_cast<uint4*>(const_cast<uint8_t*>(vt) + (c >> 3) * kBoxBytes + r * 128 +
                                  ((c & 7) << 4)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncwarp();
    }
    {
      // matrix mi: tokens (mi & 1) * 8 .., chunk 2 * cp + (mi >> 1)
      const int r = (mi & 1) * 8 + ri;
      const uint32_t rowa = vbase + r * 128;
#pragma unroll
      for (int cp = 0; cp < kKC / 2; ++cp) {
        const int c = 2 * cp + (mi >> 1);
        uint32_t y[4];
        ldmatrix_x4_trans(rowa + (c >> 3) * kBoxBytes + (((c & 7) ^ (r & 7)) << 4), y[0], y[1], y[2], y[3]);
        // chunk 2cp: tokens 0-7 in y0, 8-15 in y1; chunk 2cp+1: y2, y3.  One
        // byte permute gathers a column's 4 tokens (b0 pair, b1 pair).
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t be0, be1, bo0, bo1;
          e4m3x4_to_h2x2(__byte_perm(y[2 * h], y[2 * h + 1], 0x6420), be0, be1);
          e4m3x4_to_h2x2(__byte_perm(y[2 * h], y[2 * h + 1], 0x7531), bo0, bo1);
          mma_16816<__half>(o[4 * cp + 2 * h], pa[0], pa[1], pa[2], pa[3], be0, be1);
          mma_16816<__half>(o[4 * cp + 2 * h + 1], pa[0], pa[1], pa[2], pa[3], bo0, bo1);
        }
      }
    }
  }

  // n-tile 2c + p (p = 0 even, 1 odd columns of chunk c): accumulator column
  // j of the tile is head dimension 16c + 2j + p.
  __device__ __forceinline__ void store(float* mo, float* mm, float* ml, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int n = 0; n < kND; ++n) {
      const int d = (n >> 1) * 16 + 4 * t + (n & 1);
      mo[g * D + d] = o[n][0] + o[n][2];
      mo[g * D + d + 2] = o[n][1] + o[n][3];
    }
    float lt = l;
    lt += shfl_xor(lt, 1);
    lt += shfl_xor(lt, 2);
    if (t == 0) {
      mm[g] = m;
      ml[g] = lt;
    }
  }
};

// ---------------------------------------------------------------------------
// Fused append: the warp that will hold block `blk` (the one with the row's
// newest token) copies the new K/V row, the block id and the slot into shared
// memory (cp.async) before its pipeline starts, so the patch waits on nothing
// and no registers are held across the loop; when that block's tile lands it
// overwrites the token's row in the tile -- in the tile's own layout:
// row-major for the FMA consumer, 128-byte boxes with the 128-byte swizzle
// for the MMA consumers (e4m3 bytes for fp8 caches) -- and, in the CTA of
// head chunk 0 (`owner`), stores it into the cache, which is what
// reshape_and_cache (kv_cache_kernels.cu:34-40) does with
// slot = block_tables[s][blk] * 16 + (ctx - 1) % 16.  A slot_mapping
// entry that is negative appends nothing; one that is not that slot is
// recorded (CF_DEVERR_SLOT) and appends nothing.  Other CTAs of the same row
// may read the cache row while it is written; they overwrite it in their own
// tile.
// ---------------------------------------------------------------------------
template <typename T, typename TC, int D>
struct AppendRow {
  static constexpr bool kFp8 = std::is_same<TC, __nv_fp8_e4m3>::value;
  static constexpr int kRowBytes = D * (int)sizeof(T);         // one new K or V row
  static constexpr int kRowChunks = kRowBytes / 16;              // its 16-byte chunks
  static constexpr int kPerLane = (2 * kRowChunks + 31) / 32;    // K then V
  static constexpr int kVec = 16 / (int)sizeof(T);
  static constexpr int kOut = kVec * (int)sizeof(TC);  // cache bytes of one chunk (8 for fp8)
  // Staging area in shared memory: the K row, the V row, then four int32:
  // the block id, the slot_mapping entry, the token's position and whether
  // this CTA stores the row to the cache.
  static constexpr int kStageBytes = 2 * kRowBytes + 16;

  // Issues asynchronous copies only (nothing is held in registers and nothing
  // here waits for them), so the warp's copy pipeline starts at once and the
  // row arrives while it streams.
  __device__ __forceinline__ static void load(const AttnArgs& a, uint8_t* stage, int seq, int kvh, int pos,
                                              bool owner, int lane) {
    const size_t src = ((size_t)seq * a.num_kv_heads + kvh) * D;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int i = lane + 32 * j;
      if (i < 2 * kRowChunks) {
        const int kv = i >= kRowChunks ? 1 : 0;
        const int c = i - kv * kRowChunks;
        cp_async16(smem_addr(stage + i * 16), reinterpret_cast<const T*>(kv ? a.new_v : a.new_k) + src + c * kVec);
      }
    }
    if (lane == 0) {
      int32_t* w = reinterpret_cast<int32_t*>(stage + 2 * kRowBytes);
      cp_async4(smem_addr(w), a.block_tables + (size_t)seq * a.max_blocks_per_seq + pos / kBlockTokens);
      if (a.slot_mapping != nullptr) cp_async4(smem_addr(w + 1), a.slot_mapping + seq);
      w[2] = pos;
      w[3] = owner ? 1 : 0;
    }
    cp_async_commit();
  }

  // Called when the tile holding the token (R rows) has landed.  kTile is the
  // tile's bytes.  An fp8 cache takes each element as e4m3(x / scale),
  // rounded to nearest even and saturated to +-448, exactly as
  // reshape_and_cache_fp8 stores it.
  template <bool kMma, int kTile, int R>
  __device__ __forceinline__ static void patch(const AttnArgs& a, const uint8_t* stage, uint8_t* kt, int kvh,
                                               int lane) {
    if constexpr (kFp8) {
      patch_call<kMma, kTile, R>(a.k_cache_w, a.v_cache_w, a.slot_mapping != nullptr, a.num_kv_heads, a.k_scale,
                                 a.v_scale, stage, kt, kvh, lane);
    } else {
      patch_body<kMma, kTile, R>(a.k_cache_w, a.v_cache_w, a.slot_mapping != nullptr, a.num_kv_heads, a.k_scale,
                                 a.v_scale, stage, kt, kvh, lane);
    }
  }

  // The fp8 kernels run register-capped (four CTAs per SM): an out-of-line
  // call keeps the conversion's registers out of the streaming loop.
  template <bool kMma, int kTile, int R>
  __device__ __noinline__ static void patch_call(void* kc, void* vc, bool has_slots, int32_t num_kv_heads,
                                                 float k_scale, float v_scale, const uint8_t* stage, uint8_t* kt,
                                                 int kvh, int lane) {
    patch_body<kMma, kTile, R>(kc, vc, has_slots, num_kv_heads, k_scale, v_scale, stage, kt, kvh, lane);
  }

  template <bool kMma, int kTile, int R>
  __device__ __forceinline__ static void patch_body(void* kc, void* vc, bool has_slots, int32_t num_kv_heads,
                                                    float k_scale, float v_scale, const uint8_t* stage,
                                                    uint8_t* kt, int kvh, int lane) {
    cp_async_wait_all();
    __syncwarp();  // lane 0's block id and slot are visible to the warp
    const int32_t* w = reinterpret_cast<const int32_t*>(stage + 2 * kRowBytes);
    const int32_t phys = w[0];
    const int pos = w[2];
    const bool owner = w[3] != 0;
    const int row = pos % R;              // the token's row within the tile
    const int tok = pos % kBlockTokens;   // and within its block
    if (has_slots) {
      const int32_t slot = w[1];
      if (slot < 0) return;
      if ((int64_t)slot != (int64_t)phys * kBlockTokens + tok) {
        if (owner && lane == 0) attn_error(CF_DEVERR_SLOT);
        return;
      }
    }
    const size_t dst = (((size_t)phys * num_kv_heads + kvh) * kBlockTokens + tok) * D * sizeof(TC);
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int i = lane + 32 * j;
      if (i < 2 * kRowChunks) {
        const int kv = i >= kRowChunks ? 1 : 0;
        const int c = i - kv * kRowChunks;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + i * 16);
        const int p = c * kOut;  // byte of the chunk within the cache row
        const int off = kMma ? (p >> 7) * (kBlockTokens * 128) + row * 128 +
                                   ((((p >> 4) & 7) ^ (row & 7)) << 4) + (p & 15)
                             : row * D * (int)sizeof(TC) + p;
        uint8_t* cache = reinterpret_cast<uint8_t*>(kv ? vc : kc) + dst + p;
        if constexpr (kFp8) {
          const float sc = kv ? v_scale : k_scale;
          const uint32_t x[4] = {v.x, v.y, v.z, v.w};
          uint32_t q[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float f[4];
            unpack_word<T>(x[2 * h], f);
            unpack_word<T>(x[2 * h + 1], f + 2);
            q[h] = (uint32_t)f2_to_e4m3x2(__fdiv_rn(f[0], sc), __fdiv_rn(f[1], sc)) |
                   ((uint32_t)f2_to_e4m3x2(__fdiv_rn(f[2], sc), __fdiv_rn(f[3], sc)) << 16);
          }
          *reinterpret_cast<uint2*>(kt + kv * kTile + off) = make_uint2(q[0], q[1]);
          if (owner) *reinterpret_cast<uint2*>(cache) = make_uint2(q[0], q[1]);
        } else {
          *reinterpret_cast<uint4*>(kt + kv * kTile + off) = v;
          if (owner) *reinterpret_cast<uint4*>(cache) = v;
        }
      }
    }
    fence_proxy_async_smem();  // a later TMA write of this tile follows these stores
    __syncwarp();
  }
};

// ---------------------------------------------------------------------------
// Kernel configuration (per element type / head dim).
// ---------------------------------------------------------------------------
template <typename T, int D, int HG>
struct AttnConfig {
  // Tile rows: a 16-token block, or half of one for fp32 at D >= 128 (8 KB
  // blocks would leave room for one CTA per SM).
  static constexpr int kRows = (sizeof(T) == 4 && D >= 128) ? 8 : kBlockTokens;
  static constexpr int kTileBytes = kRows * D * (int)sizeof(T);  // one K or V tile
  static constexpr int kWarps = 4;
  // 1-byte (fp8) tiles: half the ring, so twice the CTAs fit on an SM.
  static constexpr int kStageBudget = sizeof(T) == 1 ? 48 * 1024 : 96 * 1024;
  static constexpr int kStagesRaw = kStageBudget / (kWarps * 2 * kTileBytes);
  static constexpr int kStages = kStagesRaw < 2 ? 2 : (kStagesRaw > 8 ? 8 : kStagesRaw);
  static constexpr int kTileArea = kWarps * kStages * 2 * kTileBytes;
  static constexpr int kMergeBytes = kWarps * HG * (D + 2) * 4;
  static_assert(kMergeBytes <= kTileArea, "merge area must fit in the stage area");
  static constexpr int kBarOffset = kTileArea;
  static constexpr int kFlagOffset = kBarOffset + kWarps * kStages * 8;
  static constexpr int kPbufOffset = kFlagOffset + ((kWarps * kStages * 4 + 15) / 16) * 16;
  static constexpr int kSmemBytes = kPbufOffset + kWarps * HG * kRows * 4;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack to align the base to 1 KB
  // fp8 at D=128: four CTAs (16 warps) per SM, the registers capped to fit.
  static constexpr int kMinCtas = (sizeof(T) == 1 && D == 128) ? 4 : 1;
};

template <typename T, typename TC, int D, int HG, bool kMma, bool kAppend>
__global__ void __launch_bounds__(AttnConfig<TC, D, HG>::kWarps * 32, AttnConfig<TC, D, HG>::kMinCtas)
    paged_attention_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv) {
  // T: query / output type; TC: cache type (T, or fp8 e4m3 with T 16-bit).
  using Cfg = AttnConfig<TC, D, HG>;
  constexpr bool kFp8 = std::is_same<TC, __nv_fp8_e4m3>::value;
  constexpr int R = Cfg::kRows;             // tokens per tile
  constexpr int kSubs = kBlockTokens / R;   // tiles per block
  static_assert(!kMma || R == kBlockTokens, "tensor-core tiles are whole blocks");
  using Consumer = std::conditional_t<kMma, std::conditional_t<kFp8, MmaConsumerFp8<T, D>, MmaConsumer<T, D>>,
                                      FmaConsumer<T, TC, D, HG, R>>;
  static_assert(!kMma || HG == 8, "the tensor-core consumer covers 8 query heads");
  static_assert(!kAppend || std::is_same<T, TC>::value || (kFp8 && sizeof(T) == 2),
                "the fused append writes caches of the query type, or fp8 ones");
  constexpr int NW = Cfg::kWarps;
  constexpr int S = Cfg::kStages;
  constexpr int TILE = Cfg::kTileBytes;

  const int part = blockIdx.x;
  const int kvh = blockIdx.y / a.head_chunks;
  const int chunk = blockIdx.y - kvh * a.head_chunks;
  const int seq = blockIdx.z;
  const int head0 = kvh * a.group + chunk * HG;
  const int nheads = min(HG, a.group - chunk * HG);

  // FMA consumers: this warp's first 32 block ids do not depend on the
  // context length, so load them now and the first copies wait on one memory
  // round trip, not two.  (The register-capped tensor-core consumers load
  // them after their set-up.)
  int ids_pre = 0;
  if constexpr (!kMma) {
    const int32_t* table_row = a.block_tables + (size_t)seq * a.max_blocks_per_seq;
    const int b = part * a.part_blocks + ((threadIdx.x >> 5) + (threadIdx.x & 31) * Cfg::kWarps) / kSubs;
    if (b < a.max_blocks_per_seq) ids_pre = table_row[b];
  }
  int ctx = a.context_lens[seq];
  const int ctx_cap = a.max_blocks_per_seq * kBlockTokens;
  if (ctx < 0 || ctx > ctx_cap) {
    if (threadIdx.x == 0 && part == 0 && blockIdx.y == 0) attn_error(CF_DEVERR_CONTEXT_LEN);
    ctx = ctx < 0 ? 0 : ctx_cap;
  }
  const int nblk = (ctx + kBlockTokens - 1) / kBlockTokens;
  const int nparts = nblk == 0 ? 1 : (nblk + a.part_blocks - 1) / a.part_blocks;
  if (part >= nparts) return;  // whole CTA: this sequence is shorter
  if (part == 0 && nparts > (int)gridDim.x && threadIdx.x == 0 && blockIdx.y == 0)
    attn_error(CF_DEVERR_CONTEXT_LEN);  // context_lens exceeds max_context_len
  const bool single = (nparts == 1);
  const int last_tok = (kAppend && ctx > 0) ? ctx - 1 : -1;
  const int pb0 = part * a.part_blocks;
  const int pb1 = min(nblk, pb0 + a.part_blocks);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* tiles = smem + (size_t)warp * S * 2 * TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset) + warp * S;
  int* flags = reinterpret_cast<int*>(smem + Cfg::kFlagOffset) + warp * S;
  float* pbuf = reinterpret_cast<float*>(smem + Cfg::kPbufOffset) + warp * HG * R;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  Consumer cons;
  const T* qrow = reinterpret_cast<const T*>(a.q) + ((size_t)seq * a.num_heads + head0) * D;
  // The tensor-core consumers only load Q here; the FMA consumer scales it as
  // it arrives, so it starts after the first copies are issued (below) and
  // Q's memory round trip overlaps theirs.
  if constexpr (kMma) cons.init(qrow, nheads, a.scale_log2, lane);

  // The partition's tiles (R tokens each, kSubs per block) are dealt to the
  // warps round-robin: this warp's tiles are u = warp + j*NW, j in [0, nb);
  // tile u covers block pb0 + u / kSubs, rows (u % kSubs) * R ...
  const int span = (pb1 - pb0) * kSubs;
  const int nb = span > warp ? (span - warp + NW - 1) / NW : 0;
  const int32_t* table = a.block_tables + (size_t)seq * a.max_blocks_per_seq + pb0;
  using App = AppendRow<T, TC, D>;
  if constexpr (kAppend) {
    // The warp whose tiles include the newest token's starts copying its row.
    if (last_tok >= pb0 * kBlockTokens && last_tok < pb1 * kBlockTokens &&
        (last_tok / R - pb0 * kSubs) % NW == warp) {
      // staging: App::kStageBytes past the configuration's shared memory
      App::load(a, smem + Cfg::kSmemBytes, seq, kvh, last_tok, chunk == 0, lane);
    }
  }
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.k_cache);
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.v_cache);

  auto fetch_ids = [&](int jbase) -> int {
    const int j = jbase + lane;
    return j < nb ? table[(warp + j * NW) / kSubs] : 0;
  };
  auto issue = [&](int j, int phys) {  // lane 0 only
    if (a.unarm_first_stage && j == 0) return;  // test hook: the stage never completes
    const int s = j % S;
    const uint32_t bar = smem_addr(&bars[s]);
    const int u = warp + j * NW;
    const int sub = u % kSubs;
    // a half-block tile past the context holds no tokens: nothing to load
    if (kSubs > 1 && (pb0 + u / kSubs) * kBlockTokens + sub * R >= ctx) {
      flags[s] = 0;
      mbar_arrive(bar);
      return;
    }
    if (phys < 0 || (int64_t)phys >= a.num_blocks) {
      attn_error(CF_DEVERR_BLOCK_ID);
      flags[s] = 0;
      mbar_arrive(bar);
      return;
    }
    flags[s] = 1;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, 2 * TILE);
    uint8_t* kt = tiles + (size_t)s * 2 * TILE;
    if constexpr (kMma) {
      // Boxes of 16 rows x 128 bytes (64 16-bit or 128 fp8 elements,
      // swizzled); x stays a multiple of the box width.
      constexpr int kBoxElems = 128 / (int)sizeof(TC);
      const int32_t row = (int32_t)(((int64_t)phys * a.num_kv_heads + kvh) * kBlockTokens);
#pragma unroll
      for (int b = 0; b < D / kBoxElems; ++b) {
        tma_load_2d(smem_addr(kt + b * kBlockTokens * 128), &tmk, b * kBoxElems, row, bar);
        tma_load_2d(smem_addr(kt + TILE + b * kBlockTokens * 128), &tmv, b * kBoxElems, row, bar);
      }
    } else {
      const size_t off = (((size_t)phys * a.num_kv_heads + kvh) * kBlockTokens + (size_t)sub * R) * D *
                         sizeof(TC);
      bulk_load(smem_addr(kt), kbase + off, TILE, bar);
      bulk_load(smem_addr(kt + TILE), vbase + off, TILE, bar);
    }
  };

  int ids = kMma ? fetch_ids(0) : ids_pre;  // ids_pre = fetch_ids(0) for every tile the warp uses
  const int pro = nb < S ? nb : S;
  for (int j = 0; j < pro; ++j) {
    const int phys = __shfl_sync(0xffffffffu, ids, j);
    if (lane == 0) issue(j, phys);
  }
  if constexpr (!kMma) cons.init(qrow, nheads, a.scale_log2, lane);

  // The streaming loop.  With kAppend the newest token's tile is the last
  // tile of the warp that holds it (the partition's highest tile, or the one
  // before an empty half-block tile), so the loop stops one step short and
  // that step runs peeled below, with the patch: the loop itself stays the
  // plain one (the fp8 kernels have no registers to spare in it).
  bool ok = true;
  const int nmain = kAppend ? nb - 1 : nb;
  for (int i = 0; i < nmain; ++i) {
    const int s = i % S;
    const uint32_t parity = (uint32_t)(i / S) & 1u;
    const bool ready = mbar_wait_bounded(smem_addr(&bars[s]), parity, a.wait_limit_ns);
    if (!__all_sync(0xffffffffu, ready)) {
      // A copy never completed: record it, wait (bounded) for every copy this
      // warp still has in flight so none lands after the CTA exits, and stop.
      if (lane == 0) {
        attn_error(CF_DEVERR_TIMEOUT);
        const int last = (i + S < nb ? i + S : nb);
        for (int k = i; k < last; ++k)
          mbar_wait_bounded(smem_addr(&bars[k % S]), (uint32_t)(k / S) & 1u, a.wait_limit_ns);
      }
      __syncwarp();
      ok = false;
      break;
    }
    const int u = warp + i * NW;
    const int tok0 = (pb0 + u / kSubs) * kBlockTokens + (u % kSubs) * R;  // first token of the tile
    const int ntok = min(R, ctx - tok0);
    if (flags[s]) {
      uint8_t* kt = tiles + (size_t)s * 2 * TILE;
      cons.block(kt, kt + TILE, ntok, pbuf, lane);
    }
    __syncwarp();
    const int jn = i + S;
    if (jn < nb) {
      if ((jn & 31) == 0) ids = fetch_ids(jn);
      const int phys = __shfl_sync(0xffffffffu, ids, jn & 31);
      if (lane == 0) issue(jn, phys);
    }
  }
  if constexpr (kAppend) {
    // The last step: no stage is refilled after it.
    const int i = nb - 1;
    if (ok && i >= 0) {
      const int s = i % S;
      const bool ready = mbar_wait_bounded(smem_addr(&bars[s]), (uint32_t)(i / S) & 1u, a.wait_limit_ns);
      if (!__all_sync(0xffffffffu, ready)) {
        if (lane == 0) {  // as in the loop: wait (bounded) once more for the copy in flight
          attn_error(CF_DEVERR_TIMEOUT);
          mbar_wait_bounded(smem_addr(&bars[s]), (uint32_t)(i / S) & 1u, a.wait_limit_ns);
        }
        ok = false;
      } else {
        const int u = warp + i * NW;
        const int tok0 = (pb0 + u / kSubs) * kBlockTokens + (u % kSubs) * R;
        if (flags[s]) {
          uint8_t* kt = tiles + (size_t)s * 2 * TILE;
          // whether this warp holds the newest token, recomputed here from
          // the context length so nothing extra stays live across the loop
          const int lt = ctx - 1;
          const int p1 = min((ctx + kBlockTokens - 1) / kBlockTokens, pb0 + a.part_blocks);
          if (ctx > 0 && lt >= pb0 * kBlockTokens && lt < p1 * kBlockTokens &&
              (lt / R - pb0 * kSubs) % NW == warp)
            App::template patch<kMma, TILE, R>(a, smem + Cfg::kSmemBytes, kt, kvh, lane);
          cons.block(kt, kt + TILE, min(R, ctx - tok0), pbuf, lane);
        }
      }
      __syncwarp();
    }
  }

  grid_dependency_launch();

  // Merge the warps' partial softmax states.
  __syncthreads();  // every warp is done with its stage tiles
  float* mo = reinterpret_cast<float*>(smem);
  float* mm = mo + NW * HG * D;
  float* ml = mm + NW * HG;
  cons.store(mo + warp * HG * D, mm + warp * HG, ml + warp * HG, lane);
  const int all_ok = __syncthreads_and(ok ? 1 : 0);
  if (!all_ok) {
    // a wait ran out: no output; the append's staging copies (cp.async, if
    // this thread issued any) land before the CTA leaves
    if constexpr (kAppend) cp_async_wait_all();
    return;
  }

  const size_t H = (size_t)a.num_heads;
  for (int idx = threadIdx.x; idx < nheads * D; idx += NW * 32) {
    const int h = idx / D;
    const int d = idx - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, mm[w * HG + h]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float sc = exp2f(mm[w * HG + h] - M);
        L = fmaf(ml[w * HG + h], sc, L);
        acc = fmaf(mo[(w * HG + h) * D + d], sc, acc);
      }
    }
    const float res = L > 0.f ? acc / L * a.v_scale : 0.f;
    const size_t hq = (size_t)seq * H + head0 + h;
    if (single) {
      reinterpret_cast<T*>(a.out)[hq * D + d] = from_float<T>(res);
    } else {
      const size_t pi = hq * a.num_parts + part;
      a.part_out[pi * D + d] = res;
      if (d == 0) {
        a.part_max[pi] = M * kLn2;
        a.part_sum[pi] = L;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Partition reduce: one CTA of D threads per (query head, sequence).
// out = sum_p w_p * o_p / sum_p w_p,  w_p = exp_sum_p * exp(max_p - max).
// Sequences with a single partition were written by the partition kernel.
// ---------------------------------------------------------------------------
struct ReduceArgs {
  void* out;
  const float* part_max;
  const float* part_sum;
  const float* part_out;
  const int32_t* context_lens;
  int32_t num_heads;
  int32_t max_blocks_per_seq;
  int32_t part_blocks;
  int32_t num_parts;      // scratch stride
  int32_t launched_parts; // partitions the partition kernel covered
};

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  __syncthreads();
  return r;
}

constexpr int kReduceThreads = 256;

template <typename T, int D>
__global__ void __launch_bounds__(kReduceThreads) paged_attention_reduce_kernel(const ReduceArgs r) {
  // Threads are (partition group, 4-column slice): each group walks every
  // kGroups-th partition with float4 loads (a warp reads 512 contiguous bytes
  // of one partition row), so many partition rows are in flight at once; the
  // groups' sums are added through shared memory.
  constexpr int kCols4 = D / 4;
  constexpr int kGroups = kReduceThreads / kCols4;
  grid_dependency_wait();
  const int h = blockIdx.x;
  const int seq = blockIdx.y;
  int ctx = r.context_lens[seq];
  const int cap = r.max_blocks_per_seq * kBlockTokens;
  ctx = ctx < 0 ? 0 : (ctx > cap ? cap : ctx);
  const int nblk = (ctx + kBlockTokens - 1) / kBlockTokens;
  int nparts = nblk == 0 ? 1 : (nblk + r.part_blocks - 1) / r.part_blocks;
  if (nparts <= 1) return;
  if (nparts > r.launched_parts) nparts = r.launched_parts;

  extern __shared__ float wsh[];  // nparts weights
  __shared__ float red[32];
  __shared__ float4 acc_sh[kGroups][kCols4];
  const size_t base = ((size_t)seq * r.num_heads + h) * r.num_parts;
  float lm = -INFINITY;
  for (int p = threadIdx.x; p < nparts; p += blockDim.x) lm = fmaxf(lm, r.part_max[base + p]);
  const float M = block_reduce(lm, true, red);
  float ls = 0.f;
  for (int p = threadIdx.x; p < nparts; p += blockDim.x) {
    const float w = (M == -INFINITY) ? 0.f : r.part_sum[base + p] * expf(r.part_max[base + p] - M);
    wsh[p] = w;
    ls += w;
  }
  const float L = block_reduce(ls, false, red);  // also orders the wsh writes
  const int c4 = threadIdx.x % kCols4;
  const int grp = threadIdx.x / kCols4;
  const float4* po = reinterpret_cast<const float4*>(r.part_out + base * D) + c4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int p = grp; p < nparts; p += kGroups) {
    const float4 v = po[(size_t)p * kCols4];
    const float w = wsh[p];
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  acc_sh[grp][c4] = acc;
  __syncthreads();
  if (threadIdx.x < kCols4) {
    float4 t = acc_sh[0][c4];
#pragma unroll
    for (int g = 1; g < kGroups; ++g) {
      const float4 u = acc_sh[g][c4];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    T* out = reinterpret_cast<T*>(r.out) + ((size_t)seq * r.num_heads + h) * D + c4 * 4;
    out[0] = from_float<T>(L > 0.f ? t.x / L : 0.f);
    out[1] = from_float<T>(L > 0.f ? t.y / L : 0.f);
    out[2] = from_float<T>(L > 0.f ? t.z / L : 0.f);
    out[3] = from_float<T>(L > 0.f ? t.w / L : 0.f);
  }
}

// Partition reduce for launches of at most 32 partitions (v1 splits of
// ordinary contexts): one warp per (query head, sequence), eight heads per
// CTA.  Lane p holds partition p's max and weight (one round of loads, warp
// shuffles for the max and the sum), then every lane accumulates its float4
// column slices over the partitions with the loads pipelined -- no shared
// memory, no CTA barrier.  Same merge as paged_attention_reduce_kernel:
// out = sum_p w_p o_p / sum_p w_p, w_p = exp_sum_p * exp(max_p - max).
constexpr int kReduceRowWarps = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kReduceRowWarps * 32) paged_attention_reduce_rows_kernel(const ReduceArgs r) {
  constexpr int kCols4 = D / 4;
  constexpr int kPerLane = (kCols4 + 31) / 32;
  grid_dependency_wait();
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x * kReduceRowWarps + (threadIdx.x >> 5);
  const int seq = blockIdx.y;
  if (h >= r.num_heads) return;
  int ctx = r.context_lens[seq];
  const int cap = r.max_blocks_per_seq * kBlockTokens;
  ctx = ctx < 0 ? 0 : (ctx > cap ? cap : ctx);
  const int nblk = (ctx + kBlockTokens - 1) / kBlockTokens;
  int nparts = nblk == 0 ? 1 : (nblk + r.part_blocks - 1) / r.part_blocks;
  if (nparts <= 1) return;  // written by the partition kernel
  if (nparts > r.launched_parts) nparts = r.launched_parts;
  const size_t base = ((size_t)seq * r.num_heads + h) * r.num_parts;
  const float pm = lane < nparts ? r.part_max[base + lane] : -INFINITY;
  const float ps = lane < nparts ? r.part_sum[base + lane] : 0.f;
  float M = pm;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float w = (lane < nparts && M != -INFINITY) ? ps * expf(pm - M) : 0.f;
  float L = w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  const float4* po = reinterpret_cast<const float4*>(r.part_out + base * D);
  float4 acc[kPerLane];
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int p = 0; p < nparts; ++p) {
    const float wp = __shfl_sync(0xffffffffu, w, p);
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
      const int c4 = lane + 32 * k;
      if (c4 < kCols4) {
        const float4 v = po[(size_t)p * kCols4 + c4];
        acc[k].x = fmaf(wp, v.x, acc[k].x);
        acc[k].y = fmaf(wp, v.y, acc[k].y);
        acc[k].z = fmaf(wp, v.z, acc[k].z);
        acc[k].w = fmaf(wp, v.w, acc[k].w);
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* out = reinterpret_cast<T*>(r.out) + ((size_t)seq * r.num_heads + h) * D;
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) {
    const int c4 = lane + 32 * k;
    if (c4 < kCols4) {
      out[c4 * 4 + 0] = from_float<T>(acc[k].x * inv);
      out[c4 * 4 + 1] = from_float<T>(acc[k].y * inv);
      out[c4 * 4 + 2] = from_float<T>(acc[k].z * inv);
      out[c4 * 4 + 3] = from_float<T>(acc[k].w * inv);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return (EncodeTiledFn) nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// K or V cache viewed as a 2-D tensor [rows = num_blocks*Hkv*16, D] of 16-bit
// elements, loaded in swizzled boxes of 16 rows x 64 elements (128 bytes).
bool kv_tensor_map(CUtensorMap* map, const void* base, int64_t rows, int D, int32_t dtype) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return false;
  const int eb = dtype == CF_FP8_E4M3 ? 1 : 2;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * eb};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / eb), (cuuint32_t)kBlockTokens};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType ty = dtype == CF_FP8_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dtype == CF_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, ty, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

// Per kernel instantiation and device: opt in to > 48 KB of dynamic smem.
template <typename T, typename TC, int D, int HG, bool kMma, bool kAppend>
cf_status ensure_smem(int bytes) {
  static std::once_flag flags[64];
  static cudaError_t errs[64];
  auto kern = paged_attention_kernel<T, TC, D, HG, kMma, kAppend>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  std::call_once(flags[dev], [&] {
    errs[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return cuda_status(errs[dev]);
}

struct Maps {
  CUtensorMap k, v;
};

template <typename T, typename TC, int D, int HG, bool kMma, bool kAppend>
cf_status launch_typed(const AttnLaunch& l, AttnArgs a, int grid_x, const Maps& maps) {
  using Cfg = AttnConfig<TC, D, HG>;
  const cf_paged_attention_params& p = *l.p;
  a.head_chunks = (a.group + HG - 1) / HG;
  const int smem = Cfg::kSmemAlloc + (kAppend ? AppendRow<T, TC, D>::kStageBytes : 0);
  cf_status st = ensure_smem<T, TC, D, HG, kMma, kAppend>(smem);
  if (st != CF_OK) return st;
  dim3 grid((unsigned)grid_x, (unsigned)(p.num_kv_heads * a.head_chunks), (unsigned)p.num_seqs);
  paged_attention_kernel<T, TC, D, HG, kMma, kAppend>
      <<<grid, Cfg::kWarps * 32, smem, l.stream>>>(a, maps.k, maps.v);
  st = check_launch();
  if (st != CF_OK || l.part_max == nullptr || grid_x == 1) return st;

  ReduceArgs r;
  r.out = p.output;
  r.part_max = l.part_max;
  r.part_sum = l.part_sum;
  r.part_out = l.part_out;
  r.context_lens = p.context_lens;
  r.num_heads = p.num_heads;
  r.max_blocks_per_seq = p.max_blocks_per_seq;
  r.part_blocks = a.part_blocks;
  r.num_parts = l.num_parts;
  r.launched_parts = grid_x;
  const size_t rsmem = (size_t)grid_x * sizeof(float);
  if (rsmem > 48 * 1024) return CF_ERR_UNSUPPORTED;

  cudaLaunchConfig_t cfg = {};
  cfg.stream = l.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (grid_x <= 32) {  // a warp per (head, sequence): one lane per partition
    cfg.gridDim = dim3((unsigned)((p.num_heads + kReduceRowWarps - 1) / kReduceRowWarps), (unsigned)p.num_seqs);
    cfg.blockDim = dim3(kReduceRowWarps * 32);
    return cuda_status(cudaLaunchKernelEx(&cfg, paged_attention_reduce_rows_kernel<T, D>, r));
  }
  cfg.gridDim = dim3((unsigned)p.num_heads, (unsigned)p.num_seqs);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.dynamicSmemBytes = rsmem;
  return cuda_status(cudaLaunchKernelEx(&cfg, paged_attention_reduce_kernel<T, D>, r));
}

// Which consumer runs: tensor cores for every group on fp8 caches (head_dim a
// multiple of 128) and on 16-bit caches for GQA groups of 3+ query heads or
// head_dim 128 (there the tensor-core consumer is ~1 % faster than FMA even
// for one query head per KV head: 0.345 vs 0.348 ms on 64 rows of 128-4096
// tokens, 0.360 vs 0.365 ms under the power cap), FMA otherwise.
// CF_ATTN_CONSUMER=fma|mma overrides (read per call).
bool use_mma(const cf_paged_attention_params& p, int64_t rows, bool fp8) {
  if (p.dtype == CF_F32 || p.num_blocks <= 0 || rows > INT32_MAX) return false;
  if (p.head_dim % (fp8 ? 128 : 64) != 0) return false;
  if (const char* e = std::getenv("CF_ATTN_CONSUMER")) {
    if (std::strcmp(e, "fma") == 0) return false;
    if (std::strcmp(e, "mma") == 0) return true;
  }
  // fp8 tiles cost the FMA consumer more conversion work than HBM time.
  return fp8 || p.num_heads / p.num_kv_heads >= 3 || p.head_dim == 128;
}

template <typename T, typename TC, int D, bool kAppend>
cf_status launch_dim(const AttnLaunch& l, const AttnArgs& a, int grid_x) {
  constexpr bool kFp8 = std::is_same<TC, __nv_fp8_e4m3>::value;
  const cf_paged_attention_params& p = *l.p;
  Maps maps;
  std::memset(&maps, 0, sizeof(maps));
  if constexpr (sizeof(T) == 2 && (!kFp8 || D % 128 == 0)) {
    const int32_t cdt = kFp8 ? (int32_t)CF_FP8_E4M3 : p.dtype;
    const int64_t rows = p.num_blocks * (int64_t)p.num_kv_heads * kBlockTokens;
    if (use_mma(p, rows, kFp8) && kv_tensor_map(&maps.k, p.key_cache, rows, D, cdt) &&
        kv_tensor_map(&maps.v, p.value_cache, rows, D, cdt))
      return launch_typed<T, TC, D, 8, true, kAppend>(l, a, grid_x, maps);
  }
  if (a.group == 1) return launch_typed<T, TC, D, 1, false, kAppend>(l, a, grid_x, maps);
  if (a.group == 2) return launch_typed<T, TC, D, 2, false, kAppend>(l, a, grid_x, maps);
  return launch_typed<T, TC, D, 4, false, kAppend>(l, a, grid_x, maps);
}

template <typename T, typename TC, bool kAppend>
cf_status launch_head_dim(const AttnLaunch& l, const AttnArgs& a, int grid_x) {
  if constexpr (std::is_same<TC, __nv_fp8_e4m3>::value) {
    switch (l.p->head_dim) {
      case 128: return launch_dim<T, TC, 128, kAppend>(l, a, grid_x);
      case 256: return launch_dim<T, TC, 256, kAppend>(l, a, grid_x);
      default: return CF_ERR_UNSUPPORTED;
    }
  } else {
    switch (l.p->head_dim) {
      case 64: return launch_dim<T, TC, 64, kAppend>(l, a, grid_x);
      case 128: return launch_dim<T, TC, 128, kAppend>(l, a, grid_x);
      case 256:
        if constexpr (sizeof(T) == 2) return launch_dim<T, TC, 256, kAppend>(l, a, grid_x);
        return CF_ERR_UNSUPPORTED;
      default: return CF_ERR_UNSUPPORTED;
    }
  }
}

template <typename T>
cf_status launch_type(const AttnLaunch& l, const AttnArgs& a, int grid_x) {
  if (l.cache_dtype == CF_FP8_E4M3) {
    if constexpr (sizeof(T) == 2) {
      return a.new_k != nullptr ? launch_head_dim<T, __nv_fp8_e4m3, true>(l, a, grid_x)
                                : launch_head_dim<T, __nv_fp8_e4m3, false>(l, a, grid_x);
    }
    return CF_ERR_UNSUPPORTED;
  }
  return a.new_k != nullptr ? launch_head_dim<T, T, true>(l, a, grid_x)
                            : launch_head_dim<T, T, false>(l, a, grid_x);
}

}  // namespace

bool attention_supported(int32_t head_dim, int32_t block_size, int32_t dtype) {
  if (block_size != kBlockTokens) return false;
  if (dtype == CF_F32) return head_dim == 64 || head_dim == 128;
  if (dtype == CF_F16 || dtype == CF_BF16)
    return head_dim == 64 || head_dim == 128 || head_dim == 256;
  return false;
}

bool attention_fp8_supported(int32_t head_dim, int32_t block_size, int32_t dtype) {
  return block_size == kBlockTokens && (dtype == CF_F16 || dtype == CF_BF16) &&
         (head_dim == 128 || head_dim == 256);
}

// Test hooks (cf_testing_set_pipeline_faults), read at every launch.
std::atomic<int64_t> g_test_wait_limit_ns{0};
std::atomic<int32_t> g_test_unarm_first_stage{0};

cf_status launch_paged_attention(const AttnLaunch& l) {
  const cf_paged_attention_params& p = *l.p;
  if (p.num_seqs == 0) return CF_OK;
  AttnArgs a;
  a.q = p.query;
  a.k_cache = p.key_cache;
  a.v_cache = p.value_cache;
  a.out = p.output;
  a.block_tables = p.block_tables;
  a.context_lens = p.context_lens;
  a.part_max = l.part_max;
  a.part_sum = l.part_sum;
  a.part_out = l.part_out;
  a.scale_log2 = p.scale * kLog2e * l.k_scale;
  a.v_scale = l.v_scale;
  a.k_scale = l.k_scale;
  a.num_heads = p.num_heads;
  a.num_kv_heads = p.num_kv_heads;
  a.group = p.num_heads / p.num_kv_heads;
  a.head_chunks = 1;
  a.max_blocks_per_seq = p.max_blocks_per_seq;
  a.num_blocks = p.num_blocks > 0 ? p.num_blocks : INT64_MAX;
  a.new_k = l.new_k;
  a.new_v = l.new_v;
  a.slot_mapping = l.slot_mapping;
  a.k_cache_w = const_cast<void*>(p.key_cache);
  a.v_cache_w = const_cast<void*>(p.value_cache);
  {
    const int64_t lim = g_test_wait_limit_ns.load(std::memory_order_relaxed);
    a.wait_limit_ns = lim > 0 ? (uint64_t)lim : kWaitLimitNs;
    a.unarm_first_stage = g_test_unarm_first_stage.load(std::memory_order_relaxed);
  }
  int grid_x = 1;
  if (l.part_tokens > 0 && l.part_max != nullptr) {
    a.part_blocks = l.part_tokens / kBlockTokens;
    a.num_parts = l.num_parts;
    const int need = (p.max_context_len + l.part_tokens - 1) / l.part_tokens;
    grid_x = need < 1 ? 1 : need;
    if (grid_x > l.num_parts) return CF_ERR_WORKSPACE;
  } else {
    a.part_blocks = p.max_blocks_per_seq > 0 ? p.max_blocks_per_seq : 1;
    a.num_parts = 1;
    a.part_max = a.part_sum = a.part_out = nullptr;
  }
  AttnLaunch l2 = l;
  if (a.part_max == nullptr) l2.part_max = nullptr;
  switch (p.dtype) {
    case CF_F32: return launch_type<float>(l2, a, grid_x);
    case CF_F16: return launch_type<__half>(l2, a, grid_x);
    case CF_BF16: return launch_type<__nv_bfloat16>(l2, a, grid_x);
    default: return CF_ERR_UNSUPPORTED;
  }
}

cf_status attention_read_errors(uint32_t* bits, bool clear) {
  uint32_t v = 0;
  cf_status s = cuda_status(cudaMemcpyFromSymbol(&v, g_attn_errors, sizeof(v)));
  if (s != CF_OK) return s;
  *bits |= v;
  if (clear) {
    const uint32_t zero = 0;
    s = cuda_status(cudaMemcpyToSymbol(g_attn_errors, &zero, sizeof(zero)));
  }
  return s;
}

}  // namespace cfb

// Test hook of the decode kernels' bounded waits (declared in the C ABI).
extern "C" cf_status cf_testing_set_pipeline_faults(int64_t wait_limit_ns, int32_t unarm_first_stage) {
  if (wait_limit_ns < 0 || unarm_first_stage < 0 || unarm_first_stage > 1) return CF_ERR_INVALID_ARGUMENT;
  cfb::g_test_wait_limit_ns.store(wait_limit_ns, std::memory_order_relaxed);
  cfb::g_test_unarm_first_stage.store(unarm_first_stage, std::memory_order_relaxed);
  return CF_OK;
}
