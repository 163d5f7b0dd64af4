/*
 * cf_oracle.c -- CPU restatement of CacheFlow's KV-cache kernel path.
 *
 * TEST INFRASTRUCTURE ONLY (the oracle; see cf_oracle.h).  Nothing in the
 * product links or calls this file.
 *
 * Reference lines followed (CacheFlow, src/cacheflow/cuda/):
 *   paged_attention.cuh:25-31   operand layouts
 *   paged_attention.cu:58        kv head = h / (num_heads / num_kv_heads)
 *   paged_attention.cu:75-83     block walk over block_tables, stop at ctx
 *   paged_attention.cu:85-87     K row index ((phys*Hkv + kvh)*bs + off)*D
 *   paged_attention.cu:151-153   V row index (same)
 *   paged_attention.cu:203-205   v2 partition = tokens [p*P, min((p+1)*P, ctx))
 *   paged_attention.cu:313-329   v2 reduce (restated with correct LSE weights)
 *   kv_cache_kernels.cu:34-42    slot -> (slot / bs, slot % bs) scatter
 *   kv_cache_kernels.cu:71-83    copy_blocks pairs (src, dst) = mapping[2i], [2i+1]
 *   kv_cache_kernels.cu:111-118  swap_blocks pairs, same layout
 *   kv_cache_kernels.cu:150-164  compact moves src_ids[i] -> dst_ids[i], skip src==dst
 *   memory_utils.cu:46-57        memset_blocks
 */
#include "cf_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static double half_bits_to_double(uint16_t h) {
  const int sign = (h >> 15) & 1;
  const int exp = (h >> 10) & 0x1f;
  const int man = h & 0x3ff;
  double v;
  if (exp == 0)
    v = ldexp((double)man, -24); /* subnormal */
  else if (exp == 31)
    v = man ? NAN : INFINITY;
  else
    v = ldexp((double)(man | 0x400), exp - 25);
  return sign ? -v : v;
}

static double bf16_bits_to_double(uint16_t b) {
  uint32_t w = (uint32_t)b << 16;
  float f;
  memcpy(&f, &w, sizeof f);
  return (double)f;
}

/* OCP FP8 e4m3 ("E4M3FN"): 1 sign, 4 exponent (bias 7), 3 mantissa bits;
 * exponent 0 is subnormal (m * 2^-9), S.1111.111 is NaN, no infinities;
 * largest finite 448 = 1.75 * 2^8. */
static double e4m3_bits_to_double(uint8_t b) {
  const int e = (b >> 3) & 15, m = b & 7;
  double v;
  if (e == 15 && m == 7)
    v = NAN;
  else if (e == 0)
    v = ldexp((double)m, -9);
  else
    v = ldexp((double)(8 + m), e - 10);
  return (b & 0x80) ? -v : v;
}

/* Round a float to e4m3: nearest, ties to even; magnitudes from 448 up
 * (infinities included) saturate to 448; NaN -> 0x7f. */
uint8_t cfo_e4m3_from_float(float x) {
  const uint8_t sign = signbit(x) ? 0x80 : 0;
  if (isnan(x)) return 0x7f;
  const double a = fabs((double)x);
  if (a >= 448.0) return sign | 0x7e;
  if (a < ldexp(1.0, -6)) /* subnormal quantum 2^-9; 8 * 2^-9 is the code of 2^-6 */
    return sign | (uint8_t)rint(a * 512.0);
  int e2;
  frexp(a, &e2);
  int E = e2 - 1; /* a in [2^E, 2^(E+1)) */
  double m = rint(ldexp(a, 3 - E)); /* 8..16 */
  if (m == 16.0) {
    m = 8.0;
    ++E;
  }
  return sign | (uint8_t)(((E + 7) << 3) | ((int)m - 8));
}

double cfo_load(const void* base, int64_t index, int32_t dtype) {
  switch (dtype) {
    case 0: return (double)((const float*)base)[index];
    case 1: return half_bits_to_double(((const uint16_t*)base)[index]);
    case 3: return e4m3_bits_to_double(((const uint8_t*)base)[index]);
    default: return bf16_bits_to_double(((const uint16_t*)base)[index]);
  }
}

/* ---------------------------------------------------------------- attention */

typedef struct {
  const void* q;
  const void* k;
  const void* v;
  double* out;
  const int32_t* tables;
  const int32_t* ctx;
  double scale;
  int32_t S, H, Hkv, D, bs, mbps, dtype;
  int32_t next; /* next (seq, head) pair, taken under `mu` */
  int32_t cdtype;        /* cache element type (dtype unless the caches are fp8) */
  double kscale, vscale; /* K = kscale * stored, V = vscale * stored */
  pthread_mutex_t mu;
} attn_job;

/* Logits of query head h of sequence s over tokens [t0, t1), into `sc`. */
static void logits(const attn_job* j, int s, int h, int t0, int t1, double* sc) {
  const int kvh = h / (j->H / j->Hkv);
  const int64_t qoff = ((int64_t)s * j->H + h) * j->D;
  for (int t = t0; t < t1; ++t) {
    const int blk = t / j->bs, off = t % j->bs;
    const int64_t phys = j->tables[(int64_t)s * j->mbps + blk];
    const int64_t koff = ((phys * j->Hkv + kvh) * j->bs + off) * j->D;
    double dot = 0.0;
    for (int d = 0; d < j->D; ++d)
      dot += cfo_load(j->q, qoff + d, j->dtype) * cfo_load(j->k, koff + d, j->cdtype);
    sc[t - t0] = dot * j->kscale * j->scale;
  }
}

/* Softmax-weighted V over [t0, t1) given logits; writes o[D] and returns
 * (max, sum exp(logit - max)) through *m, *l.  Empty range: o = 0, l = 0. */
static void weighted_v(const attn_job* j, int s, int h, int t0, int t1, double* sc, double* o,
                       double* m, double* l) {
  const int kvh = h / (j->H / j->Hkv);
  double mx = -INFINITY, sum = 0.0;
  for (int d = 0; d < j->D; ++d) o[d] = 0.0;
  for (int t = t0; t < t1; ++t) mx = sc[t - t0] > mx ? sc[t - t0] : mx;
  for (int t = t0; t < t1; ++t) {
    const double w = exp(sc[t - t0] - mx);
    sum += w;
    const int blk = t / j->bs, off = t % j->bs;
    const int64_t phys = j->tables[(int64_t)s * j->mbps + blk];
    const int64_t voff = ((phys * j->Hkv + kvh) * j->bs + off) * j->D;
    for (int d = 0; d < j->D; ++d) o[d] += w * j->vscale * cfo_load(j->v, voff + d, j->cdtype);
  }
  if (sum > 0)
    for (int d = 0; d < j->D; ++d) o[d] /= sum;
  *m = mx;
  *l = sum;
}

static void* attn_worker(void* arg) {
  attn_job* j = (attn_job*)arg;
  int cap = 0;
  double* sc = NULL;
  for (;;) {
    pthread_mutex_lock(&j->mu);
    const int idx = j->next++;
    pthread_mutex_unlock(&j->mu);
    if (idx >= j->S * j->H) break;
    const int s = idx / j->H, h = idx % j->H;
    const int ctx = j->ctx[s];
    if (ctx > cap) {
      free(sc);
      cap = ctx;
      sc = (double*)malloc(sizeof(double) * (size_t)cap);
    }
    double m, l;
    logits(j, s, h, 0, ctx, sc);
    weighted_v(j, s, h, 0, ctx, sc, j->out + ((int64_t)s * j->H + h) * j->D, &m, &l);
  }
  free(sc);
  return NULL;
}

static void run_attention(attn_job* jp, int32_t num_threads);

void cfo_paged_attention(const void* query, const void* key_cache, const void* value_cache,
                         double* out, const int32_t* block_tables, const int32_t* context_lens,
                         float scale, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t block_size, int32_t max_blocks_per_seq,
                         int32_t dtype, int32_t num_threads) {
  attn_job j = {query, key_cache, value_cache, out, block_tables, context_lens, (double)scale,
                num_seqs, num_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                dtype, 0};
  j.cdtype = dtype;
  j.kscale = j.vscale = 1.0;
  run_attention(&j, num_threads);
}

/* fp8 (e4m3) caches: K = k_scale * stored, V = v_scale * stored; the query
 * (and the result's type) is `dtype`. */
void cfo_paged_attention_fp8(const void* query, const void* key_cache, const void* value_cache,
                             double* out, const int32_t* block_tables, const int32_t* context_lens,
                             float scale, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t block_size, int32_t max_blocks_per_seq,
                             int32_t dtype, float k_scale, float v_scale, int32_t num_threads) {
  attn_job j = {query, key_cache, value_cache, out, block_tables, context_lens, (double)scale,
                num_seqs, num_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                dtype, 0};
  j.cdtype = 3;
  j.kscale = (double)k_scale;
  j.vscale = (double)v_scale;
  run_attention(&j, num_threads);
}

static void run_attention(attn_job* jp, int32_t num_threads) {
  attn_job j = *jp;
  pthread_mutex_init(&j.mu, NULL);
  if (num_threads <= 1) {
    attn_worker(&j);
  } else {
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)num_threads);
    for (int i = 0; i < num_threads; ++i) pthread_create(&th[i], NULL, attn_worker, &j);
    for (int i = 0; i < num_threads; ++i) pthread_join(th[i], NULL);
    free(th);
  }
  pthread_mutex_destroy(&j.mu);
}

void cfo_paged_attention_partitions(const void* query, const void* key_cache,
                                    const void* value_cache, const int32_t* block_tables,
                                    const int32_t* context_lens, float scale, int32_t num_seqs,
                                    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t block_size, int32_t max_blocks_per_seq, int32_t dtype,
                                    int32_t partition_size, int32_t num_partitions,
                                    double* max_logits, double* exp_sums, double* tmp_out) {
  attn_job j = {query, key_cache, value_cache, NULL, block_tables, context_lens, (double)scale,
                num_seqs, num_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                dtype, 0};
  j.cdtype = dtype;
  j.kscale = j.vscale = 1.0;
  double* sc = (double*)malloc(sizeof(double) * (size_t)(partition_size > 0 ? partition_size : 1));
  for (int s = 0; s < num_seqs; ++s) {
    const int ctx = context_lens[s];
    for (int h = 0; h < num_heads; ++h) {
      for (int p = 0; p < num_partitions; ++p) {
        const int t0 = p * partition_size;
        if (t0 >= ctx) break;
        const int t1 = t0 + partition_size < ctx ? t0 + partition_size : ctx;
        const int64_t flat = ((int64_t)s * num_heads + h) * num_partitions + p;
        logits(&j, s, h, t0, t1, sc);
        weighted_v(&j, s, h, t0, t1, sc, tmp_out + flat * head_dim, &max_logits[flat],
                   &exp_sums[flat]);
      }
    }
  }
  free(sc);
}

void cfo_paged_attention_reduce(const double* max_logits, const double* exp_sums,
                                const double* tmp_out, const int32_t* context_lens,
                                int32_t num_seqs, int32_t num_heads, int32_t head_dim,
                                int32_t partition_size, int32_t num_partitions, double* out) {
  for (int s = 0; s < num_seqs; ++s) {
    const int ctx = context_lens[s];
    int parts = (ctx + partition_size - 1) / partition_size;
    if (parts > num_partitions) parts = num_partitions;
    for (int h = 0; h < num_heads; ++h) {
      const int64_t base = ((int64_t)s * num_heads + h) * num_partitions;
      double* o = out + ((int64_t)s * num_heads + h) * head_dim;
      double M = -INFINITY, L = 0.0;
      for (int p = 0; p < parts; ++p) M = max_logits[base + p] > M ? max_logits[base + p] : M;
      for (int d = 0; d < head_dim; ++d) o[d] = 0.0;
      for (int p = 0; p < parts; ++p) {
        const double w = exp_sums[base + p] * exp(max_logits[base + p] - M);
        L += w;
        for (int d = 0; d < head_dim; ++d) o[d] += w * tmp_out[(base + p) * head_dim + d];
      }
      if (L > 0)
        for (int d = 0; d < head_dim; ++d) o[d] /= L;
    }
  }
}

/* ------------------------------------------------------------- cache moves */

void cfo_reshape_and_cache(const void* key, const void* value, void* key_cache,
                           void* value_cache, const int32_t* slot_mapping, int32_t num_tokens,
                           int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                           int32_t elem_bytes) {
  const int64_t row = (int64_t)head_dim * elem_bytes;
  for (int t = 0; t < num_tokens; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue; /* padding token */
    const int64_t blk = slot / block_size, off = slot % block_size;
    for (int h = 0; h < num_kv_heads; ++h) {
      const int64_t src = ((int64_t)t * num_kv_heads + h) * row;
      const int64_t dst = ((blk * num_kv_heads + h) * block_size + off) * row;
      memcpy((char*)key_cache + dst, (const char*)key + src, (size_t)row);
      memcpy((char*)value_cache + dst, (const char*)value + src, (size_t)row);
    }
  }
}

void cfo_copy_blocks(void* key_cache, void* value_cache, const int64_t* block_mapping,
                     int32_t num_pairs, int64_t block_bytes) {
  for (int i = 0; i < num_pairs; ++i) {
    const int64_t s = block_mapping[2 * i], d = block_mapping[2 * i + 1];
    memmove((char*)key_cache + d * block_bytes, (char*)key_cache + s * block_bytes,
            (size_t)block_bytes);
    memmove((char*)value_cache + d * block_bytes, (char*)value_cache + s * block_bytes,
            (size_t)block_bytes);
  }
}

void cfo_swap_blocks(const void* src_cache, void* dst_cache, const int64_t* block_mapping,
                     int32_t num_pairs, int64_t block_bytes) {
  for (int i = 0; i < num_pairs; ++i) {
    const int64_t s = block_mapping[2 * i], d = block_mapping[2 * i + 1];
    memcpy((char*)dst_cache + d * block_bytes, (const char*)src_cache + s * block_bytes,
           (size_t)block_bytes);
  }
}

/* All sources are read before any destination is written (parallel
 * assignment), which is what the concurrent reference kernel produces for
 * every plan whose destinations are not also sources. */
void cfo_compact_kv_cache(void* key_cache, void* value_cache, const int32_t* src_ids,
                          const int32_t* dst_ids, int32_t num_moves, int64_t block_bytes) {
  void* caches[2] = {key_cache, value_cache};
  char* stage = (char*)malloc((size_t)(num_moves > 0 ? num_moves : 1) * (size_t)block_bytes);
  for (int c = 0; c < 2; ++c) {
    char* base = (char*)caches[c];
    for (int i = 0; i < num_moves; ++i)
      memcpy(stage + (int64_t)i * block_bytes, base + (int64_t)src_ids[i] * block_bytes,
             (size_t)block_bytes);
    for (int i = 0; i < num_moves; ++i) {
      if (src_ids[i] == dst_ids[i]) continue;
      memcpy(base + (int64_t)dst_ids[i] * block_bytes, stage + (int64_t)i * block_bytes,
             (size_t)block_bytes);
    }
  }
  free(stage);
}

void cfo_memset_blocks(void* cache, const int32_t* block_ids, int32_t num_listed,
                       int64_t block_bytes) {
  for (int i = 0; i < num_listed; ++i)
    memset((char*)cache + (int64_t)block_ids[i] * block_bytes, 0, (size_t)block_bytes);
}

/* batch_decode.cpp:96-99: tables zero-initialised to the widest row;
 * :103 context length = position + 1; :104-105 ids copied in order;
 * :107-114 slot = table[position / bs] * bs + position % bs when the row has
 * that block.  A negative position (never produced by the reference) is an
 * empty row here. */
int32_t cfo_build_decode_inputs(const int32_t* positions, const int64_t* block_offsets,
                                const int32_t* block_ids, int32_t num_seqs,
                                int32_t max_blocks_per_seq, int32_t block_size,
                                int32_t* block_tables, int32_t* context_lens,
                                int32_t* slot_mapping) {
  int32_t cut = 0;
  for (int32_t s = 0; s < num_seqs; ++s) {
    const int64_t n = block_offsets[s + 1] - block_offsets[s];
    const int64_t keep = n < 0 ? 0 : (n < max_blocks_per_seq ? n : max_blocks_per_seq);
    if (n < 0 || n > max_blocks_per_seq) ++cut;
    int32_t* row = block_tables + (int64_t)s * max_blocks_per_seq;
    for (int64_t b = 0; b < max_blocks_per_seq; ++b)
      row[b] = b < keep ? block_ids[block_offsets[s] + b] : 0;
    const int32_t pos = positions[s];
    slot_mapping[s] = -1;
    if (pos < 0 || pos == INT32_MAX) {
      context_lens[s] = 0;
      continue;
    }
    context_lens[s] = pos + 1;
    const int64_t bi = pos / block_size;
    if (bi < keep) {
      const int64_t v = (int64_t)row[bi] * block_size + pos % block_size;
      if (v >= 0 && v <= INT32_MAX) slot_mapping[s] = (int32_t)v;
    }
  }
  return cut;
}

/* reshape_and_cache into fp8 caches: element x of the new rows (type `dtype`)
 * is stored as e4m3(float(x) / scale), the division rounded to float. */
void cfo_reshape_and_cache_fp8(const void* key, const void* value, uint8_t* key_cache,
                               uint8_t* value_cache, const int32_t* slot_mapping,
                               int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, int32_t dtype, float k_scale, float v_scale) {
  for (int32_t t = 0; t < num_tokens; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    const int64_t blk = slot / block_size, off = slot % block_size;
    for (int32_t h = 0; h < num_kv_heads; ++h) {
      const int64_t src = ((int64_t)t * num_kv_heads + h) * head_dim;
      const int64_t dst = ((blk * num_kv_heads + h) * block_size + off) * head_dim;
      for (int32_t d = 0; d < head_dim; ++d) {
        key_cache[dst + d] = cfo_e4m3_from_float((float)cfo_load(key, src + d, dtype) / k_scale);
        value_cache[dst + d] = cfo_e4m3_from_float((float)cfo_load(value, src + d, dtype) / v_scale);
      }
    }
  }
}
