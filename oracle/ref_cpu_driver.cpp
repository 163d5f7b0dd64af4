// ref_cpu_driver.cpp -- drives CacheFlow's OWN CPU decode step
// (BatchDecodeEngine::step built without CUDA, so attention runs
// execute_attention_cpu, src/cacheflow/decode/batch_decode.cpp:190-240) on a
// synthetic batch, for the reference arm / CPU baseline of bench.py.
// Compiled together with the reference sources into oracle/_ref/ by
// oracle/Makefile.  BENCH / TEST INFRASTRUCTURE ONLY.
//
// What the reference step does per sequence: build int32 block tables,
// context lengths and slot mapping on the host (prepare_kv_cache_inputs,
// :92-131), then for every (head, token) walk the block table and take a
// 128-wide dot product of the K row with itself (:213-228), softmax the
// scores (:230-237) and discard them; V, Q and the output are never touched.
// The sampler runs over a 1-entry vocabulary here (vocab is not part of the
// KV path).  Sequences are dealt to one engine per thread, longest first.
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <memory>
#include <numeric>
#include <thread>
#include <vector>

#include "cacheflow/decode/batch_decode.h"
#include "cacheflow/kv_cache/memory_pool.h"

namespace {

struct RefCpu {
  cacheflow::ModelConfig model;
  cacheflow::CacheConfig cache;
  std::unique_ptr<cacheflow::PoolManager> pools;
  std::vector<std::unique_ptr<cacheflow::BatchDecodeEngine>> engines;
  std::vector<cacheflow::DecodeBatch> batches;
  int64_t num_blocks = 0;
};

}  // namespace

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API void* refcpu_create(int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                            int64_t num_blocks, int32_t num_threads) {
  auto* r = new RefCpu();
  r->model.n_heads = num_heads;
  r->model.n_kv_heads = num_kv_heads;
  r->model.head_dim = head_dim;
  r->model.vocab_size = 1;
  r->cache.block_size = cacheflow::KV_BLOCK_SIZE;
  r->cache.num_gpu_blocks = (size_t)num_blocks;
  r->cache.num_cpu_blocks = 0;
  r->num_blocks = num_blocks;
  // The engine addresses K at the pool base and V right after all K blocks
  // (batch_decode.cpp:123-130), so one pool block holds a K and a V block.
  const size_t block_bytes =
      2ull * num_kv_heads * cacheflow::KV_BLOCK_SIZE * head_dim * sizeof(float);
  r->pools = std::make_unique<cacheflow::PoolManager>(block_bytes, (size_t)num_blocks, 0);
  const int n = num_threads > 0 ? num_threads : 1;
  for (int i = 0; i < n; ++i)
    r->engines.emplace_back(std::make_unique<cacheflow::BatchDecodeEngine>(
        r->model, r->cache, nullptr, r->pools.get()));
  r->batches.resize((size_t)n);
  return r;
}

REF_API float* refcpu_key_cache(void* h) {
  return static_cast<float*>(static_cast<RefCpu*>(h)->pools->gpu_pool().base_ptr());
}

REF_API float* refcpu_value_cache(void* h) {
  auto* r = static_cast<RefCpu*>(h);
  return refcpu_key_cache(h) + (size_t)r->num_blocks * r->model.n_kv_heads *
                                   cacheflow::KV_BLOCK_SIZE * r->model.head_dim;
}

REF_API void refcpu_set_batch(void* h, int32_t num_seqs, const int32_t* context_lens,
                              const int32_t* block_tables, int32_t max_blocks_per_seq) {
  auto* r = static_cast<RefCpu*>(h);
  std::vector<int32_t> order((size_t)num_seqs);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int32_t a, int32_t b) { return context_lens[a] > context_lens[b]; });
  std::vector<int64_t> load(r->batches.size(), 0);
  for (auto& b : r->batches) b.clear();
  for (int32_t s : order) {
    const size_t t = (size_t)(std::min_element(load.begin(), load.end()) - load.begin());
    const int32_t ctx = context_lens[s];
    const int32_t nblk = (ctx + (int32_t)cacheflow::KV_BLOCK_SIZE - 1) /
                         (int32_t)cacheflow::KV_BLOCK_SIZE;
    std::vector<cacheflow::BlockId> table(block_tables + (size_t)s * max_blocks_per_seq,
                                          block_tables + (size_t)s * max_blocks_per_seq + nblk);
    r->batches[t].add((cacheflow::SeqId)s, 0, ctx - 1, std::move(table), false);
    load[t] += ctx;
  }
}

// Runs one decode step on every engine concurrently; returns wall seconds.
REF_API double refcpu_step(void* h) {
  auto* r = static_cast<RefCpu*>(h);
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> th;
  for (size_t i = 1; i < r->engines.size(); ++i)
    th.emplace_back([r, i] { r->engines[i]->step(r->batches[i]); });
  r->engines[0]->step(r->batches[0]);
  for (auto& t : th) t.join();
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// Runs the reference's own BatchDecodeEngine::prepare_kv_cache_inputs
// (batch_decode.cpp:92-131) on a batch whose row s is at `positions[s]` and
// owns block_ids[block_offsets[s] .. block_offsets[s+1]); copies out its
// block tables ([num_seqs, *max_blocks_out], zero-padded by the reference),
// context lengths and slot mapping.  `tables_out` has room for
// num_seqs * tables_capacity entries; returns -1 if the tables do not fit.
// Slots the reference leaves unset (position past the row's blocks) hold
// whatever its uninitialised array held: the caller masks them.
REF_API int32_t refcpu_prepare_inputs(void* h, int32_t num_seqs, const int32_t* positions,
                                      const int64_t* block_offsets, const int32_t* block_ids,
                                      int32_t tables_capacity, int32_t* tables_out,
                                      int32_t* max_blocks_out, int32_t* context_lens_out,
                                      int32_t* slot_mapping_out) {
  auto* r = static_cast<RefCpu*>(h);
  cacheflow::DecodeBatch batch;
  for (int32_t s = 0; s < num_seqs; ++s) {
    std::vector<cacheflow::BlockId> table(block_ids + block_offsets[s], block_ids + block_offsets[s + 1]);
    batch.add((cacheflow::SeqId)s, 0, positions[s], std::move(table), false);
  }
  cacheflow::DecodeContext ctx;
  r->engines[0]->prepare_kv_cache_inputs(batch, ctx);
  size_t max_blocks = 0;
  for (auto& e : batch.entries) max_blocks = std::max(max_blocks, e.block_table.size());
  *max_blocks_out = (int32_t)max_blocks;
  int32_t rc = 0;
  if ((int64_t)max_blocks > tables_capacity) {
    rc = -1;
  } else {
    for (int32_t s = 0; s < num_seqs; ++s) {
      for (size_t b = 0; b < max_blocks; ++b)
        tables_out[(size_t)s * max_blocks + b] = ctx.block_tables[(size_t)s * max_blocks + b];
      context_lens_out[s] = ctx.context_lens[s];
      slot_mapping_out[s] = ctx.slot_mapping[s];
    }
  }
  delete[] ctx.block_tables;
  delete[] ctx.context_lens;
  delete[] ctx.slot_mapping;
  return rc;
}

REF_API void refcpu_destroy(void* h) { delete static_cast<RefCpu*>(h); }
