// ref_engine_driver.cpp -- CacheFlow's own host side (Scheduler, BatchManager,
// BlockManager: src/cacheflow/scheduler/*.cpp, src/cacheflow/kv_cache/
// block_manager.cpp, compiled unchanged from the reference sources by
// oracle/Makefile) driving this library through the C++ decode step of
// include/cacheflow_b200_engine.hpp.  TEST INFRASTRUCTURE ONLY (built into
// oracle/_ref/): the GPU test steps it through ctypes, keeps a host mirror of
// the pools from the block operations and rows it reports, and compares every
// step's attention output with the oracle and the device pools with the
// mirror.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include "cacheflow/kv_cache/block_manager.h"
#include "cacheflow/scheduler/batch_manager.h"
#include "cacheflow/scheduler/scheduler.h"
#include "cacheflow_b200_engine.hpp"

#define API extern "C" __attribute__((visibility("default")))

namespace {

struct Engine {
  cacheflow::ModelConfig model;
  cacheflow::CacheConfig cache;
  cacheflow::SchedulerConfig sched_cfg;
  std::unique_ptr<cacheflow::BlockManager> blocks;
  std::unique_ptr<cacheflow::Scheduler> scheduler;
  std::unique_ptr<cacheflow::BatchManager> batcher;
  std::unique_ptr<cacheflow_b200::DecodeStep> step;
  cacheflow::SchedulerOutput out;
  cacheflow::DecodeBatch batch;
};

}  // namespace

// Returns a handle (null on failure, with *status set).
API void* eng_create(int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                     int64_t num_gpu_blocks, int64_t num_cpu_blocks, int32_t max_num_seqs,
                     int32_t max_batched_tokens, int32_t max_rows, int32_t max_blocks_per_seq, void* gpu_k,
                     void* gpu_v, void* cpu_k, void* cpu_v, int32_t* status) {
  auto e = std::make_unique<Engine>();
  e->model.n_heads = num_heads;
  e->model.n_kv_heads = num_kv_heads;
  e->model.head_dim = head_dim;
  e->cache.num_gpu_blocks = (size_t)num_gpu_blocks;
  e->cache.num_cpu_blocks = (size_t)num_cpu_blocks;
  e->sched_cfg.max_num_seqs = (size_t)max_num_seqs;
  e->sched_cfg.max_num_batched_tokens = (size_t)max_batched_tokens;
  e->sched_cfg.preemption_mode = cacheflow::PreemptionMode::SWAP;
  e->blocks = std::make_unique<cacheflow::BlockManager>(e->cache, e->model);
  e->scheduler = std::make_unique<cacheflow::Scheduler>(e->sched_cfg, e->blocks.get());
  e->batcher = std::make_unique<cacheflow::BatchManager>(e->model, e->sched_cfg);
  cacheflow_b200::StepShape sh;
  sh.num_heads = num_heads;
  sh.num_kv_heads = num_kv_heads;
  sh.head_dim = head_dim;
  sh.dtype = dtype;
  sh.num_gpu_blocks = num_gpu_blocks;
  sh.num_cpu_blocks = num_cpu_blocks;
  sh.max_rows = max_rows;
  sh.max_blocks_per_seq = max_blocks_per_seq;
  e->step = std::make_unique<cacheflow_b200::DecodeStep>(sh, gpu_k, gpu_v, cpu_k, cpu_v);
  *status = e->step->init_status();
  if (*status != CF_OK) return nullptr;
  return e.release();
}

API void eng_destroy(void* h) { delete static_cast<Engine*>(h); }

// A request whose prompt is `prompt_len` tokens, generating `max_tokens`.
API void eng_add_request(void* h, uint64_t request_id, int32_t prompt_len, int32_t max_tokens) {
  auto* e = static_cast<Engine*>(h);
  std::vector<cacheflow::TokenId> prompt((size_t)prompt_len);
  for (int32_t i = 0; i < prompt_len; ++i) prompt[(size_t)i] = i + 1;
  cacheflow::SamplingParams sp;
  sp.max_tokens = max_tokens;
  e->scheduler->add_request(std::make_unique<cacheflow::SequenceGroup>(request_id, prompt, sp));
}

API int32_t eng_has_pending(void* h) { return static_cast<Engine*>(h)->scheduler->has_pending() ? 1 : 0; }

// One scheduling step: Scheduler::schedule, the block operations through the
// decode step, BatchManager::build_batch and the staging of its rows.
// counts = [rows, swaps_out, swaps_in, copies, scheduled sequences, decode
// rows, prefill chunks, fused].  Returns the cf_status of the first failure.
API int32_t eng_schedule(void* h, void* stream, int32_t* counts) {
  auto* e = static_cast<Engine*>(h);
  e->out = e->scheduler->schedule();
  cf_status st = e->step->execute_block_ops(e->out, (cudaStream_t)stream);
  if (st != CF_OK) return st;
  e->batch = e->batcher->build_batch(e->out);
  st = e->step->stage(e->batch, (cudaStream_t)stream);
  if (st != CF_OK) return st;
  counts[0] = (int32_t)e->batch.entries.size();
  counts[1] = (int32_t)e->out.block_swaps_out.size();
  counts[2] = (int32_t)e->out.block_swaps_in.size();
  counts[3] = (int32_t)e->out.block_copies.size();
  counts[4] = (int32_t)e->out.num_seqs();
  counts[5] = e->step->decode_rows();
  counts[6] = e->step->chunks();
  counts[7] = e->step->fused() ? 1 : 0;
  return CF_OK;
}

// The staged rows: sequence ids, positions and block tables ([rows,
// max_blocks], unused entries -1).
API int32_t eng_rows(void* h, uint64_t* seq_ids, int32_t* positions, int32_t* tables, int32_t max_blocks) {
  auto* e = static_cast<Engine*>(h);
  const auto& en = e->batch.entries;
  for (size_t r = 0; r < en.size(); ++r) {
    seq_ids[r] = (uint64_t)en[r].seq_id;
    positions[r] = en[r].position;
    if (en[r].block_table.size() > (size_t)max_blocks) return CF_ERR_INVALID_ARGUMENT;
    for (int32_t b = 0; b < max_blocks; ++b)
      tables[r * (size_t)max_blocks + b] = (size_t)b < en[r].block_table.size() ? en[r].block_table[b] : -1;
  }
  return CF_OK;
}

// The step's block operations as (src, dst) pairs, in execution order lists.
API void eng_block_ops(void* h, int64_t* swaps_out, int64_t* swaps_in, int64_t* copies) {
  auto* e = static_cast<Engine*>(h);
  auto put = [](const std::vector<cacheflow::SchedulerOutput::BlockOp>& ops, int64_t* dst) {
    for (size_t i = 0; i < ops.size(); ++i) {
      dst[2 * i] = ops[i].src;
      dst[2 * i + 1] = ops[i].dst;
    }
  };
  put(e->out.block_swaps_out, swaps_out);
  put(e->out.block_swaps_in, swaps_in);
  put(e->out.block_copies, copies);
}

API int32_t eng_attend(void* h, const void* query, void* output, const void* new_key, const void* new_value,
                       void* stream) {
  return static_cast<Engine*>(h)->step->attend(query, output, new_key, new_value, (cudaStream_t)stream);
}

// BatchManager::update_after_decode with one sampled token per scheduled
// sequence, then Scheduler::free_finished_requests.
API void eng_finish_step(void* h, const int32_t* tokens, int32_t n) {
  auto* e = static_cast<Engine*>(h);
  std::vector<cacheflow::TokenId> t(tokens, tokens + n);
  e->batcher->update_after_decode(e->out, t);
  e->scheduler->free_finished_requests();
}
