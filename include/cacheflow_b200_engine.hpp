// cacheflow_b200_engine.hpp -- the decode step of CacheFlow's C++ host side
// (BatchDecodeEngine::prepare_kv_cache_inputs + execute_attention,
// src/cacheflow/decode/batch_decode.cpp:92-188, and the block operations of a
// SchedulerOutput, src/cacheflow/scheduler/scheduler.h:22-29) over this
// library's C ABI.  Header-only C++17; it needs only cacheflow_b200.h and the
// CUDA runtime.
//
// What it corrects in the reference caller: the reference builds block
// tables, context lengths and slots in host memory with new[] every step and
// hands those host pointers, a null query and a null output to the kernels
// (batch_decode.cpp:100-102,138-141,170-176), and it never executes the
// scheduler's block_swaps_out / block_swaps_in / block_copies.  Here:
//   * stage(batch) packs the DecodeBatch's rows (tables, context lengths =
//     position + 1, slots) into a pinned staging buffer allocated once, and
//     sends it to device memory with one cudaMemcpyAsync on the caller's
//     stream;
//   * attend(query, output, new_key, new_value) appends every row's new
//     token to the cache and runs attention on the caller's device buffers:
//       - one row per sequence (a decode batch): the fused append + v1 launch
//         (cf_paged_attention_append_v1) with the context split over CTAs;
//       - decode rows followed by prefill chunks (BatchManager's order: a
//         prefill group's prompt tokens are consecutive entries with
//         positions 0..n-1, batch_manager.cpp:27-36): cf_reshape_and_cache,
//         v1 for the decode rows, cf_paged_prefill_attention for the chunks;
//       - anything else: cf_reshape_and_cache, then v1 over every row (one
//         query per entry, the reference's own semantics);
//   * execute_block_ops(scheduler_output) runs the step's swap-outs,
//     swap-ins and copies (cf_execute_block_ops) before the attention that
//     reads the moved blocks.
//
// Batch and SchedulerOutput are template parameters, used by the shape of
// CacheFlow's types only: batch.entries[i].{seq_id, position, block_table}
// and output.{block_swaps_out, block_swaps_in, block_copies}[i].{src, dst}.
// CacheFlow's own headers are therefore not needed to compile this file, and
// any host with the same fields can use it.
//
// Typical use inside CacheFlow (the scheduler loop of the engine):
//   cacheflow_b200::DecodeStep step(shape, k_cache, v_cache, cpu_k, cpu_v);
//   ...
//   SchedulerOutput so = scheduler.schedule();
//   step.execute_block_ops(so, stream);
//   DecodeBatch batch = batch_manager.build_batch(so);
//   step.stage(batch, stream);
//   step.attend(q_dev, out_dev, k_new_dev, v_new_dev, stream);
#pragma once

#include <cuda_runtime_api.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <unordered_set>
#include <vector>

#include "cacheflow_b200.h"

namespace cacheflow_b200 {

// Sizes of the step: the model's attention shape, the pools, and the largest
// batch that will be staged.
struct StepShape {
  int32_t num_heads = 0;
  int32_t num_kv_heads = 0;
  int32_t head_dim = 0;
  int32_t dtype = CF_BF16;  // cf_dtype of queries, outputs, new K/V rows and caches
  int32_t block_size = 16;
  int64_t num_gpu_blocks = 0;
  int64_t num_cpu_blocks = 0;      // 0: no CPU pool (no swaps)
  int32_t max_rows = 0;            // most batch entries one step holds
  int32_t max_blocks_per_seq = 0;  // longest block table
};

class DecodeStep {
 public:
  // Allocates the device and pinned staging buffers and the split-attention
  // workspace once; check init_status().
  DecodeStep(const StepShape& shape, void* gpu_key_cache, void* gpu_value_cache,
             void* cpu_key_cache = nullptr, void* cpu_value_cache = nullptr)
      : sh_(shape), k_(gpu_key_cache), v_(gpu_value_cache), ck_(cpu_key_cache), cv_(cpu_value_cache) {
    if (sh_.num_heads <= 0 || sh_.num_kv_heads <= 0 || sh_.head_dim <= 0 || sh_.max_rows <= 0 ||
        sh_.max_blocks_per_seq <= 0 || sh_.block_size <= 0 || sh_.num_gpu_blocks <= 0 || !k_ || !v_) {
      init_ = CF_ERR_INVALID_ARGUMENT;
      return;
    }
    elem_ = sh_.dtype == CF_F32 ? 4 : (sh_.dtype == CF_F16 || sh_.dtype == CF_BF16) ? 2 : 0;
    if (elem_ == 0) {
      init_ = CF_ERR_INVALID_ARGUMENT;
      return;
    }
    words_ = 2 * (size_t)sh_.max_rows * sh_.max_blocks_per_seq + 4 * (size_t)sh_.max_rows + 1;
    if (cudaMalloc(&dev_, words_ * 4) != cudaSuccess ||
        cudaMallocHost(&host_[0], words_ * 4) != cudaSuccess ||
        cudaMallocHost(&host_[1], words_ * 4) != cudaSuccess ||
        cudaEventCreateWithFlags(&copied_[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&copied_[1], cudaEventDisableTiming) != cudaSuccess) {
      (void)cudaGetLastError();
      init_ = CF_ERR_CUDA;
      return;
    }
    cf_paged_attention_params p = params(nullptr, nullptr, sh_.max_rows, sh_.max_blocks_per_seq,
                                         sh_.max_blocks_per_seq * sh_.block_size, nullptr, nullptr);
    ws_bytes_ = cf_paged_attention_v1_workspace_size(&p);
    if (ws_bytes_ > 0 && cudaMalloc(&ws_, ws_bytes_) != cudaSuccess) {
      (void)cudaGetLastError();
      init_ = CF_ERR_CUDA;
      return;
    }
    init_ = CF_OK;
  }

  ~DecodeStep() {
    if (copied_[0]) cudaEventSynchronize(copied_[0]);
    if (copied_[1]) cudaEventSynchronize(copied_[1]);
    if (ws_) cudaFree(ws_);
    if (dev_) cudaFree(dev_);
    if (host_[0]) cudaFreeHost(host_[0]);
    if (host_[1]) cudaFreeHost(host_[1]);
    if (copied_[0]) cudaEventDestroy(copied_[0]);
    if (copied_[1]) cudaEventDestroy(copied_[1]);
  }
  DecodeStep(const DecodeStep&) = delete;
  DecodeStep& operator=(const DecodeStep&) = delete;

  cf_status init_status() const { return init_; }

  // Packs the batch's rows and sends them to the device on `stream` (stage
  // and attend of consecutive steps on one stream: the device copy of the
  // rows is reused).  A row's context is position + 1 and its slot the one
  // its block table gives that position.  Returns CF_ERR_INVALID_ARGUMENT,
  // staging nothing, if the batch exceeds the shape or a row's table does not
  // cover its position.
  template <class Batch>
  cf_status stage(const Batch& batch, cudaStream_t stream) {
    if (init_ != CF_OK) return init_;
    const auto& e = batch.entries;
    const size_t n = e.size();
    if (n > (size_t)sh_.max_rows) return CF_ERR_INVALID_ARGUMENT;
    int32_t mb = 1, mctx = 0;
    std::unordered_set<uint64_t> seqs;
    bool distinct = true;
    for (size_t i = 0; i < n; ++i) {
      // a row's table must cover its position (the scheduler allocates the
      // blocks before the step, scheduler.cpp:143-152,177-184)
      if (e[i].position < 0 || (size_t)e[i].position >= e[i].block_table.size() * (size_t)sh_.block_size)
        return CF_ERR_INVALID_ARGUMENT;
      if (e[i].block_table.size() > (size_t)sh_.max_blocks_per_seq) return CF_ERR_INVALID_ARGUMENT;
      mb = e[i].block_table.size() > (size_t)mb ? (int32_t)e[i].block_table.size() : mb;
      mctx = e[i].position + 1 > mctx ? e[i].position + 1 : mctx;
      distinct = distinct && seqs.insert((uint64_t)e[i].seq_id).second;
    }
    // Prefill chunks: maximal runs of one sequence's consecutive positions
    // 0..len-1 (len >= 2) after every single decode row.
    max_q_ = 0;
    std::vector<int32_t> starts;  // first entry of each chunk
    size_t i = 0, first_chunk = n;
    bool chunked = !distinct && prefill_supported();
    while (chunked && i < n) {
      size_t j = i + 1;
      while (j < n && e[j].seq_id == e[i].seq_id && e[j].position == e[j - 1].position + 1) ++j;
      const bool is_chunk = j - i >= 2 && e[i].position == 0;
      if (is_chunk) {
        if (first_chunk == n) first_chunk = i;
        starts.push_back((int32_t)i);
      } else if (first_chunk != n || j - i != 1) {
        chunked = false;  // a decode row after a chunk, or a run that is no chunk
      }
      i = j;
    }
    if (starts.empty()) chunked = false;

    // Wait until this staging slot's previous copy has left it.
    const int slot = (int)(n_staged_++ & 1);
    if (cudaEventSynchronize(copied_[slot]) != cudaSuccess) return CF_ERR_CUDA;
    int32_t* h = static_cast<int32_t*>(host_[slot]);
    int32_t* tables = h;
    int32_t* ctx = tables + n * mb;
    int32_t* slots = ctx + n;
    const size_t nc = chunked ? starts.size() : 0;
    int32_t* c_tables = slots + n;
    int32_t* c_ctx = c_tables + nc * mb;
    int32_t* c_start = c_ctx + nc;
    const size_t used = (size_t)(c_start - h) + (nc ? nc + 1 : 0);
    std::memset(tables, 0, n * mb * sizeof(int32_t));
    for (size_t r = 0; r < n; ++r) {
      const auto& bt = e[r].block_table;
      for (size_t b = 0; b < bt.size(); ++b) tables[r * mb + b] = (int32_t)bt[b];
      const int32_t pos = e[r].position;
      ctx[r] = pos + 1;
      slots[r] = (int32_t)bt[(size_t)(pos / sh_.block_size)] * sh_.block_size + pos % sh_.block_size;
    }
    if (nc) {
      std::memset(c_tables, 0, nc * mb * sizeof(int32_t));
      for (size_t c = 0; c < nc; ++c) {
        const size_t s0 = (size_t)starts[c], s1 = c + 1 < nc ? (size_t)starts[c + 1] : n;
        std::memcpy(c_tables + c * mb, tables + s0 * mb, mb * sizeof(int32_t));
        c_ctx[c] = ctx[s1 - 1];
        c_start[c] = (int32_t)(s0 - first_chunk);
        max_q_ = (int32_t)(s1 - s0) > max_q_ ? (int32_t)(s1 - s0) : max_q_;
      }
      c_start[nc] = (int32_t)(n - first_chunk);
    }
    if (cudaMemcpyAsync(dev_, h, used * sizeof(int32_t), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaEventRecord(copied_[slot], stream) != cudaSuccess) {
      (void)cudaGetLastError();
      return CF_ERR_CUDA;
    }
    int32_t* d = static_cast<int32_t*>(dev_);
    d_tables_ = d;
    d_ctx_ = d + n * mb;
    d_slots_ = d_ctx_ + n;
    d_c_tables_ = d_slots_ + n;
    d_c_ctx_ = d_c_tables_ + nc * mb;
    d_c_start_ = d_c_ctx_ + nc;
    rows_ = (int32_t)n;
    stride_ = mb;
    max_ctx_ = mctx;
    fused_ = distinct;
    chunks_ = (int32_t)nc;
    decode_rows_ = chunked ? (int32_t)first_chunk : (int32_t)n;
    return CF_OK;
  }

  // Appends each staged row's new token (new_key / new_value [rows,
  // num_kv_heads, head_dim], device; both null if the cache already holds
  // them) and computes attention of query [rows, num_heads, head_dim] into
  // output (device), in the staged rows' order, on `stream`.
  cf_status attend(const void* query, void* output, const void* new_key, const void* new_value,
                   cudaStream_t stream) {
    if (init_ != CF_OK) return init_;
    if (rows_ == 0) return CF_OK;
    if (!query || !output || (new_key == nullptr) != (new_value == nullptr)) return CF_ERR_INVALID_ARGUMENT;
    if (fused_ && new_key) {
      cf_paged_attention_params p = params(query, output, rows_, stride_, max_ctx_, d_tables_, d_ctx_);
      return cf_paged_attention_append_v1(&p, new_key, new_value, d_slots_, ws_, ws_bytes_, stream);
    }
    if (new_key) {
      const cf_status st = cf_reshape_and_cache(new_key, new_value, k_, v_, d_slots_, rows_, sh_.num_kv_heads,
                                                sh_.head_dim, sh_.block_size, sh_.num_gpu_blocks, sh_.dtype,
                                                stream);
      if (st != CF_OK) return st;
    }
    if (decode_rows_ > 0) {
      int32_t mctx = max_ctx_;
      if (chunks_ > 0) {  // only the decode rows: their own longest context
        mctx = 0;
        for (int32_t r = 0; r < decode_rows_; ++r) mctx = host_ctx(r) > mctx ? host_ctx(r) : mctx;
      }
      cf_paged_attention_params p = params(query, output, decode_rows_, stride_, mctx, d_tables_, d_ctx_);
      const cf_status st = cf_paged_attention_v1(&p, ws_, ws_bytes_, stream);
      if (st != CF_OK) return st;
    }
    if (chunks_ > 0) {
      const size_t off = (size_t)decode_rows_ * sh_.num_heads * sh_.head_dim * elem_;
      cf_prefill_params p{};
      p.query = static_cast<const char*>(query) + off;
      p.key_cache = k_;
      p.value_cache = v_;
      p.output = static_cast<char*>(output) + off;
      p.block_tables = d_c_tables_;
      p.context_lens = d_c_ctx_;
      p.query_start = d_c_start_;
      p.scale = 1.0f / std::sqrt((float)sh_.head_dim);
      p.num_chunks = chunks_;
      p.num_heads = sh_.num_heads;
      p.num_kv_heads = sh_.num_kv_heads;
      p.head_dim = sh_.head_dim;
      p.block_size = sh_.block_size;
      p.max_query_len = max_q_;
      p.max_blocks_per_seq = stride_;
      p.num_blocks = sh_.num_gpu_blocks;
      p.dtype = sh_.dtype;
      const cf_status st = cf_paged_prefill_attention(&p, stream);
      if (st != CF_ERR_UNSUPPORTED) return st;
      // a GQA group the multi-query kernel does not take: the chunks' rows
      // one query each, like the decode rows
      cf_paged_attention_params q = params(static_cast<const char*>(query) + off,
                                           static_cast<char*>(output) + off, rows_ - decode_rows_, stride_,
                                           max_ctx_, d_tables_ + (size_t)decode_rows_ * stride_,
                                           d_ctx_ + decode_rows_);
      return cf_paged_attention_v1(&q, ws_, ws_bytes_, stream);
    }
    return CF_OK;
  }

  // Runs the scheduler's block operations of this step on `stream`:
  // swap-outs (GPU block -> CPU block), swap-ins (CPU -> GPU), then copies
  // (GPU -> GPU), K and V alike.
  template <class SchedulerOutput>
  cf_status execute_block_ops(const SchedulerOutput& so, cudaStream_t stream) {
    if (init_ != CF_OK) return init_;
    auto pairs = [](const auto& ops, std::vector<int64_t>& out) {
      out.clear();
      out.reserve(ops.size() * 2);
      for (const auto& op : ops) {
        out.push_back((int64_t)op.src);
        out.push_back((int64_t)op.dst);
      }
    };
    pairs(so.block_swaps_out, out_);
    pairs(so.block_swaps_in, in_);
    pairs(so.block_copies, cp_);
    const int64_t block_bytes = (int64_t)sh_.num_kv_heads * sh_.block_size * sh_.head_dim * elem_;
    return cf_execute_block_ops(k_, v_, ck_, cv_, block_bytes, sh_.num_gpu_blocks, sh_.num_cpu_blocks,
                                out_.data(), (int32_t)(out_.size() / 2), in_.data(), (int32_t)(in_.size() / 2),
                                cp_.data(), (int32_t)(cp_.size() / 2), stream);
  }

  // What the last stage() planned.
  int32_t rows() const { return rows_; }
  int32_t decode_rows() const { return decode_rows_; }
  int32_t chunks() const { return chunks_; }
  bool fused() const { return fused_; }
  int32_t max_context_len() const { return max_ctx_; }
  // Device copies of the staged rows (valid until the next stage()).
  const int32_t* device_block_tables() const { return d_tables_; }
  const int32_t* device_context_lens() const { return d_ctx_; }
  const int32_t* device_slot_mapping() const { return d_slots_; }
  int32_t block_table_stride() const { return stride_; }

 private:
  bool prefill_supported() const {
    return (sh_.dtype == CF_F16 || sh_.dtype == CF_BF16) && (sh_.head_dim == 64 || sh_.head_dim == 128);
  }
  int32_t host_ctx(int32_t r) const {
    const int slot = (int)((n_staged_ - 1) & 1);
    return static_cast<const int32_t*>(host_[slot])[(size_t)rows_ * stride_ + r];
  }
  cf_paged_attention_params params(const void* q, void* o, int32_t rows, int32_t stride, int32_t mctx,
                                   const int32_t* tables, const int32_t* ctx) const {
    cf_paged_attention_params p{};
    p.query = q;
    p.key_cache = k_;
    p.value_cache = v_;
    p.output = o;
    p.block_tables = tables;
    p.context_lens = ctx;
    p.scale = 1.0f / std::sqrt((float)sh_.head_dim);
    p.num_seqs = rows;
    p.num_heads = sh_.num_heads;
    p.num_kv_heads = sh_.num_kv_heads;
    p.head_dim = sh_.head_dim;
    p.block_size = sh_.block_size;
    p.max_context_len = mctx;
    p.max_blocks_per_seq = stride;
    p.num_blocks = sh_.num_gpu_blocks;
    p.dtype = sh_.dtype;
    return p;
  }

  StepShape sh_;
  void* k_;
  void* v_;
  void* ck_;
  void* cv_;
  int elem_ = 0;
  cf_status init_ = CF_ERR_INVALID_ARGUMENT;
  size_t words_ = 0;
  void* dev_ = nullptr;
  void* host_[2] = {nullptr, nullptr};
  cudaEvent_t copied_[2] = {nullptr, nullptr};
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  uint64_t n_staged_ = 0;
  int32_t* d_tables_ = nullptr;
  int32_t* d_ctx_ = nullptr;
  int32_t* d_slots_ = nullptr;
  int32_t* d_c_tables_ = nullptr;
  int32_t* d_c_ctx_ = nullptr;
  int32_t* d_c_start_ = nullptr;
  int32_t rows_ = 0, stride_ = 1, max_ctx_ = 0, chunks_ = 0, decode_rows_ = 0, max_q_ = 0;
  bool fused_ = false;
  std::vector<int64_t> out_, in_, cp_;
};

}  // namespace cacheflow_b200
