// static_scratch.cu -- paged attention v2 for callers that cannot allocate
// device memory.
//
// Some hosts hand every byte of GPU memory to their own pool before serving
// starts (CacheFlow's MemoryPool carves the whole KV budget into blocks up
// front), some run the decode step on a latency-critical thread where a
// cudaMalloc/cudaFree would stall on an implicit device synchronisation, and
// some foreign-function hosts only ever receive raw device pointers and have
// no allocator to call at all.  None of them can provide the per-partition
// scratch that cf_paged_attention_v2 takes as arguments.  This entry point
// keeps that scratch in a fixed array compiled into the library instead.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds CF_STATIC_SCRATCH_BYTES of it until the process exits.  In
// host code its name is only a stand-in for the device object, so the host
// asks the runtime for its device address (once per device, with that device
// current) and passes that address down as ordinary pointers.
#include <mutex>

#include "../../include/cacheflow_b200.h"
#include "cf_internal.h"

namespace {

constexpr size_t kScratchBytes = CF_STATIC_SCRATCH_BYTES;
constexpr int kPartitionTokens = 512;  // the partition size of cf_paged_attention_v2
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_v2_scratch[kScratchBytes];

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

// Device address of g_v2_scratch on the current device.  Only a successful
// lookup is kept: a failed one (for instance out of memory, because with lazy
// module loading the array is only placed in device memory at this first
// lookup, or a lookup attempted during stream capture) clears the runtime's
// error and is tried again on the next call.  Returns CF_OK and sets *ptr,
// or the status of the failed lookup.
cf_status scratch_address(void** ptr) {
  static std::mutex mu;
  static void* addr[kMaxDevices];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cfb::cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return CF_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_v2_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // not sticky: leave no error behind for the caller's next call
      return cfb::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    }
    addr[dev] = p;
  }
  *ptr = addr[dev];
  return CF_OK;
}

}  // namespace

extern "C" cf_status cf_paged_attention_v2_static_scratch(const cf_paged_attention_params* p,
                                                          void* stream) {
  if (p == nullptr || p->num_seqs < 0 || p->num_heads <= 0 || p->head_dim <= 0 ||
      p->max_context_len < 0)
    return CF_ERR_INVALID_ARGUMENT;
  // The shape limits of cf_paged_attention_v2 come first, so the size
  // arithmetic below works on bounded values only.
  if (!cfb::attention_supported(p->head_dim, p->block_size, p->dtype)) return CF_ERR_UNSUPPORTED;
  if (p->num_seqs > 65535 || p->num_heads > 65535) return CF_ERR_UNSUPPORTED;
  const int64_t parts = p->max_context_len > 0
                            ? ((int64_t)p->max_context_len + kPartitionTokens - 1) / kPartitionTokens
                            : 1;
  // rows < 2^16 * 2^16 * 2^22 = 2^54: no overflow in int64
  const int64_t rows = (int64_t)p->num_seqs * p->num_heads * parts;
  const int64_t per_row = (int64_t)sizeof(float) * (p->head_dim + 2);
  if (rows > (int64_t)(kScratchBytes / per_row)) return CF_ERR_WORKSPACE;  // larger than the static area
  const size_t stat_bytes = round256((size_t)rows * sizeof(float));
  const size_t need = 2 * stat_bytes + (size_t)rows * p->head_dim * sizeof(float);
  if (need > kScratchBytes) return CF_ERR_WORKSPACE;

  void* base = nullptr;
  cf_status st = scratch_address(&base);
  if (st != CF_OK) return st;
  unsigned char* b = static_cast<unsigned char*>(base);
  float* max_logits = reinterpret_cast<float*>(b);
  float* exp_sums = reinterpret_cast<float*>(b + stat_bytes);
  float* tmp_output = reinterpret_cast<float*>(b + 2 * stat_bytes);
  // The partition kernel writes every scratch entry the reduce kernel reads,
  // so nothing here has to start at zero.
  return cf_paged_attention_v2(p, exp_sums, max_logits, tmp_output, (int32_t)parts, stream);
}
