// cf_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// element types, mbarrier / bulk-copy (TMA) wrappers written as inline PTX,
// bounded waits, and the per-translation-unit device error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cacheflow_b200.h"

namespace cfb {

// ---------------------------------------------------------------------------
// Element types.  Caches hold float, __half or __nv_bfloat16; all arithmetic
// is float32.
// ---------------------------------------------------------------------------
template <typename T>
struct ElemTraits;
template <>
struct ElemTraits<float> {
  static constexpr cf_dtype kDtype = CF_F32;
};
template <>
struct ElemTraits<__half> {
  static constexpr cf_dtype kDtype = CF_F16;
};
template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr cf_dtype kDtype = CF_BF16;
};

// Unpack one 32-bit word of packed elements into floats.
template <typename T>
__device__ __forceinline__ void unpack_word(uint32_t w, float* f);
template <>
__device__ __forceinline__ void unpack_word<float>(uint32_t w, float* f) {
  f[0] = __uint_as_float(w);
}
template <>
__device__ __forceinline__ void unpack_word<__nv_bfloat16>(uint32_t w, float* f) {
  // bf16 is the high half of an fp32: widening is a shift / mask.
  f[0] = __uint_as_float(w << 16);
  f[1] = __uint_as_float(w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void unpack_word<__half>(uint32_t w, float* f) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 v = __half22float2(h);
  f[0] = v.x;
  f[1] = v.y;
}

template <typename T>
struct PerWord {
  static constexpr int kN = 4 / sizeof(T);
};

// Load N elements (N * sizeof(T) in {4, 8, 16, 32} bytes, naturally aligned)
// from shared or global memory and widen them to float.
template <typename T, int N>
__device__ __forceinline__ void load_widen(const T* p, float* f) {
  constexpr int kBytes = N * (int)sizeof(T);
  constexpr int kPerWord = PerWord<T>::kN;
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c) {
      uint4 v = reinterpret_cast<const uint4*>(p)[c];
      unpack_word<T>(v.x, f + c * 4 * kPerWord + 0 * kPerWord);
      unpack_word<T>(v.y, f + c * 4 * kPerWord + 1 * kPerWord);
      unpack_word<T>(v.z, f + c * 4 * kPerWord + 2 * kPerWord);
      unpack_word<T>(v.w, f + c * 4 * kPerWord + 3 * kPerWord);
    }
  } else if constexpr (kBytes == 8) {
    uint2 v = *reinterpret_cast<const uint2*>(p);
    unpack_word<T>(v.x, f);
    unpack_word<T>(v.y, f + kPerWord);
  } else {
    static_assert(kBytes == 4, "unsupported vector width");
    unpack_word<T>(*reinterpret_cast<const uint32_t*>(p), f);
  }
}

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ __half from_float<__half>(float x) {
  return __float2half_rn(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// ---------------------------------------------------------------------------
// Shared-memory barriers and bulk async copies (TMA), as inline PTX.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// its later async-proxy (TMA) accesses of the same buffers.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every pipeline wait gives up after this long; the kernel then records
// CF_DEVERR_TIMEOUT and returns instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Waits for phase `parity` of barrier `bar` to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Source and destination 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 2-D tiled TMA load (tensor map), completion counted on `bar`.
// x is the innermost coordinate (elements); callers keep x * sizeof(T) a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory to be
// visible / allow the next grid to begin launching.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core tiles (m16n8k16, fp32 accumulate) and their operand
// loads from shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float (&c)[4], uint32_t a0, uint32_t a1,
                                                         uint32_t a2, uint32_t a3, uint32_t b0,
                                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float (&c)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t a2, uint32_t a3, uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Packs two floats into a 16-bit pair (x in the low half), rounding to nearest.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float x, float y) {
  __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float x, float y) {
  __half2 v = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Splits x into a 16-bit head and a 16-bit remainder: x ~= hi + lo with the
// error of the remainder's rounding only.
template <typename T>
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  hi = pack2<T>(x, y);
  float h[2];
  unpack_word<T>(hi, h);  // both halves back to float
  lo = pack2<T>(x - h[0], y - h[1]);
}

// ---------------------------------------------------------------------------
// Warp helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float shfl_xor(float v, int m) {
  return __shfl_xor_sync(0xffffffffu, v, m);
}

}  // namespace cfb
