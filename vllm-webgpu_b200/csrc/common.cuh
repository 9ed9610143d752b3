// common.cuh -- shared device helpers for libggufmm (sm_100a only).
//
// GGUF block geometry follows gguf-py constants.py:4231-4245:
//   Q4_0  32 w / 18 B   Q8_0  32 w / 34 B   Q4_K 256 w / 144 B   Q6_K 256 w / 210 B
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "ggufmm.h"

namespace ggufmm {

// Programmatic dependent launch: a kernel launched with pdl_launch may start while the
// previous kernel on the stream is finishing; it must call pdl_wait() before it reads
// or overwrites anything that kernel touches. pdl_trigger() lets the next PDL kernel
// start early. Both are no-ops for a kernel launched the ordinary way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

constexpr int kQ4_0 = GGUFMM_Q4_0;
constexpr int kQ8_0 = GGUFMM_Q8_0;
constexpr int kQ4_K = GGUFMM_Q4_K;
constexpr int kQ6_K = GGUFMM_Q6_K;

template <int QT> struct QTraits;
template <> struct QTraits<kQ4_0> { static constexpr int kBlock = 32, kBytes = 18; };
template <> struct QTraits<kQ8_0> { static constexpr int kBlock = 32, kBytes = 34; };
template <> struct QTraits<kQ4_K> { static constexpr int kBlock = 256, kBytes = 144; };
template <> struct QTraits<kQ6_K> { static constexpr int kBlock = 256, kBytes = 210; };

// Device-side error word (set by bounded waits that gave up). Each
// translation unit has its own copy (no relocatable device code); the host
// reads them all through ggufmm_device_status().
static __device__ int g_device_error = 0;

// Host: read (and optionally clear) this translation unit's error word.
static inline cudaError_t tu_device_error(int* out, int clear, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear && *out) {
    static const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  return e;
}

constexpr int kErrWaitTimeout = 1;

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA) primitives. Every wait is bounded: after
// g_wait_limit polls (kWaitLimit unless lowered) the wait records kErrWaitTimeout and returns false so the
// kernel can unwind instead of hanging the GPU.
// ---------------------------------------------------------------------------
constexpr uint32_t kWaitLimit = 1u << 24;

// The poll limit in force (per translation unit, like g_device_error); the host
// lowers it with ggufmm_set_wait_limit so a test can make a wait run out quickly.
static __device__ uint32_t g_wait_limit = kWaitLimit;

static inline cudaError_t tu_set_wait_limit(uint32_t polls) {
  return cudaMemcpyToSymbol(g_wait_limit, &polls, sizeof(polls));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Returns false (and flags g_device_error) if the phase never completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case reads no limit
  const uint32_t lim = g_wait_limit;
  for (uint32_t i = 1; i < lim; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 256) __nanosleep(64);
  }
  atomicOr(&g_device_error, kErrWaitTimeout);
  return false;
}

// 1-D bulk copy global -> shared (size and both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read exactly once per call (the weight stream of a GEMV):
// evict first, so the stream does not push the small, reused activations and
// outputs out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache policy (from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// Activation loads: 16 consecutive elements of x (f32 / f16 / bf16) -> fp32.
// The caller guarantees 16-byte alignment of the first element.
// ---------------------------------------------------------------------------
template <int XT>
__device__ __forceinline__ void load_x16(const void* base, int64_t idx, float* v);

template <>
__device__ __forceinline__ void load_x16<GGUFMM_F32>(const void* base, int64_t idx, float* v) {
  const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 t = __ldg(p + i);
    v[4 * i + 0] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
}

template <>
__device__ __forceinline__ void load_x16<GGUFMM_BF16>(const void* base, int64_t idx, float* v) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + idx);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint4 t = __ldg(p + i);
    uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j + 0] = __uint_as_float(w[j] << 16);
      v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

template <>
__device__ __forceinline__ void load_x16<GGUFMM_F16>(const void* base, int64_t idx, float* v) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __half*>(base) + idx);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint4 t = __ldg(p + i);
    uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(*reinterpret_cast<__half2*>(&w[j]));
      v[8 * i + 2 * j + 0] = f.x;
      v[8 * i + 2 * j + 1] = f.y;
    }
  }
}

template <int YT>
__device__ __forceinline__ void store_y(void* base, int64_t idx, float v);
template <>
__device__ __forceinline__ void store_y<GGUFMM_F32>(void* base, int64_t idx, float v) {
  static_cast<float*>(base)[idx] = v;
}
template <>
__device__ __forceinline__ void store_y<GGUFMM_F16>(void* base, int64_t idx, float v) {
  static_cast<__half*>(base)[idx] = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void store_y<GGUFMM_BF16>(void* base, int64_t idx, float v) {
  static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void store_y_rt(void* base, int ytype, int64_t idx, float v) {
  if (ytype == GGUFMM_F32) store_y<GGUFMM_F32>(base, idx, v);
  else if (ytype == GGUFMM_F16) store_y<GGUFMM_F16>(base, idx, v);
  else store_y<GGUFMM_BF16>(base, idx, v);
}

__device__ __forceinline__ float load_y_rt(const void* base, int ytype, int64_t idx) {
  if (ytype == GGUFMM_F32) return static_cast<const float*>(base)[idx];
  if (ytype == GGUFMM_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
}

}  // namespace ggufmm
