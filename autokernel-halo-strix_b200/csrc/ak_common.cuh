// Shared device/host helpers for the libak_b200 kernels (sm_100a only).
//
// Every exported entry point is `extern "C"`, returns an int status (AK_OK on
// success) and records a thread-local message readable through ak_last_error().
// No C++ exception crosses the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "ak_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libak_b200 is built for sm_100a only"
#endif

namespace ak {

// ---------------------------------------------------------------------------
// Error plumbing (host)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define AK_REQUIRE(cond, code, ...)          \
  do {                                       \
    if (!(cond)) {                           \
      ::ak::set_error(__VA_ARGS__);          \
      return (code);                         \
    }                                        \
  } while (0)

#define AK_CHECK_LAUNCH(what)                                                    \
  do {                                                                           \
    cudaError_t _e = cudaGetLastError();                                         \
    if (_e != cudaSuccess) {                                                     \
      ::ak::set_error("%s: launch failed: %s", what, cudaGetErrorString(_e));    \
      return AK_ERR_LAUNCH;                                                      \
    }                                                                            \
  } while (0)

#define AK_CUDA_TRY(call, what)                                                  \
  do {                                                                           \
    cudaError_t _e = (call);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::ak::set_error("%s: %s", what, cudaGetErrorString(_e));                   \
      return AK_ERR_LAUNCH;                                                      \
    }                                                                            \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int elem_size(int dt) { return dt == AK_F32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == AK_F32 || dt == AK_BF16 || dt == AK_F16; }

// Number of SMs of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------------------------
// Element conversions (device)
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// A VEC-wide register fragment of T moved with one 16-byte (or smaller) access.
template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Frag {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ void load_frag(float (&dst)[VEC], const T* p) {
  Frag<T, VEC> f = *reinterpret_cast<const Frag<T, VEC>*>(p);
#pragma unroll
  for (int i = 0; i < VEC; ++i) dst[i] = to_f<T>(f.v[i]);
}

// Streaming (read-once) variant: bypasses L1 allocation.
template <typename T, int VEC>
__device__ __forceinline__ void load_frag_stream(float (&dst)[VEC], const T* p) {
  static_assert(sizeof(T) * VEC == 16, "stream loads are 16 bytes");
  int4 raw = __ldcs(reinterpret_cast<const int4*>(p));
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < VEC; ++i) dst[i] = to_f<T>(e[i]);
}

template <typename T, int VEC>
__device__ __forceinline__ void store_frag(T* p, const float (&src)[VEC]) {
  Frag<T, VEC> f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) f.v[i] = from_f<T>(src[i]);
  *reinterpret_cast<Frag<T, VEC>*>(p) = f;
}

// ---------------------------------------------------------------------------
// Math helpers (device)
// ---------------------------------------------------------------------------
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x on the SFU (PTX ex2.approx, flush-to-zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// log2(x) on the SFU (PTX lg2.approx).
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Dtype dispatch for host launchers: binds `T` to the element type of `dt`.
#define AK_DISPATCH_DTYPE(dt, T, ...)                         \
  switch (dt) {                                               \
    case AK_F32: { using T = float; __VA_ARGS__; } break;     \
    case AK_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } break; \
    case AK_F16: { using T = __half; __VA_ARGS__; } break;    \
    default: ::ak::set_error("unsupported dtype %d", (int)(dt)); return AK_ERR_DTYPE; \
  }

}  // namespace ak

// ---------------------------------------------------------------------------
// Bulk async copies (TMA engine, no multicast) + mbarrier, with bounded waits
// ---------------------------------------------------------------------------
namespace ak {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy completing on `bar` (bytes: multiple of 16,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Report a failed bounded wait through the caller's status word (nullable).
// The word may live in device memory or in mapped pinned host memory (the
// Python layer uses the latter, so the host reads it without a CUDA call); a
// plain store plus a system-scope fence works for both, where an atomic on
// host memory would need PCIe atomics.
__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) {
    *reinterpret_cast<volatile int*>(status) = code;
    __threadfence_system();
  }
}

// Bounded wait on phase `parity`.  Gives up after `max_spins` polls (the
// default is far above any legitimate copy latency), writes AK_ERR_TIMEOUT to
// *status and returns false so the kernel can finish instead of hanging the GPU.
constexpr uint32_t kMaxSpins = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status,
                                                  uint32_t max_spins = kMaxSpins) {
  for (uint32_t i = 0; i < max_spins; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
  }
  report_status(status, (int)AK_ERR_TIMEOUT);
  return false;
}

// ---- Programmatic dependent launch -----------------------------------------
// A small follow-up kernel (fixed-order reduction of per-CTA partials) is
// launched with programmatic stream serialization, so it is scheduled while the
// producing kernel drains.  The producer calls pdl_trigger() once its CTA has
// issued its last global store; the consumer calls pdl_wait() before reading the
// producer's output, which returns only when the whole producing grid has
// completed and its memory is visible.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace ak
