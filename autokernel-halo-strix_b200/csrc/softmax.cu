// Row softmax forward / backward over the last dimension, sm_100a.
//
// Forward semantics: reference.softmax_ref (reference.py:15-17), i.e.
// F.softmax(x, -1); the reference HIP kernel is kernels/hip/softmax.py:66-267.
// Backward: autograd of the same, dx = y * (dy - sum(dy*y)).
//
// Design: one warp per row with the whole row in registers (16-byte vector
// loads, one HBM read and one write in forward; two reads and one write in
// backward), fp32 max/sum with warp shuffles, exp on the SFU via ex2.approx of
// a pre-scaled argument.  Rows are grid-strided, so any row count is covered
// (the reference launcher clamps its grid to 65535 rows, softmax.py:293).
// Rows too wide for registers, or unaligned, take a CTA-per-row kernel that
// re-reads the row from L2.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kWarps = 4;

template <typename T, int VEC, int NIT, bool FULL = false>
__global__ void __launch_bounds__(kWarps * 32)
softmax_fwd_warp(T* __restrict__ y, const T* __restrict__ x, int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const T* xr = x + row * cols;
    float v[NIT][VEC];
    float m = -INFINITY;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < cols) {
        load_frag_stream<T, VEC>(v[it], xr + c);
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[it][k] = -INFINITY;
      }
#pragma unroll
      for (int k = 0; k < VEC; ++k) m = fmaxf(m, v[it][k]);
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int it = 0; it < NIT; ++it)
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        v[it][k] = ex2((v[it][k] - m) * kLog2e);
        s += v[it][k];
      }
    s = warp_sum(s);
    const float inv = 1.f / s;
    T* yr = y + row * cols;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < cols) {
        float o[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) o[k] = v[it][k] * inv;
        store_frag<T, VEC>(yr + c, o);
      }
    }
  }
}

// Two passes over the row: the first reduces sum(dy*y), the second re-reads
// y and dy (L1/L2 hits, the row was just read) and writes dx.  Keeping no row
// in registers leaves room for many resident warps, which is what a pure
// streaming kernel needs to cover HBM latency.
// FULL: cols == NIT * 32 * VEC, every lane's vectors are in range and the
// loads carry no guard (issued back to back).
template <typename T, int VEC, int NIT, bool FULL = false>
__global__ void __launch_bounds__(kWarps * 32)
softmax_bwd_warp(T* __restrict__ dx, const T* __restrict__ y, const T* __restrict__ dy,
                 int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const T* yr = y + row * cols;
    const T* gr = dy + row * cols;
    float s = 0.f;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < cols) {
        float yv[VEC], gv[VEC];
        load_frag<T, VEC>(yv, yr + c);
        load_frag<T, VEC>(gv, gr + c);
#pragma unroll
        for (int k = 0; k < VEC; ++k) s = fmaf(yv[k], gv[k], s);
      }
    }
    s = warp_sum(s);
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < cols) {
        float yv[VEC], gv[VEC], o[VEC];
        load_frag<T, VEC>(yv, yr + c);
        load_frag<T, VEC>(gv, gr + c);
#pragma unroll
        for (int k = 0; k < VEC; ++k) o[k] = yv[k] * (gv[k] - s);
        store_frag<T, VEC>(dx + row * cols + c, o);
      }
    }
  }
}

// ---- CTA-per-row fallbacks (wide or unaligned rows) -------------------------
__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  v = is_max ? warp_max(v) : warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = is_max ? -INFINITY : 0.f;
  for (int i = 0; i < nw; ++i) t = is_max ? fmaxf(t, red[i]) : t + red[i];
  return t;
}

template <typename T>
__global__ void __launch_bounds__(512)
softmax_fwd_block(T* __restrict__ y, const T* __restrict__ x, int64_t rows, int cols) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * cols;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, to_f<T>(xr[c]));
    m = block_reduce(m, red, true);
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s += ex2((to_f<T>(xr[c]) - m) * kLog2e);
    s = block_reduce(s, red, false);
    const float inv = 1.f / s;
    for (int c = threadIdx.x; c < cols; c += blockDim.x)
      y[row * cols + c] = from_f<T>(ex2((to_f<T>(xr[c]) - m) * kLog2e) * inv);
  }
}

template <typename T>
__global__ void __launch_bounds__(512)
softmax_bwd_block(T* __restrict__ dx, const T* __restrict__ y, const T* __restrict__ dy,
                  int64_t rows, int cols) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x)
      s = fmaf(to_f<T>(y[row * cols + c]), to_f<T>(dy[row * cols + c]), s);
    s = block_reduce(s, red, false);
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float yv = to_f<T>(y[row * cols + c]);
      dx[row * cols + c] = from_f<T>(yv * (to_f<T>(dy[row * cols + c]) - s));
    }
  }
}

int pick_nit(int cols, int vec) {
  const int need = (cols + 32 * vec - 1) / (32 * vec);
  const int opts[] = {1, 2, 4, 8, 16};
  for (int o : opts)
    if (o >= need) return o;
  return 0;
}

#define AK_SMX_NIT_SWITCH(nit, NIT, ...)                       \
  switch (nit) {                                               \
    case 1: { constexpr int NIT = 1; __VA_ARGS__; } break;     \
    case 2: { constexpr int NIT = 2; __VA_ARGS__; } break;     \
    case 4: { constexpr int NIT = 4; __VA_ARGS__; } break;     \
    case 8: { constexpr int NIT = 8; __VA_ARGS__; } break;     \
    case 16: { constexpr int NIT = 16; __VA_ARGS__; } break;   \
    default: break;                                            \
  }

unsigned warp_grid(int64_t rows) {
  int64_t g = (rows + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)sm_count() * 32;  // several waves of 4-warp CTAs
  return (unsigned)(g < cap ? (g < 1 ? 1 : g) : cap);
}

template <typename T>
int fwd_impl(void* y, const void* x, int64_t rows, int cols, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const int nit = (cols % VEC == 0 && aligned16(x) && aligned16(y)) ? pick_nit(cols, VEC) : 0;
  if (nit > 0) {
    if (cols == nit * 32 * VEC) {
      AK_SMX_NIT_SWITCH(nit, NIT, softmax_fwd_warp<T, VEC, NIT, true><<<warp_grid(rows), kWarps * 32, 0, st>>>(
                                      (T*)y, (const T*)x, rows, cols));
    } else {
      AK_SMX_NIT_SWITCH(nit, NIT, softmax_fwd_warp<T, VEC, NIT><<<warp_grid(rows), kWarps * 32, 0, st>>>(
                                      (T*)y, (const T*)x, rows, cols));
    }
  } else {
    const int64_t cap = (int64_t)sm_count() * 4;
    softmax_fwd_block<T><<<(unsigned)(rows < cap ? rows : cap), 512, 0, st>>>((T*)y, (const T*)x, rows, cols);
  }
  AK_CHECK_LAUNCH("ak_softmax_fwd");
  return AK_OK;
}

template <typename T>
int bwd_impl(void* dx, const void* y, const void* dy, int64_t rows, int cols, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  int nit = (cols % VEC == 0 && aligned16(dx) && aligned16(y) && aligned16(dy)) ? pick_nit(cols, VEC) : 0;
  if (nit > 0) {
    if (cols == nit * 32 * VEC) {
      AK_SMX_NIT_SWITCH(nit, NIT, softmax_bwd_warp<T, VEC, NIT, true><<<warp_grid(rows), kWarps * 32, 0, st>>>(
                                      (T*)dx, (const T*)y, (const T*)dy, rows, cols));
    } else {
      AK_SMX_NIT_SWITCH(nit, NIT, softmax_bwd_warp<T, VEC, NIT><<<warp_grid(rows), kWarps * 32, 0, st>>>(
                                      (T*)dx, (const T*)y, (const T*)dy, rows, cols));
    }
  } else {
    const int64_t cap = (int64_t)sm_count() * 4;
    softmax_bwd_block<T><<<(unsigned)(rows < cap ? rows : cap), 512, 0, st>>>((T*)dx, (const T*)y,
                                                                              (const T*)dy, rows, cols);
  }
  AK_CHECK_LAUNCH("ak_softmax_bwd");
  return AK_OK;
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_softmax_fwd(void* y, const void* x, int64_t rows, int64_t cols, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(rows >= 0 && cols > 0 && cols <= (1LL << 30), AK_ERR_SHAPE, "ak_softmax_fwd: bad shape");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(y && x, AK_ERR_ARG, "ak_softmax_fwd: null pointer");
  AK_DISPATCH_DTYPE(dt, T, return fwd_impl<T>(y, x, rows, (int)cols, (cudaStream_t)stream));
  return AK_OK;
}

extern "C" int ak_softmax_bwd(void* dx, const void* y, const void* dy, int64_t rows, int64_t cols, int dt,
                              void* stream) {
  clear_error();
  AK_REQUIRE(rows >= 0 && cols > 0 && cols <= (1LL << 30), AK_ERR_SHAPE, "ak_softmax_bwd: bad shape");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(dx && y && dy, AK_ERR_ARG, "ak_softmax_bwd: null pointer");
  AK_DISPATCH_DTYPE(dt, T, return bwd_impl<T>(dx, y, dy, rows, (int)cols, (cudaStream_t)stream));
  return AK_OK;
}
