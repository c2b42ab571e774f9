// SiLU gate multiply (the SwiGLU body) forward / backward, sm_100a.
//
// Semantics (kernels/hip/silu_gate_mul.py:102-118, backward
// kernels/hip/silu_gate_mul_backward.py:145-180 and the fp32 branch of
// _silu_gate_mul_backward, kernels/hip/_torch_ops.py:199-218):
//   y      = silu(g) * u = g * sigmoid(g) * u
//   d gate = dy * u * sigmoid(g) * (1 + g * (1 - sigmoid(g)))
//   d up   = dy * g * sigmoid(g)
// fp32 arithmetic, results rounded once to the tensor dtype.
//
// Layout: rows x cols with a row stride per operand, so gate / up may be the two
// halves of one packed (rows, 2*cols) projection output (stride 2*cols) and the
// backward may write d gate / d up straight into one packed (rows, 2*cols)
// gradient — no split copies, no concatenation.  y and dy are dense.
//
// Grid: x over 16-byte column vectors (256 threads), y over row groups of
// kRows rows, grid-strided; each thread issues all kRows rows' loads before
// using them.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kThreadsS = 256;
constexpr int kRows = 4;   // forward: rows staged per thread
constexpr int kRowsB = 2;  // backward (three operands per row)

__device__ __forceinline__ float sigmoid_f(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }

// Rows are staged as raw 16-byte vectors (4 registers each whatever the dtype)
// and unpacked to fp32 only when used.
template <typename T, int VEC>
__device__ __forceinline__ void unpack(float (&d)[VEC], const int4& raw) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int k = 0; k < VEC; ++k) d[k] = to_f<T>(e[k]);
}

template <typename T, int VEC>
__device__ __forceinline__ int4 ld_row(const T* p, int c, int cols, bool vec) {
  if (vec) return __ldcs(reinterpret_cast<const int4*>(p + c));
  int4 raw = make_int4(0, 0, 0, 0);
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int k = 0; k < VEC; ++k)
    if (c + k < cols) e[k] = p[c + k];
  return raw;
}

template <typename T, int VEC>
__device__ __forceinline__ void st_row(T* p, const float (&v)[VEC], int c, int cols, bool vec) {
  if (vec) {
    store_frag<T, VEC>(p + c, v);
  } else {
#pragma unroll
    for (int k = 0; k < VEC; ++k)
      if (c + k < cols) p[c + k] = from_f<T>(v[k]);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreadsS)
swiglu_fwd_kernel(T* __restrict__ y, const T* __restrict__ g, const T* __restrict__ u, int64_t rows, int cols,
                  int64_t ldg, int64_t ldu, bool vec) {
  const int c = (blockIdx.x * kThreadsS + threadIdx.x) * VEC;
  if (c >= cols) return;
  for (int64_t r0 = (int64_t)blockIdx.y * kRows; r0 < rows; r0 += (int64_t)gridDim.y * kRows) {
    int4 graw[kRows], uraw[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int64_t r = r0 + i < rows ? r0 + i : rows - 1;  // clamp: tail rows re-read the last one
      graw[i] = ld_row<T, VEC>(g + r * ldg, c, cols, vec);
      uraw[i] = ld_row<T, VEC>(u + r * ldu, c, cols, vec);
    }
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int64_t r = r0 + i;
      if (r >= rows) break;
      float gv[VEC], uv[VEC], o[VEC];
      unpack<T, VEC>(gv, graw[i]);
      unpack<T, VEC>(uv, uraw[i]);
#pragma unroll
      for (int k = 0; k < VEC; ++k) o[k] = gv[k] * sigmoid_f(gv[k]) * uv[k];
      st_row<T, VEC>(y + r * cols, o, c, cols, vec);
    }
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreadsS)
swiglu_bwd_kernel(T* __restrict__ dg, T* __restrict__ du, const T* __restrict__ g, const T* __restrict__ u,
                  const T* __restrict__ dy, int64_t rows, int cols, int64_t ldg, int64_t ldu, int64_t lddg,
                  int64_t lddu, bool vec) {
  const int c = (blockIdx.x * kThreadsS + threadIdx.x) * VEC;
  if (c >= cols) return;
  for (int64_t r0 = (int64_t)blockIdx.y * kRowsB; r0 < rows; r0 += (int64_t)gridDim.y * kRowsB) {
    int4 graw[kRowsB], uraw[kRowsB], yraw[kRowsB];
#pragma unroll
    for (int i = 0; i < kRowsB; ++i) {
      const int64_t r = r0 + i < rows ? r0 + i : rows - 1;
      graw[i] = ld_row<T, VEC>(g + r * ldg, c, cols, vec);
      uraw[i] = ld_row<T, VEC>(u + r * ldu, c, cols, vec);
      yraw[i] = ld_row<T, VEC>(dy + r * cols, c, cols, vec);
    }
#pragma unroll
    for (int i = 0; i < kRowsB; ++i) {
      const int64_t r = r0 + i;
      if (r >= rows) break;
      float gv[VEC], uv[VEC], yv[VEC], og[VEC], ou[VEC];
      unpack<T, VEC>(gv, graw[i]);
      unpack<T, VEC>(uv, uraw[i]);
      unpack<T, VEC>(yv, yraw[i]);
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        const float s = sigmoid_f(gv[k]);
        og[k] = yv[k] * uv[k] * s * (1.f + gv[k] * (1.f - s));
        ou[k] = yv[k] * gv[k] * s;
      }
      st_row<T, VEC>(dg + r * lddg, og, c, cols, vec);
      st_row<T, VEC>(du + r * lddu, ou, c, cols, vec);
    }
  }
}

// 16-byte vector path when every row start of every operand is 16-byte aligned.
bool rows_aligned(const void* p, int64_t ld, int es) { return aligned16(p) && (ld * es) % 16 == 0; }

dim3 swiglu_grid(int64_t rows, int cols, int vec, int rows_per) {
  const unsigned gx = (unsigned)((cols + (int64_t)kThreadsS * vec - 1) / ((int64_t)kThreadsS * vec));
  int64_t gy = (rows + rows_per - 1) / rows_per;
  const int64_t cap = (int64_t)sm_count() * 64 / (gx > 0 ? gx : 1) + 1;
  if (gy > cap) gy = cap;
  if (gy > 65535) gy = 65535;
  return dim3(gx, (unsigned)(gy < 1 ? 1 : gy));
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_silu_gate_mul_fwd(void* y, const void* gate, const void* up, int64_t rows, int64_t cols,
                                    int64_t ld_gate, int64_t ld_up, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(rows >= 0 && cols > 0 && cols < (1LL << 31) && ld_gate >= cols && ld_up >= cols, AK_ERR_SHAPE,
             "ak_silu_gate_mul_fwd: bad shape rows=%lld cols=%lld ld=(%lld, %lld)", (long long)rows,
             (long long)cols, (long long)ld_gate, (long long)ld_up);
  if (rows == 0) return AK_OK;
  AK_REQUIRE(y && gate && up, AK_ERR_ARG, "ak_silu_gate_mul_fwd: null pointer");
  const int es = elem_size(dt);
  const bool vec = rows_aligned(gate, ld_gate, es) && rows_aligned(up, ld_up, es) && rows_aligned(y, cols, es);
  AK_DISPATCH_DTYPE(dt, T, {
    constexpr int VEC = 16 / sizeof(T);
    swiglu_fwd_kernel<T, VEC><<<swiglu_grid(rows, (int)cols, VEC, kRows), kThreadsS, 0, (cudaStream_t)stream>>>(
        (T*)y, (const T*)gate, (const T*)up, rows, (int)cols, ld_gate, ld_up, vec);
  });
  AK_CHECK_LAUNCH("ak_silu_gate_mul_fwd");
  return AK_OK;
}

extern "C" int ak_silu_gate_mul_bwd(void* dgate, void* dup, const void* gate, const void* up, const void* dy,
                                    int64_t rows, int64_t cols, int64_t ld_gate, int64_t ld_up, int64_t ld_dgate,
                                    int64_t ld_dup, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(rows >= 0 && cols > 0 && cols < (1LL << 31) && ld_gate >= cols && ld_up >= cols && ld_dgate >= cols &&
                 ld_dup >= cols,
             AK_ERR_SHAPE, "ak_silu_gate_mul_bwd: bad shape");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(dgate && dup && gate && up && dy, AK_ERR_ARG, "ak_silu_gate_mul_bwd: null pointer");
  const int es = elem_size(dt);
  const bool vec = rows_aligned(gate, ld_gate, es) && rows_aligned(up, ld_up, es) && rows_aligned(dy, cols, es) &&
                   rows_aligned(dgate, ld_dgate, es) && rows_aligned(dup, ld_dup, es);
  AK_DISPATCH_DTYPE(dt, T, {
    constexpr int VEC = 16 / sizeof(T);
    swiglu_bwd_kernel<T, VEC><<<swiglu_grid(rows, (int)cols, VEC, kRowsB), kThreadsS, 0, (cudaStream_t)stream>>>(
        (T*)dgate, (T*)dup, (const T*)gate, (const T*)up, (const T*)dy, rows, (int)cols, ld_gate, ld_up, ld_dgate,
        ld_dup, vec);
  });
  AK_CHECK_LAUNCH("ak_silu_gate_mul_bwd");
  return AK_OK;
}
