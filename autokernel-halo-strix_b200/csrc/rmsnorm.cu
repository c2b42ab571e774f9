// RMSNorm forward / backward for sm_100a.
//
// Forward (reference semantics: reference.py:26-29, kernels/hip/rmsnorm.py:39-117):
//   y = x * rsqrt(mean(x^2) + eps) * w
// Backward (kernels/hip/_torch_ops.py:73-97):
//   dx = r*dy*w - x * r^3 * sum(dy*w*x)/N,   dw = sum_rows dy*x*r
// Fused residual variant (kernels/hip/fused_residual_add_rmsnorm.py,
// fused_residual_rmsnorm_backward.py): hidden = x + residual feeds the norm and
// is a second output; its backward adds grad_hidden to dx.
//
// Design: one warp per row, the row held in registers (16-byte vector loads,
// one HBM read of x / dy), fp32 accumulation, warp-shuffle reductions only.
// dw is reduced without global atomics: each CTA folds its rows into a private
// fp32 partial row (workspace), and a second tiny kernel sums the partial rows
// in a fixed order, so dw is bitwise deterministic.
#include "ak_common.cuh"

#include <mutex>

namespace ak {
namespace {

constexpr int kWarps = 8;  // rows in flight per CTA

// ----------------------------------------------------------------------------
// Forward, row in registers
// ----------------------------------------------------------------------------
// RES: fused residual add (hidden = x + res, rounded to T, stored to h_out when
// non-null, then normalised).
// FULL: N == NIT * 32 * VEC, so no lane's vector is out of range and the loads
// carry no guard (issued back to back).
// TX / TY: types of x and y when they differ from the compute / residual type T
// (mixed precision: an fp32 residual stream with 16-bit mixer outputs in and a
// 16-bit normalised output for the next autocast GEMM, rounded once).
template <typename T, typename TW, int VEC, int NIT, bool RES = false, bool FULL = false, typename TX = T,
          typename TY = T>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_warp(TY* __restrict__ y, float* __restrict__ rstd_out, const TX* __restrict__ x,
                 const TW* __restrict__ w, int64_t M, int N, float eps, const T* __restrict__ res = nullptr,
                 T* __restrict__ h_out = nullptr) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float wr[NIT][VEC];
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    const int c = (it * 32 + lane) * VEC;
    if (FULL || c < N) load_frag<TW, VEC>(wr[it], w + c);
    else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) wr[it][k] = 0.f;
    }
  }
  const float inv_n = 1.f / (float)N;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < M; row += (int64_t)gridDim.x * kWarps) {
    const TX* xr = x + row * N;
    float xv[NIT][VEC];
    float ss = 0.f;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        load_frag<TX, VEC>(xv[it], xr + c);
        if constexpr (RES) {
          float rv[VEC];
          load_frag<T, VEC>(rv, res + row * N + c);
#pragma unroll
          for (int k = 0; k < VEC; ++k) xv[it][k] = to_f<T>(from_f<T>(xv[it][k] + rv[k]));
          if (h_out != nullptr) store_frag<T, VEC>(h_out + row * N + c, xv[it]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) xv[it][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < VEC; ++k) ss = fmaf(xv[it][k], xv[it][k], ss);
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * inv_n + eps);
    if (rstd_out != nullptr && lane == 0) rstd_out[row] = r;
    TY* yr = y + row * N;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        float o[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) o[k] = xv[it][k] * r * wr[it][k];
        store_frag<TY, VEC>(yr + c, o);
      }
    }
  }
}

// Forward fallback for rows that do not fit the register path (very wide or
// unaligned rows): one CTA per row, scalar accesses, two passes (second from L2).
template <typename T, typename TW, bool RES = false, typename TX = T, typename TY = T>
__global__ void __launch_bounds__(256)
rmsnorm_fwd_block(TY* __restrict__ y, float* __restrict__ rstd_out, const TX* __restrict__ x,
                  const TW* __restrict__ w, int64_t M, int N, float eps, const T* __restrict__ res = nullptr,
                  T* __restrict__ h_out = nullptr) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const TX* xr = x + row * N;
    const T* rr = RES ? res + row * N : nullptr;
    float ss = 0.f;
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
      float v = to_f<TX>(xr[c]);
      if constexpr (RES) {
        const T h = from_f<T>(v + to_f<T>(rr[c]));
        if (h_out != nullptr) h_out[row * N + c] = h;
        v = to_f<T>(h);
      }
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float r = rsqrtf(tot / (float)N + eps);
    if (rstd_out != nullptr && threadIdx.x == 0) rstd_out[row] = r;
    TY* yr = y + row * N;
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
      float v = to_f<TX>(xr[c]);
      if constexpr (RES) v = to_f<T>(from_f<T>(v + to_f<T>(rr[c])));
      yr[c] = from_f<TY>(v * r * to_f<TW>(w[c]));
    }
    __syncthreads();
  }
}

// ----------------------------------------------------------------------------
// Backward, row in registers; per-CTA dw partial row into the workspace.
// ----------------------------------------------------------------------------
// RES: dx += gh (the gradient reaching the un-normalised output of the fused
// residual add), loaded only at store time.
// Registers hold only the row being processed (x, dy); w and the per-warp dw
// accumulators live in shared memory, each lane owning its columns (no
// atomics).  Shared layout is lane-contiguous: column (it*32 + lane)*VEC + k
// sits at slot (it*VEC + k)*32 + lane, so every access is bank-conflict free.
template <int VEC>
__device__ __forceinline__ int bwd_slot(int c) {
  const int it = c / (32 * VEC), rem = c - it * 32 * VEC;
  const int lane = rem / VEC, k = rem - lane * VEC;
  return (it * VEC + k) * 32 + lane;
}

// TG: type of dy when it differs from T (mixed precision: 16-bit gradient of a
// 16-bit normalised output).  dx2 (nullable, type TG): a second copy of dx, the
// gradient of a 16-bit fused-residual input.
template <typename T, typename TW, int VEC, int NIT, bool RES = false, bool FULL = false, typename TG = T>
__global__ void __launch_bounds__(kWarps * 32, (NIT * VEC <= 24) ? 3 : 2)
rmsnorm_bwd_warp(T* __restrict__ dx, float* __restrict__ dw_part, const TG* __restrict__ dy,
                 const T* __restrict__ x, const TW* __restrict__ w, int64_t M, int N, float eps,
                 const T* __restrict__ gh = nullptr, TG* __restrict__ dx2 = nullptr) {
  constexpr int kSlots = NIT * VEC * 32;
  extern __shared__ float s_dw[];  // [kWarps][kSlots] accumulators, then [kSlots] weights
  float* s_w = s_dw + (size_t)kWarps * kSlots;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int q = threadIdx.x; q < kSlots; q += blockDim.x) {  // every slot: columns >= N read as 0
    const int j = q >> 5, ln = q & 31, it = j / VEC, k = j - it * VEC;
    const int c = (it * 32 + ln) * VEC + k;
    s_w[q] = c < N ? to_f<TW>(w[c]) : 0.f;
  }
  float* my = s_dw + (size_t)warp * kSlots;
#pragma unroll
  for (int j = 0; j < NIT * VEC; ++j) my[j * 32 + lane] = 0.f;
  __syncthreads();
  const float inv_n = 1.f / (float)N;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < M; row += (int64_t)gridDim.x * kWarps) {
    float xv[NIT][VEC], gv[NIT][VEC];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        load_frag<T, VEC>(xv[it], x + row * N + c);
        load_frag<TG, VEC>(gv[it], dy + row * N + c);
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) { xv[it][k] = 0.f; gv[it][k] = 0.f; }
      }
    }
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        // columns >= N hold x = dy = 0 and contribute nothing
        s1 = fmaf(xv[it][k], xv[it][k], s1);
        s2 = fmaf(gv[it][k] * s_w[(it * VEC + k) * 32 + lane], xv[it][k], s2);
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float r = rsqrtf(s1 * inv_n + eps);
    const float c3 = r * r * r * s2 * inv_n;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        float o[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const int sl = (it * VEC + k) * 32 + lane;
          o[k] = r * gv[it][k] * s_w[sl] - xv[it][k] * c3;
          my[sl] = fmaf(gv[it][k], xv[it][k] * r, my[sl]);
        }
        if constexpr (RES) {
          if (gh != nullptr) {
            float hv[VEC];
            load_frag<T, VEC>(hv, gh + row * N + c);
#pragma unroll
            for (int k = 0; k < VEC; ++k) o[k] += hv[k];
          }
        }
        store_frag<T, VEC>(dx + row * N + c, o);
        if (dx2 != nullptr) store_frag<TG, VEC>(dx2 + row * N + c, o);
      }
    }
  }
  // Fold the kWarps per-warp partials in a fixed order (deterministic).
  __syncthreads();
  for (int c = threadIdx.x; c < N; c += blockDim.x) {
    const int sl = bwd_slot<VEC>(c);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += s_dw[i * kSlots + sl];
    dw_part[(int64_t)blockIdx.x * N + c] = s;
  }
  pdl_trigger();
}

// Backward with the next row's x and dy in flight (raw 16-byte vectors) while
// the current row is reduced and stored.  Same arithmetic and shared-memory
// layout as rmsnorm_bwd_warp (no residual, no second output).
template <typename T, typename TW, int VEC, int NIT, bool FULL, typename TG = T>
__global__ void __launch_bounds__(kWarps * 32, 2)
rmsnorm_bwd_pf(T* __restrict__ dx, float* __restrict__ dw_part, const TG* __restrict__ dy,
               const T* __restrict__ x, const TW* __restrict__ w, int64_t M, int N, float eps) {
  using FX = Frag<T, VEC>;
  using FG = Frag<TG, VEC>;
  constexpr int kSlots = NIT * VEC * 32;
  extern __shared__ float s_dw[];  // [kWarps][kSlots] accumulators, then [kSlots] weights
  float* s_w = s_dw + (size_t)kWarps * kSlots;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int q = threadIdx.x; q < kSlots; q += blockDim.x) {
    const int j = q >> 5, ln = q & 31, it = j / VEC, k = j - it * VEC;
    const int c = (it * 32 + ln) * VEC + k;
    s_w[q] = c < N ? to_f<TW>(w[c]) : 0.f;
  }
  float* my = s_dw + (size_t)warp * kSlots;
#pragma unroll
  for (int j = 0; j < NIT * VEC; ++j) my[j * 32 + lane] = 0.f;
  __syncthreads();
  const float inv_n = 1.f / (float)N;
  const int64_t stride = (int64_t)gridDim.x * kWarps;
  int64_t row = (int64_t)blockIdx.x * kWarps + warp;
  FX cx[NIT];
  FG cg[NIT];
  if (row < M) {
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        cx[it] = *reinterpret_cast<const FX*>(x + row * N + c);
        cg[it] = *reinterpret_cast<const FG*>(dy + row * N + c);
      }
    }
  }
  for (; row < M; row += stride) {
    const int64_t nrow = row + stride;
    FX nx[NIT];
    FG ng[NIT];
    if (nrow < M) {
#pragma unroll
      for (int it = 0; it < NIT; ++it) {
        const int c = (it * 32 + lane) * VEC;
        if (FULL || c < N) {
          nx[it] = *reinterpret_cast<const FX*>(x + nrow * N + c);
          ng[it] = *reinterpret_cast<const FG*>(dy + nrow * N + c);
        }
      }
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const float xv = to_f<T>(cx[it].v[k]), gv = to_f<TG>(cg[it].v[k]);
          s1 = fmaf(xv, xv, s1);
          s2 = fmaf(gv * s_w[(it * VEC + k) * 32 + lane], xv, s2);
        }
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float r = rsqrtf(s1 * inv_n + eps);
    const float c3 = r * r * r * s2 * inv_n;
#pragma unroll
    for (int it = 0; it < NIT; ++it) {
      const int c = (it * 32 + lane) * VEC;
      if (FULL || c < N) {
        float o[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const int sl = (it * VEC + k) * 32 + lane;
          const float xv = to_f<T>(cx[it].v[k]), gv = to_f<TG>(cg[it].v[k]);
          o[k] = r * gv * s_w[sl] - xv * c3;
          my[sl] = fmaf(gv, xv * r, my[sl]);
        }
        store_frag<T, VEC>(dx + row * N + c, o);
      }
    }
#pragma unroll
    for (int it = 0; it < NIT; ++it) { cx[it] = nx[it]; cg[it] = ng[it]; }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < N; c += blockDim.x) {
    const int sl = bwd_slot<VEC>(c);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += s_dw[i * kSlots + sl];
    dw_part[(int64_t)blockIdx.x * N + c] = s;
  }
  pdl_trigger();
}

// Backward fallback (wide / unaligned rows): one CTA per row at a time, the
// CTA owns partial row blockIdx.x of the workspace exclusively.
template <typename T, typename TW, bool RES = false, typename TG = T>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_block(T* __restrict__ dx, float* __restrict__ dw_part, const TG* __restrict__ dy,
                  const T* __restrict__ x, const TW* __restrict__ w, int64_t M, int N, float eps,
                  const T* __restrict__ gh = nullptr, TG* __restrict__ dx2 = nullptr) {
  __shared__ float red1[32], red2[32];
  float* part = dw_part + (int64_t)blockIdx.x * N;
  for (int c = threadIdx.x; c < N; c += blockDim.x) part[c] = 0.f;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * N;
    const TG* gr = dy + row * N;
    float s1 = 0.f, s2 = 0.f;
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
      const float xv = to_f<T>(xr[c]), gv = to_f<TG>(gr[c]);
      s1 = fmaf(xv, xv, s1);
      s2 = fmaf(gv * to_f<TW>(w[c]), xv, s2);
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if ((threadIdx.x & 31) == 0) { red1[threadIdx.x >> 5] = s1; red2[threadIdx.x >> 5] = s2; }
    __syncthreads();
    float t1 = 0.f, t2 = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { t1 += red1[i]; t2 += red2[i]; }
    const float r = rsqrtf(t1 / (float)N + eps);
    const float c3 = r * r * r * t2 / (float)N;
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
      const float xv = to_f<T>(xr[c]), gv = to_f<TG>(gr[c]);
      float o = r * gv * to_f<TW>(w[c]) - xv * c3;
      if constexpr (RES) {
        if (gh != nullptr) o += to_f<T>(gh[row * N + c]);
      }
      dx[row * N + c] = from_f<T>(o);
      if (dx2 != nullptr) dx2[row * N + c] = from_f<TG>(o);
      part[c] = fmaf(gv, xv * r, part[c]);
    }
    __syncthreads();
  }
}

// dw[c] = sum_g part[g][c] in a fixed order.  Block (32, 32): 32 columns x 32
// row-groups (32 loads in flight per column), folded through shared memory in
// index order.
template <typename TD>
__global__ void __launch_bounds__(1024)
rmsnorm_dw_reduce(TD* __restrict__ dw, const float* __restrict__ part, int G, int N) {
  __shared__ float s[32][33];
  pdl_wait();  // the backward kernel's partial rows are complete and visible
  const int c = blockIdx.x * 32 + threadIdx.x;
  float acc = 0.f;
  if (c < N)
#pragma unroll 8  // independent loads in flight; the adds stay in index order
    for (int g = threadIdx.y; g < G; g += 32) acc += part[(int64_t)g * N + c];
  s[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c < N) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) t += s[i][threadIdx.x];
    dw[c] = from_f<TD>(t);
  }
}

// ----------------------------------------------------------------------------
// Host dispatch
// ----------------------------------------------------------------------------
int pick_nit(int N, int vec) {
  const int need = (N + 32 * vec - 1) / (32 * vec);
  const int opts[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int o : opts)
    if (o >= need) return o;
  return 0;  // too wide for the register path
}

#define AK_NIT_SWITCH(nit, NIT, ...)              \
  switch (nit) {                                  \
    case 1: { constexpr int NIT = 1; __VA_ARGS__; } break;   \
    case 2: { constexpr int NIT = 2; __VA_ARGS__; } break;   \
    case 3: { constexpr int NIT = 3; __VA_ARGS__; } break;   \
    case 4: { constexpr int NIT = 4; __VA_ARGS__; } break;   \
    case 6: { constexpr int NIT = 6; __VA_ARGS__; } break;   \
    case 8: { constexpr int NIT = 8; __VA_ARGS__; } break;   \
    case 12: { constexpr int NIT = 12; __VA_ARGS__; } break; \
    case 16: { constexpr int NIT = 16; __VA_ARGS__; } break; \
    default: break;                               \
  }

struct RmsPlan {
  bool warp_path;
  int vec, nit, grid;
};

template <typename T, typename TW>
RmsPlan plan(int64_t M, int N, const void* a, const void* b, const void* w) {
  RmsPlan p{};
  constexpr int vec = 16 / sizeof(T);
  const bool al = aligned16(a) && aligned16(b) &&
                  (reinterpret_cast<uintptr_t>(w) % (sizeof(TW) * vec) == 0);
  p.vec = vec;
  p.nit = (N % vec == 0 && al) ? pick_nit(N, vec) : 0;
  p.warp_path = p.nit > 0;
  return p;
}

// Grid of a backward kernel capped at the CTAs that are resident at once (one
// wave: every CTA gets the same number of rows through the grid-stride loop).
template <typename K>
int resident_grid(K kern, size_t smem, int G) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int cap = per_sm * sm_count();
  return G < cap ? G : cap;
}

int bwd_grid(int64_t M, int N) {
  // at least 4 rows per warp, so the per-CTA set-up and dw fold are amortised
  const int64_t rows_per_cta = 4 * kWarps;
  int64_t g = (M + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = 3LL * sm_count();  // CTAs resident per SM on the register path
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  (void)N;
  return (int)g;
}

// TX / TY: input / output types when they differ from T (mixed precision).
template <typename T, typename TW, bool RES = false, typename TX = T, typename TY = T>
int fwd_impl(void* y, float* rstd, const void* x, const void* w, int64_t M, int N, float eps,
             cudaStream_t st, const void* res = nullptr, void* h_out = nullptr) {
  RmsPlan p = plan<T, TW>(M, N, x, y, w);
  if (RES && !(aligned16(res) && (h_out == nullptr || aligned16(h_out)))) p.warp_path = false;
  constexpr int VEC = 16 / sizeof(T);
  if (p.warp_path) {
    int64_t g = (M + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (g > cap) g = cap;
    if (N == p.nit * 32 * VEC) {
      AK_NIT_SWITCH(p.nit, NIT,
                    rmsnorm_fwd_warp<T, TW, VEC, NIT, RES, true, TX, TY><<<(unsigned)g, kWarps * 32, 0, st>>>(
                        (TY*)y, rstd, (const TX*)x, (const TW*)w, M, N, eps, (const T*)res, (T*)h_out));
    } else {
      AK_NIT_SWITCH(p.nit, NIT,
                    rmsnorm_fwd_warp<T, TW, VEC, NIT, RES, false, TX, TY><<<(unsigned)g, kWarps * 32, 0, st>>>(
                        (TY*)y, rstd, (const TX*)x, (const TW*)w, M, N, eps, (const T*)res, (T*)h_out));
    }
  } else {
    int64_t g = M;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (g > cap) g = cap;
    rmsnorm_fwd_block<T, TW, RES, TX, TY><<<(unsigned)g, 256, 0, st>>>((TY*)y, rstd, (const TX*)x, (const TW*)w,
                                                                       M, N, eps, (const T*)res, (T*)h_out);
  }
  AK_CHECK_LAUNCH("ak_rmsnorm_fwd");
  return AK_OK;
}

// TG: type of dy (and of the optional second output dx2) when it differs from T.
template <typename T, typename TW, bool RES = false, typename TG = T>
int bwd_impl(void* dx, void* dw, int dt_dw, float* ws, const void* dy, const void* x, const void* w,
             int64_t M, int N, float eps, cudaStream_t st, const void* gh = nullptr, void* dx2 = nullptr) {
  RmsPlan p = plan<T, TW>(M, N, x, dx, w);
  if (!aligned16(dy)) p.warp_path = false;
  if (dx2 != nullptr && !aligned16(dx2)) p.warp_path = false;
  if (RES && gh != nullptr && !aligned16(gh)) p.warp_path = false;
  // x and dy live in registers (w and the dw accumulators in shared memory):
  // beyond 32 elements per lane the register path spills, so wider rows take
  // the CTA fallback.
  if (p.nit * p.vec > 32) p.warp_path = false;
  constexpr int VEC = 16 / sizeof(T);
  int G = bwd_grid(M, N);
  if (M > 0) {
    if (p.warp_path) {
      const bool full = N == p.nit * 32 * VEC;
      // plain backward: the next row's x and dy are in flight while the current row is reduced
      // (bf16 [16384, 768]: 0.51 -> 0.56 of HBM); the residual / dual-output forms keep the
      // one-row kernel
      if (!RES && dx2 == nullptr) {
        AK_NIT_SWITCH(p.nit, NIT, if constexpr (NIT * VEC <= 32) {
          auto kern = full ? rmsnorm_bwd_pf<T, TW, VEC, NIT, true, TG> : rmsnorm_bwd_pf<T, TW, VEC, NIT, false, TG>;
          const size_t smem = (size_t)(kWarps + 1) * NIT * VEC * 32 * sizeof(float);
          if (smem > 48 * 1024)
            AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "ak_rmsnorm_bwd: smem attribute");
          G = resident_grid(kern, smem, G);
          kern<<<G, kWarps * 32, smem, st>>>((T*)dx, ws, (const TG*)dy, (const T*)x, (const TW*)w, M, N, eps);
        });
      } else
      AK_NIT_SWITCH(p.nit, NIT, if constexpr (NIT * VEC <= 32) {
        auto kern = full ? rmsnorm_bwd_warp<T, TW, VEC, NIT, RES, true, TG>
                         : rmsnorm_bwd_warp<T, TW, VEC, NIT, RES, false, TG>;
        const size_t smem = (size_t)(kWarps + 1) * NIT * VEC * 32 * sizeof(float);
        if (smem > 48 * 1024)
          AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "ak_rmsnorm_bwd: smem attribute");
        G = resident_grid(kern, smem, G);
        kern<<<G, kWarps * 32, smem, st>>>((T*)dx, ws, (const TG*)dy, (const T*)x, (const TW*)w, M, N, eps,
                                           (const T*)gh, (TG*)dx2);
      });
    } else {
      rmsnorm_bwd_block<T, TW, RES, TG><<<G, 256, 0, st>>>((T*)dx, ws, (const TG*)dy, (const T*)x, (const TW*)w,
                                                           M, N, eps, (const T*)gh, (TG*)dx2);
    }
    AK_CHECK_LAUNCH("ak_rmsnorm_bwd");
  }
  const int Gred = M > 0 ? G : 0;
  dim3 rb(32, 32);
  const unsigned rg = (unsigned)((N + 31) / 32);
  AK_DISPATCH_DTYPE(dt_dw, TD,
                    AK_CUDA_TRY(launch_pdl(rmsnorm_dw_reduce<TD>, dim3(rg), rb, 0, st, (TD*)dw, (const float*)ws, Gred, N),
                                "ak_rmsnorm_bwd(dw reduce)"));
  AK_CHECK_LAUNCH("ak_rmsnorm_bwd(dw reduce)");
  return AK_OK;
}

}  // namespace
}  // namespace ak

using namespace ak;

#define AK_DISPATCH_XW(dt_x, dt_w, ...)                                                   \
  do {                                                                                     \
    if (dt_x == AK_F32 && dt_w == AK_F32) { using T = float; using TW = float; __VA_ARGS__; }      \
    else if (dt_x == AK_BF16 && dt_w == AK_BF16) { using T = __nv_bfloat16; using TW = __nv_bfloat16; __VA_ARGS__; } \
    else if (dt_x == AK_BF16 && dt_w == AK_F32) { using T = __nv_bfloat16; using TW = float; __VA_ARGS__; } \
    else if (dt_x == AK_F16 && dt_w == AK_F16) { using T = __half; using TW = __half; __VA_ARGS__; } \
    else if (dt_x == AK_F16 && dt_w == AK_F32) { using T = __half; using TW = float; __VA_ARGS__; } \
    else { set_error("rmsnorm: unsupported dtype pair x=%d w=%d", dt_x, dt_w); return AK_ERR_DTYPE; } \
  } while (0)

extern "C" int ak_rmsnorm_fwd(void* y, float* rstd, const void* x, const void* w, int64_t M,
                              int64_t N, float eps, int dt_x, int dt_w, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_rmsnorm_fwd: bad shape M=%lld N=%lld",
             (long long)M, (long long)N);
  if (M == 0) return AK_OK;
  AK_REQUIRE(y && x && w, AK_ERR_ARG, "ak_rmsnorm_fwd: null pointer");
  AK_DISPATCH_XW(dt_x, dt_w, return fwd_impl<T, TW>(y, rstd, x, w, M, (int)N, eps, (cudaStream_t)stream));
  return AK_OK;
}

extern "C" int ak_rmsnorm_bwd_workspace_size(int64_t M, int64_t N, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes && M >= 0 && N > 0, AK_ERR_ARG, "ak_rmsnorm_bwd_workspace_size: bad args");
  *bytes = (size_t)bwd_grid(M, (int)N) * (size_t)N * sizeof(float);
  return AK_OK;
}

extern "C" int ak_rmsnorm_bwd(void* dx, void* dw, int dt_dw, void* workspace, size_t ws_bytes,
                              const void* dy, const void* x, const void* w, int64_t M, int64_t N,
                              float eps, int dt_x, int dt_w, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_rmsnorm_bwd: bad shape");
  AK_REQUIRE(dw && w, AK_ERR_ARG, "ak_rmsnorm_bwd: null pointer");
  AK_REQUIRE(M == 0 || (dx && dy && x), AK_ERR_ARG, "ak_rmsnorm_bwd: null pointer");
  const size_t need = (size_t)bwd_grid(M, (int)N) * (size_t)N * sizeof(float);
  AK_REQUIRE(M == 0 || (workspace && ws_bytes >= need), AK_ERR_WORKSPACE,
             "ak_rmsnorm_bwd: workspace %zu < %zu bytes", ws_bytes, need);
  AK_DISPATCH_XW(dt_x, dt_w,
                 return bwd_impl<T, TW>(dx, dw, dt_dw, (float*)workspace, dy, x, w, M, (int)N, eps,
                                        (cudaStream_t)stream));
  return AK_OK;
}

// ---- Fused residual add + RMSNorm (kernels/hip/fused_residual_add_rmsnorm.py,
// autokernel::fused_res_rmsnorm in kernels/hip/_torch_ops.py:238-296)
extern "C" int ak_fused_res_rmsnorm_fwd(void* hidden, void* normed, const void* x, const void* residual,
                                        const void* w, int64_t M, int64_t N, float eps, int dt_x, int dt_w,
                                        void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_fused_res_rmsnorm_fwd: bad shape M=%lld N=%lld",
             (long long)M, (long long)N);
  if (M == 0) return AK_OK;
  AK_REQUIRE(normed && x && residual && w, AK_ERR_ARG, "ak_fused_res_rmsnorm_fwd: null pointer");
  AK_DISPATCH_XW(dt_x, dt_w,
                 return fwd_impl<T, TW, true>(normed, nullptr, x, w, M, (int)N, eps, (cudaStream_t)stream, residual,
                                              hidden));
  return AK_OK;
}

extern "C" int ak_fused_res_rmsnorm_bwd(void* dx, void* dw, int dt_dw, void* workspace, size_t ws_bytes,
                                        const void* grad_hidden, const void* grad_normed, const void* hidden,
                                        const void* w, int64_t M, int64_t N, float eps, int dt_x, int dt_w,
                                        void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_fused_res_rmsnorm_bwd: bad shape");
  AK_REQUIRE(dw && w, AK_ERR_ARG, "ak_fused_res_rmsnorm_bwd: null pointer");
  AK_REQUIRE(M == 0 || (dx && grad_normed && hidden), AK_ERR_ARG, "ak_fused_res_rmsnorm_bwd: null pointer");
  const size_t need = (size_t)bwd_grid(M, (int)N) * (size_t)N * sizeof(float);
  AK_REQUIRE(M == 0 || (workspace && ws_bytes >= need), AK_ERR_WORKSPACE,
             "ak_fused_res_rmsnorm_bwd: workspace %zu < %zu bytes", ws_bytes, need);
  AK_DISPATCH_XW(dt_x, dt_w,
                 return bwd_impl<T, TW, true>(dx, dw, dt_dw, (float*)workspace, grad_normed, hidden, w, M, (int)N,
                                              eps, (cudaStream_t)stream, grad_hidden));
  return AK_OK;
}

// ---- Mixed precision (fp32 residual stream, 16-bit autocast activations) ----
// Dispatch over the 16-bit edge type TL (bf16 / fp16) and the weight type with an
// fp32 compute / residual type.
#define AK_DISPATCH_MIXED(dt_lo, dt_w, ...)                                                              \
  do {                                                                                                    \
    if (dt_lo == AK_BF16 && dt_w == AK_F32) { using TL = __nv_bfloat16; using TW = float; __VA_ARGS__; }   \
    else if (dt_lo == AK_F16 && dt_w == AK_F32) { using TL = __half; using TW = float; __VA_ARGS__; }      \
    else if (dt_lo == AK_BF16 && dt_w == AK_BF16) { using TL = __nv_bfloat16; using TW = __nv_bfloat16; __VA_ARGS__; } \
    else if (dt_lo == AK_F16 && dt_w == AK_F16) { using TL = __half; using TW = __half; __VA_ARGS__; }     \
    else { set_error("rmsnorm mixed: unsupported dtypes lo=%d w=%d", dt_lo, dt_w); return AK_ERR_DTYPE; } \
  } while (0)

extern "C" int ak_rmsnorm_fwd_mixed(void* y, int dt_y, const void* x, int dt_x, const void* w, int dt_w, int64_t M,
                                    int64_t N, float eps, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_rmsnorm_fwd_mixed: bad shape");
  if (M == 0) return AK_OK;
  AK_REQUIRE(y && x && w, AK_ERR_ARG, "ak_rmsnorm_fwd_mixed: null pointer");
  if (dt_y == dt_x) return ak_rmsnorm_fwd(y, nullptr, x, w, M, N, eps, dt_x, dt_w, stream);
  AK_REQUIRE(dt_x == AK_F32, AK_ERR_DTYPE, "ak_rmsnorm_fwd_mixed: x must be fp32 when y differs");
  AK_DISPATCH_MIXED(dt_y, dt_w,
                    return fwd_impl<float, TW, false, float, TL>(y, nullptr, x, w, M, (int)N, eps,
                                                                 (cudaStream_t)stream));
  return AK_OK;
}

extern "C" int ak_fused_res_rmsnorm_fwd_mixed(void* hidden, void* normed, int dt_normed, const void* x, int dt_x,
                                              const void* residual, int dt_res, const void* w, int dt_w, int64_t M,
                                              int64_t N, float eps, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_fused_res_rmsnorm_fwd_mixed: bad shape");
  if (M == 0) return AK_OK;
  AK_REQUIRE(normed && x && residual && w, AK_ERR_ARG, "ak_fused_res_rmsnorm_fwd_mixed: null pointer");
  if (dt_x == dt_res && dt_normed == dt_res)
    return ak_fused_res_rmsnorm_fwd(hidden, normed, x, residual, w, M, N, eps, dt_x, dt_w, stream);
  AK_REQUIRE(dt_res == AK_F32 && dt_x == dt_normed, AK_ERR_DTYPE,
             "ak_fused_res_rmsnorm_fwd_mixed: residual / hidden fp32, x and normed of one 16-bit type");
  AK_DISPATCH_MIXED(dt_x, dt_w,
                    return fwd_impl<float, TW, true, TL, TL>(normed, nullptr, x, w, M, (int)N, eps,
                                                             (cudaStream_t)stream, residual, hidden));
  return AK_OK;
}

extern "C" int ak_rmsnorm_bwd_mixed(void* dx, void* dx2, void* dw, int dt_dw, void* workspace, size_t ws_bytes,
                                    const void* grad_hidden, const void* dy, int dt_dy, const void* x, int dt_x,
                                    const void* w, int dt_w, int64_t M, int64_t N, float eps, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), AK_ERR_SHAPE, "ak_rmsnorm_bwd_mixed: bad shape");
  AK_REQUIRE(dw && w, AK_ERR_ARG, "ak_rmsnorm_bwd_mixed: null pointer");
  AK_REQUIRE(M == 0 || (dx && dy && x), AK_ERR_ARG, "ak_rmsnorm_bwd_mixed: null pointer");
  const size_t need = (size_t)bwd_grid(M, (int)N) * (size_t)N * sizeof(float);
  AK_REQUIRE(M == 0 || (workspace && ws_bytes >= need), AK_ERR_WORKSPACE,
             "ak_rmsnorm_bwd_mixed: workspace %zu < %zu bytes", ws_bytes, need);
  AK_REQUIRE(dt_x == AK_F32 && dt_dy != AK_F32, AK_ERR_DTYPE,
             "ak_rmsnorm_bwd_mixed: x fp32 with a 16-bit dy (equal dtypes: ak_rmsnorm_bwd / ak_fused_res_rmsnorm_bwd)");
  AK_DISPATCH_MIXED(dt_dy, dt_w, {
    if (grad_hidden != nullptr)
      return bwd_impl<float, TW, true, TL>(dx, dw, dt_dw, (float*)workspace, dy, x, w, M, (int)N, eps,
                                           (cudaStream_t)stream, grad_hidden, dx2);
    return bwd_impl<float, TW, false, TL>(dx, dw, dt_dw, (float*)workspace, dy, x, w, M, (int)N, eps,
                                          (cudaStream_t)stream, nullptr, dx2);
  });
  return AK_OK;
}

// ============================================================================
// RMSNorm backward that allocates nothing (no counterpart in the reference).
//
// Some callers cannot hand this library a workspace: code running where
// cudaMalloc is off limits (a custom allocator that owns all device memory,
// a host runtime that forbids allocation after start-up, a plugin ABI that
// passes only inputs and outputs).  ak_rmsnorm_bwd_noalloc serves them: its
// per-CTA dw partial rows live in the file-scope device array below instead
// of a caller workspace.
// ============================================================================
namespace ak {
namespace {

// 4 MiB of fp32 partial rows, resident on every GPU that loads the library.
constexpr size_t kNoAllocFloats = (size_t)1 << 20;
static __device__ __align__(256) float g_rms_noalloc_scratch[kNoAllocFloats];

// Device address of g_rms_noalloc_scratch per device (host code cannot use the
// symbol's name as a device pointer).  The array lives in the device's current
// context, so the cached address is keyed on that context: after a device reset
// (a new primary context) the first call resolves it again.
std::mutex g_noalloc_mu;
struct NoAllocSlot {
  void* ctx;
  float* ptr;
};
NoAllocSlot g_noalloc[64] = {};

typedef int (*CtxGetCurrentFn)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)

int current_context(void** ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    AK_CUDA_TRY(cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q),
                "ak_rmsnorm_bwd_noalloc: driver entry point");
    AK_REQUIRE(f != nullptr && q == cudaDriverEntryPointSuccess, AK_ERR_LAUNCH,
               "ak_rmsnorm_bwd_noalloc: cuCtxGetCurrent unavailable");
    fn = reinterpret_cast<CtxGetCurrentFn>(f);
  }
  AK_REQUIRE(fn(ctx) == 0, AK_ERR_LAUNCH, "ak_rmsnorm_bwd_noalloc: cuCtxGetCurrent failed");
  return AK_OK;
}

int noalloc_scratch(float** out) {
  int dev = 0;
  AK_CUDA_TRY(cudaGetDevice(&dev), "ak_rmsnorm_bwd_noalloc: cudaGetDevice");
  AK_REQUIRE(dev >= 0 && dev < 64, AK_ERR_ARG, "ak_rmsnorm_bwd_noalloc: device index %d out of range", dev);
  void* ctx = nullptr;
  int rc = current_context(&ctx);  // NULL until the runtime has made a context current on this thread
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc[dev].ptr == nullptr || ctx == nullptr || g_noalloc[dev].ctx != ctx) {
    void* p = nullptr;
    AK_CUDA_TRY(cudaGetSymbolAddress(&p, g_rms_noalloc_scratch), "ak_rmsnorm_bwd_noalloc: cudaGetSymbolAddress");
    if ((rc = current_context(&ctx))) return rc;  // current now
    g_noalloc[dev].ctx = ctx;
    g_noalloc[dev].ptr = static_cast<float*>(p);
  }
  *out = g_noalloc[dev].ptr;
  return AK_OK;
}

// Same kernels as ak_rmsnorm_bwd with the CTA count G chosen so that G partial
// rows of N floats fit the static scratch.  Every CTA overwrites its whole row
// before the reduction reads it, so nothing in the scratch needs clearing.
template <typename T, typename TW>
int bwd_noalloc_impl(void* dx, void* dw, int dt_dw, float* ws, int G, const void* dy, const void* x, const void* w,
                     int64_t M, int N, float eps, cudaStream_t st) {
  RmsPlan p = plan<T, TW>(M, N, x, dx, w);
  if (!aligned16(dy)) p.warp_path = false;
  if (p.nit * p.vec > 32) p.warp_path = false;
  constexpr int VEC = 16 / sizeof(T);
  if (M > 0) {
    if (p.warp_path) {
      AK_NIT_SWITCH(p.nit, NIT, if constexpr (NIT * VEC <= 32) {
        auto kern = rmsnorm_bwd_warp<T, TW, VEC, NIT>;
        const size_t smem = (size_t)(kWarps + 1) * NIT * VEC * 32 * sizeof(float);
        if (smem > 48 * 1024)
          AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "ak_rmsnorm_bwd_noalloc: smem attribute");
        G = resident_grid(kern, smem, G);
        kern<<<G, kWarps * 32, smem, st>>>((T*)dx, ws, (const T*)dy, (const T*)x, (const TW*)w, M, N, eps,
                                           nullptr, nullptr);
      });
    } else {
      rmsnorm_bwd_block<T, TW><<<G, 256, 0, st>>>((T*)dx, ws, (const T*)dy, (const T*)x, (const TW*)w, M, N, eps);
    }
    AK_CHECK_LAUNCH("ak_rmsnorm_bwd_noalloc");
  }
  dim3 rb(32, 32);
  const unsigned rg = (unsigned)((N + 31) / 32);
  AK_DISPATCH_DTYPE(dt_dw, TD,
                    AK_CUDA_TRY(launch_pdl(rmsnorm_dw_reduce<TD>, dim3(rg), rb, 0, st, (TD*)dw, (const float*)ws,
                                           M > 0 ? G : 0, N),
                                "ak_rmsnorm_bwd_noalloc(dw reduce)"));
  AK_CHECK_LAUNCH("ak_rmsnorm_bwd_noalloc(dw reduce)");
  return AK_OK;
}

}  // namespace
}  // namespace ak

extern "C" int ak_rmsnorm_bwd_noalloc(void* dx, void* dw, int dt_dw, const void* dy, const void* x, const void* w,
                                      int64_t M, int64_t N, float eps, int dt_x, int dt_w, void* stream) {
  clear_error();
  AK_REQUIRE(M >= 0 && N > 0, AK_ERR_SHAPE, "ak_rmsnorm_bwd_noalloc: bad shape");
  AK_REQUIRE((size_t)N <= kNoAllocFloats, AK_ERR_SHAPE,
             "ak_rmsnorm_bwd_noalloc: N=%lld exceeds the static scratch (%zu floats); use ak_rmsnorm_bwd",
             (long long)N, kNoAllocFloats);
  AK_REQUIRE(dw && w, AK_ERR_ARG, "ak_rmsnorm_bwd_noalloc: null pointer");
  AK_REQUIRE(M == 0 || (dx && dy && x), AK_ERR_ARG, "ak_rmsnorm_bwd_noalloc: null pointer");
  float* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  int64_t G = bwd_grid(M, (int)N);
  const int64_t fit = (int64_t)(kNoAllocFloats / (size_t)N);
  if (G > fit) G = fit;
  AK_DISPATCH_XW(dt_x, dt_w,
                 return bwd_noalloc_impl<T, TW>(dx, dw, dt_dw, ws, (int)G, dy, x, w, M, (int)N, eps,
                                                (cudaStream_t)stream));
  return AK_OK;
}
