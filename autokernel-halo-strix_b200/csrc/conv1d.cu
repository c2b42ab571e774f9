// Depthwise causal conv1d (+ optional SiLU) forward / backward, sm_100a.
//
// Semantics: the `autokernel::causal_conv1d` custom op of the reference
// (kernels/hip/_torch_ops.py:883-975, PyTorch fallback = F.conv1d on the input
// left-padded by K-1, groups = D) and causal_conv1d_fn(x, w, b, activation)
// of external/causal-conv1d as used by the Mamba block:
//   pre[b,d,t] = bias[d] + sum_k w[d,k] * x[b,d,t-K+1+k]   (x = 0 for t < 0)
//   y = silu(pre) if activation else pre
// Backward: dpre = dy * silu'(pre); dx[t] = sum_k w[k] dpre[t+K-1-k];
//           dw[d,k] = sum_{b,t} dpre[t] x[t-K+1+k];  dbias[d] = sum_{b,t} dpre[t].
//
// Layout (B, D, T), T contiguous.  One warp owns one chunk of one
// (b, d) row, 64 (fwd) / 32 (bwd) bytes of consecutive steps per lane;
// the K-1 step halo comes from the neighbouring lane by shuffle (from global
// memory at chunk edges).  dw / dbias: per-warp partials in a workspace, summed
// over batch and chunks in a fixed order (deterministic, no atomics).
#include "ak_common.cuh"

namespace ak {
namespace {

// consecutive steps per lane: BYTES of each tensor (forward: four 16-byte loads,
// backward: two per tensor, keeping its register count at 4 CTAs per SM)
constexpr int kFwdBytes = 64;
constexpr int kBwdBytes = 32;
template <typename T, int BYTES = kFwdBytes> struct Run { static constexpr int kIt = BYTES / sizeof(T); };
constexpr int kMaxK = 8;
constexpr int kWarpsC = 8;
// backward CTAs of 4 warps (64 registers, 8 CTAs per SM): shorter-lived CTAs desynchronise the
// load / compute / store phases of the resident warps a little better (0.56 -> 0.57 of HBM)
constexpr int kWarpsB = 4;
template <typename T, int BYTES> constexpr int chunk_of() { return 32 * Run<T, BYTES>::kIt; }  // steps per warp

// SiLU with the approximate divide (two MUFU ops per element instead of an IEEE
// division; for p << 0 the denominator overflows and the result is -0, the limit)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// d silu(p) / dp
__device__ __forceinline__ float dsilu_f(float p) {
  const float s = __fdividef(1.f, 1.f + __expf(-p));
  return s * (1.f + p * (1.f - s));
}

// sigmoid(x) = 0.5 + 0.5 tanh(x / 2) with the hardware tanh approximation: one MUFU op
// instead of two.  Its error (about 2^-11) is below the precision of a 16-bit result, so
// it is used only when the activations are 16-bit; fp32 keeps the two-op form.
__device__ __forceinline__ float sigmoid_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return fmaf(0.5f, t, 0.5f);
}

template <typename T>
__device__ __forceinline__ float silu_t(float x) {
  if constexpr (sizeof(T) == 2) return x * sigmoid_tanh(x);
  else return silu_f(x);
}

template <typename T>
__device__ __forceinline__ float dsilu_t(float p) {
  if constexpr (sizeof(T) == 2) {
    const float s = sigmoid_tanh(p);
    return s * (1.f + p * (1.f - s));
  } else {
    return dsilu_f(p);
  }
}

// FULL: every run is in range and 16-byte aligned (T a multiple of the chunk):
// no branch around the vector loads / stores.
template <typename T, int kIt, bool FULL = false>
__device__ __forceinline__ void load_run(float (&v)[kIt], const T* row, int t, int T_, bool vec) {
  if (FULL || (vec && t + kIt <= T_)) {
    constexpr int VEC = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < kIt; i += VEC) {
      float f[VEC];
      load_frag<T, VEC>(f, row + t + i);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[i + k] = f[k];
    }
  } else {
#pragma unroll
    for (int i = 0; i < kIt; ++i) v[i] = (t + i < T_) ? to_f<T>(row[t + i]) : 0.f;
  }
}

template <typename T, int kIt, bool FULL = false>
__device__ __forceinline__ void store_run(T* row, const float (&v)[kIt], int t, int T_, bool vec) {
  if (FULL || (vec && t + kIt <= T_)) {
    constexpr int VEC = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < kIt; i += VEC) {
      float f[VEC];
#pragma unroll
      for (int k = 0; k < VEC; ++k) f[k] = v[i + k];
      store_frag<T, VEC>(row + t + i, f);
    }
  } else {
#pragma unroll
    for (int i = 0; i < kIt; ++i)
      if (t + i < T_) row[t + i] = from_f<T>(v[i]);
  }
}

// x[t], 0 outside [0, T)
template <typename T>
__device__ __forceinline__ float ld_or0(const T* row, int t, int T_) {
  return (t >= 0 && t < T_) ? to_f<T>(row[t]) : 0.f;
}

// pre[i] = bias + sum_k w[k] x[t0 + i - (K-1) + k]; halo[j] = x[t0 - (K-1) + j]
template <int K, int kIt>
__device__ __forceinline__ void conv_run(float (&pre)[kIt], const float (&xv)[kIt], const float (&halo)[kMaxK],
                                         const float (&w)[kMaxK], float bias) {
#pragma unroll
  for (int i = 0; i < kIt; ++i) {
    float acc = bias;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int src = i - (K - 1) + k;
      acc = fmaf(w[k], src >= 0 ? xv[src] : halo[K - 1 + src], acc);
    }
    pre[i] = acc;
  }
}

// Left halo: lanes > 0 take lane-1's last K-1 steps; lane 0 uses `edge`, loaded
// from global memory before the main loads were consumed.
template <int K, int kIt>
__device__ __forceinline__ void left_halo(float (&halo)[kMaxK], const float (&xv)[kIt], const float (&edge)[kMaxK],
                                          int lane) {
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const float fromprev = __shfl_up_sync(0xffffffffu, xv[kIt - (K - 1) + j], 1);
    halo[j] = lane > 0 ? fromprev : edge[j];
  }
}

template <typename T, int K, bool FULL>
__global__ void __launch_bounds__(kWarpsC * 32)
conv1d_fwd_kernel(T* __restrict__ y, const T* __restrict__ x, const float* __restrict__ wt,
                  const float* __restrict__ bias, int64_t rows, int nch, int D, int T_, int silu, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * kWarpsC + (threadIdx.x >> 5);
  if (wid >= rows * nch) return;
  const int64_t r = wid / nch;
  constexpr int kIt = Run<T, kFwdBytes>::kIt;
  const int c0 = (int)(wid - r * nch) * chunk_of<T, kFwdBytes>();
  const int d = (int)(r % D);
  const T* xr = x + r * T_;
  const int t0 = c0 + lane * kIt;
  // issue every global load first: the run, and lane 0's halo
  float xv[kIt], edge[kMaxK];
  load_run<T, kIt, FULL>(xv, xr, t0, T_, vec);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) edge[j] = lane == 0 ? ld_or0<T>(xr, t0 - (K - 1) + j, T_) : 0.f;
  float w[kMaxK];
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = __ldg(wt + d * K + k);
  const float bs = bias ? __ldg(bias + d) : 0.f;
  float halo[kMaxK], pre[kIt];
  left_halo<K, kIt>(halo, xv, edge, lane);
  conv_run<K, kIt>(pre, xv, halo, w, bs);
  if (silu) {
#pragma unroll
    for (int i = 0; i < kIt; ++i) pre[i] = silu_t<T>(pre[i]);
  }
  store_run<T, kIt, FULL>(y + r * T_, pre, t0, T_, vec);
}

// Backward; part[row][chunk][K+1] = per-warp (dw[0..K-1], dbias) partials.
template <typename T, int K, bool FULL, int BYTES = kBwdBytes, int WARPS = kWarpsB, int MINB = 8>
__global__ void __launch_bounds__(WARPS * 32, MINB)
conv1d_bwd_kernel(T* __restrict__ dx, float* __restrict__ part, const T* __restrict__ x, const T* __restrict__ dy,
                  const float* __restrict__ wt, const float* __restrict__ bias, int64_t rows, int D, int T_, int silu,
                  int nch, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (wid >= rows * nch) return;
  const int64_t r = wid / nch;
  constexpr int kIt = Run<T, BYTES>::kIt;
  const int c0 = (int)(wid - r * nch) * chunk_of<T, BYTES>();
  const int d = (int)(r % D);
  const T* xr = x + r * T_;
  const T* gr = dy + r * T_;
  const int t0 = c0 + lane * kIt;
  const int te = t0 + kIt;  // first step after the run
  // all global loads up front: runs of x and dy, lane 0's left halo of x, and
  // lane 31's right edge (x and dy at te .. te+K-2) for the next chunk's dpre
  float xv[kIt], g[kIt], edge[kMaxK], xr_e[kMaxK], gr_e[kMaxK];
  load_run<T, kIt, FULL>(xv, xr, t0, T_, vec);
  load_run<T, kIt, FULL>(g, gr, t0, T_, vec);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    edge[j] = lane == 0 ? ld_or0<T>(xr, t0 - (K - 1) + j, T_) : 0.f;
    xr_e[j] = lane == 31 ? ld_or0<T>(xr, te + j, T_) : 0.f;
    gr_e[j] = lane == 31 ? ld_or0<T>(gr, te + j, T_) : 0.f;
  }
  float w[kMaxK];
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = __ldg(wt + d * K + k);
  const float bs = bias ? __ldg(bias + d) : 0.f;

  float halo[kMaxK], pre[kIt];
  left_halo<K, kIt>(halo, xv, edge, lane);
  conv_run<K, kIt>(pre, xv, halo, w, bs);
  if (silu) {
#pragma unroll
    for (int i = 0; i < kIt; ++i) g[i] *= dsilu_t<T>(pre[i]);
  }
  // dw, dbias over this run (steps >= T have g = 0)
  float dwacc[kMaxK], dbacc = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) dwacc[k] = 0.f;
#pragma unroll
  for (int i = 0; i < kIt; ++i) {
    dbacc += g[i];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int src = i - (K - 1) + k;
      dwacc[k] = fmaf(g[i], src >= 0 ? xv[src] : halo[K - 1 + src], dwacc[k]);
    }
  }
  // right halo of dpre (steps te .. te+K-2): the next lane's first K-1, or at
  // lane 31 recomputed from the preloaded edge
  float gh[kMaxK];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) gh[j] = __shfl_down_sync(0xffffffffu, g[j], 1);
  if (lane == 31) {
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      float acc = bs;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int s = j - (K - 1) + k;  // offset from te: < 0 -> own run, >= 0 -> edge
        acc = fmaf(w[k], s >= 0 ? xr_e[s] : xv[kIt + s], acc);
      }
      gh[j] = silu ? gr_e[j] * dsilu_t<T>(acc) : gr_e[j];
    }
  }
  float o[kIt];
#pragma unroll
  for (int i = 0; i < kIt; ++i) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int src = i + (K - 1) - k;
      acc = fmaf(w[k], src < kIt ? g[src] : gh[src - kIt], acc);
    }
    o[i] = acc;
  }
  store_run<T, kIt, FULL>(dx + r * T_, o, t0, T_, vec);
#pragma unroll
  for (int k = 0; k < K; ++k) dwacc[k] = warp_sum(dwacc[k]);
  dbacc = warp_sum(dbacc);
  if (lane == 0) {
    float* pr = part + wid * (K + 1);
#pragma unroll
    for (int k = 0; k < K; ++k) pr[k] = dwacc[k];
    pr[K] = dbacc;
  }
  pdl_trigger();
}

// One warp per channel d: lanes stride over the B * nch partial records in a
// fixed order, then a fixed butterfly (deterministic).
template <int K>
__global__ void conv1d_dw_reduce(float* __restrict__ dw, float* __restrict__ dbias, const float* __restrict__ part,
                                 int B, int D, int nch) {
  pdl_wait();  // the backward kernel's partial records are complete and visible
  const int lane = threadIdx.x & 31;
  const int d = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (d >= D) return;
  float s[K + 1];
#pragma unroll
  for (int k = 0; k <= K; ++k) s[k] = 0.f;
  const int n = B * nch;
#pragma unroll 4  // independent loads in flight; the adds stay in index order
  for (int j = lane; j < n; j += 32) {
    const int b = j / nch, c = j - b * nch;
    const float* p = part + (((int64_t)b * D + d) * nch + c) * (K + 1);
#pragma unroll
    for (int k = 0; k <= K; ++k) s[k] += p[k];
  }
#pragma unroll
  for (int k = 0; k <= K; ++k) s[k] = warp_sum(s[k]);
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) dw[d * K + k] = s[k];
    if (dbias) dbias[d] = s[K];
  }
}

#define AK_K_SWITCH(K_, KC, ...)                                  \
  switch (K_) {                                                   \
    case 2: { constexpr int KC = 2; __VA_ARGS__; } break;         \
    case 3: { constexpr int KC = 3; __VA_ARGS__; } break;         \
    case 4: { constexpr int KC = 4; __VA_ARGS__; } break;         \
    case 5: { constexpr int KC = 5; __VA_ARGS__; } break;         \
    case 6: { constexpr int KC = 6; __VA_ARGS__; } break;         \
    case 7: { constexpr int KC = 7; __VA_ARGS__; } break;         \
    case 8: { constexpr int KC = 8; __VA_ARGS__; } break;         \
    default: ::ak::set_error("causal_conv1d: kernel width %d not in [2, 8]", (int)(K_)); return AK_ERR_SHAPE; \
  }

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_causal_conv1d_fwd(void* y, const void* x, const float* weight, const float* bias, int64_t B,
                                    int64_t D, int64_t T, int64_t K, int silu, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && D > 0 && T >= 0 && T < (1LL << 31) && D < (1LL << 31), AK_ERR_SHAPE,
             "ak_causal_conv1d_fwd: bad shape");
  if (B == 0 || T == 0) return AK_OK;
  AK_REQUIRE(y && x && weight, AK_ERR_ARG, "ak_causal_conv1d_fwd: null pointer");
  const int64_t rows = B * D;
  const int chunk = 32 * kFwdBytes / elem_size(dt);
  const int nch = (int)((T + chunk - 1) / chunk);
  const bool vec = aligned16(x) && aligned16(y) && ((T * elem_size(dt)) % 16 == 0);
  const unsigned grid = (unsigned)((rows * nch + kWarpsC - 1) / kWarpsC);
  const bool full = vec && T % chunk == 0;
  AK_DISPATCH_DTYPE(dt, TT, {
    if (full)
      AK_K_SWITCH(K, KC, conv1d_fwd_kernel<TT, KC, true><<<grid, kWarpsC * 32, 0, (cudaStream_t)stream>>>(
                             (TT*)y, (const TT*)x, weight, bias, rows, nch, (int)D, (int)T, silu, vec))
    else
      AK_K_SWITCH(K, KC, conv1d_fwd_kernel<TT, KC, false><<<grid, kWarpsC * 32, 0, (cudaStream_t)stream>>>(
                             (TT*)y, (const TT*)x, weight, bias, rows, nch, (int)D, (int)T, silu, vec))
  });
  AK_CHECK_LAUNCH("ak_causal_conv1d_fwd");
  return AK_OK;
}

static size_t conv_ws_bytes(int64_t B, int64_t D, int64_t T, int64_t K) {
  const int64_t chunk = 32 * kBwdBytes / 4;  // fp32 chunk: an upper bound for every dtype
  return (size_t)B * D * ((T + chunk - 1) / chunk) * (K + 1) * sizeof(float);
}

extern "C" int ak_causal_conv1d_bwd_workspace_size(int64_t B, int64_t D, int64_t T, int64_t K, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes && B >= 0 && D > 0 && T >= 0 && K > 0, AK_ERR_ARG, "ak_causal_conv1d_bwd_workspace_size: bad args");
  *bytes = conv_ws_bytes(B, D, T, K);
  return AK_OK;
}

extern "C" int ak_causal_conv1d_bwd(void* dx, float* dweight, float* dbias, void* workspace, size_t ws_bytes,
                                    const void* x, const float* weight, const float* bias, const void* dy,
                                    int64_t B, int64_t D, int64_t T, int64_t K, int silu, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && D > 0 && T >= 0 && T < (1LL << 31) && D < (1LL << 31), AK_ERR_SHAPE,
             "ak_causal_conv1d_bwd: bad shape");
  AK_REQUIRE(dweight && weight, AK_ERR_ARG, "ak_causal_conv1d_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (B == 0 || T == 0) {
    AK_CUDA_TRY(cudaMemsetAsync(dweight, 0, (size_t)D * K * 4, st), "conv1d bwd memset");
    if (dbias) AK_CUDA_TRY(cudaMemsetAsync(dbias, 0, (size_t)D * 4, st), "conv1d bwd memset");
    return AK_OK;
  }
  AK_REQUIRE(dx && x && dy, AK_ERR_ARG, "ak_causal_conv1d_bwd: null pointer");
  const size_t need = conv_ws_bytes(B, D, T, K);
  AK_REQUIRE(workspace && ws_bytes >= need, AK_ERR_WORKSPACE, "ak_causal_conv1d_bwd: workspace %zu < %zu", ws_bytes,
             need);
  const int64_t rows = B * D;
  const int chunk = 32 * kBwdBytes / elem_size(dt);
  const int nch = (int)((T + chunk - 1) / chunk);
  const bool vec = aligned16(x) && aligned16(dx) && aligned16(dy) && ((T * elem_size(dt)) % 16 == 0);
  const unsigned grid = (unsigned)((rows * nch + kWarpsB - 1) / kWarpsB);
  float* part = (float*)workspace;
  const bool full = vec && T % chunk == 0;
  AK_DISPATCH_DTYPE(dt, TT, {
    if (full)
      AK_K_SWITCH(K, KC, conv1d_bwd_kernel<TT, KC, true><<<grid, kWarpsB * 32, 0, st>>>(
                             (TT*)dx, part, (const TT*)x, (const TT*)dy, weight, bias, rows, (int)D, (int)T, silu, nch,
                             vec))
    else
      AK_K_SWITCH(K, KC, conv1d_bwd_kernel<TT, KC, false><<<grid, kWarpsB * 32, 0, st>>>(
                             (TT*)dx, part, (const TT*)x, (const TT*)dy, weight, bias, rows, (int)D, (int)T, silu, nch,
                             vec))
  });
  AK_CHECK_LAUNCH("ak_causal_conv1d_bwd");
  AK_K_SWITCH(K, KC,
              AK_CUDA_TRY(launch_pdl(conv1d_dw_reduce<KC>, dim3((unsigned)((D + 7) / 8)), dim3(256), 0, st, dweight,
                                     dbias, (const float*)part, (int)B, (int)D, nch),
                          "ak_causal_conv1d_bwd(reduce)"));
  AK_CHECK_LAUNCH("ak_causal_conv1d_bwd(reduce)");
  return AK_OK;
}
