// Cross-entropy over materialised logit rows, sm_100a.
//
// Semantics follow cross_entropy_fwd_kernel / cross_entropy_bwd_tiny_kernel
// (kernels/ce_fused.py:122-329, 405-488):
//   x'   = softcap > 0 ? softcap * tanh(x / softcap) : x
//   lse  = log(sum exp x'),  loss = lse - (1-a) x'_y - a * mean(x')   (a = label smoothing)
//   grad = (softmax(x') - (1-a)[i==y] - a/V) * (1 - tanh^2) * scale
//   rows with y == ignore_index: loss 0, grad row 0.
// One CTA per row (grid-strided), 16-byte loads, online (max, sum) merged once
// per vector of 8/16 elements so the SFU does ~1 exp per element.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kThreads = 256;
constexpr int kBatch = 4;  // independent 16-byte loads in flight per thread

struct CeParams {
  float softcap, inv_softcap, ls, ls_uniform, target_coeff;
  int64_t ignore_index;
};

__device__ __forceinline__ float cap(float x, const CeParams& p) {
  return p.softcap > 0.f ? p.softcap * tanhf(x * p.inv_softcap) : x;
}

// Merge (m_b, s_b) into (m, s): s is a sum of exp2((x - m) * log2e).
__device__ __forceinline__ void merge(float& m, float& s, float mb, float sb) {
  const float mn = fmaxf(m, mb);
  if (mn == -INFINITY) return;
  s = s * ex2((m - mn) * kLog2e) + sb * ex2((mb - mn) * kLog2e);
  m = mn;
}

// Vector index holding the target column, or -1 (ignored row or target out of range).
__device__ __forceinline__ int target_vec(int64_t tgt, bool ignored, int V, int vec) {
  return (!ignored && tgt >= 0 && tgt < V) ? (int)(tgt / vec) : -1;
}

// o[k] -= d for the one element k == tk (unrolled select, no dynamic register index).
template <int VEC>
__device__ __forceinline__ void sub_at(float (&o)[VEC], int tk, float d) {
#pragma unroll
  for (int k = 0; k < VEC; ++k) o[k] -= (k == tk) ? d : 0.f;
}

// Gradient of one vector: o = softmax * scale - u * scale (- t * scale at the target column),
// times (1 - tanh^2) under softcap.  is_t: the vector holds the target column tk.
template <bool CAP, int VEC>
__device__ __forceinline__ void ce_grad_vec(const float (&e)[VEC], bool is_t, int tk, float off, float sc_p,
                                            float sub, float tsub, const CeParams& p, float (&o)[VEC]) {
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    if constexpr (CAP) {
      const float xc = cap(e[k], p);
      float g = fmaf(ex2(fmaf(xc, kLog2e, off)), sc_p, -sub);
      if (is_t && k == tk) g -= tsub;
      const float t = xc * p.inv_softcap;
      o[k] = g * (1.f - t * t);
    }
  }
  if constexpr (!CAP) {
    // step pairs as paired fp32 (exact per element): (x log2e + off) -> ex2 -> (* sc_p - sub)
    const float2 l2 = make_float2(kLog2e, kLog2e), off2 = make_float2(off, off);
    const float2 sc2 = make_float2(sc_p, sc_p), ms2 = make_float2(-sub, -sub);
#pragma unroll
    for (int k = 0; k < VEC; k += 2) {
      const float2 t = __ffma2_rn(make_float2(e[k], e[k + 1]), l2, off2);
      const float2 r = __ffma2_rn(make_float2(ex2(t.x), ex2(t.y)), sc2, ms2);
      o[k] = r.x;
      o[k + 1] = r.y;
    }
    if (is_t) sub_at<VEC>(o, tk, tsub);
  }
}

// One CTA per row.  Pass 1: online (max, sum of exp) with kBatch independent 16-byte loads per
// thread in flight; pass 2 (fused mode): gradient from the row re-read (an L2 hit).
// CAP: softcap active (tanh on every element and its derivative on the gradient); LS: label
// smoothing (the row sum of x' for the loss).  Without CAP, an element costs one FFMA + ex2 + add
// in pass 1 and FFMA + ex2 + FFMA in pass 2: log2(e), 1/S, the gradient scale and the uniform
// smoothing term are folded into the two FFMA constants, and the target column is corrected once
// per vector, not compared per element.
template <typename T, bool CAP, bool LS>
__global__ void __launch_bounds__(kThreads)
ce_rows_fwd_kernel(float* __restrict__ losses, float* __restrict__ lse_out, float* __restrict__ max_out,
                   float* __restrict__ sum_out, T* __restrict__ grad, const T* __restrict__ logits,
                   const int64_t* __restrict__ targets, int64_t B, int V, CeParams p, float scale_grad,
                   const float* __restrict__ scale_dev, bool vec_ok) {
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float s_m[kThreads / 32], s_s[kThreads / 32], s_x[kThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float scale = scale_grad * (scale_dev ? *scale_dev : 1.f);
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* row = logits + b * V;
    const int64_t tgt = targets[b];
    const bool ignored = (tgt == p.ignore_index);
    float m = -INFINITY, s = 0.f, sx = 0.f;
    const int nvec = vec_ok ? V / VEC : 0;
    int v = tid;
    for (; v + (kBatch - 1) * kThreads < nvec; v += kBatch * kThreads) {
      float e[kBatch][VEC];
#pragma unroll
      for (int q = 0; q < kBatch; ++q) load_frag<T, VEC>(e[q], row + (int64_t)(v + q * kThreads) * VEC);
      float lm = -INFINITY;
#pragma unroll
      for (int q = 0; q < kBatch; ++q)
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          if constexpr (CAP) e[q][k] = cap(e[q][k], p);
          lm = fmaxf(lm, e[q][k]);
          if constexpr (LS) sx += e[q][k];
        }
      const float mn = fmaxf(m, lm);
      if (mn != -INFINITY) {
        const float off = -mn * kLog2e;
        // two running partial sums (paired FFMA for the exponent arguments, paired FADD)
        const float2 l2 = make_float2(kLog2e, kLog2e), off2 = make_float2(off, off);
        float2 acc2 = make_float2(s * ex2(fmaf(m, kLog2e, off)), 0.f);
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
#pragma unroll
          for (int k = 0; k < VEC; k += 2) {
            const float2 t = __ffma2_rn(make_float2(e[q][k], e[q][k + 1]), l2, off2);
            acc2 = __fadd2_rn(acc2, make_float2(ex2(t.x), ex2(t.y)));
          }
        s = acc2.x + acc2.y;
        m = mn;
      }
    }
    for (; v < nvec; v += kThreads) {
      float e[VEC];
      load_frag<T, VEC>(e, row + (int64_t)v * VEC);
      float lm = -INFINITY;
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        if constexpr (CAP) e[k] = cap(e[k], p);
        lm = fmaxf(lm, e[k]);
        if constexpr (LS) sx += e[k];
      }
      const float mn = fmaxf(m, lm);
      if (mn != -INFINITY) {
        const float off = -mn * kLog2e;
        float acc = s * ex2(fmaf(m, kLog2e, off));
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc += ex2(fmaf(e[k], kLog2e, off));
        s = acc;
        m = mn;
      }
    }
    for (int i = nvec * VEC + tid; i < V; i += kThreads) {
      const float e = CAP ? cap(to_f<T>(row[i]), p) : to_f<T>(row[i]);
      if constexpr (LS) sx += e;
      merge(m, s, e, 1.f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, o);
      const float so = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, mo, so);
    }
    if constexpr (LS) sx = warp_sum(sx);
    if (lane == 0) { s_m[warp] = m; s_s[warp] = s; s_x[warp] = sx; }
    __syncthreads();
    float M = -INFINITY, S = 0.f, SX = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) { merge(M, S, s_m[w], s_s[w]); SX += s_x[w]; }
    __syncthreads();
    const float lse = M + lg2(S) * kLn2;
    if (tid == 0) {
      lse_out[b] = lse;
      if (max_out) max_out[b] = M;
      if (sum_out) sum_out[b] = S;
      float loss = 0.f;
      if (!ignored) {
        if (tgt < 0 || tgt >= V) {
          loss = NAN;
        } else {
          const float xt = CAP ? cap(to_f<T>(row[tgt]), p) : to_f<T>(row[tgt]);
          loss = LS ? lse - p.target_coeff * xt - p.ls * (SX / (float)V) : lse - xt;
        }
      }
      losses[b] = loss;
    }
    if (grad != nullptr) {
      T* grow = grad + b * V;
      const float off = -M * kLog2e;
      const float sc_p = scale / S;            // softmax * scale = ex2(x log2e + off) * sc_p
      const float sub = p.ls_uniform * scale;  // uniform smoothing term, scaled
      const float tsub = p.target_coeff * scale;
      const int tv = target_vec(tgt, ignored, V, VEC);
      const int tk = tv >= 0 ? (int)(tgt - (int64_t)tv * VEC) : -1;
      int v = tid;
      if (!ignored) {
        for (; v + (kBatch - 1) * kThreads < nvec; v += kBatch * kThreads) {
          float e[kBatch][VEC];
#pragma unroll
          for (int q = 0; q < kBatch; ++q) load_frag<T, VEC>(e[q], row + (int64_t)(v + q * kThreads) * VEC);
#pragma unroll
          for (int q = 0; q < kBatch; ++q) {
            float o[VEC];
            ce_grad_vec<CAP, VEC>(e[q], v + q * kThreads == tv, tk, off, sc_p, sub, tsub, p, o);
            store_frag<T, VEC>(grow + (int64_t)(v + q * kThreads) * VEC, o);
          }
        }
      }
      for (; v < nvec; v += kThreads) {
        float o[VEC];
        if (ignored) {
#pragma unroll
          for (int k = 0; k < VEC; ++k) o[k] = 0.f;
        } else {
          float e[VEC];
          load_frag<T, VEC>(e, row + (int64_t)v * VEC);
          ce_grad_vec<CAP, VEC>(e, v == tv, tk, off, sc_p, sub, tsub, p, o);
        }
        store_frag<T, VEC>(grow + (int64_t)v * VEC, o);
      }
      for (int i = nvec * VEC + tid; i < V; i += kThreads) {
        float g = 0.f;
        if (!ignored) {
          const float xc = CAP ? cap(to_f<T>(row[i]), p) : to_f<T>(row[i]);
          g = fmaf(ex2(fmaf(xc, kLog2e, off)), sc_p, -sub);
          if (i == tgt) g -= tsub;
          if constexpr (CAP) { const float t = xc * p.inv_softcap; g *= (1.f - t * t); }
        }
        grow[i] = from_f<T>(g);
      }
    }
  }
}

// Tiny-mode backward: recompute softmax from saved (row_max, row_sum), plus the
// optional z-loss gradient z_coef * lse * softmax (kernels/ce_fused.py:672-689):
//   g = (p - t[i==y] - u) * scale + z * lse * p,  times (1 - tanh^2) under softcap,
// i.e. p * (scale + z lse) - (t[i==y] + u) * scale: one FFMA around the ex2 without softcap.
template <typename T, bool CAP>
__global__ void __launch_bounds__(kThreads)
ce_rows_bwd_kernel(T* __restrict__ grad, const T* __restrict__ logits, const int64_t* __restrict__ targets,
                   const float* __restrict__ row_max, const float* __restrict__ row_sum, int64_t B, int V,
                   CeParams p, float scale_h, const float* __restrict__ scale_dev, float z_coef, bool vec_ok) {
  constexpr int VEC = 16 / sizeof(T);
  const int tid = threadIdx.x;
  const float sd = scale_dev ? *scale_dev : 1.f;
  const float scale = scale_h * sd;
  const float zc = z_coef * sd;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* row = logits + b * V;
    T* grow = grad + b * V;
    const int64_t tgt = targets[b];
    const bool ignored = (tgt == p.ignore_index);
    const float M = row_max[b];
    const float lse = M + lg2(row_sum[b]) * kLn2;
    const float off = -M * kLog2e;
    const float sc_p = (scale + zc * lse) / row_sum[b];
    const float sub = p.ls_uniform * scale;
    const float tsub = p.target_coeff * scale;
    const int tv = target_vec(tgt, ignored, V, VEC);
    const int tk = tv >= 0 ? (int)(tgt - (int64_t)tv * VEC) : -1;
    const int nvec = vec_ok ? V / VEC : 0;
    int v = tid;
    if (!ignored) {
      for (; v + (kBatch - 1) * kThreads < nvec; v += kBatch * kThreads) {
        float e[kBatch][VEC];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) load_frag<T, VEC>(e[q], row + (int64_t)(v + q * kThreads) * VEC);
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
          float o[VEC];
          ce_grad_vec<CAP, VEC>(e[q], v + q * kThreads == tv, tk, off, sc_p, sub, tsub, p, o);
          store_frag<T, VEC>(grow + (int64_t)(v + q * kThreads) * VEC, o);
        }
      }
    }
    for (; v < nvec; v += kThreads) {
      float o[VEC];
      if (ignored) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) o[k] = 0.f;
      } else {
        float e[VEC];
        load_frag<T, VEC>(e, row + (int64_t)v * VEC);
        ce_grad_vec<CAP, VEC>(e, v == tv, tk, off, sc_p, sub, tsub, p, o);
      }
      store_frag<T, VEC>(grow + (int64_t)v * VEC, o);
    }
    for (int i = nvec * VEC + tid; i < V; i += kThreads) {
      float g = 0.f;
      if (!ignored) {
        const float xc = CAP ? cap(to_f<T>(row[i]), p) : to_f<T>(row[i]);
        g = fmaf(ex2(fmaf(xc, kLog2e, off)), sc_p, -sub);
        if (i == tgt) g -= tsub;
        if constexpr (CAP) { const float t = xc * p.inv_softcap; g *= (1.f - t * t); }
      }
      grow[i] = from_f<T>(g);
    }
  }
}

// Single-CTA reductions over the row results (no host sync).
__global__ void __launch_bounds__(1024)
ce_reduce_kernel(float* __restrict__ loss_out, float* __restrict__ nvalid_out, const float* __restrict__ losses,
                 const float* __restrict__ lse, const int64_t* __restrict__ targets, int64_t B,
                 int64_t ignore_index, float zw) {
  __shared__ float r0[32], r1[32], r2[32];
  float sl = 0.f, sn = 0.f, sz = 0.f;
  for (int64_t i = threadIdx.x; i < B; i += blockDim.x) {
    const bool valid = targets[i] != ignore_index;
    if (valid) {
      sl += losses[i];
      sn += 1.f;
      if (zw > 0.f && lse) sz += lse[i] * lse[i];
    }
  }
  sl = warp_sum(sl); sn = warp_sum(sn); sz = warp_sum(sz);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { r0[w] = sl; r1[w] = sn; r2[w] = sz; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, n = 0.f, z = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { a += r0[i]; n += r1[i]; z += r2[i]; }
    n = fmaxf(n, 1.f);
    float loss = a / n;
    if (zw > 0.f) loss += zw * z / n;
    if (loss_out) loss_out[0] = loss;
    if (nvalid_out) nvalid_out[0] = n;
  }
}

__global__ void __launch_bounds__(1024)
ce_inv_valid_kernel(float* __restrict__ inv_out, const int64_t* __restrict__ targets, int64_t B,
                    int64_t ignore_index) {
  __shared__ float r[32];
  float n = 0.f;
  for (int64_t i = threadIdx.x; i < B; i += blockDim.x) n += (targets[i] != ignore_index) ? 1.f : 0.f;
  n = warp_sum(n);
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += r[i];
    inv_out[0] = 1.f / fmaxf(t, 1.f);
  }
}

CeParams make_params(float softcap, int64_t ignore_index, float ls, int64_t V) {
  CeParams p;
  p.softcap = softcap > 0.f ? softcap : 0.f;
  p.inv_softcap = softcap > 0.f ? 1.f / softcap : 0.f;
  p.ls = ls > 0.f ? ls : 0.f;
  p.ls_uniform = p.ls / (float)V;
  p.target_coeff = 1.f - p.ls;
  p.ignore_index = ignore_index;
  return p;
}

// CTAs for B rows: the CTAs resident at once (occupancy query), and the same number of rows for
// every CTA, so the rows finish in one round with no partial last wave.
template <typename K>
unsigned row_grid(K kern, int64_t B) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  if (B <= cap) return (unsigned)B;
  const int64_t per = (B + cap - 1) / cap;
  return (unsigned)((B + per - 1) / per);
}

// x *= *scale, read on the device: every CTA returns after one scalar load when the scale
// is 1 (an upstream gradient of exactly one, the usual loss.backward()), so the common
// case moves no tensor bytes and needs no host read of the scalar.
template <typename T>
__global__ void __launch_bounds__(256) scale_by_device_scalar(T* __restrict__ x, int64_t n,
                                                              const float* __restrict__ scale) {
  const float s = __ldg(scale);
  if (s == 1.f) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = from_f<T>(to_f<T>(x[i]) * s);
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_ce_rows_fwd(float* losses, float* lse, float* row_max, float* row_sum, void* grad,
                              const void* logits, const int64_t* targets, int64_t B, int64_t V, float softcap,
                              int64_t ignore_index, float label_smoothing, float scale_grad,
                              const float* scale_dev, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && V > 0 && V < (1LL << 31), AK_ERR_SHAPE, "ak_ce_rows_fwd: bad shape");
  if (B == 0) return AK_OK;
  AK_REQUIRE(losses && lse && logits && targets, AK_ERR_ARG, "ak_ce_rows_fwd: null pointer");
  const CeParams p = make_params(softcap, ignore_index, label_smoothing, V);
  const int es = elem_size(dt);
  const bool vec_ok = aligned16(logits) && (grad == nullptr || aligned16(grad)) && ((V * es) % 16 == 0);
  const bool capf = p.softcap > 0.f, lsf = p.ls > 0.f;
  AK_DISPATCH_DTYPE(dt, T, {
    auto kern = capf ? (lsf ? ce_rows_fwd_kernel<T, true, true> : ce_rows_fwd_kernel<T, true, false>)
                     : (lsf ? ce_rows_fwd_kernel<T, false, true> : ce_rows_fwd_kernel<T, false, false>);
    kern<<<row_grid(kern, B), kThreads, 0, (cudaStream_t)stream>>>(losses, lse, row_max, row_sum, (T*)grad,
                                                             (const T*)logits, targets, B, (int)V, p, scale_grad,
                                                             scale_dev, vec_ok);
  });
  AK_CHECK_LAUNCH("ak_ce_rows_fwd");
  return AK_OK;
}

extern "C" int ak_ce_rows_bwd(void* grad, const void* logits, const int64_t* targets, const float* row_max,
                              const float* row_sum, int64_t B, int64_t V, float softcap, int64_t ignore_index,
                              float label_smoothing, float scale, const float* scale_dev, float z_coef, int dt,
                              void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && V > 0 && V < (1LL << 31), AK_ERR_SHAPE, "ak_ce_rows_bwd: bad shape");
  if (B == 0) return AK_OK;
  AK_REQUIRE(grad && logits && targets && row_max && row_sum, AK_ERR_ARG, "ak_ce_rows_bwd: null pointer");
  const CeParams p = make_params(softcap, ignore_index, label_smoothing, V);
  const int es = elem_size(dt);
  const bool vec_ok = aligned16(logits) && aligned16(grad) && ((V * es) % 16 == 0);
  const bool capf = p.softcap > 0.f;
  AK_DISPATCH_DTYPE(dt, T, {
    auto kern = capf ? ce_rows_bwd_kernel<T, true> : ce_rows_bwd_kernel<T, false>;
    kern<<<row_grid(kern, B), kThreads, 0, (cudaStream_t)stream>>>((T*)grad, (const T*)logits, targets, row_max,
                                                             row_sum, B, (int)V, p, scale, scale_dev, z_coef,
                                                             vec_ok);
  });
  AK_CHECK_LAUNCH("ak_ce_rows_bwd");
  return AK_OK;
}

extern "C" int ak_ce_rows_reduce(float* loss_out, float* n_valid_out, const float* losses, const float* lse,
                                 const int64_t* targets, int64_t B, int64_t ignore_index, float z_loss_weight,
                                 void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && (B == 0 || (losses && targets)), AK_ERR_ARG, "ak_ce_rows_reduce: bad args");
  AK_REQUIRE(z_loss_weight <= 0.f || lse || B == 0, AK_ERR_ARG, "ak_ce_rows_reduce: z-loss needs lse");
  ce_reduce_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(loss_out, n_valid_out, losses, lse, targets, B,
                                                         ignore_index, z_loss_weight);
  AK_CHECK_LAUNCH("ak_ce_rows_reduce");
  return AK_OK;
}

extern "C" int ak_ce_inv_valid(float* inv_out, const int64_t* targets, int64_t B, int64_t ignore_index,
                               void* stream) {
  clear_error();
  AK_REQUIRE(inv_out && B >= 0 && (B == 0 || targets), AK_ERR_ARG, "ak_ce_inv_valid: bad args");
  ce_inv_valid_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(inv_out, targets, B, ignore_index);
  AK_CHECK_LAUNCH("ak_ce_inv_valid");
  return AK_OK;
}

extern "C" int ak_scale_by_device_scalar(void* x, int64_t n, const float* scale, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(n >= 0 && (n == 0 || (x && scale)), AK_ERR_ARG, "ak_scale_by_device_scalar: bad args");
  if (n == 0) return AK_OK;
  const int64_t g = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  AK_DISPATCH_DTYPE(dt, T,
                    scale_by_device_scalar<T><<<(unsigned)g, 256, 0, (cudaStream_t)stream>>>((T*)x, n, scale));
  AK_CHECK_LAUNCH("ak_scale_by_device_scalar");
  return AK_OK;
}
