// Rotary position embedding (interleaved pairs) forward / backward, sm_100a.
//
// Semantics: reference.rotary_embedding_ref (reference.py:63-69) and
// kernels/hip/rotary_embedding.py kernel_fn / kernel_fn_fp32 (:253-300):
//   y[..., 2i]   = x[..., 2i] * cos[n, i] - x[..., 2i+1] * sin[n, i]
//   y[..., 2i+1] = x[..., 2i] * sin[n, i] + x[..., 2i+1] * cos[n, i]
// fp32 arithmetic with fp32 cos / sin tables of shape (N, D/2), one rounding.
// The backward is the rotation by -theta on the same pairs (sign = -1):
//   dx[2i] = g[2i] c + g[2i+1] s,   dx[2i+1] = -g[2i] s + g[2i+1] c.
//
// Layout: x is read and y written through arbitrary (b, h, n) element strides
// with unit stride along D.  ak_rope_fwd / ak_rope_bwd write y dense
// (B, H, N, D), so q / k are read straight out of a fused (B, N, W) QKV
// projection and leave head-major; ak_rope_strided also takes y's strides, so
// the gradients of q, k and v are written straight into their columns of one
// packed (B, N, W) gradient (mode 0 copies without rotating, for v).  One
// thread rotates one 16-byte vector position (8 elements of a 16-bit type, 4
// of fp32) in several (b, h) planes.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kThreadsR = 256;

constexpr int kPlanesPerCta = 8;  // (b, h) planes one thread walks with the same (n, vector)

// Vector path: a thread owns one 16-byte vector position (n, j) of a (N, D)
// plane, loads its cos / sin once and applies them to kPlanesPerCta planes
// (grid.y): per plane only an address step, one load, the rotation and one
// store.  grid.x covers the N*D/VEC vector positions.
// ROT false: plain strided copy (no tables read).  DENSE: y is dense (B, H, N, D) and its
// address is one multiply-add per plane (the strided form keeps two more 64-bit strides live).
template <typename T, int VEC, bool FULL, bool ROT = true, bool DENSE = false>
__global__ void __launch_bounds__(kThreadsR, 6)
rope_kernel(T* __restrict__ y, const T* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
            int64_t planes, int H, int N, int D, int64_t sb, int64_t sh, int64_t sn_, int64_t yb, int64_t yh,
            int64_t yn, float sign, bool tab4) {
  const int vpr = D / VEC;
  const int per_plane = N * vpr;
  const int half = D / 2;
  const int idx = blockIdx.x * kThreadsR + threadIdx.x;
  if (!FULL && idx >= per_plane) return;
  const int n = idx / vpr;
  const int jb = (idx - n * vpr) * VEC;
  float c[VEC / 2], s[VEC / 2];
  const float* cr = ROT ? cs + (int64_t)n * half + jb / 2 : nullptr;
  const float* sr = ROT ? sn + (int64_t)n * half + jb / 2 : nullptr;
  if constexpr (!ROT) {
#pragma unroll
    for (int k = 0; k < VEC / 2; ++k) { c[k] = 1.f; s[k] = 0.f; }
  } else if constexpr (VEC / 2 == 4) {
    if (tab4) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(cr));
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(sr));
      c[0] = c4.x; c[1] = c4.y; c[2] = c4.z; c[3] = c4.w;
      s[0] = s4.x; s[1] = s4.y; s[2] = s4.z; s[3] = s4.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) { c[k] = __ldg(cr + k); s[k] = __ldg(sr + k); }
    }
  } else {
#pragma unroll
    for (int k = 0; k < VEC / 2; ++k) { c[k] = __ldg(cr + k); s[k] = __ldg(sr + k); }
  }
#pragma unroll
  for (int k = 0; k < VEC / 2; ++k) s[k] *= sign;
  const int64_t xo = (int64_t)n * sn_ + jb, yo = DENSE ? (int64_t)n * D + jb : (int64_t)n * yn + jb;
  const int64_t ystep = (int64_t)N * D;
  const int64_t p0 = (int64_t)blockIdx.y * kPlanesPerCta;
  const int64_t p1 = p0 + kPlanesPerCta < planes ? p0 + kPlanesPerCta : planes;
  int64_t b = p0 / H;
  int h = (int)(p0 - b * H);
  // running element pointers: + (head stride) per plane, re-based when the head index wraps
  const T* xp = x + b * sb + h * sh + xo;
  T* yp = y + (DENSE ? p0 * ystep : b * yb + h * yh) + yo;
#pragma unroll 2
  for (int64_t p = p0; p < p1; ++p) {
    if constexpr (ROT) {
      float v[VEC], o[VEC];
      load_frag<T, VEC>(v, xp);
#pragma unroll
      for (int k = 0; k < VEC / 2; ++k) {
        o[2 * k] = v[2 * k] * c[k] - v[2 * k + 1] * s[k];
        o[2 * k + 1] = v[2 * k] * s[k] + v[2 * k + 1] * c[k];
      }
      store_frag<T, VEC>(yp, o);
    } else {
      *reinterpret_cast<int4*>(yp) = *reinterpret_cast<const int4*>(xp);
    }
    if (++h == H) {
      h = 0;
      ++b;
      xp = x + b * sb + xo;
      yp = DENSE ? yp + ystep : y + b * yb + yo;
    } else {
      xp += sh;
      yp += DENSE ? ystep : yh;
    }
  }
}

// Scalar path (one pair per thread) for D not a multiple of the vector width.
template <typename T>
__global__ void __launch_bounds__(kThreadsR)
rope_pair_kernel(T* __restrict__ y, const T* __restrict__ x, const float* __restrict__ cs,
                 const float* __restrict__ sn, int64_t rows, int H, int N, int D, int64_t sb, int64_t sh,
                 int64_t sn_, int64_t yb, int64_t yh, int64_t yn, float sign, bool rot) {
  const int half = D / 2;
  const int64_t total = rows * half;
  for (int64_t t = (int64_t)blockIdx.x * kThreadsR + threadIdx.x; t < total; t += (int64_t)gridDim.x * kThreadsR) {
    const int64_t row = t / half;
    const int i = (int)(t - row * half);
    const int n = (int)(row % N);
    const int64_t bh = row / N;
    const int h = (int)(bh % H);
    const int64_t b = bh / H;
    const T* xr = x + b * sb + h * sh + (int64_t)n * sn_;
    const float x0 = to_f<T>(xr[2 * i]), x1 = to_f<T>(xr[2 * i + 1]);
    const float c = rot ? cs[(int64_t)n * half + i] : 1.f, s = rot ? sign * sn[(int64_t)n * half + i] : 0.f;
    T* yr = y + b * yb + h * yh + (int64_t)n * yn;
    yr[2 * i] = from_f<T>(x0 * c - x1 * s);
    yr[2 * i + 1] = from_f<T>(x0 * s + x1 * c);
  }
}

// sign: +1 rotate by theta, -1 by -theta, 0 copy.  y strides (yb, yh, yn); unit stride along D.
int rope_impl(void* y, const void* x, const float* cos_t, const float* sin_t, int64_t B, int64_t H, int64_t N,
              int64_t D, int64_t sb, int64_t sh, int64_t sn, int64_t yb, int64_t yh, int64_t yn, float sign, int dt,
              cudaStream_t st, const char* who) {
  AK_REQUIRE(B >= 0 && H > 0 && N > 0 && D > 0 && D % 2 == 0 && H < (1LL << 31) && N < (1LL << 31) &&
                 D < (1LL << 31),
             AK_ERR_SHAPE, "%s: bad shape B=%lld H=%lld N=%lld D=%lld (D must be even)", who, (long long)B,
             (long long)H, (long long)N, (long long)D);
  if (B == 0) return AK_OK;
  const bool rot = sign != 0.f;
  AK_REQUIRE(y && x && (!rot || (cos_t && sin_t)), AK_ERR_ARG, "%s: null pointer", who);
  const int64_t rows = B * H * N;
  const int es = elem_size(dt);
  const int vecw = 16 / es;
  const bool vec_ok = D % vecw == 0 && aligned16(x) && aligned16(y) && (sb * es) % 16 == 0 && (sh * es) % 16 == 0 &&
                      (sn * es) % 16 == 0 && (yb * es) % 16 == 0 && (yh * es) % 16 == 0 && (yn * es) % 16 == 0;
  const bool tab4 = rot && aligned16(cos_t) && aligned16(sin_t) && (D / 2) % 4 == 0;
  AK_REQUIRE(!vec_ok || N * (D / vecw) < (1LL << 31), AK_ERR_SHAPE, "%s: N*D too large", who);
  AK_REQUIRE(!vec_ok || (B * H + kPlanesPerCta - 1) / kPlanesPerCta < 65536, AK_ERR_SHAPE,
             "%s: more than %d (b, h) planes", who, 65535 * kPlanesPerCta);
  AK_DISPATCH_DTYPE(dt, T, {
    constexpr int VEC = 16 / sizeof(T);
    if (vec_ok) {
      const int64_t per_plane = N * (D / VEC);
      const unsigned gx = (unsigned)((per_plane + kThreadsR - 1) / kThreadsR);
      const int64_t planes = B * H;
      const unsigned gy = (unsigned)((planes + kPlanesPerCta - 1) / kPlanesPerCta);
      const dim3 grid(gx, gy);
      const bool full = per_plane % kThreadsR == 0;
      const bool dense = yn == D && yh == N * D && yb == H * N * D;
      auto kern = rot ? (dense ? (full ? rope_kernel<T, VEC, true, true, true> : rope_kernel<T, VEC, false, true, true>)
                               : (full ? rope_kernel<T, VEC, true, true> : rope_kernel<T, VEC, false, true>))
                      : (full ? rope_kernel<T, VEC, true, false> : rope_kernel<T, VEC, false, false>);
      kern<<<grid, kThreadsR, 0, st>>>((T*)y, (const T*)x, cos_t, sin_t, planes, (int)H, (int)N, (int)D, sb, sh, sn,
                                       yb, yh, yn, sign, tab4);
    } else {
      int64_t g = (rows * (D / 2) + kThreadsR - 1) / kThreadsR;
      const int64_t cap = (int64_t)sm_count() * 32;
      if (g > cap) g = cap;
      if (g < 1) g = 1;
      rope_pair_kernel<T><<<(unsigned)g, kThreadsR, 0, st>>>((T*)y, (const T*)x, cos_t, sin_t, rows, (int)H, (int)N,
                                                            (int)D, sb, sh, sn, yb, yh, yn, sign, rot);
    }
  });
  AK_CHECK_LAUNCH(who);
  return AK_OK;
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_rope_fwd(void* y, const void* x, const float* cos_t, const float* sin_t, int64_t B, int64_t H,
                           int64_t N, int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_n, int dt,
                           void* stream) {
  clear_error();
  return rope_impl(y, x, cos_t, sin_t, B, H, N, D, stride_b, stride_h, stride_n, H * N * D, N * D, D, 1.f, dt,
                   (cudaStream_t)stream, "ak_rope_fwd");
}

extern "C" int ak_rope_bwd(void* dx, const void* dy, const float* cos_t, const float* sin_t, int64_t B, int64_t H,
                           int64_t N, int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_n, int dt,
                           void* stream) {
  clear_error();
  return rope_impl(dx, dy, cos_t, sin_t, B, H, N, D, stride_b, stride_h, stride_n, H * N * D, N * D, D, -1.f, dt,
                   (cudaStream_t)stream, "ak_rope_bwd");
}

extern "C" int ak_rope_strided(void* y, const void* x, const float* cos_t, const float* sin_t, int64_t B, int64_t H,
                               int64_t N, int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_sn, int64_t y_sb,
                               int64_t y_sh, int64_t y_sn, int mode, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(mode == 1 || mode == -1 || mode == 0, AK_ERR_ARG, "ak_rope_strided: mode must be 1, -1 or 0, got %d",
             mode);
  return rope_impl(y, x, cos_t, sin_t, B, H, N, D, x_sb, x_sh, x_sn, y_sb, y_sh, y_sn, (float)mode, dt,
                   (cudaStream_t)stream, "ak_rope_strided");
}
