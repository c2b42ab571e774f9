// Collapsed (one state per channel) selective scan, fp32, layout (B, L, d).
//
// Reference: kernels/hip/selective_scan.py:50-163 (forward) and the sequential
// autograd fallback kernels/hip/_torch_ops.py:335-389 (backward):
//   h_t = dA_t h_{t-1} + dBx_t,  y_t = C_t h_t + D x_t
//   g_t = gy_t C_t + dA_{t+1} g_{t+1}
//   gdA_t = g_t h_{t-1},  gdBx_t = g_t,  gC_t = gy_t h_t,  gx_t = gy_t D,  gD = sum gy x
//
// Design: a CTA owns 32 adjacent channels (lane = channel, so every warp-wide
// access is one 128-byte line) of one batch row and walks L in chunks of
// 8 warps x SEG steps.  Each warp scans its SEG steps sequentially in
// registers, the 8 per-warp aggregates (prod a, local h) are combined through
// shared memory, and the chunk's carry moves on to the next chunk inside the
// CTA — no inter-CTA dependency, each input element read once in the forward.
// The backward first re-derives the chunk-start states (reads dA, dBx only),
// then sweeps the chunks in reverse with the same two-level scan for g.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kW = 8;  // warps per CTA

// All loads of a segment are unconditional (indices clamped into range, values
// masked afterwards), so a warp issues its 4*SEG loads back to back instead of
// one dependent round trip per guarded step; only the stores are guarded.
template <int SEG>
__global__ void __launch_bounds__(kW * 32)
scan1_fwd_kernel(float* __restrict__ y, float* __restrict__ carries, const float* __restrict__ dA,
                 const float* __restrict__ dBx, const float* __restrict__ Cm, const float* __restrict__ Dv,
                 const float* __restrict__ x, int L, int d, int nchunk) {
  __shared__ float sP[2][kW][32], sH[2][kW][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int64_t b = blockIdx.y;
  const bool cv = c < d;
  const float Dc = (cv && Dv) ? Dv[c] : 0.f;
  const int64_t base = b * (int64_t)L * d + (cv ? c : d - 1);
  constexpr int CH = kW * SEG;
  float carry = 0.f;
  int par = 0, ci = 0;
  for (int t0 = 0; t0 < L; t0 += CH, par ^= 1, ++ci) {
    // chunk-start state h_{t0-1} for the backward (the carry pass's output, saved here)
    if (carries != nullptr && warp == 0 && cv) carries[((int64_t)b * nchunk + ci) * d + c] = carry;
    const int tw = t0 + warp * SEG;
    float a[SEG], bb[SEG], cc[SEG], xx[SEG];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const int64_t off = base + (int64_t)min(tw + i, L - 1) * d;
      a[i] = __ldcs(dA + off);
      bb[i] = __ldcs(dBx + off);
      cc[i] = __ldcs(Cm + off);
      xx[i] = __ldcs(x + off);
    }
#pragma unroll
    for (int i = 0; i < SEG; ++i)
      if (!(cv && tw + i < L)) { a[i] = 1.f; bb[i] = 0.f; }
    float P = 1.f, H = 0.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i) { H = fmaf(a[i], H, bb[i]); P *= a[i]; }
    sP[par][warp][lane] = P;
    sH[par][warp][lane] = H;
    __syncthreads();
    float h = carry, nc = carry;
#pragma unroll
    for (int k = 0; k < kW; ++k) {
      const float pk = sP[par][k][lane], hk = sH[par][k][lane];
      if (k < warp) h = fmaf(pk, h, hk);
      nc = fmaf(pk, nc, hk);
    }
    carry = nc;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const int t = tw + i;
      h = fmaf(a[i], h, bb[i]);
      const float yv = fmaf(cc[i], h, Dc * xx[i]);
      if (cv && t < L) __stcs(y + base + (int64_t)t * d, yv);
    }
  }
}

// Pass 1 of the backward: chunk-start states h_{t0-1} -> carries[b, chunk, c].
template <int SEG>
__global__ void __launch_bounds__(kW * 32)
scan1_carry_kernel(float* __restrict__ carries, const float* __restrict__ dA, const float* __restrict__ dBx,
                   int L, int d, int nchunk) {
  __shared__ float sP[2][kW][32], sH[2][kW][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int64_t b = blockIdx.y;
  const bool cv = c < d;
  const int64_t cbase = b * (int64_t)L * d + (cv ? c : d - 1);
  constexpr int CH = kW * SEG;
  float carry = 0.f;
  int par = 0, ci = 0;
  for (int t0 = 0; t0 < L; t0 += CH, par ^= 1, ++ci) {
    if (warp == 0 && cv) carries[(b * nchunk + ci) * d + c] = carry;
    const int tw = t0 + warp * SEG;
    float av[SEG], bv[SEG];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {  // unconditional (clamped) loads, masked values
      const int64_t off = cbase + (int64_t)min(tw + i, L - 1) * d;
      av[i] = dA[off];
      bv[i] = dBx[off];
    }
    float P = 1.f, H = 0.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i)
      if (cv && tw + i < L) { H = fmaf(av[i], H, bv[i]); P *= av[i]; }
    sP[par][warp][lane] = P;
    sH[par][warp][lane] = H;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kW; ++k) carry = fmaf(sP[par][k][lane], carry, sH[par][k][lane]);
  }
}

// Pass 2: reverse sweep.  gD partial per (b, c) into gdpart[b, c].
template <int SEG>
__global__ void __launch_bounds__(kW * 32)
scan1_bwd_kernel(float* __restrict__ gdA, float* __restrict__ gdBx, float* __restrict__ gC,
                 float* __restrict__ gx, float* __restrict__ gdpart, const float* __restrict__ carries,
                 const float* __restrict__ dA, const float* __restrict__ dBx, const float* __restrict__ Cm,
                 const float* __restrict__ Dv, const float* __restrict__ x, const float* __restrict__ gy,
                 int L, int d, int nchunk) {
  __shared__ float sP[2][kW][32], sH[2][kW][32], sQ[2][kW][32], sG[2][kW][32];
  __shared__ float sD[kW][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int64_t b = blockIdx.y;
  const bool cv = c < d;
  const float Dc = (cv && Dv) ? Dv[c] : 0.f;
  const int64_t base = b * (int64_t)L * d + c;
  const int64_t cbase = b * (int64_t)L * d + (cv ? c : d - 1);  // clamped, for unconditional loads
  constexpr int CH = kW * SEG;
  float gcarry = 0.f, gdacc = 0.f;
  int par = 0;
  for (int ci = nchunk - 1; ci >= 0; --ci, par ^= 1) {
    const int t0 = ci * CH;
    const int tw = t0 + warp * SEG;
    float a[SEG + 1], bb[SEG], rb[SEG], gyv[SEG], xv[SEG];
    // unconditional (clamped) loads first, then the masks: all 5*SEG+1 loads in flight
#pragma unroll
    for (int i = 0; i <= SEG; ++i) a[i] = dA[cbase + (int64_t)min(tw + i, L - 1) * d];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const int64_t off = cbase + (int64_t)min(tw + i, L - 1) * d;
      bb[i] = dBx[off];
      gyv[i] = gy[off];
      rb[i] = Cm[off];
      xv[i] = x[off];
    }
#pragma unroll
    for (int i = 0; i <= SEG; ++i)
      if (!(cv && tw + i < L)) a[i] = (i < SEG ? 1.f : 0.f);
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const bool ok = cv && tw + i < L;
      if (!ok) { bb[i] = 0.f; gyv[i] = 0.f; xv[i] = 0.f; }
      rb[i] = gyv[i] * rb[i];
      gdacc = fmaf(gyv[i], xv[i], gdacc);
    }
    // forward aggregates (prod a, local h) and reverse aggregates (prod a', local g)
    float P = 1.f, H = 0.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i) { H = fmaf(a[i], H, bb[i]); P *= a[i]; }
    float Q = 1.f, G = 0.f;
#pragma unroll
    for (int i = SEG - 1; i >= 0; --i) { G = fmaf(a[i + 1], G, rb[i]); Q *= a[i + 1]; }
    sP[par][warp][lane] = P; sH[par][warp][lane] = H;
    sQ[par][warp][lane] = Q; sG[par][warp][lane] = G;
    __syncthreads();
    float h = cv ? carries[(b * nchunk + ci) * d + c] : 0.f;
#pragma unroll
    for (int k = 0; k < kW; ++k)
      if (k < warp) h = fmaf(sP[par][k][lane], h, sH[par][k][lane]);
    float g = gcarry, ng = gcarry;
#pragma unroll
    for (int k = kW - 1; k >= 0; --k) {
      const float qk = sQ[par][k][lane], gk = sG[par][k][lane];
      if (k > warp) g = fmaf(qk, g, gk);
      ng = fmaf(qk, ng, gk);
    }
    gcarry = ng;
    float hprev[SEG];
#pragma unroll
    for (int i = 0; i < SEG; ++i) { hprev[i] = h; h = fmaf(a[i], h, bb[i]); }
#pragma unroll
    for (int i = SEG - 1; i >= 0; --i) {
      g = fmaf(a[i + 1], g, rb[i]);
      const int t = tw + i;
      if (cv && t < L) {
        const int64_t off = base + (int64_t)t * d;
        gdA[off] = g * hprev[i];
        gdBx[off] = g;
        gC[off] = gyv[i] * fmaf(a[i], hprev[i], bb[i]);
        gx[off] = gyv[i] * Dc;
      }
    }
  }
  sD[warp][lane] = gdacc;
  __syncthreads();
  if (warp == 0 && cv) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kW; ++k) s += sD[k][lane];
    gdpart[b * d + c] = s;
  }
  pdl_trigger();
}

__global__ void scan1_gd_reduce(float* __restrict__ gD, const float* __restrict__ part, int B, int d) {
  pdl_wait();  // the backward kernel's per-(b, c) partials are complete and visible
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = 0.f;
#pragma unroll 8  // independent loads in flight; the adds stay in index order
  for (int b = 0; b < B; ++b) s += part[(int64_t)b * d + c];
  gD[c] = s;
}

constexpr int kSegF = 8, kSegB = 8;
static_assert(kSegF == kSegB, "the forward saves the backward's chunk-start states: same chunking");
inline int nchunk_bwd(int64_t L) { return (int)((L + kW * kSegB - 1) / (kW * kSegB)); }

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_scan1_fwd_ex(float* y, float* carries, const float* dA, const float* dBx, const float* C,
                               const float* D, const float* x, int64_t B, int64_t L, int64_t d, void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && L >= 0 && d >= 0 && B < 65536 && L < (1LL << 31) && d < (1LL << 31), AK_ERR_SHAPE,
             "ak_scan1_fwd: bad shape");
  if (B == 0 || L == 0 || d == 0) return AK_OK;
  AK_REQUIRE(y && dA && dBx && C && x, AK_ERR_ARG, "ak_scan1_fwd: null pointer");
  dim3 grid((unsigned)((d + 31) / 32), (unsigned)B);
  scan1_fwd_kernel<kSegF><<<grid, kW * 32, 0, (cudaStream_t)stream>>>(y, carries, dA, dBx, C, D, x, (int)L, (int)d,
                                                                      nchunk_bwd(L));
  AK_CHECK_LAUNCH("ak_scan1_fwd");
  return AK_OK;
}

extern "C" int ak_scan1_fwd(float* y, const float* dA, const float* dBx, const float* C, const float* D,
                            const float* x, int64_t B, int64_t L, int64_t d, void* stream) {
  return ak_scan1_fwd_ex(y, nullptr, dA, dBx, C, D, x, B, L, d, stream);
}

extern "C" int ak_scan1_carries_size(int64_t B, int64_t L, int64_t d, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes && B >= 0 && L >= 0 && d >= 0, AK_ERR_ARG, "ak_scan1_carries_size: bad args");
  *bytes = (size_t)B * nchunk_bwd(L) * d * sizeof(float);
  return AK_OK;
}

extern "C" int ak_scan1_bwd_workspace_size(int64_t B, int64_t L, int64_t d, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes && B >= 0 && L >= 0 && d >= 0, AK_ERR_ARG, "ak_scan1_bwd_workspace_size: bad args");
  *bytes = ((size_t)B * nchunk_bwd(L) * d + (size_t)B * d) * sizeof(float);
  return AK_OK;
}

extern "C" int ak_scan1_bwd_ex(float* gdA, float* gdBx, float* gC, float* gD, float* gx, void* workspace,
                               size_t ws_bytes, const float* carries_in, const float* dA, const float* dBx,
                               const float* C, const float* D, const float* x, const float* gy, int64_t B,
                               int64_t L, int64_t d, void* stream) {
  clear_error();
  AK_REQUIRE(B >= 0 && L >= 0 && d >= 0 && B < 65536 && L < (1LL << 31) && d < (1LL << 31), AK_ERR_SHAPE,
             "ak_scan1_bwd: bad shape");
  if (d == 0) return AK_OK;
  AK_REQUIRE(gD, AK_ERR_ARG, "ak_scan1_bwd: null gD");
  cudaStream_t st = (cudaStream_t)stream;
  if (B == 0 || L == 0) {
    AK_CUDA_TRY(cudaMemsetAsync(gD, 0, (size_t)d * sizeof(float), st), "ak_scan1_bwd: memset");
    return AK_OK;
  }
  AK_REQUIRE(gdA && gdBx && gC && gx && dA && dBx && C && x && gy, AK_ERR_ARG, "ak_scan1_bwd: null pointer");
  const int nch = nchunk_bwd(L);
  const size_t ncarry = carries_in ? 0 : (size_t)B * nch * d;
  const size_t need = (ncarry + (size_t)B * d) * sizeof(float);
  AK_REQUIRE(workspace && ws_bytes >= need, AK_ERR_WORKSPACE, "ak_scan1_bwd: workspace %zu < %zu", ws_bytes, need);
  float* gdpart = (float*)workspace + ncarry;
  dim3 grid((unsigned)((d + 31) / 32), (unsigned)B);
  const float* carries = carries_in;
  if (carries == nullptr) {  // no saved chunk-start states: re-derive them (reads dA, dBx once more)
    float* cw = (float*)workspace;
    scan1_carry_kernel<kSegB><<<grid, kW * 32, 0, st>>>(cw, dA, dBx, (int)L, (int)d, nch);
    AK_CHECK_LAUNCH("ak_scan1_bwd(carries)");
    carries = cw;
  }
  scan1_bwd_kernel<kSegB><<<grid, kW * 32, 0, st>>>(gdA, gdBx, gC, gx, gdpart, carries, dA, dBx, C, D, x, gy,
                                                    (int)L, (int)d, nch);
  AK_CHECK_LAUNCH("ak_scan1_bwd");
  AK_CUDA_TRY(launch_pdl(scan1_gd_reduce, dim3((unsigned)((d + 255) / 256)), dim3(256), 0, st, gD,
                         (const float*)gdpart, (int)B, (int)d),
              "ak_scan1_bwd(gD)");
  AK_CHECK_LAUNCH("ak_scan1_bwd(gD)");
  return AK_OK;
}

extern "C" int ak_scan1_bwd(float* gdA, float* gdBx, float* gC, float* gD, float* gx, void* workspace,
                            size_t ws_bytes, const float* dA, const float* dBx, const float* C, const float* D,
                            const float* x, const float* gy, int64_t B, int64_t L, int64_t d, void* stream) {
  return ak_scan1_bwd_ex(gdA, gdBx, gC, gD, gx, workspace, ws_bytes, nullptr, dA, dBx, C, D, x, gy, B, L, d,
                         stream);
}
