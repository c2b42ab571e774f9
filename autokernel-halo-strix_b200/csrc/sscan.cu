// Mamba-style selective scan (N states per channel), forward + backward, sm_100a.
//
// Semantics: selective_scan_ref (external/mamba/mamba_ssm/ops/selective_scan_interface.py:115-181),
// the interface SelectiveScanFn (same file, :23-83):
//   delta' = softplus(delta + bias)            (if delta_softplus, threshold 20)
//   h_t[n] = exp(delta'_t A[d,n]) h_{t-1}[n] + delta'_t B[b,g,n,t] u_t
//   y_t    = sum_n C[b,g,n,t] h_t[n] + D[d] u_t,   out = y * silu(z)
//
// Layout: u, delta, z, out (batch, dim, L) with L contiguous; B, C
// (batch, groups, N, L); A (dim, N) fp32; state fp32.
//
// Forward design.  A CTA owns `cpc` channels of one batch row (all in one
// B/C group) and walks L in chunks of 32 lanes x ITEMS steps.  The chunk's
// B and C tiles (N x chunk, shared by every channel of the CTA) are staged
// into shared memory by the bulk-copy (TMA) engine into a double buffer
// completed on mbarriers, so HBM/L2 traffic for B/C is paid once per CTA.
// Each warp scans one channel at a time: per state n every lane runs its
// ITEMS steps sequentially in registers (one SFU exp2 per step), the 32 lane
// aggregates are combined with a 5-step shuffle scan, and the chunk carry
// (one fp32 per channel and state) lives in shared memory.  The state after
// every kStateStride steps is saved for the backward.
//
// Backward design.  Same CTA/chunk structure, chunks visited in reverse.
// Per chunk and state the forward states are recomputed from the saved
// chunk-start state (no full state tensor in HBM), then the adjoint
// g_t = dy_t C_t + a_{t+1} g_{t+1} is scanned right-to-left with the same
// two-level (lane-sequential + shuffle) scheme; the adjoint carry crosses
// chunks pre-multiplied by a at the chunk's first step.  dB/dC (sums over the
// channels of a group) are reduced in shared memory across the CTA's channels
// and flushed once per chunk with fp32 global reductions; dA/dD/dbias are
// per-(batch, channel) partials reduced in a fixed order by a second kernel.
#include "ak_common.cuh"

#include <algorithm>

namespace ak {
namespace {

constexpr int kStateStride = 256;  // timesteps between saved states
constexpr int kItemsF = 16;        // forward steps per lane (chunk 512)
constexpr int kItemsB = 8;         // backward steps per lane (chunk 256 == stride)
static_assert(32 * kItemsB == kStateStride, "backward chunk must equal the state stride");
static_assert((32 * kItemsF) % kStateStride == 0, "forward chunk must be a multiple of the stride");

__device__ int g_sscan_err;  // AK_ERR_TIMEOUT if a bounded wait gave up

struct SsParams {
  const void* u;
  const void* delta;
  const float* A;
  const void* Bm;
  const void* Cm;
  const float* D;
  const void* z;
  const float* bias;
  const void* dout;
  const float* chunk_states_in;
  void* out;
  float* last_state;
  float* chunk_states;
  // backward outputs
  void* du;
  void* ddelta;
  void* dz;
  float* dB_acc;
  float* dC_acc;
  float* part;  // [batch][dim][N+2]
  int batch, dim, L, N, groups, dpg, nw, cpw, nsaved, nbuf;
  int softplus, bulk, vec_io;
};

__device__ __forceinline__ float softplus_f(float x) { return x <= 20.f ? log1pf(__expf(x)) : x; }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// Load ITEMS consecutive elements starting at position t of a length-L row.
template <typename T, int ITEMS>
__device__ __forceinline__ void load_items(float (&v)[ITEMS], const T* row, int t, int L, bool vec) {
  constexpr int VEC = 16 / sizeof(T);
  if (vec && t + ITEMS <= L) {
#pragma unroll
    for (int i = 0; i < ITEMS; i += VEC) {
      float f[VEC];
      load_frag<T, VEC>(f, row + t + i);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[i + k] = f[k];
    }
  } else {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) v[i] = (t + i < L) ? to_f<T>(row[t + i]) : 0.f;
  }
}

template <typename T, int ITEMS>
__device__ __forceinline__ void store_items(T* row, const float (&v)[ITEMS], int t, int L, bool vec) {
  constexpr int VEC = 16 / sizeof(T);
  if (vec && t + ITEMS <= L) {
#pragma unroll
    for (int i = 0; i < ITEMS; i += VEC) {
      float f[VEC];
#pragma unroll
      for (int k = 0; k < VEC; ++k) f[k] = v[i + k];
      store_frag<T, VEC>(row + t + i, f);
    }
  } else {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i)
      if (t + i < L) row[t + i] = from_f<T>(v[i]);
  }
}

// ITEMS consecutive elements of a shared-memory tile row (16-byte aligned).
template <typename T, int ITEMS>
__device__ __forceinline__ void load_smem_items(float (&v)[ITEMS], const T* p) {
  constexpr int VEC = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < ITEMS; i += VEC) {
    float f[VEC];
    load_frag<T, VEC>(f, p + i);
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[i + k] = f[k];
  }
}

// Stage the B and C tiles [N][CH] of chunk starting at t0 into buffer `buf`.
// Bulk path: one thread issues 2N row copies completing on bars[buf].
// Cooperative path (unaligned L): all threads copy; caller syncs.
template <typename T, int CH>
__device__ __forceinline__ void stage_bc(const SsParams& p, T* Bs, T* Cs, uint64_t* bars, int buf, int t0,
                                         const T* Bg, const T* Cg, bool bulk_issue) {
  const int N = p.N, L = p.L;
  const int len = min(CH, L - t0);
  T* bdst = Bs + (size_t)buf * N * CH;
  T* cdst = Cs + (size_t)buf * N * CH;
  if (p.bulk) {
    if (bulk_issue) {
      const uint32_t bytes = (uint32_t)(len * sizeof(T));
      mbar_arrive_expect_tx(&bars[buf], 2u * N * bytes);
      for (int n = 0; n < N; ++n) {
        bulk_g2s(bdst + n * CH, Bg + (int64_t)n * L + t0, bytes, &bars[buf]);
        bulk_g2s(cdst + n * CH, Cg + (int64_t)n * L + t0, bytes, &bars[buf]);
      }
    }
  } else {
    for (int idx = threadIdx.x; idx < N * CH; idx += blockDim.x) {
      const int n = idx / CH, t = idx - n * CH;
      const bool ok = t < len;
      bdst[idx] = ok ? Bg[(int64_t)n * L + t0 + t] : from_f<T>(0.f);
      cdst[idx] = ok ? Cg[(int64_t)n * L + t0 + t] : from_f<T>(0.f);
    }
  }
}

// ============================================================================
// Forward
// ============================================================================
template <typename T, int ITEMS>
__global__ void __launch_bounds__(256)
sscan_fwd_kernel(SsParams p) {
  constexpr int CH = 32 * ITEMS;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const int N = p.N, L = p.L;
  T* Bs = reinterpret_cast<T*>(smem + 128);
  T* Cs = Bs + (size_t)p.nbuf * N * CH;
  float* scarry = reinterpret_cast<float*>(Cs + (size_t)p.nbuf * N * CH);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int cpc = p.nw * p.cpw;
  const int d0 = blockIdx.x * cpc;
  const int g = d0 / p.dpg;
  const T* Bg = reinterpret_cast<const T*>(p.Bm) + ((int64_t)b * p.groups + g) * N * L;
  const T* Cg = reinterpret_cast<const T*>(p.Cm) + ((int64_t)b * p.groups + g) * N * L;
  const int nch = (L + CH - 1) / CH;

  for (int i = threadIdx.x; i < cpc * N; i += blockDim.x) scarry[i] = 0.f;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (p.bulk) {
    for (int k = 0; k < p.nbuf && k < nch; ++k) stage_bc<T, CH>(p, Bs, Cs, bars, k, k * CH, Bg, Cg, threadIdx.x == 0);
  }

  for (int k = 0; k < nch; ++k) {
    const int t0 = k * CH;
    const int buf = k % p.nbuf;
    if (p.bulk) {
      mbar_wait_bounded(&bars[buf], (uint32_t)((k / p.nbuf) & 1), &g_sscan_err);
    } else {
      stage_bc<T, CH>(p, Bs, Cs, bars, buf, t0, Bg, Cg, false);
      __syncthreads();
    }
    const T* Bt = Bs + (size_t)buf * N * CH + lane * ITEMS;
    const T* Ct = Cs + (size_t)buf * N * CH + lane * ITEMS;
    const int tl = t0 + lane * ITEMS;

    for (int j = 0; j < p.cpw; ++j) {
      const int cl = warp * p.cpw + j;
      const int d = d0 + cl;
      const int64_t chan = (int64_t)b * p.dim + d;
      float uu[ITEMS], dlt[ITEMS];
      load_items<T, ITEMS>(uu, reinterpret_cast<const T*>(p.u) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dlt, reinterpret_cast<const T*>(p.delta) + chan * L, tl, L, p.vec_io);
      const float bias = p.bias ? p.bias[d] : 0.f;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        float v = dlt[i] + bias;
        if (p.softplus) v = softplus_f(v);
        dlt[i] = (tl + i < L) ? v : 0.f;  // padded steps are the identity
      }
      float y[ITEMS];
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) y[i] = 0.f;

      for (int n = 0; n < N; ++n) {
        const float A2 = p.A[(int64_t)d * N + n] * kLog2e;
        float a[ITEMS], h[ITEMS], Bv[ITEMS];
        load_smem_items<T, ITEMS>(Bv, Bt + n * CH);
        float P = 1.f, H = 0.f;
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          a[i] = ex2(dlt[i] * A2);
          h[i] = dlt[i] * uu[i] * Bv[i];
          H = fmaf(a[i], H, h[i]);
          P *= a[i];
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float Pp = __shfl_up_sync(0xffffffffu, P, off);
          const float Hp = __shfl_up_sync(0xffffffffu, H, off);
          if (lane >= off) { H = fmaf(P, Hp, H); P *= Pp; }
        }
        const float carry = scarry[cl * N + n];
        float Pe = __shfl_up_sync(0xffffffffu, P, 1);
        float He = __shfl_up_sync(0xffffffffu, H, 1);
        if (lane == 0) { Pe = 1.f; He = 0.f; }
        const float newc = __shfl_sync(0xffffffffu, fmaf(P, carry, H), 31);
        float hh = fmaf(Pe, carry, He);
        float Cv[ITEMS];
        load_smem_items<T, ITEMS>(Cv, Ct + n * CH);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          hh = fmaf(a[i], hh, h[i]);
          y[i] = fmaf(Cv[i], hh, y[i]);
        }
        if (p.chunk_states != nullptr && ((tl + ITEMS) % kStateStride) == 0) {
          const int idx = (tl + ITEMS) / kStateStride - 1;
          if (idx < p.nsaved) p.chunk_states[(chan * p.nsaved + idx) * N + n] = hh;
        }
        if (lane == 0) scarry[cl * N + n] = newc;
      }
      // epilogue: out = (y + D u) * silu(z)
      const float Dd = p.D ? p.D[d] : 0.f;
      float o[ITEMS];
      if (p.z != nullptr) {
        float zz[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) o[i] = fmaf(Dd, uu[i], y[i]) * (zz[i] * sigmoid_f(zz[i]));
      } else {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) o[i] = fmaf(Dd, uu[i], y[i]);
      }
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.out) + chan * L, o, tl, L, p.vec_io);
    }
    __syncthreads();  // buffer `buf` fully consumed; carries visible
    if (p.bulk && k + p.nbuf < nch)
      stage_bc<T, CH>(p, Bs, Cs, bars, buf, (k + p.nbuf) * CH, Bg, Cg, threadIdx.x == 0);
  }
  if (p.last_state != nullptr) {
    for (int i = threadIdx.x; i < cpc * N; i += blockDim.x) {
      const int cl = i / N, n = i - cl * N;
      p.last_state[((int64_t)b * p.dim + d0 + cl) * N + n] = scarry[i];
    }
  }
}

// ============================================================================
// Backward
// ============================================================================
template <typename T>
__global__ void __launch_bounds__(256)
sscan_bwd_kernel(SsParams p) {
  constexpr int ITEMS = kItemsB;
  constexpr int CH = 32 * ITEMS;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const int N = p.N, L = p.L;
  T* Bs = reinterpret_cast<T*>(smem + 128);
  T* Cs = Bs + (size_t)p.nbuf * N * CH;
  float* sdB = reinterpret_cast<float*>(Cs + (size_t)p.nbuf * N * CH);  // [N][CH]
  float* sdC = sdB + N * CH;                                           // [N][CH]
  const int cpc = p.nw * p.cpw;
  float* sg = sdC + N * CH;       // adjoint carries [cpc][N] (pre-multiplied by a)
  float* sdA = sg + cpc * N;      // dA partials [cpc][N]
  float* sdD = sdA + cpc * N;     // dD partials [cpc]
  float* sdb = sdD + cpc;         // dbias partials [cpc]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * cpc;
  const int g = d0 / p.dpg;
  const T* Bg = reinterpret_cast<const T*>(p.Bm) + ((int64_t)b * p.groups + g) * N * L;
  const T* Cg = reinterpret_cast<const T*>(p.Cm) + ((int64_t)b * p.groups + g) * N * L;
  float* dBg = p.dB_acc + ((int64_t)b * p.groups + g) * N * L;
  float* dCg = p.dC_acc + ((int64_t)b * p.groups + g) * N * L;
  const int nch = (L + CH - 1) / CH;

  for (int i = threadIdx.x; i < 2 * N * CH; i += blockDim.x) sdB[i] = 0.f;
  for (int i = threadIdx.x; i < 2 * cpc * N + 2 * cpc; i += blockDim.x) sg[i] = 0.f;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (p.bulk) {
    for (int it = 0; it < p.nbuf && it < nch; ++it)
      stage_bc<T, CH>(p, Bs, Cs, bars, it, (nch - 1 - it) * CH, Bg, Cg, threadIdx.x == 0);
  }

  for (int it = 0; it < nch; ++it) {
    const int k = nch - 1 - it;
    const int t0 = k * CH;
    const int buf = it % p.nbuf;
    if (p.bulk) {
      mbar_wait_bounded(&bars[buf], (uint32_t)((it / p.nbuf) & 1), &g_sscan_err);
    } else {
      stage_bc<T, CH>(p, Bs, Cs, bars, buf, t0, Bg, Cg, false);
      __syncthreads();
    }
    const T* Bt = Bs + (size_t)buf * N * CH + lane * ITEMS;
    const T* Ct = Cs + (size_t)buf * N * CH + lane * ITEMS;
    const int tl = t0 + lane * ITEMS;

    for (int j = 0; j < p.cpw; ++j) {
      const int cl = warp * p.cpw + j;
      const int d = d0 + cl;
      const int64_t chan = (int64_t)b * p.dim + d;
      float uu[ITEMS], dlt[ITEMS], dlr[ITEMS], dy[ITEMS], dout[ITEMS];
      load_items<T, ITEMS>(uu, reinterpret_cast<const T*>(p.u) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dlr, reinterpret_cast<const T*>(p.delta) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dout, reinterpret_cast<const T*>(p.dout) + chan * L, tl, L, p.vec_io);
      const float bias = p.bias ? p.bias[d] : 0.f;
      const float Dd = p.D ? p.D[d] : 0.f;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const bool ok = tl + i < L;
        dlr[i] += bias;
        dlt[i] = ok ? (p.softplus ? softplus_f(dlr[i]) : dlr[i]) : 0.f;
        if (!ok) dout[i] = 0.f;
      }
      if (p.z != nullptr) {
        float zz[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) dy[i] = dout[i] * zz[i] * sigmoid_f(zz[i]);
      } else {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) dy[i] = dout[i];
      }
      float yacc[ITEMS], ddl[ITEMS], duacc[ITEMS];
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) { yacc[i] = Dd * uu[i]; ddl[i] = 0.f; duacc[i] = dy[i] * Dd; }

      for (int n = 0; n < N; ++n) {
        const float An = p.A[(int64_t)d * N + n];
        const float A2 = An * kLog2e;
        float a[ITEMS], h[ITEMS], Bv[ITEMS], Cv[ITEMS];
        load_smem_items<T, ITEMS>(Bv, Bt + n * CH);
        load_smem_items<T, ITEMS>(Cv, Ct + n * CH);
        // ---- forward recompute of the states inside the chunk
        float P = 1.f, H = 0.f;
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          a[i] = ex2(dlt[i] * A2);
          h[i] = dlt[i] * uu[i] * Bv[i];
          H = fmaf(a[i], H, h[i]);
          P *= a[i];
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float Pp = __shfl_up_sync(0xffffffffu, P, off);
          const float Hp = __shfl_up_sync(0xffffffffu, H, off);
          if (lane >= off) { H = fmaf(P, Hp, H); P *= Pp; }
        }
        const float hc = k > 0 ? p.chunk_states_in[(chan * p.nsaved + (k - 1)) * N + n] : 0.f;
        float Pe = __shfl_up_sync(0xffffffffu, P, 1);
        float He = __shfl_up_sync(0xffffffffu, H, 1);
        if (lane == 0) { Pe = 1.f; He = 0.f; }
        const float hin = fmaf(Pe, hc, He);
        {
          float hh = hin;
#pragma unroll
          for (int i = 0; i < ITEMS; ++i) {
            hh = fmaf(a[i], hh, h[i]);
            h[i] = hh;
            yacc[i] = fmaf(Cv[i], hh, yacc[i]);
          }
        }
        // ---- reverse scan of the adjoint g_t = dy_t C_t + a_{t+1} g_{t+1}
        const float a_next_lane = __shfl_down_sync(0xffffffffu, a[0], 1);
        const float ra_last = (lane == 31) ? 1.f : a_next_lane;
        float Q = 1.f, G = 0.f;
#pragma unroll
        for (int i = ITEMS - 1; i >= 0; --i) {
          const float ra = (i == ITEMS - 1) ? ra_last : a[i + 1];
          G = fmaf(ra, G, dy[i] * Cv[i]);
          Q *= ra;
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float Qn = __shfl_down_sync(0xffffffffu, Q, off);
          const float Gn = __shfl_down_sync(0xffffffffu, G, off);
          if (lane + off < 32) { G = fmaf(Q, Gn, G); Q *= Qn; }
        }
        const float gc = sg[cl * N + n];  // a_{t0+CH} * g_{t0+CH}
        const float Qd = __shfl_down_sync(0xffffffffu, Q, 1);
        const float Gd = __shfl_down_sync(0xffffffffu, G, 1);
        const float gfirst0 = __shfl_sync(0xffffffffu, a[0] * fmaf(Q, gc, G), 0);
        float gg = (lane == 31) ? gc : fmaf(Qd, gc, Gd);
        float dAl = 0.f;
#pragma unroll
        for (int i = ITEMS - 1; i >= 0; --i) {
          const float ra = (i == ITEMS - 1) ? ra_last : a[i + 1];
          gg = fmaf(ra, gg, dy[i] * Cv[i]);
          const float hp = (i > 0) ? h[i - 1] : hin;
          const float ea = gg * hp * a[i];  // dL/d(delta' A) of step i
          dAl = fmaf(ea, dlt[i], dAl);
          ddl[i] = fmaf(ea, An, fmaf(gg * Bv[i], uu[i], ddl[i]));
          duacc[i] = fmaf(gg * dlt[i], Bv[i], duacc[i]);
          const int ti = i * 32 + lane;  // [n][item][lane]: conflict-free shared atomics
          atomicAdd(&sdB[n * CH + ti], gg * dlt[i] * uu[i]);
          atomicAdd(&sdC[n * CH + ti], dy[i] * h[i]);
        }
        dAl = warp_sum(dAl);
        if (lane == 0) {
          sdA[cl * N + n] += dAl;
          sg[cl * N + n] = gfirst0;
        }
      }
      // ---- per-step outputs
      float dDl = 0.f, dbl = 0.f;
      float odl[ITEMS];
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const float s = p.softplus ? sigmoid_f(dlr[i]) : 1.f;
        const float v = (p.softplus && dlr[i] > 20.f) ? ddl[i] : ddl[i] * s;
        odl[i] = (tl + i < L) ? v : 0.f;
        dbl += odl[i];
        dDl = fmaf(dy[i], uu[i], dDl);
      }
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.du) + chan * L, duacc, tl, L, p.vec_io);
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.ddelta) + chan * L, odl, tl, L, p.vec_io);
      if (p.z != nullptr) {
        float zz[ITEMS], odz[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          const float sgz = sigmoid_f(zz[i]);
          odz[i] = dout[i] * yacc[i] * sgz * (1.f + zz[i] * (1.f - sgz));
        }
        store_items<T, ITEMS>(reinterpret_cast<T*>(p.dz) + chan * L, odz, tl, L, p.vec_io);
      }
      dDl = warp_sum(dDl);
      dbl = warp_sum(dbl);
      if (lane == 0) { sdD[cl] += dDl; sdb[cl] += dbl; }
    }
    __syncthreads();  // chunk consumed; sdB/sdC complete
    const int len = min(CH, L - t0);
    for (int idx = threadIdx.x; idx < N * CH; idx += blockDim.x) {
      const int n = idx / CH, t = idx - n * CH;
      const int si = n * CH + (t % ITEMS) * 32 + t / ITEMS;
      if (t < len) {
        atomicAdd(&dBg[(int64_t)n * L + t0 + t], sdB[si]);
        atomicAdd(&dCg[(int64_t)n * L + t0 + t], sdC[si]);
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 2 * N * CH; idx += blockDim.x) sdB[idx] = 0.f;
    __syncthreads();
    if (p.bulk && it + p.nbuf < nch)
      stage_bc<T, CH>(p, Bs, Cs, bars, buf, (nch - 1 - (it + p.nbuf)) * CH, Bg, Cg, threadIdx.x == 0);
  }
  for (int i = threadIdx.x; i < cpc; i += blockDim.x) {
    float* pr = p.part + ((int64_t)b * p.dim + d0 + i) * (N + 2);
    for (int n = 0; n < N; ++n) pr[n] = sdA[i * N + n];
    pr[N] = sdD[i];
    pr[N + 1] = sdb[i];
  }
}

// dA[d,n], dD[d], dbias[d] = fixed-order sums over the batch of the partials.
__global__ void sscan_bwd_reduce(float* __restrict__ dA, float* __restrict__ dD, float* __restrict__ dbias,
                                 const float* __restrict__ part, int batch, int dim, int N) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = N + 2;
  if (i >= (int64_t)dim * per) return;
  const int d = (int)(i / per), k = (int)(i - d * per);
  float s = 0.f;
  for (int b = 0; b < batch; ++b) s += part[((int64_t)b * dim + d) * per + k];
  if (k < N) dA[(int64_t)d * N + k] = s;
  else if (k == N) { if (dD) dD[d] = s; }
  else { if (dbias) dbias[d] = s; }
}

template <typename T>
__global__ void f32_to(T* __restrict__ dst, const float* __restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f<T>(src[i]);
}

// Channels per CTA: the largest candidate dividing dim/groups.
void pick_layout(int dpg, int max_cpc, int* nw, int* cpw) {
  const int cands[] = {32, 16, 8, 4, 2, 1};
  int cpc = 1;
  for (int c : cands)
    if (c <= max_cpc && dpg % c == 0) { cpc = c; break; }
  *nw = cpc < 8 ? cpc : 8;
  *cpw = cpc / *nw;
}

int validate(int64_t batch, int64_t dim, int64_t L, int64_t N, int64_t groups, int dt) {
  AK_REQUIRE(valid_dtype(dt), AK_ERR_DTYPE, "selective_scan: unsupported dtype %d", dt);
  AK_REQUIRE(batch >= 0 && batch < 65536 && dim >= 0 && L >= 0 && L < (1LL << 31), AK_ERR_SHAPE,
             "selective_scan: bad shape");
  AK_REQUIRE(N >= 1 && N <= 64, AK_ERR_SHAPE, "selective_scan: dstate must be in [1, 64], got %lld", (long long)N);
  AK_REQUIRE(groups >= 1 && dim % groups == 0, AK_ERR_SHAPE, "selective_scan: dim %% groups != 0");
  return AK_OK;
}

int nsaved_of(int64_t L) { return (int)((L + kStateStride - 1) / kStateStride); }

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_selective_scan_state_stride(void) { return kStateStride; }

extern "C" int ak_selective_scan_fwd(void* out, float* last_state, float* chunk_states, const void* u,
                                     const void* delta, const float* A, const void* Bm, const void* Cm,
                                     const float* D, const void* z, const float* delta_bias, int delta_softplus,
                                     int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate, int64_t groups,
                                     int dt, void* stream) {
  clear_error();
  int rc = validate(batch, dim, seqlen, dstate, groups, dt);
  if (rc) return rc;
  if (batch == 0 || dim == 0) return AK_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (seqlen == 0) {
    if (last_state)
      AK_CUDA_TRY(cudaMemsetAsync(last_state, 0, (size_t)batch * dim * dstate * 4, st), "selective_scan_fwd");
    return AK_OK;
  }
  AK_REQUIRE(out && u && delta && A && Bm && Cm, AK_ERR_ARG, "ak_selective_scan_fwd: null pointer");
  SsParams p{};
  p.u = u; p.delta = delta; p.A = A; p.Bm = Bm; p.Cm = Cm; p.D = D; p.z = z; p.bias = delta_bias;
  p.out = out; p.last_state = last_state; p.chunk_states = chunk_states;
  p.batch = (int)batch; p.dim = (int)dim; p.L = (int)seqlen; p.N = (int)dstate; p.groups = (int)groups;
  p.dpg = (int)(dim / groups);
  p.softplus = delta_softplus ? 1 : 0;
  p.nsaved = nsaved_of(seqlen);
  pick_layout(p.dpg, 16, &p.nw, &p.cpw);
  const int es = elem_size(dt);
  p.bulk = (((seqlen * es) % 16) == 0 && aligned16(Bm) && aligned16(Cm)) ? 1 : 0;
  p.vec_io = (((seqlen * es) % 16) == 0 && aligned16(u) && aligned16(delta) && aligned16(out) &&
              (z == nullptr || aligned16(z))) ? 1 : 0;
  constexpr int CH = 32 * kItemsF;
  size_t tile = (size_t)dstate * CH * es * 2;  // B + C, one buffer
  p.nbuf = (128 + 2 * tile + (size_t)p.nw * p.cpw * dstate * 4) <= 200 * 1024 ? 2 : 1;
  const size_t smem = 128 + p.nbuf * tile + (size_t)p.nw * p.cpw * dstate * 4;
  AK_REQUIRE(smem <= 227 * 1024, AK_ERR_SHAPE, "selective_scan_fwd: dstate too large for shared memory");
  dim3 grid((unsigned)(dim / (p.nw * p.cpw)), (unsigned)batch);
  AK_DISPATCH_DTYPE(dt, T, {
    auto kern = sscan_fwd_kernel<T, kItemsF>;
    AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "selective_scan_fwd: smem attribute");
    kern<<<grid, p.nw * 32, smem, st>>>(p);
  });
  AK_CHECK_LAUNCH("ak_selective_scan_fwd");
  return AK_OK;
}

extern "C" int ak_selective_scan_bwd_workspace_size(int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate,
                                                    int64_t groups, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes != nullptr, AK_ERR_ARG, "null bytes");
  int rc = validate(batch, dim, seqlen, dstate, groups, AK_F32);
  if (rc) return rc;
  *bytes = (2 * (size_t)batch * groups * dstate * seqlen + (size_t)batch * dim * (dstate + 2)) * sizeof(float);
  return AK_OK;
}

extern "C" int ak_selective_scan_bwd(void* du, void* ddelta, float* dA, void* dB, void* dC, float* dD, void* dz,
                                     float* ddelta_bias, void* workspace, size_t ws_bytes, const void* dout,
                                     const void* u, const void* delta, const float* A, const void* Bm,
                                     const void* Cm, const float* D, const void* z, const float* delta_bias,
                                     const float* chunk_states, int delta_softplus, int64_t batch, int64_t dim,
                                     int64_t seqlen, int64_t dstate, int64_t groups, int dt, void* stream) {
  clear_error();
  int rc = validate(batch, dim, seqlen, dstate, groups, dt);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t nbc = (size_t)batch * groups * dstate * seqlen;
  const size_t need = (2 * nbc + (size_t)batch * dim * (dstate + 2)) * sizeof(float);
  AK_REQUIRE(need == 0 || (workspace && ws_bytes >= need), AK_ERR_WORKSPACE,
             "ak_selective_scan_bwd: workspace %zu < %zu", ws_bytes, need);
  AK_REQUIRE(dim == 0 || dA, AK_ERR_ARG, "ak_selective_scan_bwd: null dA");
  if (batch == 0 || dim == 0 || seqlen == 0) {
    if (dim > 0) {
      AK_CUDA_TRY(cudaMemsetAsync(dA, 0, (size_t)dim * dstate * 4, st), "bwd memset");
      if (dD) AK_CUDA_TRY(cudaMemsetAsync(dD, 0, (size_t)dim * 4, st), "bwd memset");
      if (ddelta_bias) AK_CUDA_TRY(cudaMemsetAsync(ddelta_bias, 0, (size_t)dim * 4, st), "bwd memset");
    }
    const size_t es = (size_t)elem_size(dt);
    if (nbc && dB) AK_CUDA_TRY(cudaMemsetAsync(dB, 0, nbc * es, st), "bwd memset");
    if (nbc && dC) AK_CUDA_TRY(cudaMemsetAsync(dC, 0, nbc * es, st), "bwd memset");
    return AK_OK;
  }
  AK_REQUIRE(du && ddelta && dB && dC && dout && u && delta && A && Bm && Cm, AK_ERR_ARG,
             "ak_selective_scan_bwd: null pointer");
  AK_REQUIRE(z == nullptr || dz != nullptr, AK_ERR_ARG, "ak_selective_scan_bwd: z given without dz");
  AK_REQUIRE(seqlen <= kStateStride || chunk_states != nullptr, AK_ERR_ARG,
             "ak_selective_scan_bwd: chunk_states required for seqlen > %d", kStateStride);
  SsParams p{};
  p.u = u; p.delta = delta; p.A = A; p.Bm = Bm; p.Cm = Cm; p.D = D; p.z = z; p.bias = delta_bias;
  p.dout = dout; p.chunk_states_in = chunk_states;
  p.du = du; p.ddelta = ddelta; p.dz = dz;
  float* ws = (float*)workspace;
  p.dB_acc = ws;
  p.dC_acc = ws + nbc;
  p.part = ws + 2 * nbc;
  p.batch = (int)batch; p.dim = (int)dim; p.L = (int)seqlen; p.N = (int)dstate; p.groups = (int)groups;
  p.dpg = (int)(dim / groups);
  p.softplus = delta_softplus ? 1 : 0;
  p.nsaved = nsaved_of(seqlen);
  pick_layout(p.dpg, 32, &p.nw, &p.cpw);
  const int es = elem_size(dt);
  p.bulk = (((seqlen * es) % 16) == 0 && aligned16(Bm) && aligned16(Cm)) ? 1 : 0;
  p.vec_io = (((seqlen * es) % 16) == 0 && aligned16(u) && aligned16(delta) && aligned16(dout) && aligned16(du) &&
              aligned16(ddelta) && (z == nullptr || (aligned16(z) && aligned16(dz)))) ? 1 : 0;
  constexpr int CH = 32 * kItemsB;
  const int cpc = p.nw * p.cpw;
  const size_t tile = (size_t)dstate * CH * es * 2;
  const size_t fixed = 128 + 2 * (size_t)dstate * CH * 4 + (2 * (size_t)cpc * dstate + 2 * cpc) * 4;
  p.nbuf = (fixed + 2 * tile) <= 200 * 1024 ? 2 : 1;
  const size_t smem = fixed + p.nbuf * tile;
  AK_REQUIRE(smem <= 227 * 1024, AK_ERR_SHAPE, "selective_scan_bwd: dstate too large for shared memory");
  AK_CUDA_TRY(cudaMemsetAsync(ws, 0, 2 * nbc * sizeof(float), st), "selective_scan_bwd: workspace clear");
  dim3 grid((unsigned)(dim / cpc), (unsigned)batch);
  AK_DISPATCH_DTYPE(dt, T, {
    auto kern = sscan_bwd_kernel<T>;
    AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "selective_scan_bwd: smem attribute");
    kern<<<grid, p.nw * 32, smem, st>>>(p);
  });
  AK_CHECK_LAUNCH("ak_selective_scan_bwd");
  const int64_t nred = dim * (dstate + 2);
  sscan_bwd_reduce<<<(unsigned)((nred + 255) / 256), 256, 0, st>>>(dA, dD, ddelta_bias, p.part, (int)batch,
                                                                  (int)dim, (int)dstate);
  AK_CHECK_LAUNCH("ak_selective_scan_bwd(reduce)");
  const unsigned cg = (unsigned)std::min<int64_t>((int64_t)(nbc + 255) / 256, (int64_t)sm_count() * 8);
  AK_DISPATCH_DTYPE(dt, T, {
    f32_to<T><<<cg, 256, 0, st>>>((T*)dB, p.dB_acc, (int64_t)nbc);
    f32_to<T><<<cg, 256, 0, st>>>((T*)dC, p.dC_acc, (int64_t)nbc);
  });
  AK_CHECK_LAUNCH("ak_selective_scan_bwd(convert)");
  return AK_OK;
}
