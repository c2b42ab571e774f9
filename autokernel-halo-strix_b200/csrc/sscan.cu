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
// Work decomposition.  A CTA owns `cpc` channels of one batch row (all in one
// B/C group) and walks L in chunks of 32 lanes x ITEMS steps: lane l owns the
// ITEMS consecutive steps starting at l*ITEMS (forward: 16 when the tiles fit in
// shared memory, else 8; backward: 8).  The chunk's B and C tiles
// (N x chunk, shared by every channel of the CTA) arrive by bulk async copy
// (TMA engine, mbarrier-completed) as 16-bit values into a staging buffer and
// are converted once per CTA into an fp32 tile laid out [n][quad][lane][4], so
// each lane reads its 4-step quads with conflict-free 16-byte shared loads.
// The staging buffer is refilled with the next chunk as soon as it has been
// converted, so the copy overlaps the whole chunk's compute.  Each warp scans
// one channel at a time: per state every lane runs its ITEMS steps
// sequentially in registers (one SFU exp2 per step; the lane's decay product
// is one exp2 of the summed delta), the 32 lane aggregates are combined by a
// 5-round shuffle scan, and the chunk carry (one fp32 per channel and state)
// lives in shared memory.  With 8 steps per lane the forward processes two
// states together so their independent dependency chains interleave (16 steps
// per lane leave no registers for it).  The state after every kStateStride
// steps is saved for the backward.
//
// Small batches.  When batch * dim warps cannot fill the GPU, each channel's
// states are split over NSG warps (state_groups: 2 or 4); a warp walks N / NSG
// states, the other groups hand their partial per-step sums (y; in the
// backward also d(delta') and du) to group 0 through shared memory, and group 0
// writes the per-step outputs.  NSG is a template parameter, so the one-group
// kernels the large batches use are unaffected.
//
// Backward.  Same decomposition, chunks visited in reverse.  Per chunk and
// state the forward states are recomputed from the saved chunk-start state
// (no full state tensor in HBM), then the adjoint
// g_t = dy_t C_t + a_{t+1} g_{t+1} is scanned right-to-left with the same
// two-level scheme; the adjoint carry crosses chunks pre-multiplied by a at
// the chunk's first step.  dB/dC (sums over the channels of a group) are
// reduced in shared memory across the CTA's channels: a warp takes a per-state
// row lock and adds its values in place (plain read-modify-write; warps walk
// the states in staggered order so the locks are rarely contended), and the
// rows are flushed once per chunk with vectorised fp32 global reductions; dA/dD/dbias are per-(batch,
// channel) partials reduced in a fixed order by a second kernel.
#include "ak_common.cuh"

#include <algorithm>

namespace ak {
namespace {

constexpr int kStateStride = 256;  // timesteps between saved states
constexpr int kItems = 8;          // steps per lane: chunk = 256 steps = kStateStride
static_assert(32 * kItems == kStateStride, "chunk must equal the state stride");
constexpr int kFwdItems = 16;      // forward steps per lane when shared memory allows (chunk 512)
constexpr int kFwdInterleave = 1;  // states interleaved per pass at 16 steps per lane (registers)

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
  int batch, dim, L, N, groups, dpg, nw, cpw, nsaved;
  int nsg;  // state groups per channel: warp w works on channel slot w / nsg, states of group w % nsg
  int softplus, bulk, vec_io;
  int* status;  // caller's status word: AK_ERR_TIMEOUT when a bounded wait gave up (nullable)
};

// Channels one CTA covers: nw warps = (channel slots) x (state groups), cpw channels per slot.
__host__ __device__ inline int channels_per_cta(const SsParams& p) { return p.nw / p.nsg * p.cpw; }

__device__ __forceinline__ float softplus_f(float x) { return x <= 20.f ? log1pf(__expf(x)) : x; }

// 16-bit inputs: log2(1 + 2^(x log2 e)) ln 2 with the hardware ex2 / lg2 approximations
// (two MUFU ops instead of the library log1p); its absolute error, about 1e-7, is far below
// the precision of a 16-bit delta.  fp32 inputs keep log1pf.
template <typename T>
__device__ __forceinline__ float softplus_t(float x) {
  if constexpr (sizeof(T) == 2) return x <= 20.f ? lg2(1.f + ex2(x * kLog2e)) * kLn2 : x;
  else return softplus_f(x);
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// Load ITEMS consecutive elements starting at position t of a length-L row.
// Vector width: 16 bytes, or the lane's whole run when that is shorter (then the run
// start t * sizeof(T) is a multiple of ITEMS * sizeof(T), the access size).
template <typename T, int ITEMS>
__device__ __forceinline__ void load_items(float (&v)[ITEMS], const T* row, int t, int L, bool vec) {
  constexpr int VEC = ITEMS * sizeof(T) >= 16 ? 16 / sizeof(T) : ITEMS;
  static_assert(ITEMS % VEC == 0, "ITEMS must be a multiple of the vector width");
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
  constexpr int VEC = ITEMS * sizeof(T) >= 16 ? 16 / sizeof(T) : ITEMS;
  static_assert(ITEMS % VEC == 0, "ITEMS must be a multiple of the vector width");
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

// fp32 tile row [quad][lane][4]: the lane's ITEMS values, 4 per 16-byte load.
template <int ITEMS>
__device__ __forceinline__ void load_tile(float (&v)[ITEMS], const float* row, int lane) {
  const float4* r4 = reinterpret_cast<const float4*>(row) + lane;
#pragma unroll
  for (int q = 0; q < ITEMS / 4; ++q) {
    const float4 f = r4[q * 32];
    v[4 * q + 0] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

// Same tile row as step pairs: (v[2j], v[2j+1]) from the lane's 16-byte loads.
template <int ITEMS>
__device__ __forceinline__ void load_tile2(float2 (&v)[ITEMS / 2], const float* row, int lane) {
  const float4* r4 = reinterpret_cast<const float4*>(row) + lane;
#pragma unroll
  for (int q = 0; q < ITEMS / 4; ++q) {
    const float4 f = r4[q * 32];
    v[2 * q] = make_float2(f.x, f.y);
    v[2 * q + 1] = make_float2(f.z, f.w);
  }
}

// Issue (one thread, bulk path) or perform (all threads, unaligned rows) the
// copy of the B and C tiles [N][CH] of the chunk starting at t0 into the
// staging buffer ([2][N][CH] of T).
template <typename T, int CH>
__device__ __forceinline__ void stage_bc(const SsParams& p, T* stage, uint64_t* bar, int t0, const T* Bg,
                                         const T* Cg, bool bulk_issue) {
  const int N = p.N, L = p.L;
  const int len = min(CH, L - t0);
  T* bdst = stage;
  T* cdst = stage + (size_t)N * CH;
  if (p.bulk) {
    if (bulk_issue) {
      const uint32_t bytes = (uint32_t)(len * sizeof(T));
      mbar_arrive_expect_tx(bar, 2u * N * bytes);
      for (int n = 0; n < N; ++n) {
        bulk_g2s(bdst + n * CH, Bg + (int64_t)n * L + t0, bytes, bar);
        bulk_g2s(cdst + n * CH, Cg + (int64_t)n * L + t0, bytes, bar);
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

// Convert the staging buffer into the fp32 tiles [2][N][CH] laid out
// [n][quad][lane][4]; steps beyond the sequence end become 0.
template <typename T, int ITEMS>
__device__ __forceinline__ void convert_bc(int N, const T* src, float* tile, int len) {
  constexpr int CH = 32 * ITEMS;
  const int nquads = 2 * N * CH / 4;
  for (int qi = threadIdx.x; qi < nquads; qi += blockDim.x) {
    const int e = qi * 4;  // element index in [which][n][t]
    const int row = e / CH, t = e - row * CH;
    const int lane = t / ITEMS, i = t - lane * ITEMS;
    float4 f;
    f.x = t + 0 < len ? to_f<T>(src[e + 0]) : 0.f;
    f.y = t + 1 < len ? to_f<T>(src[e + 1]) : 0.f;
    f.z = t + 2 < len ? to_f<T>(src[e + 2]) : 0.f;
    f.w = t + 3 < len ? to_f<T>(src[e + 3]) : 0.f;
    reinterpret_cast<float4*>(tile + (size_t)row * CH)[(i / 4) * 32 + lane] = f;
  }
}

// Wait for the chunk's tiles, convert them, and (bulk path) refill the staging
// buffer with chunk `next_t0` (< 0: none).  `phase` counts completed copies.
// Returns false, the same for every thread of the CTA, when the wait ran out
// (AK_ERR_TIMEOUT is in the status word): the caller then returns at once.  The
// one copy in flight is given one more bounded wait first, so no bulk copy
// still targets this CTA's shared memory after it exits.
template <typename T, int ITEMS>
__device__ __forceinline__ bool fetch_chunk(const SsParams& p, T* stage, float* tile, uint64_t* bar, int phase,
                                            int t0, int next_t0, const T* Bg, const T* Cg) {
  constexpr int CH = 32 * ITEMS;
  if (p.bulk) {
    const bool ok = mbar_wait_bounded(bar, (uint32_t)(phase & 1), p.status);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) mbar_wait_bounded(bar, (uint32_t)(phase & 1), nullptr);
      __syncthreads();
      return false;
    }
  } else {
    stage_bc<T, CH>(p, stage, bar, t0, Bg, Cg, false);
    __syncthreads();
  }
  convert_bc<T, ITEMS>(p.N, stage, tile, min(CH, p.L - t0));
  __syncthreads();  // tile ready; staging buffer free again
  if (p.bulk && threadIdx.x == 0 && next_t0 >= 0) stage_bc<T, CH>(p, stage, bar, next_t0, Bg, Cg, true);
  return true;
}

// Inclusive scan over lanes of g -> Q g + G (right to left).
__device__ __forceinline__ void scan_down(float& Q, float& G, int lane) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float Qn = __shfl_down_sync(0xffffffffu, Q, off);
    const float Gn = __shfl_down_sync(0xffffffffu, G, off);
    if (lane + off < 32) {
      G = fmaf(Q, Gn, G);
      Q *= Qn;
    }
  }
}

// Shared memory: [0,128) mbarrier | staging 2*N*CH*sizeof(T) | fp32 tile 2*N*CH*4 | kernel arrays.
template <typename T, int CH>
__host__ __device__ inline size_t stage_bytes(int N) { return (size_t)2 * N * CH * sizeof(T); }

// ============================================================================
// Forward
// ============================================================================

// K states n0..n0+K-1 of one channel over one chunk: per lane a sequential pass
// over its ITEMS steps, a shuffle scan of the lane aggregates, the carry-in
// fix-up pass accumulating y, and the new carry.  K > 1 interleaves the K
// independent dependency chains.
template <int ITEMS, int K>
__device__ __forceinline__ void fwd_states(int n0, int N, const float (&dlt)[ITEMS], const float (&du)[ITEMS],
                                           float (&y)[ITEMS], float S, float A_l, const float* tile, int lane,
                                           float* carry_row, float* save) {
  constexpr int CH = 32 * ITEMS;
  float a[K][ITEMS], h[K][ITEMS], P[K], H[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float A2 = __shfl_sync(0xffffffffu, A_l, n0 + k) * kLog2e;  // lane n holds A[d, n]
    float2 Bv[ITEMS / 2];
    load_tile2<ITEMS>(Bv, tile + (n0 + k) * CH, lane);
    const float2 A22 = make_float2(A2, A2);
    // step pairs as paired fp32 instructions (exact per element)
#pragma unroll
    for (int j = 0; j < ITEMS / 2; ++j) {
      const float2 t = __fmul2_rn(make_float2(dlt[2 * j], dlt[2 * j + 1]), A22);
      a[k][2 * j] = ex2(t.x);
      a[k][2 * j + 1] = ex2(t.y);
      const float2 hv = __fmul2_rn(make_float2(du[2 * j], du[2 * j + 1]), Bv[j]);
      h[k][2 * j] = hv.x;
      h[k][2 * j + 1] = hv.y;
    }
    P[k] = ex2(S * A2);  // = prod of the lane's a
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    H[k] = h[k][0];
#pragma unroll
    for (int i = 1; i < ITEMS; ++i) H[k] = fmaf(a[k][i], H[k], h[k][i]);  // lane aggregate from a zero state
  }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    float Pp[K], Hp[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      Pp[k] = __shfl_up_sync(0xffffffffu, P[k], off);
      Hp[k] = __shfl_up_sync(0xffffffffu, H[k], off);
    }
    if (lane >= off) {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        H[k] = fmaf(P[k], Hp[k], H[k]);
        P[k] *= Pp[k];
      }
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float carry = carry_row[n0 + k];
    float Pe = __shfl_up_sync(0xffffffffu, P[k], 1);
    float He = __shfl_up_sync(0xffffffffu, H[k], 1);
    if (lane == 0) { Pe = 1.f; He = 0.f; }
    const float newc = __shfl_sync(0xffffffffu, fmaf(P[k], carry, H[k]), 31);
    float hh = fmaf(Pe, carry, He);
    float2 Cv[ITEMS / 2];
    load_tile2<ITEMS>(Cv, tile + (N + n0 + k) * CH, lane);
#pragma unroll
    for (int j = 0; j < ITEMS / 2; ++j) {
      float2 hv;
      hv.x = hh = fmaf(a[k][2 * j], hh, h[k][2 * j]);
      hv.y = hh = fmaf(a[k][2 * j + 1], hh, h[k][2 * j + 1]);
      const float2 yv = __ffma2_rn(Cv[j], hv, make_float2(y[2 * j], y[2 * j + 1]));
      y[2 * j] = yv.x;
      y[2 * j + 1] = yv.y;
    }
    if (save != nullptr) save[n0 + k] = hh;
    if (lane == 0) carry_row[n0 + k] = newc;
  }
}

// ITEMS steps per lane: 8 (chunk = one state stride) or 16 (chunk = two state
// strides; lanes 15 and 31 save the states, the shuffle scan is amortised over
// twice the steps).  KI states are interleaved per pass.
template <typename T, int ITEMS, int KI, int NSG>
__global__ void __launch_bounds__(256, ITEMS == 8 ? 3 : 2)
sscan_fwd_kernel(SsParams p) {
  static_assert(ITEMS * 32 % kStateStride == 0, "chunk must be a whole number of state strides");
  constexpr int CH = 32 * ITEMS;
  constexpr int kSavesPerChunk = CH / kStateStride;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  const int N = p.N, L = p.L;
  T* stage = reinterpret_cast<T*>(smem + 128);
  float* tile = reinterpret_cast<float*>(smem + 128 + stage_bytes<T, CH>(N));
  float* scarry = tile + 2 * N * CH;  // [cpc][N]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int cpc = (p.nw / NSG) * p.cpw;
  // state split: this warp walks states [nbeg, nend) of its channel; group 0 adds the other
  // groups' partial y (through ybuf) and writes the output
  const int sgi = warp % NSG, wch = warp / NSG;
  const int nper = (N + NSG - 1) / NSG;
  const int nbeg = min(N, sgi * nper), nend = min(N, nbeg + nper);
  float* ybuf = scarry + cpc * N;  // [nw / nsg][nsg - 1][ITEMS][32]
  float* ymine = sgi > 0 ? ybuf + ((wch * (NSG - 1) + sgi - 1) * ITEMS) * 32 + lane : nullptr;
  const int d0 = blockIdx.x * cpc;
  const int g = d0 / p.dpg;
  const T* Bg = reinterpret_cast<const T*>(p.Bm) + ((int64_t)b * p.groups + g) * N * L;
  const T* Cg = reinterpret_cast<const T*>(p.Cm) + ((int64_t)b * p.groups + g) * N * L;
  const int nch = (L + CH - 1) / CH;

  for (int i = threadIdx.x; i < cpc * N; i += blockDim.x) scarry[i] = 0.f;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (p.bulk && threadIdx.x == 0) stage_bc<T, CH>(p, stage, bar, 0, Bg, Cg, true);

  for (int k = 0; k < nch; ++k) {
    const int t0 = k * CH;
    if (!fetch_chunk<T, ITEMS>(p, stage, tile, bar, k, t0, k + 1 < nch ? t0 + CH : -1, Bg, Cg)) return;
    const int tl = t0 + lane * ITEMS;

    for (int j = 0; j < p.cpw; ++j) {
      const int cl = wch * p.cpw + j;
      const int d = d0 + cl;
      const int64_t chan = (int64_t)b * p.dim + d;
      float dlt[ITEMS], du[ITEMS], y[ITEMS];
      load_items<T, ITEMS>(du, reinterpret_cast<const T*>(p.u) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dlt, reinterpret_cast<const T*>(p.delta) + chan * L, tl, L, p.vec_io);
      const float bias = p.bias ? p.bias[d] : 0.f;
      const float Dd = p.D ? p.D[d] : 0.f;
      float S = 0.f;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        float v = dlt[i] + bias;
        if (p.softplus) v = softplus_t<T>(v);
        v = (tl + i < L) ? v : 0.f;  // padded steps are the identity
        dlt[i] = v;
        S += v;
        y[i] = sgi == 0 ? Dd * du[i] : 0.f;
        du[i] *= v;
      }
      const float A_l = lane < N ? p.A[(int64_t)d * N + lane] : 0.f;  // lane n holds A[d, n]
      float* carry_row = scarry + cl * N;
      // the lanes that end a state stride (lane 31, and lane 15 with 16 steps per lane) save
      // the states for the backward
      constexpr int kLanesPerStride = kStateStride / ITEMS;
      const int si = k * kSavesPerChunk + (lane + 1) / kLanesPerStride - 1;
      float* save = (p.chunk_states != nullptr && (lane + 1) % kLanesPerStride == 0 && si < p.nsaved)
                        ? p.chunk_states + (chan * p.nsaved + si) * N : nullptr;
      int n = nbeg;
      for (; n + KI <= nend; n += KI) fwd_states<ITEMS, KI>(n, N, dlt, du, y, S, A_l, tile, lane, carry_row, save);
      for (; n < nend; ++n) fwd_states<ITEMS, 1>(n, N, dlt, du, y, S, A_l, tile, lane, carry_row, save);
      if (NSG > 1) {  // uniform over the CTA: every warp runs the same cpw iterations
        if (sgi > 0) {
#pragma unroll
          for (int i = 0; i < ITEMS; ++i) ymine[i * 32] = y[i];
        }
        __syncthreads();
        if (sgi == 0) {
          for (int g2 = 0; g2 < NSG - 1; ++g2) {
            const float* yo = ybuf + ((wch * (NSG - 1) + g2) * ITEMS) * 32 + lane;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) y[i] += yo[i * 32];
          }
        }
        __syncthreads();  // ybuf free for the next channel
        if (sgi > 0) continue;
      }
      if (p.z != nullptr) {
        float zz[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) y[i] *= zz[i] * sigmoid_f(zz[i]);
      }
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.out) + chan * L, y, tl, L, p.vec_io);
    }
    __syncthreads();  // tile consumed; carries visible
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
// CTA-scope lock word in shared memory: acquire = CAS 0 -> 1 with acquire
// semantics (returns the old value), release = store 0 with release semantics.
__device__ __forceinline__ int lock_try_acquire(int* w) {
  int old;
  asm volatile("atom.acquire.cta.shared::cta.cas.b32 %0, [%1], 0, 1;"
               : "=r"(old)
               : "r"((uint32_t)__cvta_generic_to_shared(w))
               : "memory");
  return old;
}

__device__ __forceinline__ void lock_release(int* w) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], 0;" ::"r"((uint32_t)__cvta_generic_to_shared(w)) : "memory");
}

__device__ __forceinline__ void red_add_v4(float* addr, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

template <typename T, int NSG>
__global__ void __launch_bounds__(256, 2)
sscan_bwd_kernel(SsParams p) {
  constexpr int ITEMS = kItems;
  constexpr int CH = 32 * ITEMS;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  const int N = p.N, L = p.L;
  T* stage = reinterpret_cast<T*>(smem + 128);
  float* tile = reinterpret_cast<float*>(smem + 128 + stage_bytes<T, CH>(N));
  float* sdB = tile + 2 * N * CH;  // [N][ITEMS/2][32] float2 (step pairs)
  float* sdC = sdB + N * CH;       // [N][ITEMS/2][32] float2
  const int cpc = (p.nw / NSG) * p.cpw;
  float* sg = sdC + N * CH;        // adjoint carries [cpc][N] (pre-multiplied by a)
  float* sdA = sg + cpc * N;       // dA partials [cpc][N]
  float* sdD = sdA + cpc * N;      // dD partials [cpc]
  float* sdb = sdD + cpc;          // dbias partials [cpc]
  int* slock = reinterpret_cast<int*>(sdb + cpc);  // one lock word per state row of sdB / sdC
  float* xbuf = reinterpret_cast<float*>(slock + N);  // state split: [nw / nsg][nsg - 1][3][ITEMS][32]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // state split: this warp walks states [nbeg, nend) of its channel; group 0 adds the other
  // groups' partial y, d(delta') and du (through xbuf) and writes the per-step outputs
  const int sgi = warp % NSG, wch = warp / NSG;
  const int nper = (N + NSG - 1) / NSG;
  const int nbeg = min(N, sgi * nper), nend = min(N, nbeg + nper), ncnt = nend - nbeg;
  float* xmine = sgi > 0 ? xbuf + ((wch * (NSG - 1) + sgi - 1) * 3 * ITEMS) * 32 + lane : nullptr;
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
  for (int i = threadIdx.x; i < N; i += blockDim.x) slock[i] = 0;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (p.bulk && threadIdx.x == 0) stage_bc<T, CH>(p, stage, bar, (nch - 1) * CH, Bg, Cg, true);

  for (int it = 0; it < nch; ++it) {
    const int k = nch - 1 - it;
    const int t0 = k * CH;
    const int len = min(CH, L - t0);
    if (!fetch_chunk<T, ITEMS>(p, stage, tile, bar, it, t0, k > 0 ? t0 - CH : -1, Bg, Cg)) return;
    const int tl = t0 + lane * ITEMS;

    for (int j = 0; j < p.cpw; ++j) {
      const int cl = wch * p.cpw + j;
      const int d = d0 + cl;
      const int64_t chan = (int64_t)b * p.dim + d;
      float uu[ITEMS], dlt[ITEMS], dlr[ITEMS], dy[ITEMS];
      load_items<T, ITEMS>(uu, reinterpret_cast<const T*>(p.u) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dlr, reinterpret_cast<const T*>(p.delta) + chan * L, tl, L, p.vec_io);
      load_items<T, ITEMS>(dy, reinterpret_cast<const T*>(p.dout) + chan * L, tl, L, p.vec_io);  // dout for now
      const float bias = p.bias ? p.bias[d] : 0.f;
      const float Dd = (p.D && sgi == 0) ? p.D[d] : 0.f;  // the D u term belongs to group 0
      float S = 0.f;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const bool ok = tl + i < L;
        dlr[i] += bias;
        dlt[i] = ok ? (p.softplus ? softplus_f(dlr[i]) : dlr[i]) : 0.f;  // not SFU-bound here
        S += dlt[i];
      }
      // dy = dout * silu(z); the gate factor is recomputed for dz after the state loop
      if (p.z != nullptr) {
        float zz[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) dy[i] *= zz[i] * sigmoid_f(zz[i]);
      }
      // Step pairs (2j, 2j+1) as float2: the per-step products and accumulations below run as
      // paired fp32 instructions (__fmul2_rn / __ffma2_rn / __fadd2_rn, exact per element), only
      // the sequential chains and the ex2 stay scalar.
      constexpr int P = ITEMS / 2;
      float2 uu2[P], dlt2[P], dy2[P], yacc2[P], ddl2[P], duacc2[P];
#pragma unroll
      for (int j = 0; j < P; ++j) {
        uu2[j] = make_float2(uu[2 * j], uu[2 * j + 1]);
        dlt2[j] = make_float2(dlt[2 * j], dlt[2 * j + 1]);
        dy2[j] = make_float2(dy[2 * j], dy[2 * j + 1]);
        yacc2[j] = make_float2(Dd * uu[2 * j], Dd * uu[2 * j + 1]);
        ddl2[j] = make_float2(0.f, 0.f);
        duacc2[j] = make_float2(dy[2 * j] * Dd, dy[2 * j + 1] * Dd);
      }
      const float Sr = S - dlt[0];  // sum of delta' over the lane's steps 1..ITEMS-1
      // lane n holds A[d, n] and the saved chunk-start state n: one load each per
      // channel and chunk, broadcast by shuffle inside the state loop
      const float A_l = lane < N ? p.A[(int64_t)d * N + lane] : 0.f;
      const float hc_l = (k > 0 && lane < N) ? p.chunk_states_in[(chan * p.nsaved + (k - 1)) * N + lane] : 0.f;
      float dAl_keep = 0.f;  // lane n < N keeps state n's dA partial

      // warps visit their states in staggered order (the channel slot w of nw / nsg starts at
      // w * ncnt / (nw / nsg)), so two warps are rarely on the same state row of sdB / sdC at
      // once; the row lock below makes it exclusive
      const int nstart = (wch * ncnt) / (p.nw / NSG);
      for (int nn = 0; nn < ncnt; ++nn) {
        const int n = nbeg + (nn + nstart < ncnt ? nn + nstart : nn + nstart - ncnt);
        const float An = __shfl_sync(0xffffffffu, A_l, n);
        const float A2 = An * kLog2e;
        float2 a2[P], h2[P], Bv2[P], Cv2[P];
        load_tile2<ITEMS>(Bv2, tile + n * CH, lane);
        load_tile2<ITEMS>(Cv2, tile + (N + n) * CH, lane);
        // ---- forward recompute of the states inside the chunk
        const float2 A22 = make_float2(A2, A2);
#pragma unroll
        for (int j = 0; j < P; ++j) {
          const float2 t = __fmul2_rn(dlt2[j], A22);
          a2[j] = make_float2(ex2(t.x), ex2(t.y));
          h2[j] = __fmul2_rn(__fmul2_rn(dlt2[j], uu2[j]), Bv2[j]);
        }
        float H = h2[0].x;
        H = fmaf(a2[0].y, H, h2[0].y);
#pragma unroll
        for (int j = 1; j < P; ++j) {
          H = fmaf(a2[j].x, H, h2[j].x);
          H = fmaf(a2[j].y, H, h2[j].y);
        }
        float Pp = ex2(S * A2);
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float Pu = __shfl_up_sync(0xffffffffu, Pp, off);
          const float Hu = __shfl_up_sync(0xffffffffu, H, off);
          if (lane >= off) { H = fmaf(Pp, Hu, H); Pp *= Pu; }
        }
        const float hc = __shfl_sync(0xffffffffu, hc_l, n);
        float Pe = __shfl_up_sync(0xffffffffu, Pp, 1);
        float He = __shfl_up_sync(0xffffffffu, H, 1);
        if (lane == 0) { Pe = 1.f; He = 0.f; }
        const float hin = fmaf(Pe, hc, He);
        float2 hp2[P];  // the state before each step: (h[2j-1], h[2j]) with h[-1] = hin
        {
          float hh = hin;
#pragma unroll
          for (int j = 0; j < P; ++j) {
            hp2[j].x = hh;
            hh = fmaf(a2[j].x, hh, h2[j].x);
            h2[j].x = hh;
            hp2[j].y = hh;
            hh = fmaf(a2[j].y, hh, h2[j].y);
            h2[j].y = hh;
            yacc2[j] = __ffma2_rn(Cv2[j], h2[j], yacc2[j]);
          }
        }
        // ---- reverse scan of the adjoint g_t = dy_t C_t + a_{t+1} g_{t+1}
        float2 dyC2[P];
#pragma unroll
        for (int j = 0; j < P; ++j) dyC2[j] = __fmul2_rn(dy2[j], Cv2[j]);
        const float a_next_lane = __shfl_down_sync(0xffffffffu, a2[0].x, 1);
        const float ra_last = (lane == 31) ? 1.f : a_next_lane;
        float G = dyC2[P - 1].y;
        G = fmaf(a2[P - 1].y, G, dyC2[P - 1].x);
#pragma unroll
        for (int j = P - 2; j >= 0; --j) {
          G = fmaf(a2[j + 1].x, G, dyC2[j].y);
          G = fmaf(a2[j].y, G, dyC2[j].x);
        }
        float Q = ex2(Sr * A2) * ra_last;  // = prod of the lane's a_{t+1}
        scan_down(Q, G, lane);
        const float gc = sg[cl * N + n];  // a_{t0+CH} * g_{t0+CH}
        const float Qd = __shfl_down_sync(0xffffffffu, Q, 1);
        const float Gd = __shfl_down_sync(0xffffffffu, G, 1);
        const float gfirst0 = __shfl_sync(0xffffffffu, a2[0].x * fmaf(Q, gc, G), 0);
        float gg = (lane == 31) ? gc : fmaf(Qd, gc, Gd);
        float2 gsv2[P];  // the adjoint per step
        gg = fmaf(ra_last, gg, dyC2[P - 1].y);
        gsv2[P - 1].y = gg;
        gg = fmaf(a2[P - 1].y, gg, dyC2[P - 1].x);
        gsv2[P - 1].x = gg;
#pragma unroll
        for (int j = P - 2; j >= 0; --j) {
          gg = fmaf(a2[j + 1].x, gg, dyC2[j].y);
          gsv2[j].y = gg;
          gg = fmaf(a2[j].y, gg, dyC2[j].x);
          gsv2[j].x = gg;
        }
        const float2 An2 = make_float2(An, An);
        float2 dAl2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = P - 1; j >= 0; --j) {
          const float2 ea = __fmul2_rn(__fmul2_rn(gsv2[j], hp2[j]), a2[j]);  // dL/d(delta' A) per step
          dAl2 = __ffma2_rn(ea, dlt2[j], dAl2);
          const float2 gB = __fmul2_rn(gsv2[j], Bv2[j]);
          ddl2[j] = __ffma2_rn(ea, An2, __ffma2_rn(gB, uu2[j], ddl2[j]));
          duacc2[j] = __ffma2_rn(gB, dlt2[j], duacc2[j]);
        }
        float dAl = dAl2.x + dAl2.y;
        // row n of sdB / sdC under its lock: a short plain read-modify-write section
        // (no per-element atomics); [n][pair][lane] float2 slots, one 64-bit access per pair
        {
          float2 vb[P], vc[P];
#pragma unroll
          for (int j = 0; j < P; ++j) {
            vb[j] = __fmul2_rn(__fmul2_rn(gsv2[j], dlt2[j]), uu2[j]);
            vc[j] = __fmul2_rn(dy2[j], h2[j]);
          }
          bool owned = true;
          if (lane == 0) {
            uint32_t spins = 0;
            while (lock_try_acquire(&slock[n]) != 0) {
              if (++spins > kMaxSpins) { report_status(p.status, (int)AK_ERR_TIMEOUT); owned = false; break; }
              if (spins > 16) __nanosleep(20);
            }
          }
          owned = __shfl_sync(0xffffffffu, owned, 0);  // also orders the lanes after lane 0's acquire
          if (owned) {
            float2* rb = reinterpret_cast<float2*>(sdB) + n * (CH / 2) + lane;
            float2* rc = reinterpret_cast<float2*>(sdC) + n * (CH / 2) + lane;
#pragma unroll
            for (int j = 0; j < P; ++j) {
              rb[j * 32] = __fadd2_rn(rb[j * 32], vb[j]);
              rc[j * 32] = __fadd2_rn(rc[j * 32], vc[j]);
            }
          }
          __syncwarp();  // every lane's row update is ordered before lane 0's release
          if (lane == 0 && owned) lock_release(&slock[n]);
        }
        dAl = warp_sum(dAl);
        if (lane == n) dAl_keep += dAl;
        if (lane == 0) sg[cl * N + n] = gfirst0;
      }
      float yacc[ITEMS], ddl[ITEMS], duacc[ITEMS];
#pragma unroll
      for (int j = 0; j < P; ++j) {
        yacc[2 * j] = yacc2[j].x; yacc[2 * j + 1] = yacc2[j].y;
        ddl[2 * j] = ddl2[j].x; ddl[2 * j + 1] = ddl2[j].y;
        duacc[2 * j] = duacc2[j].x; duacc[2 * j + 1] = duacc2[j].y;
      }
      if (lane >= nbeg && lane < nend) sdA[cl * N + lane] += dAl_keep;  // this group's states
      if (NSG > 1) {  // uniform over the CTA: every warp runs the same cpw iterations
        if (sgi > 0) {
#pragma unroll
          for (int i = 0; i < ITEMS; ++i) {
            xmine[i * 32] = yacc[i];
            xmine[(ITEMS + i) * 32] = ddl[i];
            xmine[(2 * ITEMS + i) * 32] = duacc[i];
          }
        }
        __syncthreads();
        if (sgi == 0) {
          for (int g2 = 0; g2 < NSG - 1; ++g2) {
            const float* xo = xbuf + ((wch * (NSG - 1) + g2) * 3 * ITEMS) * 32 + lane;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
              yacc[i] += xo[i * 32];
              ddl[i] += xo[(ITEMS + i) * 32];
              duacc[i] += xo[(2 * ITEMS + i) * 32];
            }
          }
        }
        __syncthreads();  // xbuf free for the next channel
        if (sgi > 0) continue;
      }
      // ---- per-step outputs
      float dDl = 0.f, dbl = 0.f;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const float s = p.softplus ? (dlr[i] > 20.f ? 1.f : sigmoid_f(dlr[i])) : 1.f;
        const float v = (tl + i < L) ? ddl[i] * s : 0.f;
        ddl[i] = v;
        dbl += v;
        dDl = fmaf(dy[i], uu[i], dDl);
      }
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.du) + chan * L, duacc, tl, L, p.vec_io);
      store_items<T, ITEMS>(reinterpret_cast<T*>(p.ddelta) + chan * L, ddl, tl, L, p.vec_io);
      if (p.z != nullptr) {
        float zz[ITEMS], dout[ITEMS];
        load_items<T, ITEMS>(zz, reinterpret_cast<const T*>(p.z) + chan * L, tl, L, p.vec_io);
        load_items<T, ITEMS>(dout, reinterpret_cast<const T*>(p.dout) + chan * L, tl, L, p.vec_io);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          const float sgz = sigmoid_f(zz[i]);
          zz[i] = dout[i] * yacc[i] * sgz * (1.f + zz[i] * (1.f - sgz));
        }
        store_items<T, ITEMS>(reinterpret_cast<T*>(p.dz) + chan * L, zz, tl, L, p.vec_io);
      }
      dDl = warp_sum(dDl);
      dbl = warp_sum(dbl);
      if (lane == 0) { sdD[cl] += dDl; sdb[cl] += dbl; }
    }
    __syncthreads();  // chunk consumed; sdB/sdC complete
    // flush the [n][pair][lane] float2 accumulators: 4 consecutive steps per thread, v4 reductions
    const int nq = N * CH / 4;
    for (int q = threadIdx.x; q < nq; q += blockDim.x) {
      const int n = q / (CH / 4), t = (q - n * (CH / 4)) * 4;
      const int ln = t / ITEMS, i = t - ln * ITEMS;  // i even: pairs i/2 and i/2 + 1
      const float2* b2 = reinterpret_cast<const float2*>(sdB) + n * (CH / 2) + ln;
      const float2* c2 = reinterpret_cast<const float2*>(sdC) + n * (CH / 2) + ln;
      const float2 b0 = b2[(i / 2) * 32], b1 = b2[(i / 2 + 1) * 32];
      const float2 c0 = c2[(i / 2) * 32], c1 = c2[(i / 2 + 1) * 32];
      const float4 vb = make_float4(b0.x, b0.y, b1.x, b1.y);
      const float4 vc = make_float4(c0.x, c0.y, c1.x, c1.y);
      const int64_t off = (int64_t)n * L + t0 + t;
      if (t + 4 <= len && ((reinterpret_cast<uintptr_t>(dBg + off) & 15) == 0)) {
        red_add_v4(dBg + off, vb);
        red_add_v4(dCg + off, vc);
      } else {
        const float eb[4] = {vb.x, vb.y, vb.z, vb.w}, ec[4] = {vc.x, vc.y, vc.z, vc.w};
        for (int e = 0; e < 4; ++e)
          if (t + e < len) {
            atomicAdd(dBg + off + e, eb[e]);
            atomicAdd(dCg + off + e, ec[e]);
          }
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 2 * N * CH; idx += blockDim.x) sdB[idx] = 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cpc; i += blockDim.x) {
    float* pr = p.part + ((int64_t)b * p.dim + d0 + i) * (N + 2);
    for (int n = 0; n < N; ++n) pr[n] = sdA[i * N + n];
    pr[N] = sdD[i];
    pr[N + 1] = sdb[i];
  }
  pdl_trigger();
}

// dA[d,n], dD[d], dbias[d] = fixed-order sums over the batch of the partials.
__global__ void sscan_bwd_reduce(float* __restrict__ dA, float* __restrict__ dD, float* __restrict__ dbias,
                                 const float* __restrict__ part, int batch, int dim, int N) {
  pdl_wait();  // the backward kernel's partials (and dB / dC accumulators) are complete
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = N + 2;
  if (i >= (int64_t)dim * per) return;
  const int d = (int)(i / per), k = (int)(i - d * per);
  float s = 0.f;
#pragma unroll 8  // independent loads in flight; the adds stay in index order
  for (int b = 0; b < batch; ++b) s += part[((int64_t)b * dim + d) * per + k];
  if (k < N) dA[(int64_t)d * N + k] = s;
  else if (k == N) { if (dD) dD[d] = s; }
  else { if (dbias) dbias[d] = s; }
}

// dB and dC fp32 accumulators -> the output dtype (one launch for both).
template <typename T>
__global__ void f32_to2(T* __restrict__ d0, const float* __restrict__ s0, T* __restrict__ d1,
                        const float* __restrict__ s1, int64_t n) {
  pdl_wait();  // after the reduce, which itself waited for the backward kernel
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    d0[i] = from_f<T>(s0[i]);
    d1[i] = from_f<T>(s1[i]);
  }
}

// Channels per CTA: 16, halved (down to 4) while the grid would hold fewer than two CTAs per
// SM, so small batches (one batch row per GPU when the batch is sharded) still fill the GPU.
int max_channels_per_cta(int64_t batch, int64_t dim) {
  int c = 16;
  while (c > 4 && batch * (dim / c) < 2 * (int64_t)sm_count()) c /= 2;
  return c;
}

// State groups per channel: 1, or 2 / 4 when one warp per channel cannot fill the GPU
// (batch * dim warps against 16 resident warps per SM).  Each group walks N / nsg states,
// so a small batch gets more warps without repeating any exp.
int state_groups(int64_t batch, int64_t dim, int N) {
  const int64_t fill = (int64_t)sm_count() * 16;
  int g = 1;
  while (g < 4 && 2 * g <= N && batch * dim * g < fill) g *= 2;
  return g;
}

// Channels per CTA: the largest candidate dividing dim/groups; at most 8 warps per CTA,
// each (channel slot, state group) pair one warp.
void pick_layout(int dpg, int max_cpc, int nsg, int* nw, int* cpw) {
  const int cands[] = {32, 16, 8, 4, 2, 1};
  int cpc = 1;
  for (int c : cands)
    if (c <= max_cpc && dpg % c == 0) { cpc = c; break; }
  const int slots = std::max(1, 8 / nsg);
  const int sl = cpc < slots ? cpc : slots;
  *nw = sl * nsg;
  *cpw = cpc / sl;
}

int validate(int64_t batch, int64_t dim, int64_t L, int64_t N, int64_t groups, int dt) {
  AK_REQUIRE(valid_dtype(dt), AK_ERR_DTYPE, "selective_scan: unsupported dtype %d", dt);
  AK_REQUIRE(batch >= 0 && batch < 65536 && dim >= 0 && L >= 0 && L < (1LL << 31), AK_ERR_SHAPE,
             "selective_scan: bad shape");
  AK_REQUIRE(N >= 1 && N <= 32, AK_ERR_SHAPE, "selective_scan: dstate must be in [1, 32], got %lld", (long long)N);
  AK_REQUIRE(groups >= 1 && dim % groups == 0, AK_ERR_SHAPE, "selective_scan: dim %% groups != 0");
  return AK_OK;
}

int nsaved_of(int64_t L) { return (int)((L + kStateStride - 1) / kStateStride); }

// + the state-split exchange buffers: ITEMS floats per lane per non-leading group (forward),
// three such rows (y, d(delta'), du) in the backward
template <typename T, int CH>
size_t fwd_smem(int N, int cpc, int nw, int nsg) {
  return 128 + stage_bytes<T, CH>(N) + (size_t)2 * N * CH * 4 + (size_t)cpc * N * 4 +
         (size_t)(nw / nsg) * (nsg - 1) * CH * 4;
}

template <typename T, int CH>
size_t bwd_smem(int N, int cpc, int nw, int nsg) {
  return 128 + stage_bytes<T, CH>(N) + (size_t)4 * N * CH * 4 + (size_t)(2 * cpc * N + 2 * cpc) * 4 +
         (size_t)N * 4 +  // row locks
         (size_t)(nw / nsg) * (nsg - 1) * 3 * CH * 4;
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_selective_scan_state_stride(void) { return kStateStride; }

extern "C" int ak_selective_scan_fwd(void* out, float* last_state, float* chunk_states, const void* u,
                                     const void* delta, const float* A, const void* Bm, const void* Cm,
                                     const float* D, const void* z, const float* delta_bias, int delta_softplus,
                                     int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate, int64_t groups,
                                     int dt, int* status, void* stream) {
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
  p.status = status;
  p.batch = (int)batch; p.dim = (int)dim; p.L = (int)seqlen; p.N = (int)dstate; p.groups = (int)groups;
  p.dpg = (int)(dim / groups);
  p.softplus = delta_softplus ? 1 : 0;
  p.nsaved = nsaved_of(seqlen);
  p.nsg = state_groups(batch, dim, p.N);
  pick_layout(p.dpg, max_channels_per_cta(batch, dim), p.nsg, &p.nw, &p.cpw);
  const int es = elem_size(dt);
  p.bulk = (((seqlen * es) % 16) == 0 && aligned16(Bm) && aligned16(Cm)) ? 1 : 0;
  p.vec_io = (((seqlen * es) % 16) == 0 && aligned16(u) && aligned16(delta) && aligned16(out) &&
              (z == nullptr || aligned16(z))) ? 1 : 0;
  const int cpc = channels_per_cta(p);
  dim3 grid((unsigned)(dim / cpc), (unsigned)batch);
  AK_DISPATCH_DTYPE(dt, T, {
    // 16 steps per lane when the 512-step tiles fit in shared memory, else 8
    const size_t smem16 = fwd_smem<T, 32 * kFwdItems>(p.N, cpc, p.nw, p.nsg);
    const bool wide = smem16 <= 227 * 1024;
    const size_t smem = wide ? smem16 : fwd_smem<T, 32 * kItems>(p.N, cpc, p.nw, p.nsg);
    AK_REQUIRE(smem <= 227 * 1024, AK_ERR_SHAPE, "selective_scan_fwd: dstate too large for shared memory");
    auto kern = wide ? (p.nsg == 4   ? sscan_fwd_kernel<T, kFwdItems, kFwdInterleave, 4>
                        : p.nsg == 2 ? sscan_fwd_kernel<T, kFwdItems, kFwdInterleave, 2>
                                     : sscan_fwd_kernel<T, kFwdItems, kFwdInterleave, 1>)
                     : (p.nsg == 4   ? sscan_fwd_kernel<T, kItems, 2, 4>
                        : p.nsg == 2 ? sscan_fwd_kernel<T, kItems, 2, 2>
                                     : sscan_fwd_kernel<T, kItems, 2, 1>);
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
                                     int64_t seqlen, int64_t dstate, int64_t groups, int dt, int* status,
                                     void* stream) {
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
  p.status = status;
  float* ws = (float*)workspace;
  p.dB_acc = ws;
  p.dC_acc = ws + nbc;
  p.part = ws + 2 * nbc;
  p.batch = (int)batch; p.dim = (int)dim; p.L = (int)seqlen; p.N = (int)dstate; p.groups = (int)groups;
  p.dpg = (int)(dim / groups);
  p.softplus = delta_softplus ? 1 : 0;
  p.nsaved = nsaved_of(seqlen);
  p.nsg = state_groups(batch, dim, p.N);
  pick_layout(p.dpg, max_channels_per_cta(batch, dim), p.nsg, &p.nw, &p.cpw);
  const int es = elem_size(dt);
  p.bulk = (((seqlen * es) % 16) == 0 && aligned16(Bm) && aligned16(Cm)) ? 1 : 0;
  p.vec_io = (((seqlen * es) % 16) == 0 && aligned16(u) && aligned16(delta) && aligned16(dout) && aligned16(du) &&
              aligned16(ddelta) && (z == nullptr || (aligned16(z) && aligned16(dz)))) ? 1 : 0;
  constexpr int CH = 32 * kItems;
  const int cpc = channels_per_cta(p);
  AK_CUDA_TRY(cudaMemsetAsync(ws, 0, 2 * nbc * sizeof(float), st), "selective_scan_bwd: workspace clear");
  dim3 grid((unsigned)(dim / cpc), (unsigned)batch);
  AK_DISPATCH_DTYPE(dt, T, {
    const size_t smem = bwd_smem<T, CH>(p.N, cpc, p.nw, p.nsg);
    AK_REQUIRE(smem <= 227 * 1024, AK_ERR_SHAPE, "selective_scan_bwd: dstate too large for shared memory");
    auto kern = p.nsg == 4 ? sscan_bwd_kernel<T, 4> : p.nsg == 2 ? sscan_bwd_kernel<T, 2> : sscan_bwd_kernel<T, 1>;
    AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "selective_scan_bwd: smem attribute");
    kern<<<grid, p.nw * 32, smem, st>>>(p);
  });
  AK_CHECK_LAUNCH("ak_selective_scan_bwd");
  const int64_t nred = dim * (dstate + 2);
  AK_CUDA_TRY(launch_pdl(sscan_bwd_reduce, dim3((unsigned)((nred + 255) / 256)), dim3(256), 0, st, dA, dD,
                         ddelta_bias, (const float*)p.part, (int)batch, (int)dim, (int)dstate),
              "ak_selective_scan_bwd(reduce)");
  const unsigned cg = (unsigned)std::min<int64_t>((int64_t)(nbc + 255) / 256, (int64_t)sm_count() * 8);
  AK_DISPATCH_DTYPE(dt, T,
                    AK_CUDA_TRY(launch_pdl(f32_to2<T>, dim3(cg), dim3(256), 0, st, (T*)dB, (const float*)p.dB_acc,
                                           (T*)dC, (const float*)p.dC_acc, (int64_t)nbc),
                                "ak_selective_scan_bwd(convert)"));
  return AK_OK;
}
