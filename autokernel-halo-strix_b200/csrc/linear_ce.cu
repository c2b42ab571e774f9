// Fused linear + cross-entropy on sm_100a tensor cores (tcgen05 / TMEM / TMA).
//
// Semantics: kernels/hip/chunked_linear_cross_entropy.py:55-175 of the reference
// (mean CE over rows with label != ignore_index of logits = H W^T, with dH and
// dW), without its fp16 coercion, host sync, or materialised logits:
//
//   1. logits tiles = H W^T by tcgen05.mma; the epilogue reduces each 128x256
//      tile to per-row (max, sum exp) partials and picks the target logit —
//      logits never reach HBM;
//   2. a small kernel merges the partials into lse, the per-row loss and the
//      mean (n_valid counted on the device);
//   3. per chunk of rows the logits tiles are recomputed and the epilogue
//      writes G = (softmax - onehot) / n_valid directly in bf16, row-major and
//      transposed;
//   4. dH = G W and dW += G^T H by the same tcgen05 GEMM (operands pre-transposed
//      once so every GEMM reads K-major tiles).
//
// GEMM kernel: C[M,N] = A[M,K] B[N,K]^T with bf16/fp16 A, B (K contiguous) and
// fp32 accumulation in TMEM.  Persistent CTAs of 10 warps: warp 0 issues TMA
// loads (128B-swizzled 128x64 and 256x64 boxes) into a 4-stage ring, warp 1
// issues tcgen05.mma (M=128, N=256, K=16) from one thread into one of two TMEM
// accumulators (2 x 256 columns), warps 2-9 (two warpgroups, one per 128-column
// half) run the epilogue on the other accumulator via tcgen05.ld, so a tile's
// epilogue overlaps the next tile's MMAs.  All mbarrier waits are bounded (error flag + return, never a hang).
// No cluster, no TMA multicast.
#include "ak_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

namespace ak {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (2 warpgroups)
constexpr int kEpiThreads = 256;
constexpr int kHalf = BN / 2;   // columns per epilogue warpgroup
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;  // two accumulators
constexpr int kTPitch = BM + 8;    // transpose staging row pitch (16-byte aligned rows)

enum Epi : int { EPI_STATS = 0, EPI_GRAD = 1, EPI_STORE_BF16 = 2, EPI_STORE_F32 = 3 };

struct GemmArgs {
  int M, N, K;              // C is M x N; A is M x K, B is N x K
  int b_row0, a_k0, b_k0;   // coordinate offsets into the B rows and the K dimension
  // EPI_STATS
  float2* part;             // [M][ntiles] (max, sum exp2-domain)
  float* tlogit;            // [M]
  const int64_t* labels;    // [M] (already offset to the rows of this GEMM)
  int64_t ignore_index;
  // EPI_GRAD
  const float* lse;         // [M]
  const float* scale;       // device scalar: 1 / n_valid
  void* G;                  // [M][N] row-major, 16-bit
  void* GT;                 // [N][ldgt] (column block starting at gt_col0)
  int64_t ldgt, gt_col0;
  // EPI_STORE
  void* C;                  // [M][N]
  int64_t ldc;
  int accumulate;           // EPI_STORE_F32: C += acc
  int* status;              // caller's status word: AK_ERR_TIMEOUT when a bounded wait gave up
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// K-major, 128-byte swizzled operand tile: rows of 64 16-bit elements (128 B),
// 8-row swizzle atoms 1024 B apart (SBO), LBO unused (1), Blackwell version 1,
// layout type SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;           // start address
  d |= (uint64_t)1 << 16;                 // leading byte offset (16 B units)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset
  d |= (uint64_t)1 << 46;                 // version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B type, K-major both, N, M.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// The GEMM kernel
// ---------------------------------------------------------------------------
template <typename T, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
tn_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  T* sT = reinterpret_cast<T*>(smem + STAGES * STAGE_BYTES + 256);  // [2][32][kTPitch] transpose staging

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (g.M + BM - 1) / BM, ntiles = (g.N + BN - 1) / BN;
  const int ntile_total = mtiles * ntiles;
  const int ktiles = (g.K + BK - 1) / BK;  // the K tail is zero-filled by TMA in both operands

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], kEpiThreads); }
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < ntile_total; t += gridDim.x) {
        const int mt = t % mtiles, nt = t / mtiles;
        for (int kb = 0; kb < ktiles; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          mbar_wait_bounded(&empty[s], ph ^ 1u, g.status);
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          unsigned char* st = tiles + s * STAGE_BYTES;
          tma_load_2d(st, &tmA, g.a_k0 + kb * BK, mt * BM, &full[s]);
          tma_load_2d(st + A_BYTES, &tmB, g.b_k0 + kb * BK, g.b_row0 + nt * BN, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(sizeof(T) == 2 && !std::is_same<T, __half>::value, BM, BN);
      int it = 0, local = 0;
      for (int t = blockIdx.x; t < ntile_total; t += gridDim.x, ++local) {
        const int acc = local & 1;
        mbar_wait_bounded(&tempty[acc], ((uint32_t)(local >> 1) & 1u) ^ 1u, g.status);
        tc_fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < ktiles; ++kb, ++it) {
          const int s = it % STAGES;
          mbar_wait_bounded(&full[s], (uint32_t)(it / STAGES) & 1u, g.status);
          tc_fence_after();
          const unsigned char* st = tiles + s * STAGE_BYTES;
          const uint64_t ad = smem_desc_sw128(st), bd = smem_desc_sw128(st + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // advance 32 B (16 elements) inside the swizzle row
            mma_f16(dcol, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb | k) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5 own TMEM lanes 32*(warp%4) ...
    const int quad = warp & 3;
    const int eg = (warp - 2) >> 2;           // epilogue warpgroup: column half
    T* sTg = sT + eg * 32 * kTPitch;
    const int rl = quad * 32 + lane;  // row within the tile
    int local = 0;
    for (int t = blockIdx.x; t < ntile_total; t += gridDim.x, ++local) {
      const int mt = t % mtiles, nt = t / mtiles;
      const int acc = local & 1;
      mbar_wait_bounded(&tfull[acc], (uint32_t)(local >> 1) & 1u, g.status);
      tc_fence_after();
      const int row = mt * BM + rl;
      const bool rv = row < g.M;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      const int col0 = nt * BN;
      if constexpr (EPI == EPI_STATS) {
        const int64_t lab = rv ? g.labels[row] : -1;
        float m = -INFINITY, s = 0.f;  // s: sum of exp2(x*log2e - m) with m in log2 units
        for (int c = eg * kHalf; c < (eg + 1) * kHalf; c += 32) {
          float v[32];
          tmem_ld32(tbase + (uint32_t)c, v);
          if (g.G != nullptr) {
            // logits kept in 16 bits for the gradient pass; the statistics use the
            // same rounded values so that softmax and lse stay consistent
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = to_f<T>(from_f<T>(v[j]));
            const int cbase = col0 + c;
            T* lrow = reinterpret_cast<T*>(g.G) + (int64_t)row * g.N;
            if (rv && cbase + 32 <= g.N) {
#pragma unroll
              for (int q = 0; q < 32; q += 8) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[q + e];
                store_frag<T, 8>(lrow + cbase + q, f);
              }
            } else if (rv) {
              for (int j = 0; j < 32; ++j)
                if (cbase + j < g.N) lrow[cbase + j] = from_f<T>(v[j]);
            }
          }
          float lm = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = col0 + c + j;
            v[j] = (col < g.N) ? v[j] * kLog2e : -INFINITY;
            lm = fmaxf(lm, v[j]);
            if (col == lab && rv) g.tlogit[row] = v[j] * kLn2;
          }
          const float mn = fmaxf(m, lm);
          if (mn != -INFINITY) {
            float a = s * ex2(m - mn);
#pragma unroll
            for (int j = 0; j < 32; ++j) a += ex2(v[j] - mn);
            s = a;
            m = mn;
          }
        }
        if (rv) g.part[(int64_t)row * (2 * ntiles) + 2 * nt + eg] = make_float2(m, s);
      } else if constexpr (EPI == EPI_GRAD) {
        const int64_t lab = rv ? g.labels[row] : g.ignore_index;
        const bool ign = (lab == g.ignore_index);
        const float sc = ign ? 0.f : *g.scale;
        const float lse2 = rv ? g.lse[row] * kLog2e : 0.f;
        T* grow = reinterpret_cast<T*>(g.G) + (int64_t)row * g.N;
        T* gt = reinterpret_cast<T*>(g.GT);
        for (int c = eg * kHalf; c < (eg + 1) * kHalf; c += 32) {
          float v[32];
          tmem_ld32(tbase + (uint32_t)c, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = col0 + c + j;
            float gv = ex2(fmaf(v[j], kLog2e, -lse2)) * sc;
            if (col == lab) gv -= sc;
            v[j] = gv;
          }
          const int cbase = col0 + c;
          if (rv) {
            if (cbase + 32 <= g.N) {
#pragma unroll
              for (int q = 0; q < 32; q += 8) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[q + e];
                store_frag<T, 8>(grow + cbase + q, f);
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (cbase + j < g.N) grow[cbase + j] = from_f<T>(v[j]);
            }
          }
          // G^T: transpose the 128x32 block through shared memory, then 16-byte
          // coalesced stores of 8 consecutive rows per thread.
#pragma unroll
          for (int j = 0; j < 32; ++j) sTg[j * kTPitch + rl] = from_f<T>(v[j]);
          asm volatile("bar.sync %0, 128;" ::"r"(1 + eg) : "memory");
          const int e = (threadIdx.x - 64) & 127;
#pragma unroll
          for (int q = e; q < 32 * (BM / 8); q += 128) {
            const int cj = q / (BM / 8), rc = q - cj * (BM / 8);
            const int r0 = mt * BM + rc * 8;
            if (cbase + cj < g.N && r0 < g.M)
              *reinterpret_cast<int4*>(gt + (int64_t)(cbase + cj) * g.ldgt + g.gt_col0 + r0) =
                  *reinterpret_cast<const int4*>(sTg + cj * kTPitch + rc * 8);
          }
          asm volatile("bar.sync %0, 128;" ::"r"(1 + eg) : "memory");
        }
      } else {
        for (int c = eg * kHalf; c < (eg + 1) * kHalf; c += 32) {
          float v[32];
          tmem_ld32(tbase + (uint32_t)c, v);
          const int cbase = col0 + c;
          if (!rv) continue;
          if constexpr (EPI == EPI_STORE_BF16) {
            T* crow = reinterpret_cast<T*>(g.C) + (int64_t)row * g.ldc;
            if (cbase + 32 <= g.N) {
#pragma unroll
              for (int q = 0; q < 32; q += 8) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[q + e];
                store_frag<T, 8>(crow + cbase + q, f);
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (cbase + j < g.N) crow[cbase + j] = from_f<T>(v[j]);
            }
          } else {
            float* crow = reinterpret_cast<float*>(g.C) + (int64_t)row * g.ldc;
            if (cbase + 32 <= g.N) {
#pragma unroll
              for (int q = 0; q < 32; q += 4) {
                float4* p4 = reinterpret_cast<float4*>(crow + cbase + q);
                float4 o = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                if (g.accumulate) {
                  const float4 old = *p4;
                  o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
                }
                *p4 = o;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (cbase + j < g.N) crow[cbase + j] = v[j] + (g.accumulate ? crow[cbase + j] : 0.f);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
}

// ---------------------------------------------------------------------------
// Side kernels
// ---------------------------------------------------------------------------
// Merge the per-tile partials: lse (natural log), per-row loss, and the mean.
__global__ void __launch_bounds__(256)
lce_rows_reduce(float* __restrict__ lse, float* __restrict__ losses, const float2* __restrict__ part,
                const float* __restrict__ tlogit, const int64_t* __restrict__ labels, int M, int ntiles,
                int64_t ignore_index) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int t = lane; t < ntiles; t += 32) {
    const float2 p = part[(int64_t)warp * ntiles + t];
    const float mn = fmaxf(m, p.x);
    if (mn != -INFINITY) { s = s * ex2(m - mn) + p.y * ex2(p.x - mn); m = mn; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o), so = __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, mo);
    if (mn != -INFINITY) { s = s * ex2(m - mn) + so * ex2(mo - mn); m = mn; }
  }
  if (lane == 0) {
    const float l = (m + lg2(s)) * kLn2;
    lse[warp] = l;
    const bool ign = labels[warp] == ignore_index;
    losses[warp] = ign ? 0.f : l - tlogit[warp];
  }
}

__global__ void __launch_bounds__(1024)
lce_mean(float* __restrict__ loss, float* __restrict__ inv_valid, const float* __restrict__ losses,
         const int64_t* __restrict__ labels, int64_t M, int64_t ignore_index) {
  __shared__ float r0[32], r1[32];
  float a = 0.f, n = 0.f;
#pragma unroll 4
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) {
    const int64_t lb = labels[i];
    const float li = losses[i];  // unconditional: both loads in flight together
    if (lb != ignore_index) { a += li; n += 1.f; }
  }
  a = warp_sum(a);
  n = warp_sum(n);
  if ((threadIdx.x & 31) == 0) { r0[threadIdx.x >> 5] = a; r1[threadIdx.x >> 5] = n; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float A = 0.f, Nn = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { A += r0[i]; Nn += r1[i]; }
    Nn = fmaxf(Nn, 1.f);
    loss[0] = A / Nn;
    inv_valid[0] = 1.f / Nn;
  }
}

// out[c][r] = in[r][c] for a 16-bit [R][Cc] matrix (32x32 tiles through shared memory).
template <typename T>
__global__ void transpose16(T* __restrict__ out, const T* __restrict__ in, int64_t R, int64_t Cc) {
  __shared__ T tile[32][33];
  const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < Cc) tile[i][threadIdx.x] = in[r * Cc + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < Cc) out[c * R + r] = tile[threadIdx.x][i];
  }
}

// In place over 16-bit logits L[M][V]: L = (softmax(L) - onehot(label)) / n_valid,
// zero rows for ignored labels.  V % 8 == 0.  A CTA walks whole rows (the row's
// lse and label stay in registers, no per-vector division); each thread loads
// kGradBatch 16-byte vectors before using any of them.
constexpr int kGradBatch = 4;

template <typename T>
__global__ void __launch_bounds__(256)
lce_grad_inplace(T* __restrict__ L, const float* __restrict__ lse, const int64_t* __restrict__ labels,
                 const float* __restrict__ inv_valid, int64_t M, int64_t V, int64_t ignore_index) {
  const float sc0 = *inv_valid;
  const int nv = (int)(V / 8);
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t lab = labels[row];
    const float sc = (lab == ignore_index) ? 0.f : sc0;
    const float l2 = lse[row] * kLog2e;
    T* Lr = L + row * V;
    for (int v0 = threadIdx.x; v0 < nv; v0 += kGradBatch * 256) {
      float f[kGradBatch][8];
#pragma unroll
      for (int u = 0; u < kGradBatch; ++u)
        if (v0 + u * 256 < nv) load_frag<T, 8>(f[u], Lr + (int64_t)(v0 + u * 256) * 8);
#pragma unroll
      for (int u = 0; u < kGradBatch; ++u) {
        const int v = v0 + u * 256;
        if (v >= nv) break;
        const int64_t col = (int64_t)v * 8;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float gv = ex2(fmaf(f[u][k], kLog2e, -l2)) * sc;
          if (col + k == lab) gv -= sc;
          f[u][k] = gv;
        }
        store_frag<T, 8>(Lr + col, f[u]);
      }
    }
  }
}

template <typename T>
__global__ void cast_f32(T* __restrict__ dst, const float* __restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f<T>(src[i]);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int make_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows, bool bf16) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  // Resolved through the runtime so the library does not link libcuda directly.
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    AK_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                "linear_ce: driver entry point");
    AK_REQUIRE(fn != nullptr && q == cudaDriverEntryPointSuccess, AK_ERR_LAUNCH,
               "linear_ce: cuTensorMapEncodeTiled unavailable");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                            2, const_cast<void*>(base), dims, strides, box, estr,
                                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AK_REQUIRE(r == CUDA_SUCCESS, AK_ERR_ARG, "linear_ce: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AK_OK;
}

constexpr size_t kSmem = (size_t)STAGES * STAGE_BYTES + 1024 + 256 + 2 * 32 * kTPitch * 2;

template <typename T, int EPI>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  auto kern = tn_gemm_kernel<T, EPI>;
  AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem),
              "linear_ce: smem attribute");
  const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, sm_count()));
  kern<<<grid, kThreads, kSmem, st>>>(ta, tb, g);
  AK_CHECK_LAUNCH("linear_ce: tcgen05 gemm");
  return AK_OK;
}

struct Ws {
  float2* part;
  float* tlogit;
  float* losses;
  float* inv_valid;
  void* WT;
  void* HT;
  void* G;
  void* GT;
  float* dWacc;
  size_t bytes;
};

// Rows per gradient chunk: large chunks keep the dH / dW GEMMs several waves deep.
int64_t chunk_rows(int64_t N) { return std::min<int64_t>(N, 32768); }

Ws carve(void* base, int64_t N, int64_t D, int64_t V) {
  Ws w{};
  const int64_t ntiles = (V + BN - 1) / BN;
  const int64_t Nc = chunk_rows(N);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 255) & ~size_t(255);
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off += bytes;
    return p;
  };
  w.part = reinterpret_cast<float2*>(take((size_t)N * ntiles * 2 * sizeof(float2)));  // one per column half
  w.tlogit = reinterpret_cast<float*>(take((size_t)N * 4));
  w.losses = reinterpret_cast<float*>(take((size_t)N * 4));
  w.inv_valid = reinterpret_cast<float*>(take(4));
  w.WT = take((size_t)D * V * 2);
  w.HT = take((size_t)D * N * 2);
  w.G = take((size_t)Nc * V * 2);
  w.GT = take((size_t)V * Nc * 2);
  w.dWacc = reinterpret_cast<float*>(take((size_t)V * D * 4));
  w.bytes = off + 256;
  return w;
}

template <typename T>
int run(float* loss, float* lse, void* dH, void* dW, const Ws& w, const void* H, const void* W,
        const int64_t* labels, int64_t N, int64_t D, int64_t V, int64_t ignore_index, int* status,
        cudaStream_t st) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const int ntiles = (int)((V + BN - 1) / BN);
  // 0. K-major copies of W^T and H^T for the gradient GEMMs
  {
    dim3 b(32, 8);
    transpose16<T><<<dim3((unsigned)((D + 31) / 32), (unsigned)((V + 31) / 32)), b, 0, st>>>((T*)w.WT, (const T*)W, V, D);
    transpose16<T><<<dim3((unsigned)((D + 31) / 32), (unsigned)((N + 31) / 32)), b, 0, st>>>((T*)w.HT, (const T*)H, N, D);
    AK_CHECK_LAUNCH("linear_ce: transpose");
  }
  CUtensorMap tH, tW, tG, tWT, tGT, tHT;
  int rc;
  if ((rc = make_tmap(&tH, H, N, D, BM, bf16))) return rc;
  if ((rc = make_tmap(&tW, W, V, D, BN, bf16))) return rc;
  if ((rc = make_tmap(&tWT, w.WT, D, V, BN, bf16))) return rc;
  if ((rc = make_tmap(&tHT, w.HT, D, N, BN, bf16))) return rc;
  // 1. logits tiles -> per-row partial (max, sum exp)
  {
    GemmArgs g{};
    g.status = status;
    g.M = (int)N; g.N = (int)V; g.K = (int)D;
    g.part = w.part; g.tlogit = w.tlogit; g.labels = labels; g.ignore_index = ignore_index;
    if ((rc = launch_gemm<T, EPI_STATS>(tH, tW, g, st))) return rc;
  }
  // 2. lse, per-row loss, mean and 1/n_valid on the device
  lce_rows_reduce<<<(unsigned)((N * 32 + 255) / 256), 256, 0, st>>>(lse, w.losses, w.part, w.tlogit, labels, (int)N,
                                                                    2 * ntiles, ignore_index);
  lce_mean<<<1, 1024, 0, st>>>(loss, w.inv_valid, w.losses, labels, N, ignore_index);
  AK_CHECK_LAUNCH("linear_ce: reduce");
  // 3-4. per row chunk: G tiles, dH = G W, dW += G^T H
  const int64_t Nc = chunk_rows(N);
  for (int64_t r0 = 0; r0 < N; r0 += Nc) {
    const int64_t nr = std::min(Nc, N - r0);
    CUtensorMap tHc;
    if ((rc = make_tmap(&tHc, static_cast<const T*>(H) + r0 * D, nr, D, BM, bf16))) return rc;
    if ((rc = make_tmap(&tG, w.G, nr, V, BM, bf16))) return rc;
    if ((rc = make_tmap(&tGT, w.GT, V, nr, BM, bf16))) return rc;
    {
      GemmArgs g{};
    g.status = status;
      g.M = (int)nr; g.N = (int)V; g.K = (int)D;
      g.labels = labels + r0; g.ignore_index = ignore_index;
      g.lse = lse + r0; g.scale = w.inv_valid;
      g.G = w.G; g.GT = w.GT; g.ldgt = nr; g.gt_col0 = 0;
      if ((rc = launch_gemm<T, EPI_GRAD>(tHc, tW, g, st))) return rc;
    }
    if (dH) {  // dH[r0:r0+nr] = G W  (A = G [nr, V], B = W^T [D, V])
      GemmArgs g{};
    g.status = status;
      g.M = (int)nr; g.N = (int)D; g.K = (int)V;
      g.C = static_cast<T*>(dH) + r0 * D; g.ldc = D;
      if ((rc = launch_gemm<T, EPI_STORE_BF16>(tG, tWT, g, st))) return rc;
    }
    if (dW) {  // dW += G^T H  (A = G^T [V, nr], B = H^T [D, N] columns r0..r0+nr)
      GemmArgs g{};
    g.status = status;
      g.M = (int)V; g.N = (int)D; g.K = (int)nr; g.b_k0 = (int)r0;
      g.C = w.dWacc; g.ldc = D; g.accumulate = r0 > 0;
      if ((rc = launch_gemm<T, EPI_STORE_F32>(tGT, tHT, g, st))) return rc;
    }
  }
  if (dW) {
    const int64_t n = V * D;
    cast_f32<T><<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8), 256, 0, st>>>((T*)dW, w.dWacc, n);
    AK_CHECK_LAUNCH("linear_ce: dW cast");
  }
  return AK_OK;
}

int check_shape(int64_t N, int64_t D, int64_t V, int dt) {
  AK_REQUIRE(dt == AK_BF16 || dt == AK_F16, AK_ERR_DTYPE, "linear_ce: tensor-core path takes bf16 or fp16");
  AK_REQUIRE(N > 0 && D > 0 && V > 0, AK_ERR_SHAPE, "linear_ce: empty problem");
  AK_REQUIRE(D % 8 == 0 && D <= (1 << 20), AK_ERR_SHAPE, "linear_ce: hidden size must be a multiple of 8");
  AK_REQUIRE(V % 8 == 0 && N % 8 == 0, AK_ERR_SHAPE, "linear_ce: rows and vocab must be multiples of 8");
  AK_REQUIRE(N < (1LL << 31) && V < (1LL << 31), AK_ERR_SHAPE, "linear_ce: too large");
  return AK_OK;
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_linear_ce_workspace_size(int64_t N, int64_t D, int64_t V, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes != nullptr, AK_ERR_ARG, "null bytes");
  AK_REQUIRE(N > 0 && D > 0 && V > 0, AK_ERR_SHAPE, "linear_ce: empty problem");
  *bytes = carve(nullptr, N, D, V).bytes;
  return AK_OK;
}

extern "C" int ak_linear_ce_fwdbwd(float* loss, float* lse, void* dH, void* dW, void* workspace, size_t ws_bytes,
                                   const void* H, const void* W, const int64_t* labels, int64_t N, int64_t D,
                                   int64_t V, int64_t ignore_index, int dt, int* status, void* stream) {
  clear_error();
  int rc = check_shape(N, D, V, dt);
  if (rc) return rc;
  AK_REQUIRE(loss && lse && H && W && labels, AK_ERR_ARG, "ak_linear_ce_fwdbwd: null pointer");
  AK_REQUIRE(aligned16(H) && aligned16(W) && (!dH || aligned16(dH)), AK_ERR_ARG,
             "ak_linear_ce_fwdbwd: H, W, dH must be 16-byte aligned");
  const Ws need = carve(nullptr, N, D, V);
  AK_REQUIRE(workspace && ws_bytes >= need.bytes, AK_ERR_WORKSPACE, "ak_linear_ce_fwdbwd: workspace %zu < %zu",
             ws_bytes, need.bytes);
  void* base = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const Ws w = carve(base, N, D, V);
  cudaStream_t st = (cudaStream_t)stream;
  if (dt == AK_BF16) return run<__nv_bfloat16>(loss, lse, dH, dW, w, H, W, labels, N, D, V, ignore_index, status, st);
  return run<__half>(loss, lse, dH, dW, w, H, W, labels, N, D, V, ignore_index, status, st);
}

extern "C" int ak_linear_ce_logits_grad_workspace_size(int64_t N, int64_t V, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes != nullptr && N > 0 && V > 0, AK_ERR_ARG, "linear_ce: bad args");
  const int64_t ntiles = (V + BN - 1) / BN;
  *bytes = (size_t)N * ntiles * 2 * sizeof(float2) + (size_t)N * 8 + 1024;
  return AK_OK;
}

extern "C" int ak_linear_ce_logits_grad(float* loss, float* lse, void* G, void* workspace, size_t ws_bytes,
                                        const void* H, const void* W, const int64_t* labels, int64_t N, int64_t D,
                                        int64_t V, int64_t ignore_index, int dt, int* status, void* stream) {
  clear_error();
  int rc = check_shape(N, D, V, dt);
  if (rc) return rc;
  AK_REQUIRE(loss && lse && G && H && W && labels, AK_ERR_ARG, "ak_linear_ce_logits_grad: null pointer");
  AK_REQUIRE(aligned16(H) && aligned16(W) && aligned16(G), AK_ERR_ARG, "ak_linear_ce_logits_grad: unaligned");
  size_t need = 0;
  ak_linear_ce_logits_grad_workspace_size(N, V, &need);
  AK_REQUIRE(workspace && ws_bytes >= need, AK_ERR_WORKSPACE, "ak_linear_ce_logits_grad: workspace %zu < %zu",
             ws_bytes, need);
  const int ntiles = (int)((V + BN - 1) / BN);
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  float2* part = reinterpret_cast<float2*>(base);
  float* tlogit = reinterpret_cast<float*>(part + (size_t)N * ntiles * 2);
  float* losses = tlogit + N;
  float* inv_valid = losses + N;  // one float after the per-row losses
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf16 = dt == AK_BF16;
  CUtensorMap tH, tW;
  if ((rc = make_tmap(&tH, H, N, D, BM, bf16))) return rc;
  if ((rc = make_tmap(&tW, W, V, D, BN, bf16))) return rc;
  GemmArgs g{};
    g.status = status;
  g.M = (int)N; g.N = (int)V; g.K = (int)D;
  g.part = part; g.tlogit = tlogit; g.labels = labels; g.ignore_index = ignore_index; g.G = G;
  if (bf16) rc = launch_gemm<__nv_bfloat16, EPI_STATS>(tH, tW, g, st);
  else rc = launch_gemm<__half, EPI_STATS>(tH, tW, g, st);
  if (rc) return rc;
  lce_rows_reduce<<<(unsigned)((N * 32 + 255) / 256), 256, 0, st>>>(lse, losses, part, tlogit, labels, (int)N,
                                                                    2 * ntiles, ignore_index);
  lce_mean<<<1, 1024, 0, st>>>(loss, inv_valid, losses, labels, N, ignore_index);
  const unsigned grid = (unsigned)std::min<int64_t>(N, (int64_t)sm_count() * 8);
  if (bf16)
    lce_grad_inplace<__nv_bfloat16><<<grid, 256, 0, st>>>((__nv_bfloat16*)G, lse, labels, inv_valid, N, V,
                                                         ignore_index);
  else
    lce_grad_inplace<__half><<<grid, 256, 0, st>>>((__half*)G, lse, labels, inv_valid, N, V, ignore_index);
  AK_CHECK_LAUNCH("ak_linear_ce_logits_grad");
  return AK_OK;
}
