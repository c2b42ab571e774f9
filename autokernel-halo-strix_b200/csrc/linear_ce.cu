// Fused linear + cross-entropy on sm_100a tensor cores (tcgen05 / TMEM / TMA).
//
// Semantics: kernels/hip/chunked_linear_cross_entropy.py:55-175 of the reference
// (mean CE over rows with label != ignore_index of logits = H W^T, with dH and
// dW), without its fp16 coercion, host sync or cuBLAS GEMMs.  Per chunk of up to
// kChunkRows rows:
//
//   1. logits = H_c W^T on the tensor cores; the epilogue reduces each tile to
//      per-row (max, sum exp) partials, picks the target logit and stores the
//      16-bit logits into the chunk buffer G_c;
//   2. a row kernel merges the partials into lse and the per-row loss;
//   3. a streaming kernel turns G_c in place into softmax - onehot (unscaled: the
//      dW / dH epilogues apply 1 / n_valid to the fp32 accumulators);
//   4. one grouped launch of the same GEMM kernel computes dW (+)= G_c^T H_c and
//      dH_c = G_c W, reading G_c, H and W in their row-major layouts (the
//      operands whose contiguous dimension is M or N use MN-major shared-memory
//      descriptors, so nothing is transposed).
//
// Full logits never exist: G_c holds kChunkRows rows at most.  Why G_c is
// materialised at all: an accumulator for dH (128 rows x D = 768 fp32) or dW
// (128 vocab rows x 768) does not fit the 512 TMEM columns next to a logits
// tile, and keeping one of them outside TMEM costs more HBM traffic than
// writing and re-reading G_c once.
//
// GEMM kernel: C[M,N] = A[M,K] B[N,K]^T, bf16/fp16 operands, fp32 accumulation.
// Clusters of two CTAs on a TPC issue tcgen05.mma.cta_group::2 (M = 256 split
// over the pair, N = 256): each CTA stages its 128 rows of A and its 128 rows of
// B per 64-deep K block by TMA (no multicast) and accumulates its 128 x 256
// half of the tile in its own TMEM.  Per CTA: warp 0 issues TMA into a 6-stage
// ring (both CTAs' copies complete on the leader CTA's barrier), warp 1 of the
// leader issues the MMAs from one thread into one of two TMEM accumulators,
// warps 2-9 (two warpgroups, one per 128-column half) run the epilogue on the
// other accumulator, so a tile's epilogue overlaps the next tile's MMAs.
// Persistent: each CTA pair walks the tiles of up to two problems (the dW and
// dH contractions share one launch; their short- and long-K tiles are
// list-scheduled, see sched_tile).  Every mbarrier wait is bounded: on a
// timeout AK_ERR_TIMEOUT goes to the caller's status word, the CTA stops
// issuing loads and MMAs, drains what it issued, frees TMEM and finishes.
#include "ak_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

namespace ak {
namespace {

constexpr int BM = 128;            // rows of A per CTA (256 per CTA pair)
constexpr int BN = 256;            // tile columns (each CTA stages half of B)
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int kEpiGroups = 2;      // epilogue warpgroups, one per 128-column half of the tile
constexpr int kEpiWarps = 4 * kEpiGroups;
constexpr int kThreads = 32 * (2 + kEpiWarps);  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kGroupCols = BN / kEpiGroups;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = (BN / 2) * BK * 2;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA
constexpr int TMEM_COLS = 2 * BN;  // two accumulators
constexpr int64_t kChunkRows = 16384;
constexpr int kTileOverheadK = 4;  // per-tile cost beyond its K blocks, in K blocks (list schedule)

enum Epi : int { EPI_STATS = 0, EPI_STORE = 1, EPI_NONE = 2 };  // EPI_NONE: accumulate only (timing)

struct Prob {
  int M, N, K;
  int a_mn, b_mn;           // 1: the operand's M (N) dimension is contiguous in memory
  int epi;
  int mtiles, ntiles, tiles;
  // EPI_STATS: per-row (max, sum exp2) partial per 128-column half, target logit,
  // and optionally the 16-bit logits (C, ldc)
  float2* part;             // [M][kEpiGroups * ntiles]
  float* tlogit;            // [M]
  const int64_t* labels;    // [M]
  int64_t ignore_index;
  // EPI_STORE: C = acc (+ add_f32) (+ C if accumulate), fp32 (c_f32) or 16-bit
  void* C;
  int64_t ldc;
  const float* add_f32;     // nullable, same layout as C
  const float* scale;       // nullable device scalar multiplying acc (before add_f32 / accumulate)
  int c_f32, accumulate;
};

// Two problems whose tiles differ in K (dW's short-K tiles and dH's long-K ones)
// are list-scheduled: the long tiles first, round robin, then every pair takes
// the next short tile whenever it becomes free.  lp = the long problem (-1: one
// class, plain round robin); cL / cS = tile costs in K blocks (+ a per-tile
// overhead), which fix the order in which pairs become free.
struct Group {
  Prob p[2];
  int nprob, total;
  int* status;
  int lp, nL, nS, cL, cS;
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Cluster-wide barrier.  The warp reconverges first: in the producer and MMA
// warps one lane runs the pipeline while the others wait here.
__device__ __forceinline__ void cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}

// Tiled 2-D TMA load into this CTA's shared memory; the transaction bytes are
// counted on `bar`, which may be the peer CTA's barrier (cluster address).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 128-byte swizzled operand tile descriptor.  K-major: rows of 64 16-bit K
// elements (128 B), 8-row atoms 1024 B apart (SBO), LBO unused.  MN-major: rows
// of 64 contiguous M (or N) elements per K index, 8-K-row atoms 1024 B apart
// (SBO), and the next 64 M (N) elements `mn_block` bytes further (LBO).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, bool mn, uint32_t mn_block) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((mn ? (mn_block >> 4) : 1u) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B type, majorness, N, M.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int m, int n, int a_mn, int b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma2(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (cluster address: this CTA's or the peer's) once every
// tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void commit2(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on a barrier given by cluster address (this CTA's or the peer's).  The
// default CTA-scope release: the arrival only has to follow this thread's TMEM
// reads (completed by tcgen05.wait::ld and fenced by tcgen05.fence), not make
// its global stores visible, which a cluster-scope release would wait for.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded waits.  The first wait of a CTA that runs out reports AK_ERR_TIMEOUT
// and raises the CTA's abort flag; every later wait of that CTA then returns at
// once, so a broken pipeline ends the kernel after one time-out instead of one
// per stage.  `cluster` waits also acquire what the peer CTA released before
// arriving.
struct Waiter {
  int* status;
  volatile int* abort;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait in one launch

template <bool kCluster>
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const Waiter& w) {
  if (*w.abort) return false;
  if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
    if ((i & 255u) == 0) {
      if (*w.abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) break;
    }
  }
  *w.abort = 1;
  report_status(w.status, (int)AK_ERR_TIMEOUT);
  return false;
}

// Abort-path drains.  drain_bar: a bounded wait on one phase that ignores the
// abort flag (the MMA issuer's last commit, so TMEM is never freed under a
// running MMA).  drain_grace: the producer's loads still in flight land on the
// leader CTA's barrier, which a peer CTA cannot poll, so it waits a fixed 1 ms
// (a tile load takes microseconds) before leaving the loop.
__device__ __forceinline__ bool drain_bar(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    __nanosleep(256);
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

__device__ __forceinline__ void drain_grace() {
  const uint64_t t0 = global_ns();
  while (global_ns() - t0 < 1000000ull) __nanosleep(1000);
}

// 32 consecutive fp32 columns of this thread's TMEM lane, as an asynchronous
// load (tmem_ld_issue) completed by tmem_ld_wait.  The wait names the
// destination registers as in-out operands, so no use of them can be moved
// above it; a load of the next columns can run while the current ones are used.
struct Tm32 {
  uint32_t r[32];
};

__device__ __forceinline__ void tmem_ld_issue(uint32_t taddr, Tm32& t) {
  uint32_t* r = t.r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait(Tm32& t) {
  uint32_t* r = t.r;
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// ---- 16-bit row tiles through shared memory -------------------------------
// A warp's 32 rows x 64 columns (one row per lane, two 32-column halves) are
// written to a 4 KB tile (row r at r * 128 B, 16-byte chunk c stored at chunk
// position c ^ (r & 7): conflict-free on both sides) and leave as 16-byte
// global stores that cover four full 128-byte lines per instruction, instead
// of 32 partial lines when every lane stores its own row.
constexpr int kStageWarpBytes = 32 * 128;

template <typename T>
__device__ __forceinline__ void stage_put(uint32_t stg, int lane, int half, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    Frag<T, 8> f;
#pragma unroll
    for (int e = 0; e < 8; ++e) f.v[e] = from_f<T>(v[8 * q + e]);
    const uint4 u = *reinterpret_cast<const uint4*>(&f);
    const uint32_t pos = (uint32_t)((4 * half + q) ^ (lane & 7));
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stg + (uint32_t)lane * 128u + pos * 16u),
                 "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                 : "memory");
  }
}

// Rows row0 .. row0+31 (those below nrows), 64 columns starting at col.
template <typename T>
__device__ __forceinline__ void stage_flush(uint32_t stg, int lane, T* C, int64_t ldc, int64_t row0, int nrows,
                                            int col) {
  const int q = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int R = 4 * i + (lane >> 3);
    uint4 u;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "r"(stg + (uint32_t)R * 128u + (uint32_t)((q ^ (R & 7)) * 16))
                 : "memory");
    if (R < nrows) *reinterpret_cast<uint4*>(C + (row0 + R) * ldc + col + 8 * q) = u;
  }
}

// Global tile index -> (problem, m tile, n tile).  Tiles are visited in groups
// of kGroupM m tiles: inside a group the m tile varies fastest, so the ~74 CTA
// pairs working at one time cover a compact block of about 8 m tiles x 9 n
// tiles, and both operands' tiles are reused from L2 instead of one of them
// streaming from HBM once per tile row or column.
constexpr int kGroupM = 8;

__device__ __forceinline__ void decode_tile(const Group& g, int t, int& pi, int& mt, int& nt) {
  pi = (g.nprob > 1 && t >= g.p[0].tiles) ? 1 : 0;
  const Prob& P = pi ? g.p[1] : g.p[0];
  const int l = pi ? t - g.p[0].tiles : t;
  const int per_group = kGroupM * P.ntiles;
  const int grp = l / per_group, r = l - grp * per_group;
  const int m0 = grp * kGroupM;
  const int gm = min(kGroupM, P.mtiles - m0);
  mt = m0 + r % gm;
  nt = r / gm;
}

// The tile of this pair's k-th turn (decode_tile's numbering), or -1 when it has no more.
// Long tiles: pair + k * npairs.  Short tiles: pair p makes its j-th grab at time
// tau = nl(p) * cL + j * cS, and grabs are served in (time, pair) order, so the
// grab's short index is the number of grabs of all pairs that come before it: the
// first r pairs (q + 1 long tiles) start at (q + 1) * cL, the others at q * cL.
// Every role of both CTAs computes the same sequence, so nothing is exchanged.
__device__ __forceinline__ int sched_tile(const Group& g, int pair, int npairs, int k) {
  if (g.lp < 0) {
    const int t = pair + k * npairs;
    return t < g.total ? t : -1;
  }
  const int q = g.nL / npairs, r = g.nL - q * npairs;
  const int nl = q + (pair < r ? 1 : 0);
  if (k < nl) {
    const int l = pair + k * npairs;
    return g.lp == 0 ? l : g.p[0].tiles + l;
  }
  const int64_t cL = g.cL, cS = g.cS;
  const int64_t tau = (int64_t)nl * cL + (int64_t)(k - nl) * cS;
  const int64_t xa = tau - (int64_t)(q + 1) * cL, xb = tau - (int64_t)q * cL;
  const int64_t na = xa <= 0 ? 0 : (xa + cS - 1) / cS, nb = xb <= 0 ? 0 : (xb + cS - 1) / cS;
  int64_t sidx = (int64_t)r * na + (int64_t)(npairs - r) * nb;
  if (xa >= 0 && xa % cS == 0) sidx += min(pair, r);
  if (xb >= 0 && xb % cS == 0) sidx += max(0, pair - r);
  if (sidx >= g.nS) return -1;
  return g.lp == 0 ? g.p[0].tiles + (int)sidx : (int)sidx;
}

// This pair's tile after `prev` (its k-th turn).  kList = false: plain round robin,
// the loop the single-class launches compile to; true: sched_tile.
template <bool kList>
__device__ __forceinline__ int next_tile(const Group& g, int pair, int npairs, int k, int prev) {
  if constexpr (kList) {
    return sched_tile(g, pair, npairs, k);
  } else {
    const int t = k == 0 ? pair : prev + npairs;
    return t < g.total ? t : -1;
  }
}

// ---------------------------------------------------------------------------
// Epilogues (one lane = one row of the warp's 32; a warpgroup = 128 rows x its columns)
// ---------------------------------------------------------------------------
// Softmax statistics of 32 logits of this lane's row (natural units in v).
__device__ __forceinline__ void stats_chunk(const float (&v)[32], int cbase, int N, float& m, float& s) {
  // the maximum is taken on the raw logits (log2 e > 0 and rounding are monotone, so it equals
  // the maximum of the scaled ones); each exponent argument is then one paired FMA x log2e - m
  float2 v2[16];
  const float2 l2e = make_float2(kLog2e, kLog2e);
#pragma unroll
  for (int j = 0; j < 16; ++j) v2[j] = make_float2(v[2 * j], v[2 * j + 1]);
  if (cbase + 32 > N) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (cbase + 2 * j >= N) v2[j].x = -INFINITY;
      if (cbase + 2 * j + 1 >= N) v2[j].y = -INFINITY;
    }
  }
  float lm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 16; ++j) lm = fmaxf(lm, fmaxf(v2[j].x, v2[j].y));
  const float mn = fmaxf(m, lm * kLog2e);
  if (mn != -INFINITY) {
    const float2 neg = make_float2(-mn, -mn);
    float2 a2 = make_float2(s * ex2(m - mn), 0.f);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 d = __ffma2_rn(v2[j], l2e, neg);
      a2 = __fadd2_rn(a2, make_float2(ex2(d.x), ex2(d.y)));
    }
    s = a2.x + a2.y;
    m = mn;
  }
}

template <typename T>
__device__ __forceinline__ void put_row16(T* crow, int cbase, int N, const float (&v)[32]) {
  if (cbase + 32 <= N) {
#pragma unroll
    for (int q = 0; q < 32; q += 8) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = v[q + e];
      store_frag<T, 8>(crow + cbase + q, f);
    }
  } else {
    for (int j = 0; j < 32; ++j)
      if (cbase + j < N) crow[cbase + j] = from_f<T>(v[j]);
  }
}

// Per-row (max, sum exp2) partial of this warpgroup's 128 columns, the target
// logit and, with P.C, the 16-bit logits.  TMEM loads run one 32-column chunk
// ahead of the arithmetic.
template <typename T>
__device__ __forceinline__ void epi_stats(const Prob& P, uint32_t tbase, int row0, int lane, int64_t lab,
                                          int col0, int eg, uint32_t stg) {
  const int row = row0 + lane;
  const bool rv = row < P.M;
  const int nrows = min(32, P.M - row0);
  float m = -INFINITY, s = 0.f;  // s: sum of exp2(x log2e - m), m in log2 units
  T* C = reinterpret_cast<T*>(P.C);
  const int c0 = eg * kGroupCols;
  Tm32 buf[2];
  __syncwarp();
  tmem_ld_issue(tbase + (uint32_t)c0, buf[0]);
  tmem_ld_wait(buf[0]);
#pragma unroll
  for (int k = 0; k < kGroupCols / 32; ++k) {
    if (k + 1 < kGroupCols / 32) tmem_ld_issue(tbase + (uint32_t)(c0 + 32 * (k + 1)), buf[(k + 1) & 1]);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(buf[k & 1].r[j]);
    const int cbase = col0 + c0 + 32 * k;
    if (C != nullptr) {
      // logits kept in 16 bits for the gradient pass (the statistics use the fp32 values)
      if (col0 + c0 + 32 * (k | 1) + 32 <= P.N) {  // this 64-column block is inside the matrix
        stage_put<T>(stg, lane, k & 1, v);
        if (k & 1) {
          __syncwarp();
          stage_flush<T>(stg, lane, C, P.ldc, row0, nrows, cbase - 32);
          __syncwarp();
        }
      } else if (rv) {
        put_row16<T>(C + (int64_t)row * P.ldc, cbase, P.N, v);
      }
    }
    // the target logit: one range check per chunk (a row's target lies in one chunk of its
    // V / 32), then a predicated store per column, which keeps v in registers
    const int rel = (int)(lab - cbase);
    if ((unsigned)rel < 32u) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == rel) P.tlogit[row] = v[j];
    }
    stats_chunk(v, cbase, P.N, m, s);
    if (k + 1 < kGroupCols / 32) tmem_ld_wait(buf[(k + 1) & 1]);
  }
  if (rv) P.part[(int64_t)row * (kEpiGroups * P.ntiles) + kEpiGroups * (col0 / BN) + eg] = make_float2(m, s);
}

// C = acc * scale (+ add_f32) (+ C if accumulate), fp32 or 16-bit (staged rows).
template <typename T>
__device__ __forceinline__ void epi_store(const Prob& P, uint32_t tbase, int row0, int lane, int col0, int eg,
                                          uint32_t stg) {
  const int row = row0 + lane;
  const bool rv = row < P.M;
  const int nrows = min(32, P.M - row0);
  const int c0 = eg * kGroupCols;
  const float sc = P.scale != nullptr ? *P.scale : 1.f;
  Tm32 buf[2];
  __syncwarp();
  tmem_ld_issue(tbase + (uint32_t)c0, buf[0]);
  tmem_ld_wait(buf[0]);
#pragma unroll
  for (int k = 0; k < kGroupCols / 32; ++k) {
    if (k + 1 < kGroupCols / 32) tmem_ld_issue(tbase + (uint32_t)(c0 + 32 * (k + 1)), buf[(k + 1) & 1]);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(buf[k & 1].r[j]) * sc;
    const int cbase = col0 + c0 + 32 * k;
    const int64_t off = (int64_t)row * P.ldc + cbase;
    const bool full = cbase + 32 <= P.N;
    if (P.add_f32 != nullptr && rv) {
      const float* a = P.add_f32 + off;
      if (full) {
#pragma unroll
        for (int q = 0; q < 32; q += 4) {
          const float4 o = *reinterpret_cast<const float4*>(a + q);
          v[q] += o.x; v[q + 1] += o.y; v[q + 2] += o.z; v[q + 3] += o.w;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (cbase + j < P.N) v[j] += a[j];
      }
    }
    if (P.c_f32) {
      if (rv) {
        float* crow = reinterpret_cast<float*>(P.C) + off;
        if (full) {
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            float4* p4 = reinterpret_cast<float4*>(crow + q);
            float4 o = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
            if (P.accumulate) {
              const float4 old = *p4;
              o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
            }
            *p4 = o;
          }
        } else {
          for (int j = 0; j < 32; ++j)
            if (cbase + j < P.N) crow[j] = v[j] + (P.accumulate ? crow[j] : 0.f);
        }
      }
    } else {
      T* C = reinterpret_cast<T*>(P.C);
      if (col0 + c0 + 32 * (k | 1) + 32 <= P.N) {
        stage_put<T>(stg, lane, k & 1, v);
        if (k & 1) {
          __syncwarp();
          stage_flush<T>(stg, lane, C, P.ldc, row0, nrows, cbase - 32);
          __syncwarp();
        }
      } else if (rv) {
        put_row16<T>(C + (int64_t)row * P.ldc, cbase, P.N, v);
      }
    }
    if (k + 1 < kGroupCols / 32) tmem_ld_wait(buf[(k + 1) & 1]);
  }
}

// ---------------------------------------------------------------------------
// The GEMM kernel (clusters of 2 CTAs)
// ---------------------------------------------------------------------------
template <typename T, bool kList>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc_gemm2_kernel(const __grid_constant__ CUtensorMap tA0, const __grid_constant__ CUtensorMap tB0,
                const __grid_constant__ CUtensorMap tA1, const __grid_constant__ CUtensorMap tB1,
                const __grid_constant__ Group g) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);  // leader: TMA bytes of both CTAs
  uint64_t* empty = full + STAGES;                                             // each CTA: its stage is free
  uint64_t* tfull = empty + STAGES;   // [2] each CTA: accumulator ready
  uint64_t* tempty = tfull + 2;       // [2] leader: both CTAs' epilogues done with the accumulator
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);

  const Waiter wt{g.status, abort_flag};
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 2 * kEpiWarps); }
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = peer_addr(smem_u32(&full[0]), 0);  // the leader's barriers
      int it = 0;
      bool live = true;
      for (int k = 0, t = -1; live && (t = next_tile<kList>(g, pair, npairs, k, t)) >= 0; ++k) {
        int pi, mt, nt;
        decode_tile(g, t, pi, mt, nt);
        const Prob& P = pi ? g.p[1] : g.p[0];
        const CUtensorMap* mA = pi ? &tA1 : &tA0;
        const CUtensorMap* mB = pi ? &tB1 : &tB0;
        const int m0 = mt * (2 * BM) + (int)rank * BM;
        const int n0 = nt * BN + (int)rank * (BN / 2);
        const int ktiles = (P.K + BK - 1) / BK;  // the K tail is zero-filled by TMA in both operands
        for (int kb = 0; kb < ktiles; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!wait_bar<false>(&empty[s], ph ^ 1u, wt)) { live = false; break; }  // issue no more loads
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
          const uint32_t bar = full0 + (uint32_t)(s * 8);
          const uint32_t st = smem_u32(tiles + s * STAGE_BYTES);
          const int k0 = kb * BK;
          if (P.a_mn) {
            tma_load_2d(st, mA, m0, k0, bar);
            tma_load_2d(st + A_BYTES / 2, mA, m0 + 64, k0, bar);
          } else {
            tma_load_2d(st, mA, k0, m0, bar);
          }
          if (P.b_mn) {
            tma_load_2d(st + A_BYTES, mB, n0, k0, bar);
            tma_load_2d(st + A_BYTES + B_BYTES / 2, mB, n0 + 64, k0, bar);
          } else {
            tma_load_2d(st + A_BYTES, mB, k0, n0, bar);
          }
        }
      }
      if (!live || *wt.abort) drain_grace();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only)
    if (rank == 0 && lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t peer_empty0 = peer_addr(smem_u32(&empty[0]), 1);
      const uint32_t peer_tfull0 = peer_addr(smem_u32(&tfull[0]), 1);
      int it = 0, local = 0;
      int last_it = -1;  // the last stage consumption whose commit was issued
      bool live = true;
      for (int t = -1; live && (t = next_tile<kList>(g, pair, npairs, local, t)) >= 0; ++local) {
        int pi, mt, nt;
        decode_tile(g, t, pi, mt, nt);
        const Prob& P = pi ? g.p[1] : g.p[0];
        const uint32_t idesc = make_idesc(kBf16, 2 * BM, BN, P.a_mn, P.b_mn);
        // K = 16 steps inside a 64-deep stage: 32 B along a K-major row, or two
        // 8-row atoms (2048 B) of an MN-major tile
        const uint32_t astep = P.a_mn ? (2048u >> 4) : 2u, bstep = P.b_mn ? (2048u >> 4) : 2u;
        const int acc = local & 1;
        if (!wait_bar<true>(&tempty[acc], ((uint32_t)(local >> 1) & 1u) ^ 1u, wt)) { live = false; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)(acc * BN);
        const int ktiles = (P.K + BK - 1) / BK;
        for (int kb = 0; kb < ktiles; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_bar<false>(&full[s], (uint32_t)(it / STAGES) & 1u, wt)) { live = false; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(tiles + s * STAGE_BYTES);
          const uint64_t ad = smem_desc_sw128(st, P.a_mn, A_BYTES / 2);
          const uint64_t bd = smem_desc_sw128(st + A_BYTES, P.b_mn, B_BYTES / 2);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma2(dcol, ad + (uint64_t)(astep * k), bd + (uint64_t)(bstep * k), idesc, (kb | k) ? 1u : 0u);
          commit2(smem_u32(&empty[s]));
          commit2(peer_empty0 + (uint32_t)(s * 8));
          last_it = it;
        }
        if (!live) break;
        commit2(smem_u32(&tfull[acc]));
        commit2(peer_tfull0 + (uint32_t)(acc * 8));
      }
      // after an abort: commits arrive in order, so the last one completing means every MMA
      // issued so far has finished with TMEM and shared memory
      if ((!live || *wt.abort) && last_it >= 0)
        drain_bar(&empty[last_it % STAGES], (uint32_t)(last_it / STAGES) & 1u);
    }
  } else {
    // ---------------- epilogue (both CTAs): warps 2..9 own TMEM lanes 32*(warp%4) ...
    const int quad = warp & 3;
    const int eg = (warp - 2) >> 2;  // epilogue warpgroup: column half
    const uint32_t stg = smem_u32(smem + STAGES * STAGE_BYTES + 256) + (uint32_t)((warp - 2) * kStageWarpBytes);
    const uint32_t tempty0 = peer_addr(smem_u32(&tempty[0]), 0);
    int local = 0;
    for (int t = -1; (t = next_tile<kList>(g, pair, npairs, local, t)) >= 0; ++local) {
      int pi, mt, nt;
      decode_tile(g, t, pi, mt, nt);
      const Prob& P = pi ? g.p[1] : g.p[0];
      const int acc = local & 1;
      const int row0 = mt * (2 * BM) + (int)rank * BM + quad * 32;  // this warp's 32 rows
      // the row's label is loaded before the wait, so its latency hides behind the MMAs
      const int64_t lab = (P.epi == EPI_STATS && row0 + lane < P.M) ? P.labels[row0 + lane] : -1;
      if (!wait_bar<false>(&tfull[acc], (uint32_t)(local >> 1) & 1u, wt)) break;  // no accumulator to read
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      if (P.epi == EPI_STATS) epi_stats<T>(P, tbase, row0, lane, lab, nt * BN, eg, stg);
      else if (P.epi == EPI_STORE) epi_store<T>(P, tbase, row0, lane, nt * BN, eg, stg);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));
    }
  }
  tc_fence_before();
  cluster_sync();  // every MMA has completed and been read; no more remote arrivals
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
}

// ---------------------------------------------------------------------------
// Side kernels
// ---------------------------------------------------------------------------
// 1 / max(1, number of rows whose label is not ignore_index), on the device.
__global__ void __launch_bounds__(1024)
lce_inv_valid(float* __restrict__ inv_valid, const int64_t* __restrict__ labels, int64_t M, int64_t ignore_index) {
  __shared__ float r[32];
  float n = 0.f;
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) n += (labels[i] != ignore_index) ? 1.f : 0.f;
  n = warp_sum(n);
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += r[i];
    inv_valid[0] = 1.f / fmaxf(s, 1.f);
  }
}

// Merge the per-tile partials: lse (natural log) and the per-row loss.
__global__ void __launch_bounds__(256)
lce_rows_reduce(float* __restrict__ lse, float* __restrict__ losses, const float2* __restrict__ part,
                const float* __restrict__ tlogit, const int64_t* __restrict__ labels, int M, int nparts,
                int64_t ignore_index) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int t = lane; t < nparts; t += 32) {
    const float2 p = part[(int64_t)warp * nparts + t];
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

// loss[0] = inv_valid * sum of the per-row losses (ignored rows hold 0), fixed order.
__global__ void __launch_bounds__(1024)
lce_loss(float* __restrict__ loss, const float* __restrict__ losses, const float* __restrict__ inv_valid, int64_t M) {
  __shared__ float r[32];
  float a = 0.f;
#pragma unroll 4
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) a += losses[i];
  a = warp_sum(a);
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += r[i];
    loss[0] = s * inv_valid[0];
  }
}

// In place over 16-bit logits L[M][V]: L = (softmax(L) - onehot(label)) * scale
// (scale: a device scalar, or 1 when it is null), zero rows for ignored labels.  V % 8 == 0.  A CTA walks whole rows (the row's
// lse and label stay in registers); each thread loads kGradBatch 16-byte vectors
// before using any of them.
constexpr int kGradBatch = 4;

template <typename T>
__global__ void __launch_bounds__(256)
lce_grad_inplace(T* __restrict__ L, const float* __restrict__ lse, const int64_t* __restrict__ labels,
                 const float* __restrict__ scale, int64_t M, int64_t V, int64_t ignore_index) {
  const float sc0 = scale != nullptr ? *scale : 1.f;
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tensor map over a row-major [rows][cols] 16-bit matrix.  K-major operands
// (cols = K) load 64 x 128 boxes; MN-major operands (cols = M or N) load 64 x 64
// boxes, two per operand and stage.
int make_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, bool mn, bool bf16) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64u, mn ? 64u : 128u};
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
  const CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AK_REQUIRE(r == CUDA_SUCCESS, AK_ERR_ARG, "linear_ce: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AK_OK;
}

constexpr size_t kSmem = (size_t)STAGES * STAGE_BYTES + 256 + (size_t)kEpiWarps * kStageWarpBytes + 1024;

// One GEMM operand: a row-major [rows][cols] matrix read K-major (cols = K) or
// MN-major (cols = M or N).
struct Operand {
  const void* base;
  int64_t rows, cols;
  int mn;
};

void finish_prob(Prob& P) {
  P.mtiles = (P.M + 2 * BM - 1) / (2 * BM);
  P.ntiles = (P.N + BN - 1) / BN;
  P.tiles = P.mtiles * P.ntiles;
}

std::mutex g_pairs_mu;
int g_pairs_cache[64] = {0};

// CTA pairs that fit on the device at once (one CTA per SM).
template <typename T>
int resident_pairs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return std::max(1, sm_count() / 2);
  std::lock_guard<std::mutex> lock(g_pairs_mu);
  if (g_pairs_cache[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)sm_count());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_gemm2_kernel<T, false>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    g_pairs_cache[dev] = std::max(1, n);
  }
  return g_pairs_cache[dev];
}

template <typename T>
int launch_group(const Operand* A, const Operand* B, Group& g, cudaStream_t st) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap maps[4];
  int rc;
  for (int i = 0; i < g.nprob; ++i) {
    if ((rc = make_tmap(&maps[2 * i], A[i].base, A[i].rows, A[i].cols, A[i].mn, bf16))) return rc;
    if ((rc = make_tmap(&maps[2 * i + 1], B[i].base, B[i].rows, B[i].cols, B[i].mn, bf16))) return rc;
    g.p[i].a_mn = A[i].mn;
    g.p[i].b_mn = B[i].mn;
    finish_prob(g.p[i]);
  }
  if (g.nprob == 1) { maps[2] = maps[0]; maps[3] = maps[1]; }
  g.total = g.p[0].tiles + (g.nprob > 1 ? g.p[1].tiles : 0);
  g.lp = -1;
  if (g.nprob == 2 && g.p[0].tiles > 0 && g.p[1].tiles > 0) {
    const int k0 = (g.p[0].K + BK - 1) / BK, k1 = (g.p[1].K + BK - 1) / BK;
    if (k0 != k1) {
      g.lp = k0 > k1 ? 0 : 1;
      g.nL = g.p[g.lp].tiles;
      g.nS = g.p[1 - g.lp].tiles;
      g.cL = std::max(k0, k1) + kTileOverheadK;
      g.cS = std::min(k0, k1) + kTileOverheadK;
    }
  }
  if (g.total == 0) return AK_OK;
  auto kern = g.lp >= 0 ? tc_gemm2_kernel<T, true> : tc_gemm2_kernel<T, false>;
  AK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem),
              "linear_ce: smem attribute");
  const int pairs = std::max(1, std::min(g.total, resident_pairs<T>()));
  kern<<<2 * pairs, kThreads, kSmem, st>>>(maps[0], maps[1], maps[2], maps[3], g);
  AK_CHECK_LAUNCH("linear_ce: tcgen05 gemm");
  return AK_OK;
}

// Workspace: per-row statistics of one chunk, the chunk's 16-bit logits /
// gradient G_c, and (several chunks only) the fp32 dW accumulator.
struct Ws {
  float2* part;
  float* tlogit;
  float* losses;
  float* inv_valid;
  void* G;
  float* dWacc;
  size_t bytes;
};

int64_t chunk_rows(int64_t N) { return std::min<int64_t>(N, kChunkRows); }

Ws carve(void* base, int64_t N, int64_t D, int64_t V, bool need_dw) {
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
  w.part = reinterpret_cast<float2*>(take((size_t)Nc * ntiles * kEpiGroups * sizeof(float2)));
  w.tlogit = reinterpret_cast<float*>(take((size_t)N * 4));
  w.losses = reinterpret_cast<float*>(take((size_t)N * 4));
  w.inv_valid = reinterpret_cast<float*>(take(4));
  w.G = take((size_t)Nc * V * 2);
  w.dWacc = (need_dw && N > Nc) ? reinterpret_cast<float*>(take((size_t)V * D * 4)) : nullptr;
  w.bytes = off + 256;
  return w;
}

// Logits GEMM with statistics over rows [r0, r0 + nr) (16-bit logits into Gc when
// it is given), then lse and the per-row loss.
template <typename T>
int stats_pass(const Ws& w, float* lse, void* Gc, const void* H, const void* W, const int64_t* labels, int64_t r0,
               int64_t nr, int64_t D, int64_t V, int64_t ignore_index, int* status, cudaStream_t st) {
  Operand A[1] = {{static_cast<const T*>(H) + r0 * D, nr, D, 0}};
  Operand B[1] = {{W, V, D, 0}};
  Group g{};
  g.nprob = 1;
  g.status = status;
  Prob& P = g.p[0];
  P.M = (int)nr; P.N = (int)V; P.K = (int)D;
  P.epi = EPI_STATS;
  P.part = w.part; P.tlogit = w.tlogit + r0; P.labels = labels + r0; P.ignore_index = ignore_index;
  P.C = Gc; P.ldc = V;
  int rc = launch_group<T>(A, B, g, st);
  if (rc) return rc;
  const int nparts = kEpiGroups * (int)((V + BN - 1) / BN);
  lce_rows_reduce<<<(unsigned)((nr * 32 + 255) / 256), 256, 0, st>>>(lse + r0, w.losses + r0, w.part,
                                                                     w.tlogit + r0, labels + r0, (int)nr, nparts,
                                                                     ignore_index);
  AK_CHECK_LAUNCH("linear_ce: row reduce");
  return AK_OK;
}

template <typename T>
int grad_inplace(void* Gc, const float* lse, const int64_t* labels, const float* scale, int64_t nr, int64_t V,
                 int64_t ignore_index, cudaStream_t st) {
  const unsigned grid = (unsigned)std::min<int64_t>(nr, (int64_t)sm_count() * 8);
  lce_grad_inplace<T><<<grid, 256, 0, st>>>((T*)Gc, lse, labels, scale, nr, V, ignore_index);
  AK_CHECK_LAUNCH("linear_ce: gradient");
  return AK_OK;
}

template <typename T>
int run(float* loss, float* lse, void* dH, void* dW, const Ws& w, const void* H, const void* W,
        const int64_t* labels, const float* inv_valid_in, int64_t N, int64_t D, int64_t V, int64_t ignore_index,
        int* status, cudaStream_t st) {
  const float* inv = inv_valid_in;
  if (inv == nullptr) {
    lce_inv_valid<<<1, 1024, 0, st>>>(w.inv_valid, labels, N, ignore_index);
    AK_CHECK_LAUNCH("linear_ce: valid rows");
    inv = w.inv_valid;
  }
  const int64_t Nc = chunk_rows(N);
  int rc;
  for (int64_t r0 = 0; r0 < N; r0 += Nc) {
    const int64_t nr = std::min(Nc, N - r0);
    const bool first = r0 == 0, last = r0 + nr >= N;
    const bool grads = dH != nullptr || dW != nullptr;
    if ((rc = stats_pass<T>(w, lse, grads ? w.G : nullptr, H, W, labels, r0, nr, D, V, ignore_index, status, st)))
      return rc;
    if (!grads) continue;
    // G_c = softmax - onehot, unscaled: 1 / n_valid would push 16-bit values towards
    // underflow; the GEMM epilogues apply it to the fp32 accumulators instead
    if ((rc = grad_inplace<T>(w.G, lse + r0, labels + r0, nullptr, nr, V, ignore_index, st))) return rc;
    // one launch: dW (+)= G_c^T H_c (problem 0, many short-K tiles) and dH_c = G_c W
    // (problem 1, few long-K tiles, spread over the pairs after the dW tiles)
    Operand A[2], B[2];
    Group g{};
    g.status = status;
    int np = 0;
    if (dW) {
      A[np] = {w.G, nr, V, 1};                                // G_c^T: M = V contiguous
      B[np] = {static_cast<const T*>(H) + r0 * D, nr, D, 1};  // H_c^T: N = D contiguous
      Prob& P = g.p[np++];
      P.M = (int)V; P.N = (int)D; P.K = (int)nr;
      P.epi = EPI_STORE;
      P.ldc = D;
      P.scale = inv;
      if (first && last) {  // one chunk: the 16-bit dW directly
        P.C = dW;
      } else if (!last) {   // fp32 accumulator
        P.C = w.dWacc; P.c_f32 = 1; P.accumulate = first ? 0 : 1;
      } else {              // last chunk: accumulator + this chunk -> 16-bit dW
        P.C = dW; P.add_f32 = w.dWacc;
      }
    }
    if (dH) {
      A[np] = {w.G, nr, V, 0};  // G_c: K = V contiguous
      B[np] = {W, V, D, 1};     // W^T: N = D contiguous
      Prob& P = g.p[np++];
      P.M = (int)nr; P.N = (int)D; P.K = (int)V;
      P.epi = EPI_STORE;
      P.C = static_cast<T*>(dH) + r0 * D; P.ldc = D;
      P.scale = inv;
    }
    g.nprob = np;
    if ((rc = launch_group<T>(A, B, g, st))) return rc;
  }
  lce_loss<<<1, 1024, 0, st>>>(loss, w.losses, inv, N);
  AK_CHECK_LAUNCH("linear_ce: loss");
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
  *bytes = carve(nullptr, N, D, V, true).bytes;
  return AK_OK;
}

extern "C" int ak_linear_ce_fwdbwd(float* loss, float* lse, void* dH, void* dW, void* workspace, size_t ws_bytes,
                                   const void* H, const void* W, const int64_t* labels, const float* inv_valid,
                                   int64_t N, int64_t D, int64_t V, int64_t ignore_index, int dt, int* status,
                                   void* stream) {
  clear_error();
  int rc = check_shape(N, D, V, dt);
  if (rc) return rc;
  AK_REQUIRE(loss && lse && H && W && labels, AK_ERR_ARG, "ak_linear_ce_fwdbwd: null pointer");
  AK_REQUIRE(aligned16(H) && aligned16(W) && (!dH || aligned16(dH)) && (!dW || aligned16(dW)), AK_ERR_ARG,
             "ak_linear_ce_fwdbwd: H, W, dH, dW must be 16-byte aligned");
  const Ws need = carve(nullptr, N, D, V, dW != nullptr);
  AK_REQUIRE(workspace && ws_bytes >= need.bytes, AK_ERR_WORKSPACE, "ak_linear_ce_fwdbwd: workspace %zu < %zu",
             ws_bytes, need.bytes);
  void* base = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const Ws w = carve(base, N, D, V, dW != nullptr);
  cudaStream_t st = (cudaStream_t)stream;
  if (dt == AK_BF16)
    return run<__nv_bfloat16>(loss, lse, dH, dW, w, H, W, labels, inv_valid, N, D, V, ignore_index, status, st);
  return run<__half>(loss, lse, dH, dW, w, H, W, labels, inv_valid, N, D, V, ignore_index, status, st);
}

extern "C" int ak_tc_gemm(void* C, int dt_c, const void* A, const void* B, int64_t M, int64_t N, int64_t K,
                          int a_mn, int b_mn, int dt, int* status, void* stream) {
  clear_error();
  AK_REQUIRE(dt == AK_BF16 || dt == AK_F16, AK_ERR_DTYPE, "ak_tc_gemm: operands must be bf16 or fp16");
  AK_REQUIRE(dt_c == dt || dt_c == AK_F32, AK_ERR_DTYPE, "ak_tc_gemm: C is fp32 or the operand type");
  AK_REQUIRE(M >= 0 && N >= 0 && K >= 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), AK_ERR_SHAPE,
             "ak_tc_gemm: bad shape");
  if (M == 0 || N == 0) return AK_OK;
  AK_REQUIRE(K > 0, AK_ERR_SHAPE, "ak_tc_gemm: K must be positive");
  AK_REQUIRE(A && B, AK_ERR_ARG, "ak_tc_gemm: null pointer");
  AK_REQUIRE(aligned16(A) && aligned16(B) && aligned16(C), AK_ERR_ARG, "ak_tc_gemm: pointers must be 16-byte aligned");
  AK_REQUIRE((a_mn ? M : K) % 8 == 0 && (b_mn ? N : K) % 8 == 0 && N % 8 == 0, AK_ERR_SHAPE,
             "ak_tc_gemm: contiguous dimensions and N must be multiples of 8");
  Operand As[1] = {{A, a_mn ? K : M, a_mn ? M : K, a_mn ? 1 : 0}};
  Operand Bs[1] = {{B, b_mn ? K : N, b_mn ? N : K, b_mn ? 1 : 0}};
  Group g{};
  g.nprob = 1;
  g.status = status;
  Prob& P = g.p[0];
  P.M = (int)M; P.N = (int)N; P.K = (int)K;
  P.epi = C != nullptr ? EPI_STORE : EPI_NONE;
  P.C = C; P.ldc = N; P.c_f32 = dt_c == AK_F32 ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (dt == AK_BF16) return launch_group<__nv_bfloat16>(As, Bs, g, st);
  return launch_group<__half>(As, Bs, g, st);
}

extern "C" int ak_linear_ce_logits_grad_workspace_size(int64_t N, int64_t V, size_t* bytes) {
  clear_error();
  AK_REQUIRE(bytes != nullptr && N > 0 && V > 0, AK_ERR_ARG, "linear_ce: bad args");
  const int64_t ntiles = (V + BN - 1) / BN;
  *bytes = (size_t)N * ntiles * kEpiGroups * sizeof(float2) + (size_t)N * 8 + 1024;
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
  Ws w{};
  w.part = reinterpret_cast<float2*>(base);
  w.tlogit = reinterpret_cast<float*>(w.part + (size_t)N * ntiles * kEpiGroups);
  w.losses = w.tlogit + N;
  w.inv_valid = w.losses + N;  // one float after the per-row losses
  cudaStream_t st = (cudaStream_t)stream;
  lce_inv_valid<<<1, 1024, 0, st>>>(w.inv_valid, labels, N, ignore_index);
  AK_CHECK_LAUNCH("ak_linear_ce_logits_grad");
  if (dt == AK_BF16) {
    if ((rc = stats_pass<__nv_bfloat16>(w, lse, G, H, W, labels, 0, N, D, V, ignore_index, status, st))) return rc;
    if ((rc = grad_inplace<__nv_bfloat16>(G, lse, labels, w.inv_valid, N, V, ignore_index, st))) return rc;
  } else {
    if ((rc = stats_pass<__half>(w, lse, G, H, W, labels, 0, N, D, V, ignore_index, status, st))) return rc;
    if ((rc = grad_inplace<__half>(G, lse, labels, w.inv_valid, N, V, ignore_index, st))) return rc;
  }
  lce_loss<<<1, 1024, 0, st>>>(loss, w.losses, w.inv_valid, N);
  AK_CHECK_LAUNCH("ak_linear_ce_logits_grad");
  return AK_OK;
}
