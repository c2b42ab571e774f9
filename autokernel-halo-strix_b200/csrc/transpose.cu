// Batched last-two-dims transpose, sm_100a: out[b][c][r] = in[b][r][c].
//
// The hybrid's Mamba block moves activations between the (B, T, D) layout of the
// projections and the (B, D, T) layout of the conv / scan kernels
// (mamba_simple-style `.transpose(1, 2)` + `.contiguous()`).  PyTorch's strided
// copy does these at under 1 TB/s; this kernel stages 64 x 64 tiles through
// padded shared memory with 16-byte global loads and stores on both sides.
//
// Both sides take a batch stride and a leading (row) stride in elements, so the
// input may be a column slice of a wider tensor (one half of the in_proj output)
// and the output may be written into a slice of a wider tensor (one half of a
// packed gradient).  Unit stride along the last dimension on both sides.
#include "ak_common.cuh"

namespace ak {
namespace {

constexpr int kTile = 64;
constexpr int kThreadsT = 256;

// Vector path: R % VEC == 0 and C % VEC == 0 and every row start 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kThreadsT)
transpose_vec_kernel(T* __restrict__ out, const T* __restrict__ in, int R, int C, int64_t isb, int64_t ild,
                     int64_t osb, int64_t old) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int kPad = 4 / sizeof(T) > 0 ? 4 / sizeof(T) : 1;  // one 4-byte word of padding per row
  __shared__ T tile[kTile][kTile + kPad];
  const int64_t b = blockIdx.z;
  const int r0 = blockIdx.y * kTile, c0 = blockIdx.x * kTile;
  const T* ib = in + b * isb;
  T* ob = out + b * osb;
  constexpr int kVecPerRow = kTile / VEC;
  constexpr int kVecs = kTile * kVecPerRow;
  // load: row r of the tile = input row r0 + r, columns c0 .. c0+63
#pragma unroll
  for (int v = threadIdx.x; v < kVecs; v += kThreadsT) {
    const int r = v / kVecPerRow, cv = (v - r * kVecPerRow) * VEC;
    if (r0 + r < R && c0 + cv < C) {
      const int4 raw = *reinterpret_cast<const int4*>(ib + (int64_t)(r0 + r) * ild + c0 + cv);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < VEC; ++k) tile[r][cv + k] = e[k];
    }
  }
  __syncthreads();
  // store: output row c0 + c holds input column c: gather VEC tile rows per vector
#pragma unroll
  for (int v = threadIdx.x; v < kVecs; v += kThreadsT) {
    const int c = v / kVecPerRow, rv = (v - c * kVecPerRow) * VEC;
    if (c0 + c < C && r0 + rv < R) {
      int4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int k = 0; k < VEC; ++k) e[k] = tile[rv + k][c];
      *reinterpret_cast<int4*>(ob + (int64_t)(c0 + c) * old + r0 + rv) = raw;
    }
  }
}

// Scalar path for ragged shapes or unaligned rows.
template <typename T>
__global__ void __launch_bounds__(kThreadsT)
transpose_scalar_kernel(T* __restrict__ out, const T* __restrict__ in, int R, int C, int64_t isb, int64_t ild,
                        int64_t osb, int64_t old) {
  __shared__ T tile[32][33];
  const int64_t b = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int i = ty; i < 32; i += 8)
    if (r0 + i < R && c0 + tx < C) tile[i][tx] = in[b * isb + (int64_t)(r0 + i) * ild + c0 + tx];
  __syncthreads();
  for (int i = ty; i < 32; i += 8)
    if (c0 + i < C && r0 + tx < R) out[b * osb + (int64_t)(c0 + i) * old + r0 + tx] = tile[tx][i];
}

}  // namespace
}  // namespace ak

using namespace ak;

extern "C" int ak_transpose(void* out, const void* in, int64_t batch, int64_t R, int64_t C, int64_t in_bstride,
                            int64_t in_ld, int64_t out_bstride, int64_t out_ld, int dt, void* stream) {
  clear_error();
  AK_REQUIRE(batch >= 0 && batch < 65536 && R >= 0 && C >= 0 && R < (1LL << 31) && C < (1LL << 31) && in_ld >= C &&
                 out_ld >= R,
             AK_ERR_SHAPE, "ak_transpose: bad shape batch=%lld R=%lld C=%lld ld=(%lld, %lld)", (long long)batch,
             (long long)R, (long long)C, (long long)in_ld, (long long)out_ld);
  if (batch == 0 || R == 0 || C == 0) return AK_OK;
  AK_REQUIRE(out && in, AK_ERR_ARG, "ak_transpose: null pointer");
  const int es = elem_size(dt);
  const int vec = 16 / es;
  const bool vec_ok = R % vec == 0 && C % vec == 0 && aligned16(in) && aligned16(out) && (in_ld * es) % 16 == 0 &&
                      (out_ld * es) % 16 == 0 && (in_bstride * es) % 16 == 0 && (out_bstride * es) % 16 == 0;
  cudaStream_t st = (cudaStream_t)stream;
  AK_DISPATCH_DTYPE(dt, T, {
    if (vec_ok) {
      dim3 grid((unsigned)((C + kTile - 1) / kTile), (unsigned)((R + kTile - 1) / kTile), (unsigned)batch);
      transpose_vec_kernel<T><<<grid, kThreadsT, 0, st>>>((T*)out, (const T*)in, (int)R, (int)C, in_bstride, in_ld,
                                                          out_bstride, out_ld);
    } else {
      dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32), (unsigned)batch);
      transpose_scalar_kernel<T><<<grid, kThreadsT, 0, st>>>((T*)out, (const T*)in, (int)R, (int)C, in_bstride,
                                                             in_ld, out_bstride, out_ld);
    }
  });
  AK_CHECK_LAUNCH("ak_transpose");
  return AK_OK;
}
