/*
 * ak_b200.h — C ABI of libak_b200.so, the sm_100a (B200) kernels behind the
 * autokernel drop-in Python API.
 *
 * Conventions shared by every entry point:
 *   - `extern "C"`, no C++ exceptions cross the boundary.
 *   - Return AK_OK (0) on success, a nonzero ak_status otherwise; the reason
 *     is available from ak_last_error() on the calling thread.
 *   - All tensor arguments are raw device pointers to caller-owned, densely
 *     packed row-major buffers (the Python layer allocates outputs and
 *     workspaces with PyTorch).  Nothing here allocates device memory.
 *   - `stream` is a cudaStream_t passed as void*; every call is asynchronous
 *     on that stream (NULL = legacy default stream).
 *   - Element types are given by ak_dtype codes.
 *   - Functions keep no mutable global state beyond a per-device attribute
 *     cache, so they are reentrant and thread-safe.
 *   - Kernels that wait on asynchronous copies or on each other (the mamba
 *     scan and the tensor-core linear + CE) bound every wait.  When a wait runs
 *     out they write AK_ERR_TIMEOUT to the caller's `status` word (nullable; a
 *     device int, or a pinned host int whose device address comes from
 *     ak_status_device_pointer), stop issuing work, wait (again bounded) for
 *     the copies and tensor-core operations they already issued, free their
 *     tensor memory and finish without hanging; their outputs are then invalid.  The word is only ever written on failure, so the caller
 *     zeroes it once and reads it after the stream has passed the call.
 *
 * Each declaration names the reference interface it replaces, as a path inside
 * the joelhenwang/autokernel-halo-strix project.
 */
#ifndef AK_B200_H
#define AK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AK_API __attribute__((visibility("default")))
#else
#define AK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum { AK_F32 = 0, AK_BF16 = 1, AK_F16 = 2 } ak_dtype;

typedef enum {
  AK_OK = 0,
  AK_ERR_ARG = 1,       /* invalid pointer / size / alignment */
  AK_ERR_DTYPE = 2,     /* unsupported dtype combination */
  AK_ERR_SHAPE = 3,     /* unsupported shape */
  AK_ERR_LAUNCH = 4,    /* CUDA launch or runtime error */
  AK_ERR_TIMEOUT = 5,   /* a bounded device-side wait gave up */
  AK_ERR_WORKSPACE = 6  /* workspace smaller than the *_workspace_size query */
} ak_status;

/* Library version, (major << 16) | (minor << 8) | patch. */
AK_API int ak_version(void);
/* Message for the last failing call on this thread ("" if none). */
AK_API const char* ak_last_error(void);

/* Device address of a pinned (cudaHostAlloc) host word, for use as the
 * `status` argument: kernels then report straight into host memory, so the
 * host can read a timeout without a CUDA call or a stream sync.  No
 * counterpart in the reference, whose kernels have no bounded waits; it turns
 * the device-side failure into the RuntimeError its TORCH_CHECKs raise
 * (kernels/hip/rmsnorm.py:119-123). */
AK_API int ak_status_device_pointer(void* host_word, void** dev_ptr);

/* Test hook for the status path: launches one thread that waits on an
 * mbarrier nothing completes, with a limit of max_spins polls (1..2^20), so
 * the wait runs out and *status receives AK_ERR_TIMEOUT.  Asynchronous. */
AK_API int ak_test_bounded_wait(int* status, int max_spins, void* stream);

/* ------------------------------------------------------------------------ *
 * RMSNorm
 * ------------------------------------------------------------------------ */

/* y[M,N] = x * rsqrt(mean(x^2, -1) + eps) * w.   x, y: dt_x; w: dt_w.
 * rstd (nullable, fp32 [M]) receives rsqrt(mean(x^2)+eps).
 * Replaces rmsnorm_hip / kernel_fn (kernels/hip/rmsnorm.py:119-177) and the
 * torch.ops.autokernel.rmsnorm forward (kernels/hip/_torch_ops.py:56-59). */
AK_API int ak_rmsnorm_fwd(void* y, float* rstd, const void* x, const void* w,
                   int64_t M, int64_t N, float eps, int dt_x, int dt_w,
                   void* stream);

/* Workspace bytes needed by ak_rmsnorm_bwd for an [M, N] problem. */
AK_API int ak_rmsnorm_bwd_workspace_size(int64_t M, int64_t N, size_t* bytes);

/* dx[M,N] (dt_x) and dw[N] (dt_dw) of the RMSNorm above, given dy (dt_x).
 * dw is a deterministic column reduction (no atomics).
 * Replaces rmsnorm_backward_hip / kernel_fn (kernels/hip/rmsnorm_backward.py:191-281)
 * and _rmsnorm_backward (kernels/hip/_torch_ops.py:73-97). */
AK_API int ak_rmsnorm_bwd(void* dx, void* dw, int dt_dw, void* workspace, size_t ws_bytes,
                   const void* dy, const void* x, const void* w,
                   int64_t M, int64_t N, float eps, int dt_x, int dt_w,
                   void* stream);

/* ak_rmsnorm_bwd without a workspace argument, for callers that cannot
 * allocate device memory (e.g. hosts whose own allocator owns all of it, or
 * plugin ABIs that pass only inputs and outputs).  No counterpart in the
 * reference.  The dw partial rows live in a 4 MiB static device array
 * (2^20 floats) that every GPU loading the library keeps until exit; N up to
 * 2^20 is accepted, larger N returns AK_ERR_SHAPE.  The first call on a device
 * looks up that array's device address (cudaGetSymbolAddress), so make it
 * before any stream capture; the address is cached per device and context and
 * looked up again after a device reset gives the device a new context.  All calls share the array: calls that overlap
 * on the GPU (different streams, or several host threads) race on it and must
 * be serialised by the caller.  Allocates nothing. */
AK_API int ak_rmsnorm_bwd_noalloc(void* dx, void* dw, int dt_dw, const void* dy,
                   const void* x, const void* w, int64_t M, int64_t N, float eps,
                   int dt_x, int dt_w, void* stream);

/* ------------------------------------------------------------------------ *
 * Row softmax over the last dimension
 * ------------------------------------------------------------------------ */

/* y[rows,cols] = softmax(x) along cols.  fp32 accumulation.
 * Replaces softmax_hip / kernel_fn (kernels/hip/softmax.py:273-360). */
AK_API int ak_softmax_fwd(void* y, const void* x, int64_t rows, int64_t cols, int dt,
                   void* stream);

/* dx = y * (dy - sum(dy * y)).  The reference has no backward kernel; this is
 * the autograd of reference.softmax_ref (reference.py:15-17). */
AK_API int ak_softmax_bwd(void* dx, const void* y, const void* dy, int64_t rows,
                   int64_t cols, int dt, void* stream);

/* ------------------------------------------------------------------------ *
 * Cross-entropy over logit rows
 * ------------------------------------------------------------------------ */

/* Per-row online-softmax cross entropy on logits[B, V] (dt), targets int64[B].
 * Outputs (fp32 [B]): losses, lse; row_max/row_sum nullable.
 * If grad != NULL, writes grad[B, V] (dt) =
 *   (softmax - (1-a)*onehot - a/V) * softcap' * scale,
 * where scale = scale_grad * (scale_dev ? *scale_dev : 1).
 * Ignored rows (target == ignore_index) get loss 0 and a zero grad row.
 * Replaces cross_entropy_fwd_hip (kernels/ce_fused.py:122-382). */
AK_API int ak_ce_rows_fwd(float* losses, float* lse, float* row_max, float* row_sum,
                   void* grad, const void* logits, const int64_t* targets,
                   int64_t B, int64_t V, float softcap, int64_t ignore_index,
                   float label_smoothing, float scale_grad,
                   const float* scale_dev, int dt, void* stream);

/* grad[B,V] from saved row_max/row_sum (tiny mode), optionally adding the
 * z-loss term z_coef * lse * softmax (z_coef = 0 disables it).
 * Replaces cross_entropy_bwd_tiny_hip (kernels/ce_fused.py:405-522) and the
 * z-loss branch of _CrossEntropyHIP.backward (kernels/ce_fused.py:672-689). */
AK_API int ak_ce_rows_bwd(void* grad, const void* logits, const int64_t* targets,
                   const float* row_max, const float* row_sum, int64_t B,
                   int64_t V, float softcap, int64_t ignore_index,
                   float label_smoothing, float scale, const float* scale_dev,
                   float z_coef, int dt, void* stream);

/* loss_out[0] = sum(losses * valid) / max(1, n_valid) (+ z_w * sum(lse^2*valid)/n)
 * computed on device; n_valid_out (nullable) receives max(1, n_valid).
 * Replaces the host-side reductions of _CrossEntropyHIP.forward
 * (kernels/ce_fused.py:593-629). */
AK_API int ak_ce_rows_reduce(float* loss_out, float* n_valid_out, const float* losses,
                      const float* lse, const int64_t* targets, int64_t B,
                      int64_t ignore_index, float z_loss_weight, void* stream);

/* inv_out[0] = 1 / max(1, count(targets != ignore_index)).  Device-side
 * replacement of the `.item()` sync in _ChunkedLinearCrossEntropy.forward
 * (kernels/hip/chunked_linear_cross_entropy.py:71-74). */
AK_API int ak_ce_inv_valid(float* inv_out, const int64_t* targets, int64_t B,
                    int64_t ignore_index, void* stream);

/* x[i] *= scale[0] for i < n (x of dtype dt), with the scalar read on the device:
 * nothing is written when it is 1.  Device-side replacement of the
 * `grad_output.item() == 1.0` fast-path check before the gradient scaling in
 * the backward of the chunked linear + CE
 * (kernels/hip/chunked_linear_cross_entropy.py:152-169), so the backward needs
 * no host sync and can be captured in a CUDA graph. */
AK_API int ak_scale_by_device_scalar(void* x, int64_t n, const float* scale, int dt,
                                     void* stream);

/* ------------------------------------------------------------------------ *
 * Fused linear + cross-entropy on the tensor cores (tcgen05 / TMEM / TMA)
 * ------------------------------------------------------------------------ */

/* Workspace bytes for ak_linear_ce_fwdbwd on H[N, D], W[V, D]. */
AK_API int ak_linear_ce_workspace_size(int64_t N, int64_t D, int64_t V, size_t* bytes);

/* loss[0] = mean over rows with labels != ignore_index of CE(H W^T) (fp32),
 * lse[N] fp32 per-row logsumexp, and the gradients of that mean: dH[N, D] (dt,
 * nullable) and dW[V, D] (dt, nullable).  H, W: bf16 or fp16 (dt), row-major;
 * labels int64[N].  N, D, V multiples of 8.
 * inv_valid (nullable, device fp32 scalar): 1 / n_valid to use instead of this
 * call's own count of valid rows.  A caller that shards the rows over ranks
 * passes 1 / (valid rows of all ranks); the loss and dW of each rank are then
 * partial sums whose all-reduce (SUM) is the loss and dW of the whole batch,
 * and dH is final.
 * All three contractions run on the library's tcgen05 GEMM (CTA pairs, TMA
 * operands, TMEM accumulators): per chunk of at most 16384 rows the logits GEMM
 * reduces its tiles to softmax statistics and keeps 16-bit logits only for that
 * chunk, which becomes G = (softmax - onehot) / n_valid in place and feeds
 * dW += G^T H and dH = G W in one grouped launch.  Full [N, V] logits are never
 * stored.  Replaces _ChunkedLinearCrossEntropy.forward / .backward
 * (kernels/hip/chunked_linear_cross_entropy.py:55-175) for softcap = 0,
 * label_smoothing = 0, z_loss_weight = 0. */
AK_API int ak_linear_ce_fwdbwd(float* loss, float* lse, void* dH, void* dW, void* workspace,
                   size_t ws_bytes, const void* H, const void* W, const int64_t* labels,
                   const float* inv_valid, int64_t N, int64_t D, int64_t V,
                   int64_t ignore_index, int dt, int* status, void* stream);

/* C[M, N] = A B^T on the tensor cores (the GEMM behind the linear + CE entries),
 * fp32 accumulation.  A is M x K and B is N x K, bf16 or fp16 (dt), each given
 * row-major either K-contiguous (a_mn / b_mn = 0: A[M][K], B[N][K]) or
 * M / N-contiguous (1: A stored [K][M], B stored [K][N]), so transposed
 * operands need no copy.  C is row-major [M][N], fp32 or dt (dt_c).
 * Contiguous dimensions and N must be multiples of 8.  C = NULL runs the
 * contraction and discards the result (measures the main loop alone).  No counterpart in the
 * reference, whose chunked linear + CE calls torch GEMMs
 * (kernels/hip/chunked_linear_cross_entropy.py:95-132). */
AK_API int ak_tc_gemm(void* C, int dt_c, const void* A, const void* B, int64_t M,
                      int64_t N, int64_t K, int a_mn, int b_mn, int dt, int* status,
                      void* stream);

/* Workspace bytes for ak_linear_ce_logits_grad. */
AK_API int ak_linear_ce_logits_grad_workspace_size(int64_t N, int64_t V, size_t* bytes);

/* Forward half of the fused linear + CE for callers that run the two gradient
 * GEMMs themselves: the tcgen05 logits GEMM writes G[N, V] (dt, caller buffer)
 * and per-row softmax statistics in its epilogue; then loss[0], lse[N] and, in
 * place, G = (softmax - onehot) / n_valid (zero rows for ignored labels).
 * dH = G W and dW = G^T H are plain GEMMs.
 * Replaces the per-chunk F.linear + cross_entropy_fwd_hip of
 * _ChunkedLinearCrossEntropy.forward (kernels/hip/chunked_linear_cross_entropy.py:95-110). */
AK_API int ak_linear_ce_logits_grad(float* loss, float* lse, void* G, void* workspace,
                   size_t ws_bytes, const void* H, const void* W, const int64_t* labels,
                   int64_t N, int64_t D, int64_t V, int64_t ignore_index, int dt,
                   int* status, void* stream);

/* ------------------------------------------------------------------------ *
 * Collapsed (single-state) selective scan, fp32, layout (B, L, d)
 * ------------------------------------------------------------------------ */

/* h_t = dA_t*h_{t-1} + dBx_t;  y_t = C_t*h_t + D*x_t   (h_{-1} = 0).
 * Replaces selective_scan_hip / kernel_fn (kernels/hip/selective_scan.py:165-241)
 * and torch.ops.autokernel.selective_scan (kernels/hip/_torch_ops.py:312-318). */
AK_API int ak_scan1_fwd(float* y, const float* dA, const float* dBx, const float* C,
                 const float* D, const float* x, int64_t B, int64_t L, int64_t d,
                 void* stream);

AK_API int ak_scan1_bwd_workspace_size(int64_t B, int64_t L, int64_t d, size_t* bytes);

/* Gradients of ak_scan1_fwd given gy.  gD is reduced deterministically.
 * Replaces selective_scan_backward_hip / kernel_fn
 * (kernels/hip/selective_scan_backward.py:314-421) and _selective_scan_backward
 * (kernels/hip/_torch_ops.py:335-389). */
AK_API int ak_scan1_bwd(float* gdA, float* gdBx, float* gC, float* gD, float* gx,
                 void* workspace, size_t ws_bytes, const float* dA,
                 const float* dBx, const float* C, const float* D, const float* x,
                 const float* gy, int64_t B, int64_t L, int64_t d, void* stream);

/* Forward that also saves the backward's chunk-start states: carries (nullable)
 * receives h at the start of every 64-step chunk, B * ceil(L/64) * d floats
 * (ak_scan1_carries_size).  ak_scan1_fwd is this call with carries = NULL. */
AK_API int ak_scan1_carries_size(int64_t B, int64_t L, int64_t d, size_t* bytes);
AK_API int ak_scan1_fwd_ex(float* y, float* carries, const float* dA, const float* dBx,
                           const float* C, const float* D, const float* x, int64_t B,
                           int64_t L, int64_t d, void* stream);

/* Backward given the carries saved by ak_scan1_fwd_ex (carries_in non-NULL): the
 * pass that re-derives them from dA and dBx is skipped, and the workspace needs
 * only B * d floats.  With carries_in = NULL it is ak_scan1_bwd.  The
 * reference's sequential backward (kernels/hip/_torch_ops.py:335-389) keeps
 * the forward states; this keeps one state per 64 steps. */
AK_API int ak_scan1_bwd_ex(float* gdA, float* gdBx, float* gC, float* gD, float* gx,
                           void* workspace, size_t ws_bytes, const float* carries_in,
                           const float* dA, const float* dBx, const float* C,
                           const float* D, const float* x, const float* gy, int64_t B,
                           int64_t L, int64_t d, void* stream);

/* ------------------------------------------------------------------------ *
 * Mamba-style selective scan, layout (batch, dim, L), N states per channel
 * ------------------------------------------------------------------------ */

/* Timesteps between two saved states in `chunk_states`.  The forward saves the
 * state after every `ak_selective_scan_state_stride()` steps (and after the
 * last step): n_saved = ceil(L / stride). */
AK_API int ak_selective_scan_state_stride(void);

/* delta' = softplus?(delta + delta_bias);  per state n:
 *   h_t[n] = exp(delta'_t * A[d,n]) h_{t-1}[n] + delta'_t * B[b,g,n,t] * u_t
 *   y_t = sum_n C[b,g,n,t] h_t[n] + D[d] u_t;  out = y * silu(z)  (if z)
 * u, delta, z, out: (batch, dim, L) dt; A: fp32 (dim, dstate);
 * B, C: (batch, groups, dstate, L) dt, g = d / (dim / groups); 1 <= dstate <= 32;
 * D, delta_bias: fp32 (dim) nullable; last_state: fp32 (batch, dim, dstate)
 * nullable; chunk_states: fp32 (batch, dim, n_saved, dstate) nullable
 * (required for the backward).
 * Replaces selective_scan_cuda.fwd as called by SelectiveScanFn.forward
 * (external/mamba/mamba_ssm/ops/selective_scan_interface.py:23-53), with the
 * semantics of selective_scan_ref (same file, lines 115-181). */
AK_API int ak_selective_scan_fwd(void* out, float* last_state, float* chunk_states,
                          const void* u, const void* delta, const float* A,
                          const void* Bm, const void* Cm, const float* D,
                          const void* z, const float* delta_bias,
                          int delta_softplus, int64_t batch, int64_t dim,
                          int64_t seqlen, int64_t dstate, int64_t groups, int dt,
                          int* status, void* stream);

AK_API int ak_selective_scan_bwd_workspace_size(int64_t batch, int64_t dim,
                                         int64_t seqlen, int64_t dstate,
                                         int64_t groups, size_t* bytes);

/* Gradients of ak_selective_scan_fwd w.r.t. u, delta, A, B, C, D, z,
 * delta_bias (dD, dz, ddelta_bias nullable when the input was absent).
 * du, ddelta, dB, dC, dz: dt; dA, dD, ddelta_bias: fp32.
 * Replaces selective_scan_cuda.bwd as called by SelectiveScanFn.backward
 * (external/mamba/mamba_ssm/ops/selective_scan_interface.py:56-83). */
AK_API int ak_selective_scan_bwd(void* du, void* ddelta, float* dA, void* dB, void* dC,
                          float* dD, void* dz, float* ddelta_bias,
                          void* workspace, size_t ws_bytes, const void* dout,
                          const void* u, const void* delta, const float* A,
                          const void* Bm, const void* Cm, const float* D,
                          const void* z, const float* delta_bias,
                          const float* chunk_states, int delta_softplus,
                          int64_t batch, int64_t dim, int64_t seqlen,
                          int64_t dstate, int64_t groups, int dt, int* status,
                          void* stream);

/* ---- Fused residual add + RMSNorm (dual output) --------------------------
 * hidden = x + residual (rounded to dt_x); normed = hidden * rsqrt(mean(hidden^2)
 * + eps) * w.  hidden is nullable (single-output form).  x, residual, hidden,
 * normed: (M, N) dt_x; w: (N) dt_w, with the (dt_x, dt_w) pairs of
 * ak_rmsnorm_fwd.  Replaces fused_residual_add_rmsnorm_hip /
 * fused_residual_add_rmsnorm_dual_hip (kernels/hip/fused_residual_add_rmsnorm.py:
 * 340-418) behind autokernel::fused_res_rmsnorm (kernels/hip/_torch_ops.py:238-251). */
AK_API int ak_fused_res_rmsnorm_fwd(void* hidden, void* normed, const void* x,
                                    const void* residual, const void* w,
                                    int64_t M, int64_t N, float eps, int dt_x,
                                    int dt_w, void* stream);

/* Backward: dx (= d residual) = grad_hidden + RMSNorm-backward(hidden, w,
 * grad_normed); dw (dt_dw) = sum over rows of grad_normed * hidden * rstd.
 * grad_hidden nullable (zero).  Workspace: ak_rmsnorm_bwd_workspace_size(M, N).
 * Replaces fused_residual_rmsnorm_backward_hip
 * (kernels/hip/fused_residual_rmsnorm_backward.py:248-300) and the fp32 branch
 * of _fused_res_rmsnorm_backward (kernels/hip/_torch_ops.py:262-290). */
AK_API int ak_fused_res_rmsnorm_bwd(void* dx, void* dw, int dt_dw, void* workspace,
                                    size_t ws_bytes, const void* grad_hidden,
                                    const void* grad_normed, const void* hidden,
                                    const void* w, int64_t M, int64_t N, float eps,
                                    int dt_x, int dt_w, void* stream);

/* ---- SiLU gate multiply (SwiGLU body) -------------------------------------
 * y = silu(gate) * up over rows x cols; gate / up rows start ld_gate / ld_up
 * elements apart (cols for dense tensors, 2*cols for the halves of one packed
 * gate_up projection); y is dense (ld = cols).  All dt.
 * Replaces silu_gate_mul_hip (kernels/hip/silu_gate_mul.py:102-118) behind
 * autokernel::silu_gate_mul (kernels/hip/_torch_ops.py:181-186). */
AK_API int ak_silu_gate_mul_fwd(void* y, const void* gate, const void* up,
                                int64_t rows, int64_t cols, int64_t ld_gate,
                                int64_t ld_up, int dt, void* stream);

/* d gate = dy * up * silu'(gate), d up = dy * silu(gate); dgate / dup rows
 * ld_dgate / ld_dup apart (2*cols writes one packed d gate_up).  Replaces
 * silu_gate_mul_backward_hip (kernels/hip/silu_gate_mul_backward.py:145-180)
 * and the fp32 branch of _silu_gate_mul_backward (_torch_ops.py:199-218). */
AK_API int ak_silu_gate_mul_bwd(void* dgate, void* dup, const void* gate,
                                const void* up, const void* dy, int64_t rows,
                                int64_t cols, int64_t ld_gate, int64_t ld_up,
                                int64_t ld_dgate, int64_t ld_dup, int dt,
                                void* stream);

/* ---- Rotary position embedding (interleaved pairs) ------------------------
 * y[b,h,n,2i]   = x[.,2i] cos[n,i] - x[.,2i+1] sin[n,i]
 * y[b,h,n,2i+1] = x[.,2i] sin[n,i] + x[.,2i+1] cos[n,i]
 * x: element (b, h, n, d) at x + b*stride_b + h*stride_h + n*stride_n + d
 * (any strides with unit stride along D, e.g. q / k inside a fused QKV
 * projection); y: dense (B, H, N, D); cos_t / sin_t: fp32 (N, D/2).  D even.
 * Replaces rotary_embedding_hip / rotary_embedding_fp32_hip
 * (kernels/hip/rotary_embedding.py:253-300) behind autokernel::rotary_emb_fp32
 * (kernels/hip/_torch_ops.py:117-131). */
AK_API int ak_rope_fwd(void* y, const void* x, const float* cos_t,
                       const float* sin_t, int64_t B, int64_t H, int64_t N,
                       int64_t D, int64_t stride_b, int64_t stride_h,
                       int64_t stride_n, int dt, void* stream);

/* Gradient of ak_rope_fwd: dx = rotation of dy by -theta on the same pairs
 * (dy read through the given strides, dx dense).  Replaces
 * rotary_embedding_backward_hip (kernels/hip/rotary_embedding_backward.py:126-170)
 * and _rotary_backward (kernels/hip/_torch_ops.py:140-162), which assume the
 * rotate-half pairing with full-width tables. */
AK_API int ak_rope_bwd(void* dx, const void* dy, const float* cos_t,
                       const float* sin_t, int64_t B, int64_t H, int64_t N,
                       int64_t D, int64_t stride_b, int64_t stride_h,
                       int64_t stride_n, int dt, void* stream);

/* Strided form of both: x element (b, h, n, d) at x + b*x_sb + h*x_sh + n*x_sn + d,
 * y element at y + b*y_sb + h*y_sh + n*y_sn + d.  mode 1 = ak_rope_fwd's rotation,
 * -1 = ak_rope_bwd's, 0 = plain copy (cos_t / sin_t may be NULL).  Used for the
 * gradient of a fused QKV projection: dq and dk are rotated back and dv copied
 * straight into their columns of one packed (B, N, W) gradient, the work the
 * reference's autograd does with separate slice, fill and add kernels around
 * autokernel::rotary_emb_fp32 (kernels/hip/_torch_ops.py:117-162). */
AK_API int ak_rope_strided(void* y, const void* x, const float* cos_t,
                           const float* sin_t, int64_t B, int64_t H, int64_t N,
                           int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_sn,
                           int64_t y_sb, int64_t y_sh, int64_t y_sn, int mode,
                           int dt, void* stream);

/* ---- Batched last-two-dims transpose ---------------------------------------
 * out[b][c][r] = in[b][r][c] for b < batch, r < R, c < C; element (b, r, c) of
 * `in` at in + b*in_bstride + r*in_ld + c, element (b, c, r) of `out` at
 * out + b*out_bstride + c*out_ld + r (strides in elements, unit last stride).
 * Replaces the `.transpose(1, 2).contiguous()` layout copies between the
 * (B, T, D) projections and the (B, D, T) conv / scan operands of the Mamba
 * block (external/mamba/mamba_ssm/modules/mamba_simple.py forward). */
AK_API int ak_transpose(void* out, const void* in, int64_t batch, int64_t R,
                        int64_t C, int64_t in_bstride, int64_t in_ld,
                        int64_t out_bstride, int64_t out_ld, int dt,
                        void* stream);

/* ---- Mixed-precision RMSNorm (fp32 residual stream, 16-bit activations) ----
 * No reference counterpart: under bf16/fp16 autocast the reference computes the
 * norm in fp32 and the next GEMM casts its output; these entries write the
 * 16-bit output directly (the same single rounding) and take 16-bit gradients.
 * Mixed combinations: compute / residual fp32, the 16-bit side bf16 or fp16,
 * w fp32 or of the 16-bit type.  Equal dtypes route to the plain entries.
 *
 * ak_rmsnorm_fwd_mixed: y (dt_y) = rmsnorm(x fp32) * w.
 * ak_fused_res_rmsnorm_fwd_mixed: hidden (fp32) = x (16-bit) + residual (fp32);
 *   normed (16-bit, = dt_x) = rmsnorm(hidden) * w.
 * ak_rmsnorm_bwd_mixed: x fp32 (the normalised input / hidden), dy 16-bit:
 *   dx (fp32) = [grad_hidden fp32, nullable] + rmsnorm backward; dx2 (16-bit,
 *   nullable) = dx rounded (the gradient of a 16-bit fused-residual input);
 *   dw (dt_dw).  Workspace: ak_rmsnorm_bwd_workspace_size(M, N). */
AK_API int ak_rmsnorm_fwd_mixed(void* y, int dt_y, const void* x, int dt_x,
                                const void* w, int dt_w, int64_t M, int64_t N,
                                float eps, void* stream);
AK_API int ak_fused_res_rmsnorm_fwd_mixed(void* hidden, void* normed, int dt_normed,
                                          const void* x, int dt_x, const void* residual,
                                          int dt_res, const void* w, int dt_w,
                                          int64_t M, int64_t N, float eps, void* stream);
AK_API int ak_rmsnorm_bwd_mixed(void* dx, void* dx2, void* dw, int dt_dw, void* workspace,
                                size_t ws_bytes, const void* grad_hidden, const void* dy,
                                int dt_dy, const void* x, int dt_x, const void* w, int dt_w,
                                int64_t M, int64_t N, float eps, void* stream);

/* ---- Depthwise causal conv1d (+ optional SiLU) --------------------------
 * y[b,d,t] = act(bias[d] + sum_k w[d,k] x[b,d,t-K+1+k]), x = 0 before t = 0;
 * act = SiLU when silu != 0, identity otherwise.  x, y: (B, D, T) dt, T
 * contiguous; weight: fp32 (D, K), 2 <= K <= 8; bias: fp32 (D) nullable.
 * Replaces the forward of autokernel::causal_conv1d
 * (kernels/hip/_torch_ops.py:883-902: F.pad + F.conv1d groups=D, or
 * causal_conv1d_fn) and causal_conv1d_fn(x, w, b, activation="silu") as
 * called from the Mamba block. */
AK_API int ak_causal_conv1d_fwd(void* y, const void* x, const float* weight,
                                const float* bias, int64_t B, int64_t D,
                                int64_t T, int64_t K, int silu, int dt,
                                void* stream);

AK_API int ak_causal_conv1d_bwd_workspace_size(int64_t B, int64_t D, int64_t T,
                                               int64_t K, size_t* bytes);

/* Gradients of ak_causal_conv1d_fwd: dx (B, D, T) dt; dweight fp32 (D, K);
 * dbias fp32 (D) nullable.  Deterministic (fixed-order weight reduction).
 * Replaces _causal_conv1d_shim_backward (kernels/hip/_torch_ops.py:910-965). */
AK_API int ak_causal_conv1d_bwd(void* dx, float* dweight, float* dbias,
                                void* workspace, size_t ws_bytes, const void* x,
                                const float* weight, const float* bias,
                                const void* dy, int64_t B, int64_t D, int64_t T,
                                int64_t K, int silu, int dt, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AK_B200_H */
