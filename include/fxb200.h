/*
 * fxb200.h - C ABI of libfxb200.so, the sm_100a (B200) kernels behind the
 * fxlm / fxgpu operator surface.
 *
 * The reference launches runtime-compiled HIP kernels through ctypes
 * (ml/fxgpu/hip_kernel.py:50-145: compile_kernel / compile_module / launch).
 * This library is built ahead of time and exposes one plain C function per
 * operation instead. Conventions:
 *   - every pointer is a device pointer owned by the caller; the library
 *     never allocates or frees device memory (workspaces are passed in, their
 *     sizes come from the *_workspace functions);
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); no function
 *     synchronises the host except fxb_device_error;
 *   - functions return FXB_OK (0) or a negative FXB_E* code; the message of
 *     the last failure on the calling thread is returned by fxb_last_error().
 *     Nothing exits, aborts or traps.
 *   - dtype codes: FXB_DTYPE_F32 / F16 / BF16.
 */
#ifndef FXB200_H
#define FXB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FXB_OK 0
#define FXB_EINVAL (-1)      /* bad shape / stride / alignment / pointer */
#define FXB_EUNSUPPORTED (-2) /* valid request this build does not implement */
#define FXB_ECUDA (-3)       /* CUDA runtime / driver error (see fxb_last_error) */

#define FXB_DTYPE_F32 0
#define FXB_DTYPE_F16 1
#define FXB_DTYPE_BF16 2

/* ------------------------------------------------------------------ misc */

/* Library version (major*10000 + minor*100 + patch). */
int fxb_version(void);

/* Message of the last failed call on this thread ("" if none).
 * Replaces the RuntimeError text of _chk, ml/fxgpu/hip_kernel.py:45-47. */
const char* fxb_last_error(void);

/* Reads (and with clear != 0 resets) the device error word that kernels set
 * when a bounded wait expires (bit 1 GEMM, 2 attention, 4 gather, 8 cross-
 * entropy). Synchronises
 * the current device. No reference counterpart (the reference has no bounded
 * waits). */
int fxb_device_error(int32_t* code, int32_t clear);

/* Number of streaming multiprocessors of the current device (grid sizing). */
int fxb_num_sms(int32_t* out);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t fxb_launch_count(void);

/* ABI self-check for bindings: sizeof(fxb_gemm_args) for which == 0,
 * sizeof(fxb_attn_args) for which == 1, 0 otherwise. */
size_t fxb_abi_struct_size(int32_t which);

/* ------------------------------------------------------------------ RMSNorm */

/* y = x * rsqrt(mean(x^2) + eps) * w, rstd saved (fp32, one per row).
 * x, y: (rows, D) contiguous; w: (D,). D % 8 == 0, D <= 8192.
 * Replaces rms_norm_fwd (ml/fxlm/kernels/norm.hip:33) as launched by
 * _RMSNorm.forward (ml/fxlm/norm.py:45-60). */
int fxb_rmsnorm_fwd(int32_t dtype, const void* x, const void* w, void* y, float* rstd,
                    int64_t rows, int32_t D, float eps, void* stream);

/* Bytes of fp32 workspace fxb_rmsnorm_bwd needs for the dw partial sums. */
size_t fxb_rmsnorm_bwd_workspace(int64_t rows, int32_t D);

/* dx = rstd*w*dy - x*rstd^3*sum(x*w*dy)/D (+ dres when dres != NULL: the
 * gradient reaching x through a residual connection, summed in the same pass);
 * dw = sum_rows x*rstd*dy.
 * dw (dtype dw_dtype, e.g. an fp32 flat-gradient slot) is written
 * (dw_accumulate == 0) or added to (dw_accumulate != 0). Any D the forward
 * takes (D % 8 == 0, D <= 8192): rows of up to 2048 16-bit (1024 fp32)
 * elements are handled a warp per row, longer rows a block per row.
 * Deterministic: per-block partials, then a fixed-order sum.
 * Replaces rms_norm_bwd_dx + rms_norm_bwd_dw + part.sum(0)
 * (ml/fxlm/kernels/norm.hip:64,102; ml/fxlm/norm.py:62-84). */
int fxb_rmsnorm_bwd(int32_t dtype, const void* x, const void* w, const float* rstd,
                    const void* dy, const void* dres, void* dx, void* dw, int32_t dw_dtype,
                    int32_t dw_accumulate, float* workspace, int64_t rows, int32_t D,
                    void* stream);

/* fxb_rmsnorm_bwd without a workspace argument: the call allocates nothing.
 * It has no counterpart in the reference; this entry exists for callers
 * that cannot allocate device memory on the call path, e.g. a host runtime
 * with a fixed memory budget that owns no allocator, or code that must not
 * call cudaMalloc / cudaFree (which synchronise the device).
 * Same math, arguments and results as fxb_rmsnorm_bwd (identical block count,
 * so identical dw). The dw partials live in a file-scope device array of
 * fxb_rmsnorm_bwd_static_max_bytes() bytes (4 MiB), one per device:
 *  - the first call on a device looks up that array's address
 *    (cudaGetSymbolAddress) and caches it (again after the device's context
 *    was replaced, e.g. by cudaDeviceReset); make that first call before any
 *    stream capture;
 *  - a call whose partials need more than the array holds
 *    (fxb_rmsnorm_bwd_workspace(rows, D) > the maximum) returns FXB_EINVAL;
 *  - nothing in the array has to start at zero (each block writes all of its
 *    partials before they are read);
 *  - every call on a device shares the array, so two calls that overlap in
 *    time (different streams or host threads) race on it: issue them in order
 *    on one stream. */
size_t fxb_rmsnorm_bwd_static_max_bytes(void);
int fxb_rmsnorm_bwd_static(int32_t dtype, const void* x, const void* w, const float* rstd,
                           const void* dy, const void* dres, void* dx, void* dw,
                           int32_t dw_dtype, int32_t dw_accumulate, int64_t rows, int32_t D,
                           void* stream);

/* ------------------------------------------------------------------ cross entropy */

/* Row-wise softmax cross entropy with the gradient written in the same pass.
 *   row_loss[r] = logsumexp(row) - row[target]   (0 for rows that are not valid)
 *   grad[r,:]   = (softmax(row) - onehot(target)) * (*mul)   (0 for ignored rows)
 * A row is valid when target != ignore_index and 0 <= target < V. The caller
 * sums row_loss (fixed order, deterministic) where the reference accumulated
 * one scalar with atomics.
 * grad may be NULL (loss only) or equal to logits (in place).
 * logits/grad: (rows, V) with row stride ld (elements); target int64 (rows,);
 * row_loss fp32 (rows,); mul is an fp32 device scalar (no host sync).
 * Replaces ce_fwd_grad (ml/fxlm/kernels/ce.hip:32) as launched by _ce_rows
 * (ml/fxlm/cross_entropy.py:47-59). */
int fxb_ce_fwd_grad(int32_t dtype, const void* logits, int64_t ld, const int64_t* target,
                    void* grad, float* row_loss, const float* mul, int64_t rows, int32_t V,
                    int64_t ignore_index, void* stream);

/* ------------------------------------------------------------------ FlatAdamW */

/* scratch[0] += sum(g^2); flags |= 1 if any g is non-finite. g: flat (n,).
 * Replaces adamw_sumsq (ml/fxlm/kernels/optim.hip:26) over the per-tensor
 * TensorList of FlatAdamW._chunks (ml/fxlm/optim.py:107-144). */
int fxb_adamw_sumsq(int32_t gdtype, const void* grad, int64_t n, float* scratch,
                    int32_t* flags, void* stream);

/* Same result as fxb_adamw_sumsq, summed in a fixed order: per-block partial
 * sums go to the workspace `ws` (fxb_adamw_sumsq_ws_bytes() bytes, 4-byte
 * aligned, zero-filled once before its first use; every call leaves its
 * ticket counter at zero) and the block that finishes last adds them in
 * block order. The
 * norm is then bitwise reproducible, so data-parallel ranks holding the same
 * reduced gradient take bitwise identical optimizer steps. One workspace per
 * stream (concurrent calls must not share it). No reference counterpart: the
 * reference accumulates with atomicAdd (ml/fxlm/kernels/optim.hip:71). */
size_t fxb_adamw_sumsq_ws_bytes(void);
int fxb_adamw_sumsq_det(int32_t gdtype, const void* grad, int64_t n, float* scratch,
                        int32_t* flags, void* ws, void* stream);

/* One thread: found_inf = flags || !isfinite(scratch[0]);
 * norm = sqrt(scratch[0]) / scale; scratch[1] = clip coefficient
 * min(1, max_norm/(norm+1e-6)) (0 when found_inf); step += !found_inf;
 * flags and scratch[0] reset for the next step.
 * Replaces adamw_final (ml/fxlm/kernels/optim.hip:77-93). */
int fxb_adamw_final(float* scratch, int32_t* flags, int32_t* step, float* found_inf,
                    float* norm_out, const float* scale, float max_norm, void* stream);

/* Flat decoupled-weight-decay AdamW over n elements (skipped when *found_inf):
 *   g = grad * scratch[1] / scale; w -= lr*wd*w (segments with seg_wd != 0);
 *   m = b1*m + (1-b1) g; v = b2*v + (1-b2) g^2;
 *   w -= lr * (m / (1-b1^step)) / (sqrt(v / (1-b2^step)) + eps);
 *   master = w; param = (pdtype) w; grad = 0 (the gradient is consumed, also
 *   when the step is skipped, so the buffer is ready for the next backward).
 * Segments: seg_end[i] (exclusive, device int64, ascending, multiples of 8) and
 * seg_wd[i] (device int32), nseg <= 1024.
 * lr_dev: when non-NULL the learning rate is read from this device fp32
 * scalar and `lr` is ignored, so a captured CUDA graph can follow a schedule
 * (the host updates the scalar between replays).
 * Replaces adamw_update (ml/fxlm/kernels/optim.hip:96-162). */
int fxb_adamw_update(int32_t gdtype, int32_t pdtype, const void* grad, float* master,
                     float* m, float* v, void* param, int64_t n, const int64_t* seg_end,
                     const int32_t* seg_wd, int32_t nseg, const float* scratch,
                     const float* found_inf, const float* scale, const int32_t* step,
                     float lr, const float* lr_dev, float beta1, float beta2, float eps,
                     float weight_decay, void* stream);

/* ------------------------------------------------------------------ GEMM */

/* Epilogues applied to acc = sum_k A[m,k] * B[n,k] (fp32 in tensor memory). */
#define FXB_EPI_STORE 0     /* C = alpha*acc */
#define FXB_EPI_RESIDUAL 1  /* C = alpha*acc + R  (R may alias C: accumulate) */
#define FXB_EPI_GELU 2      /* Z = acc ; C = gelu_tanh(acc) */
#define FXB_EPI_DGELU 3     /* C = acc * gelu_tanh'(R)   (R = pre-activation) */
#define FXB_EPI_BIAS 4      /* C = acc + bias[n] */
#define FXB_EPI_BIAS_GELU 5 /* Z = acc + bias[n] ; C = gelu_tanh(Z) */
#define FXB_EPI_BIAS_SILU 6 /* Z = acc + bias[n] ; C = silu(Z) */
#define FXB_EPI_ACCUM_F32 7 /* C(fp32) += alpha*acc (red.add; enables split-K) */
#define FXB_EPI_DSILU 8     /* C = acc * silu'(R)        (R = pre-activation) */
#define FXB_EPI_GELU_DERIV 9 /* C = gelu_tanh(p) ; Z = gelu_tanh'(p), p = acc rounded to C's type */
#define FXB_EPI_MUL 10      /* C = alpha*acc*R  (with Z of FXB_EPI_GELU_DERIV as R: the
                               GELU backward without recomputing the activation) */

typedef struct fxb_gemm_args {
  int32_t dtype;     /* A/B dtype: FXB_DTYPE_BF16 / FXB_DTYPE_F16 (tensor cores) or
                        FXB_DTYPE_F32 (fp32 parity mode: C, R, Z, bias fp32 too) */
  int32_t M, N, K;
  const void* A;     /* a_trans == 0: (M,K) row stride lda; 1: (K,M) row stride lda */
  int64_t lda;
  int32_t a_trans;
  const void* B;     /* b_trans == 0: (N,K) row stride ldb; 1: (K,N) row stride ldb */
  int64_t ldb;
  int32_t b_trans;
  void* C;           /* (M,N) row stride ldc, dtype c_dtype */
  int64_t ldc;
  int32_t c_dtype;
  int32_t epilogue;  /* FXB_EPI_* */
  float alpha;
  const void* R;     /* residual / pre-activation input, dtype c_dtype, row stride ldr */
  int64_t ldr;
  void* Z;           /* second output (pre-activation), dtype c_dtype, row stride ldz */
  int64_t ldz;
  const void* bias;  /* (N,), dtype c_dtype */
  /* Optional scratch (NULL: none) of workspace_bytes >= fxb_gemm_workspace_size()
   * bytes, 16-byte aligned, whose first 4096 bytes (arrival counters) are
   * zero-filled once before its first use (the kernels leave them at zero). With it, tiles that would leave most of the
   * last wave idle are split along K and their pieces reduced through it; it
   * must not be shared by calls that can run concurrently (one per stream). */
  void* workspace;
  int64_t workspace_bytes;
} fxb_gemm_args;

/* tcgen05 / TMEM GEMM with TMA-fed operands. Requires K % 8 == 0 for K-major
 * operands and M (resp. N) % 8 == 0 for transposed ones (16-byte TMA rows),
 * 16-byte aligned bases, N % 8 == 0 for C.
 * dtype FXB_DTYPE_F32 runs an fp32 SIMT kernel instead (every epilogue, exact
 * tanh / exp, no shape or alignment constraints beyond positive leading
 * dimensions): the 1e-5 fp32 parity mode, not a fast path.
 * Replaces the rocBLAS matmuls on the hot path: nn.Linear qkv/proj/fc/fc2
 * (ml/fxlm/model.py:48-51,61,69-71), the linear-CE chunk mm's
 * (ml/fxlm/cross_entropy.py:131-135,180) and the fxgpu dW mm
 * (ml/fxgpu/fused_linear.py:94). */
int fxb_gemm(const fxb_gemm_args* args, void* stream);

/* Bytes of fxb_gemm_args.workspace that enable the tail split on the current
 * device. No reference counterpart (the reference's rocBLAS calls own their
 * scratch). */
size_t fxb_gemm_workspace_size(void);

/* The tile configuration fxb_gemm would use for this problem on the current
 * device: *pair = 1 for the CTA-pair (cta_group::2, 256-row) kernel, 0 for the
 * single-CTA (128-row) kernel; *bn = tile width; *splits = split-K factor
 * (> 1 for FXB_EPI_ACCUM_F32), or for the other epilogues the number of K
 * pieces of each tail tile when a workspace is given (1: no tail split).
 * Diagnostic; no reference counterpart. */
int fxb_gemm_plan(int32_t M, int32_t N, int32_t K, int32_t epilogue, int32_t* pair,
                  int32_t* bn, int32_t* splits);

/* Loss-only linear cross entropy with the logits kept on chip:
 *   row_loss[r] = logsumexp_v(x_r . w_v) - x_r . w_{target[r]}
 * (0 for rows whose target is ignore_index or outside [0, V)). The tcgen05
 * GEMM of x (N, D) by w (V, D)^T reduces each accumulator tile in tensor
 * memory to per-row (max, sum of exp) pairs and the target column's value
 * (fp32, before any rounding), so no (N, V) logits are written; a second
 * kernel merges the pairs per row. x, w bf16 or f16, 16-byte aligned, D and
 * V multiples of 8; workspace of fxb_linear_ce_loss_workspace(N, V) bytes,
 * 16-byte aligned. The caller sums row_loss (fixed order) and divides by the
 * number of valid rows.
 * Replaces the loss-only chunk loop of _linear_ce_loss_only
 * (ml/fxlm/cross_entropy.py:170-183: mm to a logits chunk, then ce_fwd_grad
 * without gradient, ml/fxlm/kernels/ce.hip:32). */
size_t fxb_linear_ce_loss_workspace(int64_t N, int32_t V);
int fxb_linear_ce_loss(int32_t dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                       const int64_t* target, float* row_loss, void* workspace, int64_t N,
                       int32_t D, int32_t V, int64_t ignore_index, void* stream);

/* ------------------------------------------------------------------ attention */

typedef struct fxb_attn_args {
  int32_t dtype;          /* FXB_DTYPE_BF16 or FXB_DTYPE_F16 */
  int32_t B, T, H, D;     /* D = head dim (64 or 128) */
  float scale;
  int32_t causal;
  /* (B,T,H,D) views with unit stride on D; strides in elements (b, t, h) */
  const void* q; int64_t q_sb, q_st, q_sh;
  const void* k; int64_t k_sb, k_st, k_sh;
  const void* v; int64_t v_sb, v_st, v_sh;
  void* o;       int64_t o_sb, o_st, o_sh;   /* forward output; backward input */
  float* lse;                                /* (B,H,T) natural-log LSE of scaled scores */
  const void* dout; int64_t do_sb, do_st, do_sh;
  void* dq;      int64_t dq_sb, dq_st, dq_sh;
  void* dk;      int64_t dk_sb, dk_st, dk_sh;
  void* dv;      int64_t dv_sb, dv_st, dv_sh;
  float* workspace;                          /* backward: fxb_attn_bwd_workspace bytes */
} fxb_attn_args;

/* Causal / non-causal flash-attention forward: o = softmax(q k^T * scale) v,
 * lse = logsumexp of the scaled scores (natural log). dtype bf16 / f16 run
 * the tcgen05 kernel (strides multiples of 8 elements, 16-byte aligned
 * bases); dtype f32 runs an fp32 SIMT kernel (the 1e-5 parity mode; any
 * positive strides). Head dim 64 or 128.
 * Replaces attn_fwd (ml/fxlm/kernels/attention.hip:104) as launched by _fwd
 * (ml/fxlm/attention.py:87-104). */
int fxb_attn_fwd(const fxb_attn_args* args, void* stream);

/* Workspace bytes for fxb_attn_bwd (delta = rowsum(dO*O), fp32 dQ staging). */
size_t fxb_attn_bwd_workspace(int32_t B, int32_t T, int32_t H, int32_t D);

/* Flash-attention backward: dq, dk, dv from q, k, v, o, lse, dout (head dim
 * 64 or 128; bf16 / f16 on tensor cores, f32 as the forward).
 * Replaces attn_bwd_prep + attn_bwd_dkv + attn_bwd_dq
 * (ml/fxlm/kernels/attention.hip:229,256,411) as launched by _bwd
 * (ml/fxlm/attention.py:107-134). */
int fxb_attn_bwd(const fxb_attn_args* args, void* stream);

/* ------------------------------------------------------------------ embedding / glue */

/* out[b,t,:] = tok[idx[b,t],:] + pos[t,:]. idx int64 (B*T). Rows of out are D
 * contiguous; dtype bf16, f16 or f32; D % 8 == 0, 16-byte aligned buffers. Replaces tok_emb(idx) + pos_emb[:T] (ml/fxlm/model.py:118). */
int fxb_embedding_fwd(int32_t dtype, const int64_t* idx, const void* tok, const void* pos,
                      void* out, int64_t B, int64_t T, int32_t D, int64_t V, void* stream);

/* dtok_ws[idx[b,t],:] += dout[b,t,:], dpos_ws[t,:] += dout[b,t,:] (fp32
 * workspaces, zeroed by the caller, 16-byte aligned; fp32 vector reductions).
 * Backward of ml/fxlm/model.py:118. */
int fxb_embedding_bwd(int32_t dtype, const int64_t* idx, const void* dout, float* dtok_ws,
                      float* dpos_ws, int64_t B, int64_t T, int32_t D, int64_t V,
                      void* stream);

/* dst[i] = (accumulate ? dst[i] : 0) + src[i] * (scale ? *scale : 1) for i < n.
 * dst dtype ddtype, src dtype sdtype, scale an fp32 device scalar or NULL.
 * Carries the linear-CE backward rescale (ml/fxlm/cross_entropy.py:140-149). */
int fxb_axpy(int32_t ddtype, void* dst, int32_t sdtype, const void* src, const float* scale,
             int32_t accumulate, int64_t n, void* stream);

/* ------------------------------------------------------------------ fxgpu window model */

/* Xg[b, :] = X[idx[b] : idx[b] + window, :] flattened window-major (K = window*F),
 * i.e. Xg[b, w*F + f] = X[idx[b] + w, f]. X (R, F) row-major (bf16, f16 or
 * f32), F % 8 == 0,
 * idx int32; windows that leave [0, R) are written as zeros.
 * Replaces the A-operand gather and the Xg write-out of gather_gemm
 * (ml/fxgpu/gather_gemm.hip:17-180, launched by ml/fxgpu/fused_linear.py:76-85);
 * the GEMM itself runs through fxb_gemm with FXB_EPI_BIAS*. */
int fxb_gather_windows(int32_t dtype, const void* X, int64_t R, int32_t F, const int32_t* idx,
                       int32_t B, int32_t window, void* Xg, void* stream);

/* out[c] (fp32) = (accumulate ? out[c] : 0) + sum_r g[r, c]; g (rows, cols) row-major
 * (may be NULL when rows == 0). Deterministic (fixed summation order, no atomics).
 * The bias gradient db = g.sum(0) of ml/fxgpu/fused_linear.py:95. */
int fxb_colsum(int32_t dtype, const void* g, int64_t rows, int32_t cols, float* out,
               int32_t accumulate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FXB200_H */
