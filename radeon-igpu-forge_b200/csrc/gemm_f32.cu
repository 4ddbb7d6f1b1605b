// fp32 GEMM for the parity mode (fxb_gemm with dtype FXB_DTYPE_F32).
//
// The reference's fp32 path is PyTorch's own fp32 matmul (its selftest and
// model torch path, ml/fxlm/selftest.py:301-333); parity there is 1e-5, which
// the 16-bit tensor-core kernels cannot meet and tf32 would not either. This
// is a plain SIMT kernel with fp32 fused multiply-adds: 128 x 64 output tiles,
// 256 threads each owning 8 x 4 outputs, 16-deep K slices staged in shared
// memory (stored K-major so each thread reads its 8 A rows and 4 B columns as
// vectors). Every epilogue of the tensor-core GEMM is supported with the same
// meaning, computed in fp32 with the accurate tanhf / expf (no hardware
// approximations). Accuracy, not speed, is its purpose: it runs at a few
// percent of the tensor-core kernel's rate.
#include "common.cuh"
#include "internal.h"

namespace {

constexpr int BM = 128, BN = 64, BKF = 16, TM = 8, TN = 4;
constexpr int kThreads = (BM / TM) * (BN / TN);  // 256

struct F32Args {
  int M, N, K;
  const float* A; int64_t lda; int at;
  const float* B; int64_t ldb; int bt;
  float* C; int64_t ldc;
  int epi; float alpha;
  const float* R; int64_t ldr;
  float* Z; int64_t ldz;
  const float* bias;
};

__device__ float gelu_acc(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}
__device__ float gelu_grad_acc(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float t = tanhf(k0 * (x + k1 * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}
__device__ float silu_acc(float x) { return x / (1.f + expf(-x)); }
__device__ float silu_grad_acc(float x) {
  const float s = 1.f / (1.f + expf(-x));
  return s * (1.f + x * (1.f - s));
}

__device__ void epilogue(const F32Args& p, int m, int n, float acc) {
  float* c = p.C + (int64_t)m * p.ldc + n;
  switch (p.epi) {
    case FXB_EPI_STORE: *c = p.alpha * acc; break;
    case FXB_EPI_RESIDUAL: *c = p.alpha * acc + p.R[(int64_t)m * p.ldr + n]; break;
    case FXB_EPI_GELU: p.Z[(int64_t)m * p.ldz + n] = acc; *c = gelu_acc(acc); break;
    case FXB_EPI_DGELU: *c = acc * gelu_grad_acc(p.R[(int64_t)m * p.ldr + n]); break;
    case FXB_EPI_BIAS: *c = acc + p.bias[n]; break;
    case FXB_EPI_BIAS_GELU: {
      const float z = acc + p.bias[n];
      p.Z[(int64_t)m * p.ldz + n] = z;
      *c = gelu_acc(z);
      break;
    }
    case FXB_EPI_BIAS_SILU: {
      const float z = acc + p.bias[n];
      p.Z[(int64_t)m * p.ldz + n] = z;
      *c = silu_acc(z);
      break;
    }
    case FXB_EPI_ACCUM_F32: *c += p.alpha * acc; break;  // one thread per element: no race
    case FXB_EPI_DSILU: *c = acc * silu_grad_acc(p.R[(int64_t)m * p.ldr + n]); break;
    case FXB_EPI_GELU_DERIV:
      *c = gelu_acc(acc);
      p.Z[(int64_t)m * p.ldz + n] = gelu_grad_acc(acc);
      break;
    case FXB_EPI_MUL: *c = p.alpha * acc * p.R[(int64_t)m * p.ldr + n]; break;
    default: break;
  }
}

// opA(A)[m, k] and opB(B)[n, k] with bounds (zero outside)
__device__ __forceinline__ float ldA(const F32Args& p, int m, int k) {
  if (m >= p.M || k >= p.K) return 0.f;
  return p.at ? p.A[(int64_t)k * p.lda + m] : p.A[(int64_t)m * p.lda + k];
}
__device__ __forceinline__ float ldB(const F32Args& p, int n, int k) {
  if (n >= p.N || k >= p.K) return 0.f;
  return p.bt ? p.B[(int64_t)k * p.ldb + n] : p.B[(int64_t)n * p.ldb + k];
}

__global__ void __launch_bounds__(kThreads) gemm_f32_kernel(const F32Args p) {
  pdl_trigger();
  pdl_wait();  // operands come from earlier kernels on the stream
  // rows padded by 4 floats: the k-fastest stores of K-major operands hit
  // 2-way bank conflicts instead of 16-way; rows stay 16-byte aligned
  __shared__ __align__(16) float sA[BKF][BM + 4];
  __shared__ __align__(16) float sB[BKF][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);  // 16 x 16 threads
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < p.K; k0 += BKF) {
    // A slice: BM x BKF = 2048 values, 8 per thread; along k for K-major A
    // (consecutive threads read consecutive k) and along m for transposed A
#pragma unroll
    for (int u = 0; u < (BM * BKF) / kThreads; ++u) {
      const int e = u * kThreads + tid;
      int mm, kk;
      if (p.at) { mm = e % BM; kk = e / BM; } else { kk = e % BKF; mm = e / BKF; }
      sA[kk][mm] = ldA(p, m0 + mm, k0 + kk);
    }
#pragma unroll
    for (int u = 0; u < (BN * BKF) / kThreads; ++u) {
      const int e = u * kThreads + tid;
      int nn, kk;
      if (p.bt) { nn = e % BN; kk = e / BN; } else { kk = e % BKF; nn = e / BKF; }
      sB[kk][nn] = ldB(p, n0 + nn, k0 + kk);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BKF; ++kk) {
      float a[TM], b[TN];
      const float4 a0 = *reinterpret_cast<const float4*>(&sA[kk][ty * TM]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sA[kk][ty * TM + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sB[kk][tx * TN]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty * TM + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx * TN + j;
      if (n < p.N) epilogue(p, m, n, acc[i][j]);
    }
  }
}

}  // namespace

namespace fxb {

// Called by fxb_gemm for dtype FXB_DTYPE_F32 (arguments already validated
// for pointers and the epilogue's required inputs).
int gemm_f32(const fxb_gemm_args* a, cudaStream_t st) {
  if (a->c_dtype != FXB_DTYPE_F32)
    return set_error(FXB_EINVAL, "gemm fp32: C must be fp32 (c_dtype %d)", a->c_dtype);
  F32Args p;
  p.M = a->M; p.N = a->N; p.K = a->K;
  p.A = static_cast<const float*>(a->A); p.lda = a->lda; p.at = a->a_trans;
  p.B = static_cast<const float*>(a->B); p.ldb = a->ldb; p.bt = a->b_trans;
  p.C = static_cast<float*>(a->C); p.ldc = a->ldc;
  p.epi = a->epilogue; p.alpha = a->alpha;
  p.R = static_cast<const float*>(a->R); p.ldr = a->ldr;
  p.Z = static_cast<float*>(a->Z); p.ldz = a->ldz;
  p.bias = static_cast<const float*>(a->bias);
  const dim3 grid((unsigned)((a->N + BN - 1) / BN), (unsigned)((a->M + BM - 1) / BM));
  if (grid.y > 65535u) return set_error(FXB_EINVAL, "gemm fp32: M=%d too large", a->M);
  pdl_launch(gemm_f32_kernel, grid, dim3(kThreads), 0, st, p);
  return check_launch("gemm_f32");
}

}  // namespace fxb
