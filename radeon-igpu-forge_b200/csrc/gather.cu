// fxgpu window gather and bias-gradient column sum (HBM-bound).
//
// The reference's gather_gemm kernel (ml/fxgpu/gather_gemm.hip:17-180) reads
// A[b, k] = X[idx[b] + k / F, k % F] on the fly and also writes that gathered
// row to Xg (:88-89) for the weight gradient. Because X is row-major (R, F),
// the window of row b is the contiguous span X[idx[b]*F, (idx[b]+W)*F), so
// the gather is a row-wise copy; the GEMM then reads Xg through TMA. The bias
// gradient db = sum_b g[b, :] (ml/fxgpu/fused_linear.py:95) is a column sum.
#include "common.cuh"
#include "internal.h"

namespace {

// one warp per output row, 16-byte vectors (F % 8 == 0 => row starts aligned)
template <typename T>
__global__ void gather_windows_kernel(const T* __restrict__ X, int64_t R, int F,
                                      const int* __restrict__ idx, int B, int window,
                                      T* __restrict__ Xg) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const int lane = threadIdx.x & 31;
  const int64_t K = (int64_t)window * F;
  const int64_t nvec = K / 8;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < B; b += nw) {
    const int64_t s = idx[b];
    const bool ok = s >= 0 && s + window <= R;  // out-of-range windows are zero-filled
    const uint4* src = reinterpret_cast<const uint4*>(X + (ok ? s : 0) * F);
    uint4* dst = reinterpret_cast<uint4*>(Xg + b * K);
    for (int64_t v = lane; v < nvec; v += 32) dst[v] = ok ? src[v] : make_uint4(0, 0, 0, 0);
  }
}

// out[c] (fp32) (+)= sum_r g[r, c]; block = 32 columns x 8 row-groups
template <typename T>
__global__ void colsum_kernel(const T* __restrict__ g, int64_t rows, int cols,
                              float* __restrict__ out, int accumulate) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  __shared__ float part[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < cols)
    for (int64_t r = threadIdx.y; r < rows; r += 8) s += to_f<T>(g[r * cols + c]);
  part[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k][threadIdx.x];
    out[c] = accumulate ? out[c] + t : t;
  }
}

}  // namespace

extern "C" {

int fxb_gather_windows(int32_t dtype, const void* X, int64_t R, int32_t F, const int32_t* idx,
                       int32_t B, int32_t window, void* Xg, void* stream) {
  if (dtype != FXB_DTYPE_F16 && dtype != FXB_DTYPE_BF16)
    return fxb::set_error(FXB_EUNSUPPORTED, "gather_windows: dtype %d (16-bit only)", dtype);
  if (F <= 0 || F % 8 != 0)
    return fxb::set_error(FXB_EINVAL, "gather_windows: F=%d must be a positive multiple of 8", F);
  if (R < 0 || B < 0 || window <= 0 || !idx || !X || !Xg)
    return fxb::set_error(FXB_EINVAL, "gather_windows: bad arguments");
  if (!fxb::aligned16(X) || !fxb::aligned16(Xg))
    return fxb::set_error(FXB_EINVAL, "gather_windows: X and Xg must be 16-byte aligned");
  if (B == 0) return FXB_OK;
  int64_t want = ((int64_t)B + 7) / 8;
  int64_t cap = (int64_t)fxb::num_sms() * 16;
  int blocks = (int)(want < cap ? want : cap);
  cudaStream_t st = fxb::as_stream(stream);
  if (dtype == FXB_DTYPE_F16)
    fxb::pdl_launch(gather_windows_kernel<__half>, blocks, 256, 0, st, static_cast<const __half*>(X), R, F, idx, B,
                                                          window, static_cast<__half*>(Xg));
  else
    fxb::pdl_launch(gather_windows_kernel<__nv_bfloat16>, blocks, 256, 0, st, 
        static_cast<const __nv_bfloat16*>(X), R, F, idx, B, window, static_cast<__nv_bfloat16*>(Xg));
  return fxb::check_launch("gather_windows");
}

int fxb_colsum(int32_t dtype, const void* g, int64_t rows, int32_t cols, float* out,
               int32_t accumulate, void* stream) {
  if (fxb::dtype_size(dtype) == 0 || rows < 0 || cols <= 0 || !g || !out)
    return fxb::set_error(FXB_EINVAL, "colsum: bad arguments");
  dim3 block(32, 8), grid((cols + 31) / 32);
  cudaStream_t st = fxb::as_stream(stream);
  switch (dtype) {
    case FXB_DTYPE_F16:
      fxb::pdl_launch(colsum_kernel<__half>, grid, block, 0, st, static_cast<const __half*>(g), rows, cols, out, accumulate);
      break;
    case FXB_DTYPE_BF16:
      fxb::pdl_launch(colsum_kernel<__nv_bfloat16>, grid, block, 0, st, static_cast<const __nv_bfloat16*>(g), rows, cols, out, accumulate);
      break;
    default:
      fxb::pdl_launch(colsum_kernel<float>, grid, block, 0, st, static_cast<const float*>(g), rows, cols, out, accumulate);
  }
  return fxb::check_launch("colsum");
}

}  // extern "C"
