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

// one warp per output row, 16-byte vectors (F % 8 == 0 => row starts aligned,
// for 16-bit and fp32 elements alike)
template <typename T>
__global__ void gather_windows_kernel(const T* __restrict__ X, int64_t R, int F,
                                      const int* __restrict__ idx, int B, int window,
                                      T* __restrict__ Xg) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const int lane = threadIdx.x & 31;
  const int64_t K = (int64_t)window * F;
  const int64_t nvec = K * (int64_t)sizeof(T) / 16;  // 16-byte vectors per window
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

// Same sum when a row is a whole number of 16-byte vectors: block b owns the
// E = 16 / sizeof(T) columns of vector b and all rows, so the sum needs no
// cross-block step (deterministic, no workspace). Thread t reads rows t,
// t + blockDim.x, ... with four 16-byte loads in flight, then the block adds
// its threads' sums in a fixed tree order (warp shuffles, then the warps'
// partials in warp order).
template <typename T>
__global__ void __launch_bounds__(1024, 1)
colsum_vec_kernel(const T* __restrict__ g, int64_t rows, int cols, float* __restrict__ out,
                  int accumulate) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = 16 / sizeof(T);
  __shared__ float part[32][E];
  const int64_t vecs_per_row = cols / E;
  const uint4* src = reinterpret_cast<const uint4*>(g) + blockIdx.x;
  float s[E];
#pragma unroll
  for (int j = 0; j < E; ++j) s[j] = 0.f;
  const int64_t step = blockDim.x;
  int64_t r = threadIdx.x;
  for (; r + 3 * step < rows; r += 4 * step) {
    uint4 u[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) u[k] = src[(r + k * step) * vecs_per_row];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const T* h = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
      for (int j = 0; j < E; ++j) s[j] += to_f<T>(h[j]);
    }
  }
  for (; r < rows; r += step) {
    const uint4 u = src[r * vecs_per_row];
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < E; ++j) s[j] += to_f<T>(h[j]);
  }
#pragma unroll
  for (int j = 0; j < E; ++j) s[j] = warp_sum(s[j]);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < E; ++j) part[wid][j] = s[j];
  }
  __syncthreads();
  if (threadIdx.x < E) {
    const int nw = (blockDim.x + 31) >> 5;
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += part[w][threadIdx.x];
    const int64_t c = (int64_t)blockIdx.x * E + threadIdx.x;
    out[c] = accumulate ? out[c] + t : t;
  }
}

// Narrow outputs (fewer columns than one 16-byte vector, e.g. the single
// output of a regression head): block c sums column c over all rows with
// eight loads in flight per thread, then the same fixed-order block sum.
template <typename T>
__global__ void __launch_bounds__(1024, 1)
colsum_col_kernel(const T* __restrict__ g, int64_t rows, int cols, float* __restrict__ out,
                  int accumulate) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  __shared__ float part[32];
  const int c = blockIdx.x;
  const int64_t step = blockDim.x;
  float s = 0.f;
  int64_t r = threadIdx.x;
  for (; r + 7 * step < rows; r += 8 * step) {
    T v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = g[(r + k * step) * cols + c];
#pragma unroll
    for (int k = 0; k < 8; ++k) s += to_f<T>(v[k]);
  }
  for (; r < rows; r += step) s += to_f<T>(g[r * cols + c]);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += part[w];
    out[c] = accumulate ? out[c] + t : t;
  }
}

template <typename T>
void launch_colsum(const T* g, int64_t rows, int cols, float* out, int accumulate, cudaStream_t st) {
  constexpr int E = 16 / sizeof(T);
  const int threads = rows >= 1024 ? 1024 : (int)((rows + 31) / 32) * 32;
  if (cols % E == 0 && fxb::aligned16(g) && rows > 0) {
    fxb::pdl_launch(colsum_vec_kernel<T>, cols / E, threads, 0, st, g, rows, cols, out, accumulate);
    return;
  }
  if (cols < E && rows > 0) {
    fxb::pdl_launch(colsum_col_kernel<T>, cols, threads, 0, st, g, rows, cols, out, accumulate);
    return;
  }
  dim3 block(32, 8), grid((cols + 31) / 32);
  fxb::pdl_launch(colsum_kernel<T>, grid, block, 0, st, g, rows, cols, out, accumulate);
}

}  // namespace

extern "C" {

int fxb_gather_windows(int32_t dtype, const void* X, int64_t R, int32_t F, const int32_t* idx,
                       int32_t B, int32_t window, void* Xg, void* stream) {
  if (fxb::dtype_size(dtype) == 0)
    return fxb::set_error(FXB_EINVAL, "gather_windows: bad dtype %d", dtype);
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
  else if (dtype == FXB_DTYPE_BF16)
    fxb::pdl_launch(gather_windows_kernel<__nv_bfloat16>, blocks, 256, 0, st, 
        static_cast<const __nv_bfloat16*>(X), R, F, idx, B, window, static_cast<__nv_bfloat16*>(Xg));
  else
    fxb::pdl_launch(gather_windows_kernel<float>, blocks, 256, 0, st,
        static_cast<const float*>(X), R, F, idx, B, window, static_cast<float*>(Xg));
  return fxb::check_launch("gather_windows");
}

int fxb_colsum(int32_t dtype, const void* g, int64_t rows, int32_t cols, float* out,
               int32_t accumulate, void* stream) {
  if (fxb::dtype_size(dtype) == 0 || rows < 0 || cols <= 0 || !out || (rows > 0 && !g))
    return fxb::set_error(FXB_EINVAL, "colsum: bad arguments");
  cudaStream_t st = fxb::as_stream(stream);
  if (rows == 0) {  // empty sum: out = 0 (or unchanged when accumulating)
    if (accumulate) return FXB_OK;
    return fxb::check_cuda(cudaMemsetAsync(out, 0, (size_t)cols * sizeof(float), st), "colsum memset");
  }
  switch (dtype) {
    case FXB_DTYPE_F16:
      launch_colsum(static_cast<const __half*>(g), rows, cols, out, accumulate, st);
      break;
    case FXB_DTYPE_BF16:
      launch_colsum(static_cast<const __nv_bfloat16*>(g), rows, cols, out, accumulate, st);
      break;
    default:
      launch_colsum(static_cast<const float*>(g), rows, cols, out, accumulate, st);
  }
  return fxb::check_launch("colsum");
}

}  // extern "C"
