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

// Same sum when a row is a whole number of 16-byte vectors. A cluster of
// kColsumCluster CTAs owns a group of cv consecutive vectors (cv * E columns);
// its CTAs split the rows into equal ranges. Within a CTA, thread t reads
// vector t % cv of rows t / cv, t / cv + 256 / cv, ... (a warp reads whole
// cv * 16-byte row segments, four loads in flight), and the CTA adds its
// threads' sums over the row offsets in a fixed order into a shared partial.
// After a cluster barrier CTA 0 adds the CTAs' partials, read through
// distributed shared memory, in rank order, and writes the columns: the sum
// needs no workspace and no atomics, so it is the same on every run. cv is
// chosen so that the clusters cover the SMs with row segments of >= 32 bytes.
constexpr int kColsumCluster = 8;
constexpr int kColsumThreads = 256;

template <typename T>
__global__ void __cluster_dims__(kColsumCluster, 1, 1) __launch_bounds__(kColsumThreads)
colsum_cluster_kernel(const T* __restrict__ g, int64_t rows, int cols, int cv,
                      float* __restrict__ out, int accumulate) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = 16 / sizeof(T);
  __shared__ float part[kColsumThreads * E];  // [row offset][vector][element]
  __shared__ float cta_sum[32 * E];            // cv <= 32 vectors of E columns
  const int nvec = cols / E;
  const int rank = (int)cluster_ctarank();
  const int grp = (int)(blockIdx.x / kColsumCluster);
  const int tid = threadIdx.x;
  const int tv = tid % cv, tr = tid / cv, rstep = kColsumThreads / cv;
  const int vec = grp * cv + tv;
  const int64_t per = (rows + kColsumCluster - 1) / kColsumCluster;
  const int64_t r0 = (int64_t)rank * per;
  const int64_t r1 = r0 + per < rows ? r0 + per : rows;
  float s[E];
#pragma unroll
  for (int j = 0; j < E; ++j) s[j] = 0.f;
  if (vec < nvec) {
    const uint4* src = reinterpret_cast<const uint4*>(g) + vec;
    int64_t r = r0 + tr;
    for (; r + 3 * rstep < r1; r += 4 * rstep) {
      uint4 u[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) u[k] = src[(r + (int64_t)k * rstep) * nvec];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const T* h = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
        for (int j = 0; j < E; ++j) s[j] += to_f<T>(h[j]);
      }
    }
    for (; r < r1; r += rstep) {
      const uint4 u = src[r * nvec];
      const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < E; ++j) s[j] += to_f<T>(h[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < E; ++j) part[(tr * cv + tv) * E + j] = s[j];
  __syncthreads();
  // this CTA's sum of (vector tv, element j) over its row offsets, in order
  const int ncol = cv * E;
  if (tid < ncol) {
    float t = 0.f;
    for (int k = 0; k < rstep; ++k) t += part[k * ncol + tid];
    cta_sum[tid] = t;
  }
  cluster_sync();  // every CTA's cta_sum is written and visible to the cluster
  if (rank == 0 && tid < ncol) {
    const int c = grp * ncol + tid;
    float t = 0.f;
    const uint32_t a = smem_u32(&cta_sum[tid]);
    for (int q = 0; q < kColsumCluster; ++q) {
      float v;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(mapa_shared(a, (uint32_t)q)) : "memory");
      t += v;
    }
    if (c < cols) out[c] = accumulate ? out[c] + t : t;
  }
  cluster_sync();  // the partials stay in place until CTA 0 has read them
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
    // vectors per cluster: >= 2 (32-byte row segments), growing with the
    // width so that about 16 clusters (128 CTAs) share the columns
    const int nvec = cols / E;
    int cv = 2;
    while (cv < 32 && (nvec + cv - 1) / cv > 16) cv *= 2;
    const int clusters = (nvec + cv - 1) / cv;
    fxb::pdl_launch(colsum_cluster_kernel<T>, clusters * kColsumCluster, kColsumThreads, 0, st, g, rows,
                    cols, cv, out, accumulate);
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
