// RMSNorm forward / backward for sm_100a (HBM-bound).
//
// Math follows the reference kernels ml/fxlm/kernels/norm.hip:33-59 (fwd),
// :64-95 (dx) and :102-127 (dw partials), which compute in fp32 over 16-bit
// inputs. Layout differs: one warp owns a row (one block, for long rows), the
// row lives in registers as 16-byte vectors (one HBM read of x, one write of
// y), and the dw reduction is a per-block partial followed by a fixed-order
// column sum (deterministic).
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kWarps = 8;  // warps per block

template <typename T> struct Vec {
  static constexpr int N = 16 / sizeof(T);  // elements per 16-byte vector
};

template <typename T> FXB_DEV void load_vec(const T* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    const float* q = reinterpret_cast<const float*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = q[i];
  } else {
    unpack8<T>(u, f);
  }
}
template <typename T> FXB_DEV void store_vec(T* p, const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    float* q = reinterpret_cast<float*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = f[i];
  } else {
    u = pack8<T>(f);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

// VPL = 16-byte vectors per lane (row length D <= VPL * 32 * Vec<T>::N).
// Each warp takes two rows per pass (rows r and r + the grid's warp count)
// and issues all of their loads before using any, so that enough bytes are
// in flight per SM at the step's small row counts.
template <typename T, int VPL>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                   float* __restrict__ rstd, int64_t rows, int D, float eps) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int nvec = D / E;
  float wv[VPL][E];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    int v = i * 32 + lane;
    if (v < nvec) load_vec<T>(w + (int64_t)v * E, wv[i]);
  }
  const int64_t warp0 = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  for (int64_t r0 = warp0; r0 < rows; r0 += 2 * nwarps) {
    const int64_t r1 = r0 + nwarps;
    const bool two = r1 < rows;  // warp-uniform
    float xv[2][VPL][E];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const T* xr = x + (k ? r1 : r0) * D;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        int v = i * 32 + lane;
        if (v < nvec && (k == 0 || two)) {
          load_vec<T>(xr + (int64_t)v * E, xv[k][i]);
        } else {
#pragma unroll
          for (int j = 0; j < E; ++j) xv[k][i][j] = 0.f;
        }
      }
    }
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int i = 0; i < VPL; ++i)
#pragma unroll
        for (int j = 0; j < E; ++j) ss[k] += xv[k][i][j] * xv[k][i][j];
    ss[0] = warp_sum(ss[0]);
    ss[1] = warp_sum(ss[1]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      const int64_t r = k ? r1 : r0;
      const float rs = rsqrtf(ss[k] / (float)D + eps);
      if (lane == 0) rstd[r] = rs;
      T* yr = y + r * D;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        int v = i * 32 + lane;
        if (v < nvec) {
          float o[E];
#pragma unroll
          for (int j = 0; j < E; ++j) o[j] = xv[k][i][j] * rs * wv[i][j];
          store_vec<T>(yr + (int64_t)v * E, o);
        }
      }
    }
  }
}

// dx per row + per-block dw partial (part[blockIdx.x, :]). Each warp takes
// two rows at a time and issues all of their loads (x, dy, dres) before using
// any, so that enough bytes are in flight to keep HBM busy with one block
// per SM or two.
template <typename T> FXB_DEV void unpack_vec(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    unpack8<T>(u, f);
  }
}

template <typename T, int VPL>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                   const float* __restrict__ rstd, const T* __restrict__ dy,
                   const T* __restrict__ dres, T* __restrict__ dx,
                   float* __restrict__ part, int64_t rows, int D) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = Vec<T>::N;
  extern __shared__ float sdw[];  // kWarps x D
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int nvec = D / E;
  float wv[VPL][E], acc[VPL][E];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    int v = i * 32 + lane;
#pragma unroll
    for (int j = 0; j < E; ++j) acc[i][j] = wv[i][j] = 0.f;  // lanes past D keep zeros
    if (v < nvec) load_vec<T>(w + (int64_t)v * E, wv[i]);
  }
  const float invD = 1.f / (float)D;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  const int64_t stride = (int64_t)gridDim.x * kWarps * 2;
  for (int64_t r0 = ((int64_t)blockIdx.x * kWarps + wid) * 2; r0 < rows; r0 += stride) {
    const bool two = r0 + 1 < rows;  // warp-uniform
    uint4 xp[2][VPL], gp[2][VPL], dp[2][VPL];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t r = r0 + k;
      const bool rv = k == 0 || two;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int v = i * 32 + lane;
        const bool ok = rv && v < nvec;
        xp[k][i] = ok ? *reinterpret_cast<const uint4*>(x + r * D + (int64_t)v * E) : zero;
        gp[k][i] = ok ? *reinterpret_cast<const uint4*>(dy + r * D + (int64_t)v * E) : zero;
        dp[k][i] = (ok && dres) ? *reinterpret_cast<const uint4*>(dres + r * D + (int64_t)v * E) : zero;
      }
    }
    float rs[2], t[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      rs[k] = (k == 0 || two) ? rstd[r0 + k] : 0.f;
      float tt = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        float xv[E], gv[E];
        unpack_vec<T>(xp[k][i], xv);
        unpack_vec<T>(gp[k][i], gv);
#pragma unroll
        for (int j = 0; j < E; ++j) tt += xv[j] * wv[i][j] * gv[j];
      }
      t[k] = tt;
    }
    t[0] = warp_sum(t[0]);
    t[1] = warp_sum(t[1]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      const int64_t r = r0 + k;
      const float corr = rs[k] * rs[k] * rs[k] * t[k] * invD;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int v = i * 32 + lane;
        if (v < nvec) {
          float xv[E], gv[E], dv[E], o[E];
          unpack_vec<T>(xp[k][i], xv);
          unpack_vec<T>(gp[k][i], gv);
          unpack_vec<T>(dp[k][i], dv);  // zero without a residual gradient
#pragma unroll
          for (int j = 0; j < E; ++j) {
            o[j] = rs[k] * wv[i][j] * gv[j] - xv[j] * corr + dv[j];
            acc[i][j] += xv[j] * rs[k] * gv[j];
          }
          store_vec<T>(dx + r * D + (int64_t)v * E, o);
        }
      }
    }
  }
  // fixed-order reduction of the warps' partials
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    int v = i * 32 + lane;
    if (v < nvec) {
#pragma unroll
      for (int j = 0; j < E; ++j) sdw[wid * D + v * E + j] = acc[i][j];
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += sdw[k * D + d];
    part[(int64_t)blockIdx.x * D + d] = s;
  }
}

// ---------------------------------------------------------------- long rows
// Rows longer than one warp's registers hold (the forward: more than 8
// vectors per lane, D > 2048 in 16-bit, D > 1024 in fp32; the backward, which
// keeps two rows of x, dy and dres per warp in flight: more than 4, D > 1024 /
// D > 512; up to the ABI's D <= 8192): one block
// of kRowThreads threads owns a row, each thread VPT 16-byte vectors at
// stride kRowThreads (coalesced). The row sums go through warp shuffles and a
// kWarps-slot shared array that alternates between two copies by row parity,
// so one barrier per row suffices: a warp can only overwrite a copy after
// every warp has passed the barrier of the row in between, i.e. after all of
// them finished reading it.
constexpr int kRowThreads = kWarps * 32;

FXB_DEV float block_row_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kWarps; ++k) s += red[k];  // same order in every thread
  return s;
}

template <typename T, int VPT>
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_fwd_row_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                       float* __restrict__ rstd, int64_t rows, int D, float eps) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = Vec<T>::N;
  __shared__ float red[2][kWarps];
  const int nvec = D / E;
  float wv[VPT][E];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = i * kRowThreads + threadIdx.x;
    if (v < nvec) load_vec<T>(w + (int64_t)v * E, wv[i]);
  }
  int par = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, par ^= 1) {
    const T* xr = x + r * D;
    float xv[VPT][E];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = i * kRowThreads + threadIdx.x;
      if (v < nvec) {
        load_vec<T>(xr + (int64_t)v * E, xv[i]);
#pragma unroll
        for (int j = 0; j < E; ++j) ss += xv[i][j] * xv[i][j];
      }
    }
    ss = block_row_sum(ss, red[par]);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (threadIdx.x == 0) rstd[r] = rs;
    T* yr = y + r * D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = i * kRowThreads + threadIdx.x;
      if (v < nvec) {
        float o[E];
#pragma unroll
        for (int j = 0; j < E; ++j) o[j] = xv[i][j] * rs * wv[i][j];
        store_vec<T>(yr + (int64_t)v * E, o);
      }
    }
  }
}

// dx per row, as rmsnorm_bwd_kernel, and the block's dw partial kept in
// registers (each thread owns fixed columns), written once at the end.
template <typename T, int VPT>
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_bwd_row_kernel(const T* __restrict__ x, const T* __restrict__ w,
                       const float* __restrict__ rstd, const T* __restrict__ dy,
                       const T* __restrict__ dres, T* __restrict__ dx,
                       float* __restrict__ part, int64_t rows, int D) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = Vec<T>::N;
  __shared__ float red[2][kWarps];
  const int nvec = D / E;
  float wv[VPT][E], acc[VPT][E];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = i * kRowThreads + threadIdx.x;
#pragma unroll
    for (int j = 0; j < E; ++j) acc[i][j] = wv[i][j] = 0.f;
    if (v < nvec) load_vec<T>(w + (int64_t)v * E, wv[i]);
  }
  const float invD = 1.f / (float)D;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  int par = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, par ^= 1) {
    uint4 xp[VPT], gp[VPT], dp[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = i * kRowThreads + threadIdx.x;
      const bool ok = v < nvec;
      const int64_t off = r * D + (int64_t)v * E;
      xp[i] = ok ? *reinterpret_cast<const uint4*>(x + off) : zero;
      gp[i] = ok ? *reinterpret_cast<const uint4*>(dy + off) : zero;
      dp[i] = (ok && dres) ? *reinterpret_cast<const uint4*>(dres + off) : zero;
    }
    const float rs = rstd[r];
    float tt = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float xv[E], gv[E];
      unpack_vec<T>(xp[i], xv);
      unpack_vec<T>(gp[i], gv);
#pragma unroll
      for (int j = 0; j < E; ++j) tt += xv[j] * wv[i][j] * gv[j];
    }
    const float t = block_row_sum(tt, red[par]);
    const float corr = rs * rs * rs * t * invD;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = i * kRowThreads + threadIdx.x;
      if (v < nvec) {
        float xv[E], gv[E], dv[E], o[E];
        unpack_vec<T>(xp[i], xv);
        unpack_vec<T>(gp[i], gv);
        unpack_vec<T>(dp[i], dv);  // zero without a residual gradient
#pragma unroll
        for (int j = 0; j < E; ++j) {
          o[j] = rs * wv[i][j] * gv[j] - xv[j] * corr + dv[j];
          acc[i][j] += xv[j] * rs * gv[j];
        }
        store_vec<T>(dx + r * D + (int64_t)v * E, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = i * kRowThreads + threadIdx.x;
    if (v < nvec) {
      float4* p = reinterpret_cast<float4*>(part + (int64_t)blockIdx.x * D + (int64_t)v * E);
#pragma unroll
      for (int j = 0; j < E / 4; ++j)
        p[j] = make_float4(acc[i][4 * j], acc[i][4 * j + 1], acc[i][4 * j + 2], acc[i][4 * j + 3]);
    }
  }
}

// dw[d] = (acc ? dw[d] : 0) + sum_b part[b, d]   (fixed order over b)
template <typename T>
__global__ void rmsnorm_dw_reduce_kernel(const float* __restrict__ part, int nparts, int D,
                                         T* __restrict__ dw, int accumulate) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  // block (32 columns) x (32 row groups); row group y sums partials y, y + 32,
  // ... (four loads in flight), then the 32 group sums are added in a fixed
  // order (deterministic). 32 row groups keep the chain short: the reduction
  // is latency-bound (a few hundred partials of a few KB).
  constexpr int RG = 32;
  __shared__ float grp[RG][33];
  const int d = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (d < D) {
    float s4[4] = {0.f, 0.f, 0.f, 0.f};  // four loads in flight, fixed assignment
    int b = threadIdx.y;
    for (; b + 3 * RG < nparts; b += 4 * RG)
#pragma unroll
      for (int u = 0; u < 4; ++u) s4[u] += part[(int64_t)(b + RG * u) * D + d];
    for (; b < nparts; b += RG) s4[0] += part[(int64_t)b * D + d];
    s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }
  grp[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && d < D) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < RG; ++k) t += grp[k][threadIdx.x];
    if (accumulate) t += to_f<T>(dw[d]);
    dw[d] = from_f<T>(t);
  }
}

template <typename T>
int launch_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int D, float eps,
               cudaStream_t st) {
  constexpr int E = Vec<T>::N;
  const int vpl = (D / E + 31) / 32;
  int64_t blocks64 = (rows + 2 * kWarps - 1) / (2 * kWarps);  // two rows per warp
  int cap = fxb::num_sms() * 16;
  int blocks = (int)(blocks64 < cap ? blocks64 : cap);
  if (blocks < 1) blocks = 1;
  auto X = static_cast<const T*>(x);
  auto W = static_cast<const T*>(w);
  auto Y = static_cast<T*>(y);
#define FXB_RMS_FWD(V)                                                            \
  case V:                                                                         \
    fxb::pdl_launch(rmsnorm_fwd_kernel<T, V>, blocks, kWarps * 32, 0, st, X, W, Y, rstd, rows, D, eps); \
    break;
  if (vpl > 8) {  // long rows: a block per row
    const int nvec = D / E;
    const int64_t cap = (int64_t)fxb::num_sms() * 4;
    const int rb = (int)(rows < cap ? rows : cap);
    if (nvec <= 2 * kRowThreads)
      fxb::pdl_launch(rmsnorm_fwd_row_kernel<T, 2>, rb, kRowThreads, 0, st, X, W, Y, rstd, rows, D, eps);
    else if (nvec <= 4 * kRowThreads)
      fxb::pdl_launch(rmsnorm_fwd_row_kernel<T, 4>, rb, kRowThreads, 0, st, X, W, Y, rstd, rows, D, eps);
    else if (nvec <= 8 * kRowThreads)
      fxb::pdl_launch(rmsnorm_fwd_row_kernel<T, 8>, rb, kRowThreads, 0, st, X, W, Y, rstd, rows, D, eps);
    else
      return fxb::set_error(FXB_EUNSUPPORTED, "rmsnorm: D=%d too large", D);
    return fxb::check_launch("rmsnorm_fwd_row");
  }
  switch (vpl) {
    FXB_RMS_FWD(1) FXB_RMS_FWD(2) FXB_RMS_FWD(3) FXB_RMS_FWD(4) FXB_RMS_FWD(5) FXB_RMS_FWD(6)
    FXB_RMS_FWD(7) FXB_RMS_FWD(8)
    default:
      return fxb::set_error(FXB_EUNSUPPORTED, "rmsnorm: D=%d too large", D);
  }
#undef FXB_RMS_FWD
  return fxb::check_launch("rmsnorm_fwd");
}

// rows of at most 4 vectors per lane take the warp-per-row kernels (beyond
// that their two rows in flight per warp spill registers)
template <typename T> constexpr int kWarpRowMaxD = 4 * 32 * Vec<T>::N;

// long-row backward: two blocks per SM, one row per block at a time
int row_blocks(int64_t rows) {
  const int64_t cap = (int64_t)fxb::num_sms() * 2;
  const int64_t b = rows < cap ? rows : cap;
  return b < 1 ? 1 : (int)b;
}

// The warp-row backward kernels of the wider rows hold two rows of x, dy and
// dres per warp in registers (up to ~240 per thread), so fewer blocks than
// bwd_blocks' two per SM may be resident at once. The grid is cut to the
// blocks that are resident together: one wave instead of two, and fewer dw
// partials for the column reduction (the workspace is sized for the larger
// grid, so it always suffices).
template <typename K> int resident_grid(K k, size_t smem, int blocks) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kWarps * 32, smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();  // leave no sticky error behind; keep the grid as it is
    return blocks;
  }
  const int cap = fxb::num_sms() * per_sm;
  return blocks < cap ? blocks : cap;
}

int bwd_blocks(int64_t rows) {
  // two blocks per SM, each warp two rows per pass with all their loads in
  // flight: enough bytes outstanding for HBM, and few dw partials to reduce
  int64_t want = (rows + kWarps * 2 - 1) / (kWarps * 2);
  int cap = fxb::num_sms() * 2;
  int b = (int)(want < cap ? want : cap);
  return b < 1 ? 1 : b;
}

template <typename T>
int launch_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres,
               void* dx, void* dw,
               int dw_dtype, int acc, float* ws, int64_t rows, int D, cudaStream_t st) {
  constexpr int E = Vec<T>::N;
  const int vpl = (D / E + 31) / 32;
  const bool long_rows = D > kWarpRowMaxD<T>;
  int blocks = long_rows ? row_blocks(rows) : bwd_blocks(rows);
  const size_t smem = (size_t)kWarps * D * sizeof(float);
  auto X = static_cast<const T*>(x);
  auto W = static_cast<const T*>(w);
  auto G = static_cast<const T*>(dy);
  auto DX = static_cast<T*>(dx);
#define FXB_RMS_BWD(V)                                                                   \
  case V: {                                                                              \
    auto k = rmsnorm_bwd_kernel<T, V>;                                                   \
    if (smem > 48 * 1024)                                                                \
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
    blocks = resident_grid(k, smem, blocks);                                             \
    fxb::pdl_launch(k, blocks, kWarps * 32, smem, st, X, W, rstd, G, static_cast<const T*>(dres), DX, ws, rows, D); \
    break;                                                                               \
  }
  if (long_rows) {
    const int nvec = D / E;
    auto DR = static_cast<const T*>(dres);
    if (nvec <= kRowThreads)
      fxb::pdl_launch(rmsnorm_bwd_row_kernel<T, 1>, blocks, kRowThreads, 0, st, X, W, rstd, G, DR, DX, ws, rows, D);
    else if (nvec <= 2 * kRowThreads)
      fxb::pdl_launch(rmsnorm_bwd_row_kernel<T, 2>, blocks, kRowThreads, 0, st, X, W, rstd, G, DR, DX, ws, rows, D);
    else if (nvec <= 4 * kRowThreads)
      fxb::pdl_launch(rmsnorm_bwd_row_kernel<T, 4>, blocks, kRowThreads, 0, st, X, W, rstd, G, DR, DX, ws, rows, D);
    else if (nvec <= 8 * kRowThreads)
      fxb::pdl_launch(rmsnorm_bwd_row_kernel<T, 8>, blocks, kRowThreads, 0, st, X, W, rstd, G, DR, DX, ws, rows, D);
    else
      return fxb::set_error(FXB_EUNSUPPORTED, "rmsnorm bwd: D=%d too large", D);
  } else {
    switch (vpl) {
      FXB_RMS_BWD(1) FXB_RMS_BWD(2) FXB_RMS_BWD(3) FXB_RMS_BWD(4)
      default:
        return fxb::set_error(FXB_EUNSUPPORTED, "rmsnorm bwd: D=%d not supported", D);
    }
  }
#undef FXB_RMS_BWD
  int r = fxb::check_launch("rmsnorm_bwd");
  if (r) return r;
  const dim3 g((D + 31) / 32), blk(32, 32);
  switch (dw_dtype) {
    case FXB_DTYPE_BF16:
      fxb::pdl_launch(rmsnorm_dw_reduce_kernel<__nv_bfloat16>, g, blk, 0, st, ws, blocks, D, static_cast<__nv_bfloat16*>(dw), acc);
      break;
    case FXB_DTYPE_F16:
      fxb::pdl_launch(rmsnorm_dw_reduce_kernel<__half>, g, blk, 0, st, ws, blocks, D, static_cast<__half*>(dw), acc);
      break;
    default:
      fxb::pdl_launch(rmsnorm_dw_reduce_kernel<float>, g, blk, 0, st, ws, blocks, D, static_cast<float*>(dw), acc);
  }
  return fxb::check_launch("rmsnorm_dw_reduce");
}

// ---------------------------------------------------------------- static scratch
// fxb_rmsnorm_bwd_static keeps its dw partials in this file-scope array (one
// copy per device) instead of a caller-provided workspace. Every call on a
// device shares it. Nothing in it has to start at zero: each backward block
// writes all D of its partials before the column reduction reads them.
constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
__device__ __align__(256) float g_rms_scratch[kStaticScratchBytes / sizeof(float)];

std::mutex g_scratch_mu;
float* g_scratch_ptr[64] = {nullptr};
uintptr_t g_scratch_ctx[64] = {0};

// Address of g_rms_scratch on the current device; looked up on the first call
// on a device (and again if that device's context was replaced, e.g. after a
// cudaDeviceReset), never allocated.
int static_scratch(float** out) {
  int dev = 0;
  int r = fxb::check_cuda(cudaGetDevice(&dev), "rmsnorm bwd static: cudaGetDevice");
  if (r) return r;
  if (dev < 0 || dev >= 64)
    return fxb::set_error(FXB_EUNSUPPORTED, "rmsnorm bwd static: device ordinal %d >= 64", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const uintptr_t ctx = fxb::context_token();
  if (!g_scratch_ptr[dev] || ctx == 0 || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    r = fxb::check_cuda(cudaGetSymbolAddress(&p, g_rms_scratch),
                        "rmsnorm bwd static: cudaGetSymbolAddress(scratch)");
    if (r) return r;
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_scratch_ctx[dev] = fxb::context_token();
  }
  *out = g_scratch_ptr[dev];
  return FXB_OK;
}

int check_common(int32_t dtype, const void* x, const void* w, int64_t rows, int32_t D) {
  if (fxb::dtype_size(dtype) == 0) return fxb::set_error(FXB_EINVAL, "rmsnorm: bad dtype %d", dtype);
  if (D <= 0 || D % 8 != 0 || D > 8192)
    return fxb::set_error(FXB_EINVAL, "rmsnorm: D=%d needs D %% 8 == 0 and D <= 8192", D);
  if (rows < 0) return fxb::set_error(FXB_EINVAL, "rmsnorm: rows=%lld", (long long)rows);
  if (!fxb::aligned16(x) || !fxb::aligned16(w))
    return fxb::set_error(FXB_EINVAL, "rmsnorm: x and w must be 16-byte aligned");
  return FXB_OK;
}

}  // namespace

extern "C" {

int fxb_rmsnorm_fwd(int32_t dtype, const void* x, const void* w, void* y, float* rstd,
                    int64_t rows, int32_t D, float eps, void* stream) {
  int r = check_common(dtype, x, w, rows, D);
  if (r) return r;
  if (!fxb::aligned16(y)) return fxb::set_error(FXB_EINVAL, "rmsnorm: y must be 16-byte aligned");
  if (rows == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  switch (dtype) {
    case FXB_DTYPE_BF16: return launch_fwd<__nv_bfloat16>(x, w, y, rstd, rows, D, eps, st);
    case FXB_DTYPE_F16: return launch_fwd<__half>(x, w, y, rstd, rows, D, eps, st);
    default: return launch_fwd<float>(x, w, y, rstd, rows, D, eps, st);
  }
}

size_t fxb_rmsnorm_bwd_workspace(int64_t rows, int32_t D) {
  // the dtype is not an argument: rows longer than fp32's warp-row limit may
  // take either kernel, so size for the larger (long-row) grid
  const int blocks = D > kWarpRowMaxD<float> ? row_blocks(rows) : bwd_blocks(rows);
  return (size_t)blocks * (size_t)(D > 0 ? D : 0) * sizeof(float);
}

int fxb_rmsnorm_bwd(int32_t dtype, const void* x, const void* w, const float* rstd,
                    const void* dy, const void* dres, void* dx, void* dw, int32_t dw_dtype,
                    int32_t dw_accumulate,
                    float* workspace, int64_t rows, int32_t D, void* stream) {
  int r = check_common(dtype, x, w, rows, D);
  if (r) return r;
  if (fxb::dtype_size(dw_dtype) == 0) return fxb::set_error(FXB_EINVAL, "rmsnorm bwd: bad dw dtype");
  if (!fxb::aligned16(dy) || !fxb::aligned16(dx) || (dres && !fxb::aligned16(dres)))
    return fxb::set_error(FXB_EINVAL, "rmsnorm bwd: dy, dres and dx must be 16-byte aligned");
  if (!workspace || !dw) return fxb::set_error(FXB_EINVAL, "rmsnorm bwd: workspace/dw NULL");
  cudaStream_t st = fxb::as_stream(stream);
  if (rows == 0) {
    if (dw_accumulate) return FXB_OK;
    return fxb::check_cuda(cudaMemsetAsync(dw, 0, (size_t)D * fxb::dtype_size(dw_dtype), st),
                           "rmsnorm bwd memset");
  }
  switch (dtype) {
    case FXB_DTYPE_BF16:
      return launch_bwd<__nv_bfloat16>(x, w, rstd, dy, dres, dx, dw, dw_dtype, dw_accumulate, workspace, rows, D, st);
    case FXB_DTYPE_F16:
      return launch_bwd<__half>(x, w, rstd, dy, dres, dx, dw, dw_dtype, dw_accumulate, workspace, rows, D, st);
    default:
      return launch_bwd<float>(x, w, rstd, dy, dres, dx, dw, dw_dtype, dw_accumulate, workspace, rows, D, st);
  }
}

size_t fxb_rmsnorm_bwd_static_max_bytes(void) { return kStaticScratchBytes; }

int fxb_rmsnorm_bwd_static(int32_t dtype, const void* x, const void* w, const float* rstd,
                           const void* dy, const void* dres, void* dx, void* dw,
                           int32_t dw_dtype, int32_t dw_accumulate, int64_t rows, int32_t D,
                           void* stream) {
  int r = check_common(dtype, x, w, rows, D);
  if (r) return r;
  const size_t need = fxb_rmsnorm_bwd_workspace(rows, D);
  if (need > kStaticScratchBytes)
    return fxb::set_error(FXB_EINVAL,
                          "rmsnorm bwd static: rows=%lld D=%d need %zu bytes of scratch, the "
                          "static array holds %zu; use fxb_rmsnorm_bwd with a workspace",
                          (long long)rows, D, need, kStaticScratchBytes);
  float* scratch = nullptr;
  r = static_scratch(&scratch);
  if (r) return r;
  return fxb_rmsnorm_bwd(dtype, x, w, rstd, dy, dres, dx, dw, dw_dtype, dw_accumulate, scratch,
                         rows, D, stream);
}

}  // extern "C"
