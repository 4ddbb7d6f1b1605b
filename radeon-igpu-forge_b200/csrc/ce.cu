// Fused softmax cross-entropy forward + gradient for sm_100a (HBM-bound).
//
// Semantics follow ce_fwd_grad (ml/fxlm/kernels/ce.hip:32-116): per row,
// logsumexp in fp32, row loss lse - x[target] for valid rows (the reference
// atomically adds it into one scalar, ce.hip:89-92; here each row's loss is
// stored and the caller sums them in a fixed order, so the result does not
// depend on scheduling), grad = (softmax - onehot) * (*mul), zero for rows
// whose target is ignore_index or out of [0, V) (ce.hip:43,97-115). The B200 layout keeps
// the whole row in registers (16-byte vectors), so logits are read from HBM
// once and the gradient written once; the gradient may overwrite the logits.
#include "common.cuh"
#include "internal.h"

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T> struct CEVec { static constexpr int N = 16 / sizeof(T); };

template <typename T> FXB_DEV void ld_vec(const T* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    const float* q = reinterpret_cast<const float*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = q[i];
  } else {
    unpack8<T>(u, f);
  }
}
template <typename T> FXB_DEV void st_vec(T* p, const float* f) {
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

// 16-byte vector v of a row staged in shared memory, as floats / from floats
template <typename T> FXB_DEV void unpack_row(const uint8_t* row, int v, float* f) {
  const uint4 u = reinterpret_cast<const uint4*>(row)[v];
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    unpack8<T>(u, f);
  }
}
template <typename T> FXB_DEV void pack_row(uint8_t* row, int v, const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                   __float_as_uint(f[3]));
  } else {
    u = pack8<T>(f);
  }
  reinterpret_cast<uint4*>(row)[v] = u;
}

// Block-wide (or warp-wide when NT == 32) max and sum.
template <int NT> FXB_DEV float block_max(float v, float* red) {
  v = warp_max(v);
  if constexpr (NT == 32) return v;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < NT / 32) ? red[lane] : -INFINITY;
  return warp_max(r);
}
template <int NT> FXB_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  if constexpr (NT == 32) return v;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < NT / 32) ? red[lane] : 0.f;
  return warp_sum(r);
}

// NT threads per row (32 = warp per row, else block per row); VPT vectors per
// thread cache the row. Rows handled grid-stride.
template <typename T, int NT, int VPT>
__global__ void __launch_bounds__(NT == 32 ? 256 : NT)
ce_cached_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ target,
                 T* grad, float* __restrict__ row_loss, const float* __restrict__ mul,
                 int64_t rows, int V, int64_t ignore_index) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  constexpr int E = CEVec<T>::N;
  __shared__ float red[32];
  const int nvec = V / E;
  const int tid = (NT == 32) ? (threadIdx.x & 31) : threadIdx.x;
  const int64_t group = (NT == 32) ? ((int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5))
                                   : (int64_t)blockIdx.x;
  const int64_t ngroups = (NT == 32) ? ((int64_t)gridDim.x * (blockDim.x / 32)) : (int64_t)gridDim.x;
  const float gm = grad ? *mul : 0.f;
  for (int64_t r = group; r < rows; r += ngroups) {
    const T* row = logits + r * ld;
    float xv[VPT][E];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int v = i * NT + tid;
      if (v < nvec) {
        ld_vec<T>(row + (int64_t)v * E, xv[i]);
#pragma unroll
        for (int j = 0; j < E; ++j) mx = fmaxf(mx, xv[i][j]);
      }
    }
    mx = block_max<NT>(mx, red);
    const float mxl = mx * kLog2e;
    const int64_t t = target[r];
    const bool valid = (t != ignore_index) && (t >= 0) && (t < (int64_t)V);
    float s = 0.f, xt = 0.f;
    bool owner = false;  // this thread holds column t in its registers
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int v = i * NT + tid;
      if (v < nvec) {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if ((int64_t)(v * E + j) == t) { xt = xv[i][j]; owner = true; }
          xv[i][j] = exp2f(fmaf(xv[i][j], kLog2e, -mxl));  // now holds exp(x - max)
          s += xv[i][j];
        }
      }
    }
    s = block_sum<NT>(s, red);
    // the logit of the target comes from registers: with grad == logits the
    // row in memory is being overwritten by other threads below
    if (valid && owner) row_loss[r] = mx + log2f(s) * kLn2 - xt;
    if (!valid && tid == 0) row_loss[r] = 0.f;
    if (grad) {
      const float scale = valid ? gm / s : 0.f;
      const float sub = valid ? gm : 0.f;
      T* grow = grad + r * ld;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        int v = i * NT + tid;
        if (v < nvec) {
          float o[E];
#pragma unroll
          for (int j = 0; j < E; ++j) {
            o[j] = xv[i][j] * scale;
            if ((int64_t)(v * E + j) == t) o[j] -= sub;
          }
          st_vec<T>(grow + (int64_t)v * E, o);
        }
      }
    }
    if constexpr (NT != 32) __syncthreads();  // red[] reuse across rows
  }
}

// Rows of up to kSmemRowMax bytes (V = 32768 in 16-bit is 64 KB): the row is
// brought into shared memory by one bulk asynchronous copy, three passes run
// out of shared memory (the row maximum; exp(x - max) once per element, summed
// and, with a gradient, kept in place; the gradient scaled in place), and one
// bulk copy stores the gradient row. One exponential per element keeps the
// special-function pipe at half the load of an online max / sum followed by
// a second exponential pass. (With a gradient the kept exp(x - max) is
// rounded to the row type before it is scaled.) Three blocks per SM keep
// loads, arithmetic and stores of different rows overlapped; the logits are
// read from HBM once and the gradient written once.
constexpr int kSmemRowMax = 72 * 1024;
constexpr int kSmemThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kSmemThreads)
ce_smem_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ target,
               T* grad, float* __restrict__ row_loss, const float* __restrict__ mul,
               int64_t rows, int V, int64_t ignore_index, int* err) {
  constexpr int E = CEVec<T>::N;
  constexpr int NW = kSmemThreads / 32;
  extern __shared__ __align__(128) uint8_t srow_raw[];
  __shared__ __align__(8) uint64_t full_bar;
  __shared__ float red_m[NW], red_s[NW];
  __shared__ float s_xt;
  const uint32_t srow = smem_u32(srow_raw);
  const uint32_t bar = smem_u32(&full_bar);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nvec = V / E;
  const uint32_t row_bytes = (uint32_t)V * sizeof(T);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const float gm = grad ? *mul : 0.f;
  uint32_t phase = 0;
  bool ok = true;
  if (tid == 0 && (int64_t)blockIdx.x < rows) {
    mbar_expect_tx(bar, row_bytes);
    bulk_load_g2s(srow, logits + (int64_t)blockIdx.x * ld, row_bytes, bar);
  }
  for (int64_t r = blockIdx.x; r < rows && ok; r += gridDim.x) {
    ok = mbar_wait(bar, phase, err, FXB_DERR_CE_WAIT);
    phase ^= 1;
    if (!ok) break;  // uniform: every thread saw the same barrier
    const int64_t t = target[r];
    const bool valid = (t != ignore_index) && (t >= 0) && (t < (int64_t)V);
    // the target logit, read before pass 2 overwrites the row
    if (tid == 0) s_xt = valid ? to_f<T>(reinterpret_cast<const T*>(srow_raw)[t]) : 0.f;
    // pass 1: row maximum (no exponentials)
    float m = -INFINITY;
    for (int v = tid; v < nvec; v += kSmemThreads) {
      float f[E];
      unpack_row<T>(srow_raw, v, f);
#pragma unroll
      for (int j = 0; j < E; ++j) m = fmaxf(m, f[j]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red_m[wid] = m;
    __syncthreads();
    float M = red_m[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, red_m[w]);
    // pass 2: one exp2 per element; its sum, and (with a gradient) the value
    // exp(x - M) kept in place for pass 3
    const float Ml = (M == -INFINITY) ? 0.f : M * kLog2e;  // all -inf: every term is 0
    float s = 0.f;
    for (int v = tid; v < nvec; v += kSmemThreads) {
      float f[E];
      unpack_row<T>(srow_raw, v, f);
      float e4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < E; ++j) {
        f[j] = exp2f(fmaf(f[j], kLog2e, -Ml));
        e4[j & 3] += f[j];
      }
      s += (e4[0] + e4[1]) + (e4[2] + e4[3]);
      if (grad) pack_row<T>(srow_raw, v, f);
    }
    s = warp_sum(s);
    if (lane == 0) red_s[wid] = s;
    __syncthreads();
    float S = red_s[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) S += red_s[w];
    const float xt = s_xt;
    if (tid == 0) row_loss[r] = valid ? M + log2f(S) * kLn2 - xt : 0.f;
    if (grad) {
      // pass 3: gradient in place in shared memory, then one bulk store
      const float scale = valid ? gm / S : 0.f;
      for (int v = tid; v < nvec; v += kSmemThreads) {
        float f[E];
        unpack_row<T>(srow_raw, v, f);
#pragma unroll
        for (int j = 0; j < E; ++j) {
          f[j] *= scale;
          if ((int64_t)(v * E + j) == t && valid) f[j] -= gm;
        }
        pack_row<T>(srow_raw, v, f);
      }
      fence_proxy_async_smem();
    }
    __syncthreads();  // row consumed (and the gradient staged)
    if (tid == 0) {
      if (grad) {
        bulk_store_s2g(grad + r * ld, srow, row_bytes);
        bulk_commit();
        bulk_wait_read0();  // the buffer is free once the store has read it
      }
      const int64_t rn = r + gridDim.x;
      if (rn < rows) {
        mbar_expect_tx(bar, row_bytes);
        bulk_load_g2s(srow, logits + rn * ld, row_bytes, bar);
      }
    }
  }
  if (tid == 0) bulk_wait_all0();
}

// Generic path (any V, any alignment): block per row, three streaming passes.
template <typename T>
__global__ void __launch_bounds__(256)
ce_generic_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ target,
                  T* grad, float* __restrict__ row_loss, const float* __restrict__ mul,
                  int64_t rows, int V, int64_t ignore_index) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  __shared__ float red[32];
  const float gm = grad ? *mul : 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = logits + r * ld;
    float mx = -INFINITY;
    for (int d = threadIdx.x; d < V; d += 256) mx = fmaxf(mx, to_f<T>(row[d]));
    const int64_t t = target[r];
    const bool valid = (t != ignore_index) && (t >= 0) && (t < (int64_t)V);
    // read before the barrier inside block_sum: later passes may overwrite the row
    const float xt = (valid && threadIdx.x == 0) ? to_f<T>(row[t]) : 0.f;
    mx = block_max<256>(mx, red);
    const float mxl = mx * kLog2e;
    float s = 0.f;
    for (int d = threadIdx.x; d < V; d += 256) s += exp2f(fmaf(to_f<T>(row[d]), kLog2e, -mxl));
    s = block_sum<256>(s, red);
    if (threadIdx.x == 0) row_loss[r] = valid ? mx + log2f(s) * kLn2 - xt : 0.f;
    if (grad) {
      const float scale = valid ? gm / s : 0.f;
      T* grow = grad + r * ld;
      for (int d = threadIdx.x; d < V; d += 256) {
        float p = exp2f(fmaf(to_f<T>(row[d]), kLog2e, -mxl)) * scale;
        if (valid && d == t) p -= gm;
        grow[d] = from_f<T>(p);
      }
    }
    __syncthreads();
  }
}

template <typename T>
int launch_ce(const void* lg, int64_t ld, const int64_t* tg, void* gr, float* loss,
              const float* mul, int64_t rows, int V, int64_t ign, cudaStream_t st) {
  constexpr int E = CEVec<T>::N;
  auto L = static_cast<const T*>(lg);
  auto G = static_cast<T*>(gr);
  const int sms = fxb::num_sms();
  const bool vec_ok = (V % E == 0) && (ld % E == 0) && fxb::aligned16(lg) && (!gr || fxb::aligned16(gr));
  const int nvec = V / E;
  if (vec_ok && nvec <= 32 * 8) {
    // warp per row, 8 rows per block
    int vpt = (nvec + 31) / 32;
    int64_t want = (rows + 7) / 8;
    int blocks = (int)(want < (int64_t)sms * 32 ? want : (int64_t)sms * 32);
#define FXB_CE_W(VP) case VP: fxb::pdl_launch(ce_cached_kernel<T, 32, VP>, blocks, 256, 0, st, L, ld, tg, G, loss, mul, rows, V, ign); break;
    switch (vpt) { FXB_CE_W(1) FXB_CE_W(2) FXB_CE_W(3) FXB_CE_W(4) FXB_CE_W(5) FXB_CE_W(6) FXB_CE_W(7) FXB_CE_W(8) }
#undef FXB_CE_W
    return fxb::check_launch("ce_fwd_grad(warp)");
  }
  const size_t row_bytes = (size_t)V * sizeof(T);
  if (vec_ok && row_bytes > 32 * 1024 && row_bytes <= (size_t)kSmemRowMax && (ld * sizeof(T)) % 16 == 0) {
    int* err = fxb::dev_error_ptr();
    if (!err) return FXB_ECUDA;
    auto k = ce_smem_kernel<T>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      int r = fxb::check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   kSmemRowMax), "ce smem attribute");
      if (r) return r;
      attr_set[dev] = true;
    }
    int blocks = (int)(rows < (int64_t)sms * 3 ? rows : (int64_t)sms * 3);
    fxb::pdl_launch(k, blocks, kSmemThreads, row_bytes, st, L, ld, tg, G, loss, mul, rows, V, ign, err);
    return fxb::check_launch("ce_fwd_grad(smem)");
  }
  if (vec_ok && nvec <= 512 * 16) {
    int vpt = (nvec + 511) / 512;
    int blocks = (int)(rows < (int64_t)sms * 8 ? rows : (int64_t)sms * 8);
#define FXB_CE_B(VP) case VP: fxb::pdl_launch(ce_cached_kernel<T, 512, VP>, blocks, 512, 0, st, L, ld, tg, G, loss, mul, rows, V, ign); break;
    switch (vpt) {
      FXB_CE_B(1) FXB_CE_B(2) FXB_CE_B(3) FXB_CE_B(4) FXB_CE_B(5) FXB_CE_B(6) FXB_CE_B(7) FXB_CE_B(8)
      default:
        if (vpt <= 12) { fxb::pdl_launch(ce_cached_kernel<T, 512, 12>, blocks, 512, 0, st, L, ld, tg, G, loss, mul, rows, V, ign); }
        else { fxb::pdl_launch(ce_cached_kernel<T, 512, 16>, blocks, 512, 0, st, L, ld, tg, G, loss, mul, rows, V, ign); }
    }
#undef FXB_CE_B
    return fxb::check_launch("ce_fwd_grad(block)");
  }
  int blocks = (int)(rows < (int64_t)sms * 8 ? rows : (int64_t)sms * 8);
  fxb::pdl_launch(ce_generic_kernel<T>, blocks, 256, 0, st, L, ld, tg, G, loss, mul, rows, V, ign);
  return fxb::check_launch("ce_fwd_grad(generic)");
}

}  // namespace

extern "C" int fxb_ce_fwd_grad(int32_t dtype, const void* logits, int64_t ld,
                               const int64_t* target, void* grad, float* row_loss,
                               const float* mul, int64_t rows, int32_t V, int64_t ignore_index,
                               void* stream) {
  if (fxb::dtype_size(dtype) == 0) return fxb::set_error(FXB_EINVAL, "ce: bad dtype %d", dtype);
  if (V <= 0 || rows < 0 || ld < V)
    return fxb::set_error(FXB_EINVAL, "ce: bad shape rows=%lld V=%d ld=%lld", (long long)rows, V,
                          (long long)ld);
  if (!logits || !target || !row_loss || (grad && !mul))
    return fxb::set_error(FXB_EINVAL, "ce: NULL pointer");
  if (rows == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  switch (dtype) {
    case FXB_DTYPE_BF16:
      return launch_ce<__nv_bfloat16>(logits, ld, target, grad, row_loss, mul, rows, V, ignore_index, st);
    case FXB_DTYPE_F16:
      return launch_ce<__half>(logits, ld, target, grad, row_loss, mul, rows, V, ignore_index, st);
    default:
      return launch_ce<float>(logits, ld, target, grad, row_loss, mul, rows, V, ignore_index, st);
  }
}
