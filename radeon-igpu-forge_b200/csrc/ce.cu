// Fused softmax cross-entropy forward + gradient for sm_100a (HBM-bound).
//
// Semantics follow ce_fwd_grad (ml/fxlm/kernels/ce.hip:32-116): per row,
// logsumexp in fp32, row loss lse - x[target] for valid rows (the reference
// atomically adds it into one scalar, ce.hip:89-92; here each row's loss is
// stored and the caller sums them in a fixed order, so the result does not
// depend on scheduling), grad = (softmax - onehot) * (*mul), zero for rows
// whose target is ignore_index or out of [0, V) (ce.hip:43,97-115). The B200
// layout keeps a row in registers (16-byte vectors) up to 8K-16K columns, or in
// a ring of shared-memory row buffers (32-72 KB rows, V = 32768 in 16-bit), so
// logits are read from HBM once and the gradient written once; the gradient
// may overwrite the logits.
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

// Rows of up to kSmemRowMax bytes (V = 32768 in 16-bit is 64 KB) go through
// a ring of three row buffers in shared memory, one persistent block per SM
// (rows blockIdx.x, blockIdx.x + gridDim.x, ...). A producer warp keeps the
// ring moving with bulk asynchronous copies: it stores each finished gradient
// row and, once that store has read its buffer, loads the row three places
// further into it. So while the 16 compute warps work on row k, the gradient
// of row k-1 drains and rows k+1 and k+2 are loaded or loading: HBM sees a
// steady stream of reads and writes instead of each row's load, arithmetic
// and store in turn. Per row, each compute thread works on its own 16-byte
// vectors:
//  - pass A: its maximum m_t (16-bit rows: paired max on the packed halves,
//    exact), then exp(x - m_t) once per element, summed, and with a gradient
//    kept in place (rounded to the row type);
//  - one barrier of the compute warps combines the (m_t, sum) pairs into the
//    row's maximum M and S = sum exp(x - M) (each warp combines the per-warp
//    pairs itself, in the same order, so every thread holds the same M, S);
//  - pass B (with a gradient): grad = kept * (mul / S) * exp(m_t - M), and
//    minus mul at the target.
// The logits are read from HBM once and the gradient written once (in place
// allowed). Exponentials: ex2.approx for 16-bit rows (rounded to 8 or 11
// bits afterwards), exp2f for fp32 rows.
constexpr int kSmemRowMax = 72 * 1024;
constexpr int kRingCompute = 512;  // compute threads (warps 0-15)
constexpr int kRingWarps = kRingCompute / 32;
constexpr int kRingThreads = kRingCompute + 32;  // + the producer warp
constexpr int kRingBufs = 3;

// running maximum over the 16-byte vectors of a thread (16-bit rows: paired
// max on the packed halves)
template <typename T> struct RowMax {
  uint32_t p = std::is_same<T, __half>::value ? 0xfc00fc00u : 0xff80ff80u;  // a pair of -inf
  float f = -INFINITY;
  FXB_DEV void max2(uint32_t w) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) asm("max.bf16x2 %0, %0, %1;" : "+r"(p) : "r"(w));
    else asm("max.f16x2 %0, %0, %1;" : "+r"(p) : "r"(w));
  }
  FXB_DEV void add(const uint4& u) {
    if constexpr (sizeof(T) == 2) {
      max2(u.x); max2(u.y); max2(u.z); max2(u.w);
    } else {
      f = fmaxf(fmaxf(f, __uint_as_float(u.x)),
                fmaxf(__uint_as_float(u.y), fmaxf(__uint_as_float(u.z), __uint_as_float(u.w))));
    }
  }
  FXB_DEV float get() const {
    if constexpr (sizeof(T) == 2) {
      const float2 v = unpack2<T>(p);
      return fmaxf(v.x, v.y);
    } else {
      return f;
    }
  }
};

template <typename T> FXB_DEV float ce_exp2(float x) {
  if constexpr (sizeof(T) == 2) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
  } else {
    return exp2f(x);
  }
}

// barrier of the compute warps (named barrier 1) that also ANDs a predicate
FXB_DEV bool compute_bar_and(bool v) {
  int r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\t"
               "selp.s32 %0, 1, 0, q;\n\t}"
               : "=r"(r) : "r"((int)v), "n"(kRingCompute) : "memory");
  return r != 0;
}

template <typename T>
__global__ void __launch_bounds__(kRingThreads, 1)
ce_ring_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ target,
               T* grad, float* __restrict__ row_loss, const float* __restrict__ mul,
               int64_t rows, int V, int64_t ignore_index, uint32_t buf_bytes, int* err) {
  constexpr int E = CEVec<T>::N;
  extern __shared__ __align__(128) uint8_t ring_raw[];
  __shared__ __align__(8) uint64_t full_bar[kRingBufs], done_bar[kRingBufs];
  __shared__ float red_m[kRingWarps], red_s[kRingWarps];
  __shared__ float s_xt;
  const uint32_t ring = smem_u32(ring_raw);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nvec = V / E;
  const uint32_t row_bytes = (uint32_t)V * sizeof(T);
  const int64_t r0 = blockIdx.x, G = gridDim.x;
  const int64_t nk = (rows - r0 + G - 1) / G;  // rows of this block (>= 1)
  if (tid == 0) {
    for (int i = 0; i < kRingBufs; ++i) {
      mbar_init(smem_u32(&full_bar[i]), 1);  // the row's bulk load landed
      mbar_init(smem_u32(&done_bar[i]), 1);  // the compute warps are done with the row
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream

  if (wid == kRingWarps) {
    // ------------------------------------------------ producer (lane 0)
    if (lane == 0) {
      auto load = [&](int64_t u) {
        const uint32_t bar = smem_u32(&full_bar[u % kRingBufs]);
        mbar_expect_tx(bar, row_bytes);
        bulk_load_g2s(ring + (uint32_t)(u % kRingBufs) * buf_bytes, logits + (r0 + u * G) * ld, row_bytes, bar);
      };
      int64_t loaded = 0;
      for (; loaded < kRingBufs && loaded < nk; ++loaded) load(loaded);
      for (int64_t u = 0; u < nk; ++u) {
        const int b = (int)(u % kRingBufs);
        if (!mbar_wait(smem_u32(&done_bar[b]), (uint32_t)((u / kRingBufs) & 1), err, FXB_DERR_CE_WAIT)) break;
        if (grad) {
          bulk_store_s2g(grad + (r0 + u * G) * ld, ring + (uint32_t)b * buf_bytes, row_bytes);
          bulk_commit();
        }
        if (loaded < nk) {
          if (grad) bulk_wait_read0();  // the store has read the buffer that the next load fills
          load(loaded++);
        }
      }
      // every load issued has landed (after an expired wait too) and every
      // store has completed before shared memory goes away
      for (int64_t u = loaded > kRingBufs ? loaded - kRingBufs : 0; u < loaded; ++u)
        mbar_wait(smem_u32(&full_bar[u % kRingBufs]), (uint32_t)((u / kRingBufs) & 1), err, FXB_DERR_CE_WAIT);
      bulk_wait_all0();
    }
    __syncwarp();
    return;
  }

  // ------------------------------------------------ compute warps 0-15
  const float gm = grad ? *mul : 0.f;
  int64_t t_next = target[r0];
  for (int64_t k = 0; k < nk; ++k) {
    const int64_t r = r0 + k * G;
    const int b = (int)(k % kRingBufs);
    uint8_t* srow = ring_raw + b * buf_bytes;
    const int64_t t = t_next;
    if (k + 1 < nk) t_next = target[r + G];  // one row ahead
    const bool got = mbar_wait(smem_u32(&full_bar[b]), (uint32_t)((k / kRingBufs) & 1), err, FXB_DERR_CE_WAIT);
    if (!compute_bar_and(got)) break;
    const bool valid = (t != ignore_index) && (t >= 0) && (t < (int64_t)V);
    const int tv = valid ? (int)(t / E) : -1;  // the vector holding the target
    const int tj = valid ? (int)(t - (int64_t)tv * E) : 0;
    // pass A
    RowMax<T> rm;
    for (int v = tid; v < nvec; v += kRingCompute) rm.add(reinterpret_cast<const uint4*>(srow)[v]);
    const float m_t = rm.get();
    const float ml = (m_t == -INFINITY) ? 0.f : m_t * kLog2e;  // all -inf: every term is 0
    float s_t = 0.f;
    for (int v = tid; v < nvec; v += kRingCompute) {
      float f[E];
      unpack_row<T>(srow, v, f);
      if (v == tv) {
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (j == tj) s_xt = f[j];  // the target logit, before it is overwritten
      }
      float e4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < E; ++j) {
        f[j] = ce_exp2<T>(fmaf(f[j], kLog2e, -ml));
        e4[j & 3] += f[j];
      }
      s_t += (e4[0] + e4[1]) + (e4[2] + e4[3]);
      if (grad) pack_row<T>(srow, v, f);
    }
    // (m_t, s_t) -> per-warp pairs -> the row's M and S
    float mw = m_t;
#pragma unroll
    for (int o = 16; o; o >>= 1) mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, o));
    const float rel = (m_t == -INFINITY) ? 0.f : exp2f((m_t - mw) * kLog2e);
    const float sw = warp_sum(s_t * rel);
    if (lane == 0) {
      red_m[wid] = mw;
      red_s[wid] = sw;
    }
    named_bar_sync(1, kRingCompute);
    const float pm = lane < kRingWarps ? red_m[lane] : -INFINITY;
    const float M = warp_max(pm);
    const float S = warp_sum(pm == -INFINITY ? 0.f : red_s[lane & (kRingWarps - 1)] * exp2f((pm - M) * kLog2e));
    if (tid == 0) row_loss[r] = valid ? M + log2f(S) * kLn2 - s_xt : 0.f;
    if (grad) {
      // pass B: the gradient in place, stored by the producer
      const float sc = (valid && m_t != -INFINITY) ? gm / S * exp2f((m_t - M) * kLog2e) : 0.f;
      for (int v = tid; v < nvec; v += kRingCompute) {
        float f[E];
        unpack_row<T>(srow, v, f);
#pragma unroll
        for (int j = 0; j < E; ++j) f[j] *= sc;
        if (v == tv) {
#pragma unroll
          for (int j = 0; j < E; ++j)
            if (j == tj) f[j] -= gm;
        }
        pack_row<T>(srow, v, f);
      }
    }
    // this thread's shared-memory accesses of the row come before the
    // producer's bulk copies out of / into the buffer
    fence_proxy_async_smem();
    named_bar_sync(1, kRingCompute);  // row consumed, gradient staged, s_xt / red_* free for the next row
    if (tid == 0) mbar_arrive(smem_u32(&done_bar[b]));
  }
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
    auto k = ce_ring_kernel<T>;
    const uint32_t buf_bytes = (uint32_t)((row_bytes + 127) / 128 * 128);
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      int r = fxb::check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   kRingBufs * kSmemRowMax), "ce ring attribute");
      if (r) return r;
      attr_set[dev] = true;
    }
    int blocks = (int)(rows < (int64_t)sms ? rows : (int64_t)sms);
    fxb::pdl_launch(k, blocks, kRingThreads, (size_t)kRingBufs * buf_bytes, st, L, ld, tg, G, loss, mul, rows,
                    V, ign, buf_bytes, err);
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
