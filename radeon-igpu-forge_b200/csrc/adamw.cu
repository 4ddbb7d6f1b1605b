// FlatAdamW kernels for sm_100a (HBM-bound).
//
// Semantics follow ml/fxlm/kernels/optim.hip: adamw_sumsq (:26-75, sum of
// squared grads + non-finite flag), adamw_final (:77-93, found_inf / norm /
// clip / step), adamw_update (:96-162, decoupled weight decay on ndim>=2
// params, m/v update, bias correction with powf, fp32 master + low-precision
// copy). The reference walks a list of per-parameter gradient tensors; here
// gradients live in one flat buffer with the same offsets as the master, so
// each kernel is a single grid-stride pass over 4-element vectors, and the
// per-parameter weight-decay flag becomes a sorted segment table.
#include "common.cuh"
#include "internal.h"

namespace {

// Four consecutive elements per access (16 bytes fp32, 8 bytes 16-bit): the
// 32 lanes of a warp touch 32 consecutive 4-element units, so every warp
// instruction covers one contiguous 512 (or 256) byte span.
template <typename G> FXB_DEV void load4(const G* p, float* f) {
  if constexpr (sizeof(G) == 4) {
    float4 a = *reinterpret_cast<const float4*>(p);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  } else {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    float2 a = unpack2<G>(u.x), b = unpack2<G>(u.y);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
}
template <typename P> FXB_DEV void store4(P* p, const float* f) {
  if constexpr (sizeof(P) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack2<P>(f[0], f[1]), pack2<P>(f[2], f[3]));
  }
}

// Deterministic sum: per-block partials in a caller workspace, summed in
// block order by the block that finishes last (ticket counter), so identical
// gradients give a bitwise identical norm on every data-parallel rank.
constexpr int kSumsqMaxBlocks = 2048;
struct SumsqWs {
  float part[kSumsqMaxBlocks];
  unsigned int ticket;  // zero between calls
};

template <typename G>
__global__ void __launch_bounds__(256)
adamw_sumsq_kernel(const G* __restrict__ g, int64_t n, float* __restrict__ scratch,
                   int* __restrict__ flags, SumsqWs* __restrict__ ws) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  float ss = 0.f;
  int bad = 0;
  const int64_t nunits = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < nunits; i += 4 * stride) {  // four loads in flight
    float f[4][4];
#pragma unroll
    for (int k = 0; k < 4; ++k) load4<G>(g + (i + k * stride) * 4, f[k]);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ss += f[k][j] * f[k][j];
        bad |= !isfinite(f[k][j]);
      }
  }
  for (; i < nunits; i += stride) {
    float f[4];
    load4<G>(g + i * 4, f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ss += f[j] * f[j];
      bad |= !isfinite(f[j]);
    }
  }
  // tail (n not a multiple of 4)
  if (blockIdx.x == 0) {
    for (int64_t i = nunits * 4 + threadIdx.x; i < n; i += blockDim.x) {
      float f = to_f<G>(g[i]);
      ss += f * f;
      bad |= !isfinite(f);
    }
  }
  __shared__ float sred[8];
  __shared__ int bred[8];
  ss = warp_sum(ss);
#pragma unroll
  for (int o = 16; o; o >>= 1) bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { sred[wid] = ss; bred[wid] = bad; }
  __syncthreads();
  if (wid == 0) {
    ss = lane < 8 ? sred[lane] : 0.f;
    bad = lane < 8 ? bred[lane] : 0;
    ss = warp_sum(ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    if (lane == 0) {
      if (bad) atomicOr(flags, 1);
      if (ws == nullptr) {
        if (ss != 0.f) atomicAdd(&scratch[0], ss);
      } else {
        ws->part[blockIdx.x] = ss;
      }
    }
  }
  if (ws == nullptr) return;
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    __threadfence();  // this block's partial before its ticket
    s_last = atomicAdd(&ws->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float t = 0.f;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) t += __ldcg(&ws->part[b]);
  __shared__ float tred[8];
  t = warp_sum(t);
  if (lane == 0) tred[wid] = t;
  __syncthreads();
  if (wid == 0) {
    t = warp_sum(lane < 8 ? tred[lane] : 0.f);
    if (lane == 0) {
      scratch[0] += t;
      ws->ticket = 0u;  // ready for the next call
    }
  }
}

__global__ void adamw_final_kernel(float* scratch, int* flags, int* step, float* found_inf,
                                   float* norm_out, const float* scale, float max_norm) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int bad = (*flags != 0) || !isfinite(scratch[0]);
  *found_inf = bad ? 1.f : 0.f;
  const float norm = sqrtf(scratch[0]) / (*scale);
  *norm_out = norm;
  scratch[1] = bad ? 0.f : fminf(1.f, max_norm / (norm + 1e-6f));
  if (!bad) *step += 1;
  *flags = 0;
  scratch[0] = 0.f;
}

constexpr int kMaxSeg = 1024;

template <typename G, typename P>
__global__ void __launch_bounds__(256)
adamw_update_kernel(G* __restrict__ g, float* __restrict__ master, float* __restrict__ m,
                    float* __restrict__ v, P* __restrict__ p, int64_t n,
                    const int64_t* __restrict__ seg_end, const int* __restrict__ seg_wd, int nseg,
                    const float* __restrict__ scratch, const float* __restrict__ found_inf,
                    const float* __restrict__ scale_p, const int* __restrict__ step_p, float lr_arg,
                    const float* __restrict__ lr_dev,
                    float b1, float b2, float eps, float wd) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const int64_t nunits = n >> 2;  // n % 8 == 0
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  if (*found_inf != 0.f) {
    // step skipped: master / m / v untouched, the gradient is still consumed
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < nunits; u += stride)
      store4<G>(g + u * 4, zero4);
    return;
  }
  __shared__ int64_t s_end[kMaxSeg];
  __shared__ int s_wd[kMaxSeg];
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) {
    s_end[i] = seg_end[i];
    s_wd[i] = seg_wd[i];
  }
  __syncthreads();
  const float inv = scratch[1] / (*scale_p);  // clip coefficient / loss scale
  const int step = *step_p;
  const float bc1 = 1.f - powf(b1, (float)step);
  const float bc2 = 1.f - powf(b2, (float)step);
  const float inv_bc1 = 1.f / bc1, inv_bc2 = 1.f / bc2;
  const float b1c = 1.f - b1, b2c = 1.f - b2;
  const float lr = lr_dev ? *lr_dev : lr_arg;
  const float lrwd = lr * wd;
  // Each thread walks its units in increasing order, so the segment cursor
  // only moves forward (segment boundaries are multiples of 8 elements). Two
  // units per iteration: all eight loads are issued before any arithmetic.
  int seg = 0;
  auto wd_of = [&](int64_t e0) {
    while (seg < nseg - 1 && s_end[seg] <= e0) ++seg;
    return s_wd[seg] != 0;
  };
  auto update4 = [&](int64_t e0, bool wd_on, float* gv, float* mw, float* mv, float* vv) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gg = gv[j] * inv;
      float w = mw[j];
      if (wd_on) w -= lrwd * w;
      const float a = mv[j] * b1 + b1c * gg;
      const float b = vv[j] * b2 + b2c * gg * gg;
      mv[j] = a;
      vv[j] = b;
      w -= lr * (a * inv_bc1) / (sqrtf(b * inv_bc2) + eps);
      mw[j] = w;
    }
    store4<G>(g + e0, zero4);  // gradient consumed
    store4<float>(master + e0, mw);
    store4<float>(m + e0, mv);
    store4<float>(v + e0, vv);
    store4<P>(p + e0, mw);
  };
  int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; u + stride < nunits; u += 2 * stride) {
    const int64_t e0 = u * 4, e1 = (u + stride) * 4;
    float g0[4], w0[4], m0[4], v0[4], g1[4], w1[4], m1[4], v1[4];
    load4<G>(g + e0, g0); load4<float>(master + e0, w0); load4<float>(m + e0, m0); load4<float>(v + e0, v0);
    load4<G>(g + e1, g1); load4<float>(master + e1, w1); load4<float>(m + e1, m1); load4<float>(v + e1, v1);
    const bool wd0 = wd_of(e0);
    update4(e0, wd0, g0, w0, m0, v0);
    const bool wd1 = wd_of(e1);
    update4(e1, wd1, g1, w1, m1, v1);
  }
  if (u < nunits) {
    const int64_t e0 = u * 4;
    float g0[4], w0[4], m0[4], v0[4];
    load4<G>(g + e0, g0); load4<float>(master + e0, w0); load4<float>(m + e0, m0); load4<float>(v + e0, v0);
    update4(e0, wd_of(e0), g0, w0, m0, v0);
  }
}

template <typename G, typename P>
int launch_update(const void* g, float* master, float* m, float* v, void* p, int64_t n,
                  const int64_t* se, const int* sw, int nseg, const float* scratch,
                  const float* fi, const float* sc, const int* stp, float lr, const float* lrd,
                  float b1, float b2,
                  float eps, float wd, cudaStream_t st) {
  int64_t units = n >> 2;
  int64_t want = (units + 255) / 256;
  int64_t cap = (int64_t)fxb::num_sms() * 8;
  int blocks = (int)(want < cap ? want : cap);
  if (blocks < 1) blocks = 1;
  fxb::pdl_launch(adamw_update_kernel<G, P>, blocks, 256, 0, st, static_cast<G*>(const_cast<void*>(g)), master, m, v,
                                                    static_cast<P*>(p), n, se, sw, nseg, scratch,
                                                    fi, sc, stp, lr, lrd, b1, b2, eps, wd);
  return fxb::check_launch("adamw_update");
}

template <typename G>
int dispatch_update_p(int32_t pdtype, const void* g, float* master, float* m, float* v, void* p,
                      int64_t n, const int64_t* se, const int* sw, int nseg, const float* scratch,
                      const float* fi, const float* sc, const int* stp, float lr, const float* lrd,
                      float b1,
                      float b2, float eps, float wd, cudaStream_t st) {
  switch (pdtype) {
    case FXB_DTYPE_BF16:
      return launch_update<G, __nv_bfloat16>(g, master, m, v, p, n, se, sw, nseg, scratch, fi, sc, stp, lr, lrd, b1, b2, eps, wd, st);
    case FXB_DTYPE_F16:
      return launch_update<G, __half>(g, master, m, v, p, n, se, sw, nseg, scratch, fi, sc, stp, lr, lrd, b1, b2, eps, wd, st);
    default:
      return launch_update<G, float>(g, master, m, v, p, n, se, sw, nseg, scratch, fi, sc, stp, lr, lrd, b1, b2, eps, wd, st);
  }
}

}  // namespace

extern "C" {

static int sumsq_launch(int32_t gdtype, const void* grad, int64_t n, float* scratch, int32_t* flags,
                        SumsqWs* ws, void* stream) {
  if (fxb::dtype_size(gdtype) == 0) return fxb::set_error(FXB_EINVAL, "adamw_sumsq: bad dtype");
  if (n < 0 || !scratch || !flags) return fxb::set_error(FXB_EINVAL, "adamw_sumsq: bad args");
  if (n == 0) return FXB_OK;
  if (!fxb::aligned16(grad)) return fxb::set_error(FXB_EINVAL, "adamw_sumsq: grad not 16-byte aligned");
  cudaStream_t st = fxb::as_stream(stream);
  int64_t want = ((n >> 2) + 255) / 256;
  int64_t cap = (int64_t)fxb::num_sms() * 8;
  if (cap > kSumsqMaxBlocks) cap = kSumsqMaxBlocks;
  int blocks = (int)(want < cap ? want : cap);
  if (blocks < 1) blocks = 1;
  switch (gdtype) {
    case FXB_DTYPE_BF16:
      fxb::pdl_launch(adamw_sumsq_kernel<__nv_bfloat16>, blocks, 256, 0, st, static_cast<const __nv_bfloat16*>(grad), n, scratch, flags, ws);
      break;
    case FXB_DTYPE_F16:
      fxb::pdl_launch(adamw_sumsq_kernel<__half>, blocks, 256, 0, st, static_cast<const __half*>(grad), n, scratch, flags, ws);
      break;
    default:
      fxb::pdl_launch(adamw_sumsq_kernel<float>, blocks, 256, 0, st, static_cast<const float*>(grad), n, scratch, flags, ws);
  }
  return fxb::check_launch("adamw_sumsq");
}

int fxb_adamw_sumsq(int32_t gdtype, const void* grad, int64_t n, float* scratch, int32_t* flags,
                    void* stream) {
  return sumsq_launch(gdtype, grad, n, scratch, flags, nullptr, stream);
}

size_t fxb_adamw_sumsq_ws_bytes(void) { return sizeof(SumsqWs); }

int fxb_adamw_sumsq_det(int32_t gdtype, const void* grad, int64_t n, float* scratch,
                        int32_t* flags, void* ws, void* stream) {
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 3u))
    return fxb::set_error(FXB_EINVAL, "adamw_sumsq_det: workspace NULL or not 4-byte aligned");
  return sumsq_launch(gdtype, grad, n, scratch, flags, static_cast<SumsqWs*>(ws), stream);
}

int fxb_adamw_final(float* scratch, int32_t* flags, int32_t* step, float* found_inf,
                    float* norm_out, const float* scale, float max_norm, void* stream) {
  if (!scratch || !flags || !step || !found_inf || !norm_out || !scale)
    return fxb::set_error(FXB_EINVAL, "adamw_final: NULL pointer");
  fxb::pdl_launch(adamw_final_kernel, 1, 32, 0, fxb::as_stream(stream), scratch, flags, step, found_inf,
                                                          norm_out, scale, max_norm);
  return fxb::check_launch("adamw_final");
}

int fxb_adamw_update(int32_t gdtype, int32_t pdtype, const void* grad, float* master, float* m,
                     float* v, void* param, int64_t n, const int64_t* seg_end,
                     const int32_t* seg_wd, int32_t nseg, const float* scratch,
                     const float* found_inf, const float* scale, const int32_t* step, float lr,
                     const float* lr_dev,
                     float beta1, float beta2, float eps, float weight_decay, void* stream) {
  if (fxb::dtype_size(gdtype) == 0 || fxb::dtype_size(pdtype) == 0)
    return fxb::set_error(FXB_EINVAL, "adamw_update: bad dtype");
  if (n < 0 || (n & 7) != 0)
    return fxb::set_error(FXB_EINVAL, "adamw_update: n=%lld must be a multiple of 8", (long long)n);
  if (nseg < 1 || nseg > kMaxSeg)
    return fxb::set_error(FXB_EINVAL, "adamw_update: nseg=%d outside [1, %d]", nseg, kMaxSeg);
  if (!fxb::aligned16(grad) || !fxb::aligned16(master) || !fxb::aligned16(m) ||
      !fxb::aligned16(v) || !fxb::aligned16(param))
    return fxb::set_error(FXB_EINVAL, "adamw_update: buffers must be 16-byte aligned");
  if (!seg_end || !seg_wd || !scratch || !found_inf || !scale || !step)
    return fxb::set_error(FXB_EINVAL, "adamw_update: NULL pointer");
  if (n == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  switch (gdtype) {
    case FXB_DTYPE_BF16:
      return dispatch_update_p<__nv_bfloat16>(pdtype, grad, master, m, v, param, n, seg_end, seg_wd, nseg, scratch, found_inf, scale, step, lr, lr_dev, beta1, beta2, eps, weight_decay, st);
    case FXB_DTYPE_F16:
      return dispatch_update_p<__half>(pdtype, grad, master, m, v, param, n, seg_end, seg_wd, nseg, scratch, found_inf, scale, step, lr, lr_dev, beta1, beta2, eps, weight_decay, st);
    default:
      return dispatch_update_p<float>(pdtype, grad, master, m, v, param, n, seg_end, seg_wd, nseg, scratch, found_inf, scale, step, lr, lr_dev, beta1, beta2, eps, weight_decay, st);
  }
}

}  // extern "C"
