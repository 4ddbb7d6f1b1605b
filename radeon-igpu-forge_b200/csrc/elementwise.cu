// Embedding gather/scatter and the scaled-add used by the linear-CE backward.
//
// fxb_embedding_fwd/bwd implement tok_emb(idx) + pos_emb[:T] and its backward
// (ml/fxlm/model.py:118); fxb_axpy carries the rescale that
// _LinearCE.backward applies to the gradients it computed in forward
// (ml/fxlm/cross_entropy.py:140-149).
#include "common.cuh"
#include "internal.h"

namespace {

// fp32 vector reduction into global memory (four consecutive floats)
FXB_DEV void red_add4(float* addr, const float* f) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(f[0]), "f"(f[1]),
               "f"(f[2]), "f"(f[3])
               : "memory");
}

template <typename T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const T* __restrict__ tok,
                                     const T* __restrict__ pos, T* __restrict__ out, int64_t rows,
                                     int64_t T_, int D, int64_t V) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  // one warp per token row, 8 elements per lane-step (D % 8 == 0)
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nw) {
    int64_t id = idx[r];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);  // out-of-range ids clamp (no fault)
    const int64_t t = r % T_;
    const T* a = tok + id * D;
    const T* b = pos + t * D;
    T* o = out + r * D;
    for (int d = lane * 8; d < D; d += 256) {
      float fa[8], fb[8];
      load8<T>(a + d, fa);
      load8<T>(b + d, fb);
#pragma unroll
      for (int j = 0; j < 8; ++j) fa[j] += fb[j];
      store8<T>(o + d, fa);
    }
  }
}

template <typename T>
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ idx, const T* __restrict__ dout,
                                     float* __restrict__ dtok, float* __restrict__ dpos,
                                     int64_t rows, int64_t T_, int D, int64_t V) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nw) {
    int64_t id = idx[r];
    const bool ok = id >= 0 && id < V;
    const int64_t t = r % T_;
    const T* g = dout + r * D;
    for (int d = lane * 8; d < D; d += 256) {
      float f[8];
      load8<T>(g + d, f);
      if (ok && dtok) {
        red_add4(dtok + id * D + d, f);
        red_add4(dtok + id * D + d + 4, f + 4);
      }
      if (dpos) {
        red_add4(dpos + t * D + d, f);
        red_add4(dpos + t * D + d + 4, f + 4);
      }
    }
  }
}

template <typename DT, typename ST>
__global__ void axpy_kernel(DT* __restrict__ dst, const ST* __restrict__ src,
                            const float* __restrict__ scale, int acc, int64_t n) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const float s = scale ? *scale : 1.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float v = to_f<ST>(src[i]) * s;
    if (acc) v += to_f<DT>(dst[i]);
    dst[i] = from_f<DT>(v);
  }
}

template <typename DT>
int axpy_src(int32_t sdt, void* dst, const void* src, const float* scale, int acc, int64_t n,
             cudaStream_t st) {
  int64_t want = (n + 255) / 256;
  int64_t cap = (int64_t)fxb::num_sms() * 16;
  int blocks = (int)(want < cap ? want : cap);
  if (blocks < 1) blocks = 1;
  DT* d = static_cast<DT*>(dst);
  switch (sdt) {
    case FXB_DTYPE_BF16:
      fxb::pdl_launch(axpy_kernel<DT, __nv_bfloat16>, blocks, 256, 0, st, d, static_cast<const __nv_bfloat16*>(src), scale, acc, n);
      break;
    case FXB_DTYPE_F16:
      fxb::pdl_launch(axpy_kernel<DT, __half>, blocks, 256, 0, st, d, static_cast<const __half*>(src), scale, acc, n);
      break;
    default:
      fxb::pdl_launch(axpy_kernel<DT, float>, blocks, 256, 0, st, d, static_cast<const float*>(src), scale, acc, n);
  }
  return fxb::check_launch("axpy");
}

int emb_blocks(int64_t rows) {
  int64_t want = (rows + 7) / 8;
  int64_t cap = (int64_t)fxb::num_sms() * 16;
  int b = (int)(want < cap ? want : cap);
  return b < 1 ? 1 : b;
}

}  // namespace

extern "C" {

int fxb_embedding_fwd(int32_t dtype, const int64_t* idx, const void* tok, const void* pos,
                      void* out, int64_t B, int64_t T, int32_t D, int64_t V, void* stream) {
  if (fxb::dtype_size(dtype) == 0)
    return fxb::set_error(FXB_EINVAL, "embedding_fwd: bad dtype %d", dtype);
  if (D <= 0 || D % 8 || B < 0 || T <= 0 || V <= 0)
    return fxb::set_error(FXB_EINVAL, "embedding_fwd: bad shape");
  if (!fxb::aligned16(tok) || !fxb::aligned16(pos) || !fxb::aligned16(out))
    return fxb::set_error(FXB_EINVAL, "embedding_fwd: buffers must be 16-byte aligned");
  const int64_t rows = B * T;
  if (rows == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  if (dtype == FXB_DTYPE_BF16)
    fxb::pdl_launch(embedding_fwd_kernel<__nv_bfloat16>, emb_blocks(rows), 256, 0, st, 
        idx, static_cast<const __nv_bfloat16*>(tok), static_cast<const __nv_bfloat16*>(pos),
        static_cast<__nv_bfloat16*>(out), rows, T, D, V);
  else if (dtype == FXB_DTYPE_F16)
    fxb::pdl_launch(embedding_fwd_kernel<__half>, emb_blocks(rows), 256, 0, st, 
        idx, static_cast<const __half*>(tok), static_cast<const __half*>(pos),
        static_cast<__half*>(out), rows, T, D, V);
  else
    fxb::pdl_launch(embedding_fwd_kernel<float>, emb_blocks(rows), 256, 0, st,
        idx, static_cast<const float*>(tok), static_cast<const float*>(pos),
        static_cast<float*>(out), rows, T, D, V);
  return fxb::check_launch("embedding_fwd");
}

int fxb_embedding_bwd(int32_t dtype, const int64_t* idx, const void* dout, float* dtok_ws,
                      float* dpos_ws, int64_t B, int64_t T, int32_t D, int64_t V, void* stream) {
  if (fxb::dtype_size(dtype) == 0)
    return fxb::set_error(FXB_EINVAL, "embedding_bwd: bad dtype %d", dtype);
  if (D <= 0 || D % 8 || B < 0 || T <= 0 || V <= 0)
    return fxb::set_error(FXB_EINVAL, "embedding_bwd: bad shape");
  if (!fxb::aligned16(dout) || (dtok_ws && !fxb::aligned16(dtok_ws)) ||
      (dpos_ws && !fxb::aligned16(dpos_ws)))
    return fxb::set_error(FXB_EINVAL, "embedding_bwd: dout / dtok_ws / dpos_ws must be 16-byte aligned");
  const int64_t rows = B * T;
  if (rows == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  if (dtype == FXB_DTYPE_BF16)
    fxb::pdl_launch(embedding_bwd_kernel<__nv_bfloat16>, emb_blocks(rows), 256, 0, st, 
        idx, static_cast<const __nv_bfloat16*>(dout), dtok_ws, dpos_ws, rows, T, D, V);
  else if (dtype == FXB_DTYPE_F16)
    fxb::pdl_launch(embedding_bwd_kernel<__half>, emb_blocks(rows), 256, 0, st, 
        idx, static_cast<const __half*>(dout), dtok_ws, dpos_ws, rows, T, D, V);
  else
    fxb::pdl_launch(embedding_bwd_kernel<float>, emb_blocks(rows), 256, 0, st,
        idx, static_cast<const float*>(dout), dtok_ws, dpos_ws, rows, T, D, V);
  return fxb::check_launch("embedding_bwd");
}

int fxb_axpy(int32_t ddtype, void* dst, int32_t sdtype, const void* src, const float* scale,
             int32_t accumulate, int64_t n, void* stream) {
  if (fxb::dtype_size(ddtype) == 0 || fxb::dtype_size(sdtype) == 0)
    return fxb::set_error(FXB_EINVAL, "axpy: bad dtype");
  if (n < 0 || !dst || !src) return fxb::set_error(FXB_EINVAL, "axpy: bad args");
  if (n == 0) return FXB_OK;
  cudaStream_t st = fxb::as_stream(stream);
  switch (ddtype) {
    case FXB_DTYPE_BF16: return axpy_src<__nv_bfloat16>(sdtype, dst, src, scale, accumulate, n, st);
    case FXB_DTYPE_F16: return axpy_src<__half>(sdtype, dst, src, scale, accumulate, n, st);
    default: return axpy_src<float>(sdtype, dst, src, scale, accumulate, n, st);
  }
}

}  // extern "C"
