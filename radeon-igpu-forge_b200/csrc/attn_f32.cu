// fp32 flash attention for the parity mode (fxb_attn_fwd / fxb_attn_bwd with
// dtype FXB_DTYPE_F32).
//
// Same semantics as the tensor-core kernels and the reference
// (ml/fxlm/kernels/attention.hip:104-534): o = softmax(q k^T * scale, causal:
// key <= query) v with the natural-log logsumexp saved per row; backward
// delta = rowsum(dO * O), P = exp(s*scale - lse), dS = P * (dP - delta),
// dV = P^T dO, dK = scale * dS^T Q, dQ = scale * dS K. Everything is fp32
// with the accurate expf / logf, for the 1e-5 fp32 parity bar that 16-bit
// tensor-core operands cannot meet. Plain SIMT: one warp per query row
// (forward, dQ) or key row (dK / dV), each lane owning DH/32 head dims, dot
// products reduced across the warp, keys (queries) walked four at a time
// with an online softmax. Accuracy, not speed, is its purpose.
#include "common.cuh"
#include "internal.h"

namespace {

struct View {  // (B, T, H, D) tensor with element strides, D contiguous
  const float* p;
  int64_t sb, st, sh;
  __device__ __forceinline__ const float* row(int b, int t, int h) const {
    return p + b * sb + (int64_t)t * st + h * sh;
  }
};
struct OutView {
  float* p;
  int64_t sb, st, sh;
  __device__ __forceinline__ float* row(int b, int t, int h) const {
    return p + b * sb + (int64_t)t * st + h * sh;
  }
};

struct F32Attn {
  int B, T, H, causal;
  float scale;
  View q, k, v, o, dout;
  OutView out, dq, dk, dv;
  float* lse;
  const float* lse_in;
  float* delta;
};

constexpr int kWarps = 8;  // warps per block

template <int E> __device__ __forceinline__ void load_row(const float* r, int lane, float* f) {
#pragma unroll
  for (int e = 0; e < E; ++e) f[e] = r[lane + 32 * e];
}
template <int E> __device__ __forceinline__ float dot_part(const float* a, const float* b) {
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) s = fmaf(a[e], b[e], s);
  return s;
}

// forward: warp per (b, h, query row)
template <int DH>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_f32_kernel(const F32Attn p) {
  pdl_trigger();
  pdl_wait();  // q / k / v come from earlier kernels on the stream
  constexpr int E = DH / 32;
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= (int64_t)p.B * p.H * p.T) return;
  const int t = (int)(w % p.T);
  const int bh = (int)(w / p.T);
  const int b = bh / p.H, h = bh - b * p.H;
  float q[E], acc[E];
  load_row<E>(p.q.row(b, t, h), lane, q);
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int nk = p.causal ? t + 1 : p.T;
  for (int j0 = 0; j0 < nk; j0 += 4) {
    float s[4], vv[4][E];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u < nk ? j0 + u : nk - 1;
      float kk[E];
      load_row<E>(p.k.row(b, j, h), lane, kk);
      load_row<E>(p.v.row(b, j, h), lane, vv[u]);
      s[u] = dot_part<E>(q, kk);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) s[u] = warp_sum(s[u]) * p.scale;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u >= nk) break;
      const float mn = fmaxf(m, s[u]);
      const float a = expf(m - mn);  // 0 on the first key (m = -inf)
      const float e = expf(s[u] - mn);
      l = l * a + e;
#pragma unroll
      for (int d = 0; d < E; ++d) acc[d] = fmaf(e, vv[u][d], acc[d] * a);
      m = mn;
    }
  }
  const float inv = 1.f / l;
  float* o = p.out.row(b, t, h);
#pragma unroll
  for (int e = 0; e < E; ++e) o[lane + 32 * e] = acc[e] * inv;
  if (lane == 0) p.lse[(int64_t)bh * p.T + t] = m + logf(l);
}

// delta[bh, t] = sum_d dO * O
template <int DH>
__global__ void __launch_bounds__(kWarps * 32) attn_delta_f32_kernel(const F32Attn p) {
  pdl_trigger();
  pdl_wait();
  constexpr int E = DH / 32;
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= (int64_t)p.B * p.H * p.T) return;
  const int t = (int)(w % p.T);
  const int bh = (int)(w / p.T);
  const int b = bh / p.H, h = bh - b * p.H;
  float o[E], g[E];
  load_row<E>(p.o.row(b, t, h), lane, o);
  load_row<E>(p.dout.row(b, t, h), lane, g);
  const float d = warp_sum(dot_part<E>(o, g));
  if (lane == 0) p.delta[w] = d;
}

// dQ: warp per (b, h, query row i), walking its keys
template <int DH>
__global__ void __launch_bounds__(kWarps * 32) attn_dq_f32_kernel(const F32Attn p) {
  pdl_trigger();
  pdl_wait();
  constexpr int E = DH / 32;
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= (int64_t)p.B * p.H * p.T) return;
  const int i = (int)(w % p.T);
  const int bh = (int)(w / p.T);
  const int b = bh / p.H, h = bh - b * p.H;
  float q[E], g[E], acc[E];
  load_row<E>(p.q.row(b, i, h), lane, q);
  load_row<E>(p.dout.row(b, i, h), lane, g);
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  const float lse = p.lse_in[w], dl = p.delta[w];
  const int nk = p.causal ? i + 1 : p.T;
  for (int j0 = 0; j0 < nk; j0 += 4) {
    float s[4], dp[4], kk[4][E];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u < nk ? j0 + u : nk - 1;
      float vv[E];
      load_row<E>(p.k.row(b, j, h), lane, kk[u]);
      load_row<E>(p.v.row(b, j, h), lane, vv);
      s[u] = dot_part<E>(q, kk[u]);
      dp[u] = dot_part<E>(g, vv);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[u] = warp_sum(s[u]);
      dp[u] = warp_sum(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u >= nk) break;
      const float pr = expf(s[u] * p.scale - lse);
      const float ds = pr * (dp[u] - dl);
#pragma unroll
      for (int d = 0; d < E; ++d) acc[d] = fmaf(ds, kk[u][d], acc[d]);
    }
  }
  float* o = p.dq.row(b, i, h);
#pragma unroll
  for (int e = 0; e < E; ++e) o[lane + 32 * e] = acc[e] * p.scale;
}

// dK, dV: warp per (b, h, key row j), walking the queries that see it
template <int DH>
__global__ void __launch_bounds__(kWarps * 32) attn_dkdv_f32_kernel(const F32Attn p) {
  pdl_trigger();
  pdl_wait();
  constexpr int E = DH / 32;
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= (int64_t)p.B * p.H * p.T) return;
  const int j = (int)(w % p.T);
  const int bh = (int)(w / p.T);
  const int b = bh / p.H, h = bh - b * p.H;
  float kk[E], vv[E], ak[E], av[E];
  load_row<E>(p.k.row(b, j, h), lane, kk);
  load_row<E>(p.v.row(b, j, h), lane, vv);
#pragma unroll
  for (int e = 0; e < E; ++e) ak[e] = av[e] = 0.f;
  const int i_begin = p.causal ? j : 0;
  const int64_t rbase = (int64_t)bh * p.T;
  for (int i0 = i_begin; i0 < p.T; i0 += 4) {
    float s[4], dp[4], qq[4][E], gg[4][E];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u < p.T ? i0 + u : p.T - 1;
      load_row<E>(p.q.row(b, i, h), lane, qq[u]);
      load_row<E>(p.dout.row(b, i, h), lane, gg[u]);
      s[u] = dot_part<E>(qq[u], kk);
      dp[u] = dot_part<E>(gg[u], vv);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[u] = warp_sum(s[u]);
      dp[u] = warp_sum(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u;
      if (i >= p.T) break;
      const float pr = expf(s[u] * p.scale - p.lse_in[rbase + i]);
      const float ds = pr * (dp[u] - p.delta[rbase + i]);
#pragma unroll
      for (int d = 0; d < E; ++d) {
        av[d] = fmaf(pr, gg[u][d], av[d]);
        ak[d] = fmaf(ds, qq[u][d], ak[d]);
      }
    }
  }
  float* ok = p.dk.row(b, j, h);
  float* ov = p.dv.row(b, j, h);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    ok[lane + 32 * e] = ak[e] * p.scale;
    ov[lane + 32 * e] = av[e];
  }
}

View view(const void* ptr, int64_t sb, int64_t st, int64_t sh) {
  return View{static_cast<const float*>(ptr), sb, st, sh};
}
OutView oview(void* ptr, int64_t sb, int64_t st, int64_t sh) {
  return OutView{static_cast<float*>(ptr), sb, st, sh};
}

bool pos(int64_t a, int64_t b, int64_t c) { return a > 0 && b > 0 && c > 0; }

int check_f32(const fxb_attn_args* a, bool bwd) {
  if (a->D != 64 && a->D != 128)
    return fxb::set_error(FXB_EINVAL, "attn: head_dim %d not supported (64 or 128)", a->D);
  if (a->B < 1 || a->T < 1 || a->H < 1)
    return fxb::set_error(FXB_EINVAL, "attn: bad shape B=%d T=%d H=%d", a->B, a->T, a->H);
  if (!a->q || !a->k || !a->v || !a->o || !a->lse)
    return fxb::set_error(FXB_EINVAL, "attn: NULL q/k/v/o/lse");
  if (!pos(a->q_sb, a->q_st, a->q_sh) || !pos(a->k_sb, a->k_st, a->k_sh) ||
      !pos(a->v_sb, a->v_st, a->v_sh) || !pos(a->o_sb, a->o_st, a->o_sh))
    return fxb::set_error(FXB_EINVAL, "attn: strides must be positive");
  if (bwd) {
    if (!a->dout || !a->dq || !a->dk || !a->dv || !a->workspace)
      return fxb::set_error(FXB_EINVAL, "attn bwd: NULL dout/dq/dk/dv/workspace");
    if (!pos(a->do_sb, a->do_st, a->do_sh) || !pos(a->dq_sb, a->dq_st, a->dq_sh) ||
        !pos(a->dk_sb, a->dk_st, a->dk_sh) || !pos(a->dv_sb, a->dv_st, a->dv_sh))
      return fxb::set_error(FXB_EINVAL, "attn bwd: strides must be positive");
  }
  if ((int64_t)a->B * a->H * a->T / kWarps >= (int64_t(1) << 31))
    return fxb::set_error(FXB_EINVAL, "attn: B*H*T too large");
  return FXB_OK;
}

F32Attn params(const fxb_attn_args* a) {
  F32Attn p;
  p.B = a->B; p.T = a->T; p.H = a->H;
  p.causal = a->causal ? 1 : 0;
  p.scale = a->scale;
  p.q = view(a->q, a->q_sb, a->q_st, a->q_sh);
  p.k = view(a->k, a->k_sb, a->k_st, a->k_sh);
  p.v = view(a->v, a->v_sb, a->v_st, a->v_sh);
  p.o = view(a->o, a->o_sb, a->o_st, a->o_sh);
  p.out = oview(a->o, a->o_sb, a->o_st, a->o_sh);
  p.dout = view(a->dout, a->do_sb, a->do_st, a->do_sh);
  p.dq = oview(a->dq, a->dq_sb, a->dq_st, a->dq_sh);
  p.dk = oview(a->dk, a->dk_sb, a->dk_st, a->dk_sh);
  p.dv = oview(a->dv, a->dv_sb, a->dv_st, a->dv_sh);
  p.lse = a->lse;
  p.lse_in = a->lse;
  p.delta = a->workspace;
  return p;
}

}  // namespace

namespace fxb {

int attn_fwd_f32(const fxb_attn_args* a, cudaStream_t st) {
  int r = check_f32(a, false);
  if (r) return r;
  const F32Attn p = params(a);
  const unsigned grid = (unsigned)(((int64_t)a->B * a->H * a->T + kWarps - 1) / kWarps);
  if (a->D == 64) pdl_launch(attn_fwd_f32_kernel<64>, grid, kWarps * 32, 0, st, p);
  else pdl_launch(attn_fwd_f32_kernel<128>, grid, kWarps * 32, 0, st, p);
  return check_launch("attn_fwd_f32");
}

int attn_bwd_f32(const fxb_attn_args* a, cudaStream_t st) {
  int r = check_f32(a, true);
  if (r) return r;
  const F32Attn p = params(a);
  const unsigned grid = (unsigned)(((int64_t)a->B * a->H * a->T + kWarps - 1) / kWarps);
  if (a->D == 64) {
    pdl_launch(attn_delta_f32_kernel<64>, grid, kWarps * 32, 0, st, p);
    if ((r = check_launch("attn_delta_f32"))) return r;
    pdl_launch(attn_dq_f32_kernel<64>, grid, kWarps * 32, 0, st, p);
    if ((r = check_launch("attn_dq_f32"))) return r;
    pdl_launch(attn_dkdv_f32_kernel<64>, grid, kWarps * 32, 0, st, p);
  } else {
    pdl_launch(attn_delta_f32_kernel<128>, grid, kWarps * 32, 0, st, p);
    if ((r = check_launch("attn_delta_f32"))) return r;
    pdl_launch(attn_dq_f32_kernel<128>, grid, kWarps * 32, 0, st, p);
    if ((r = check_launch("attn_dq_f32"))) return r;
    pdl_launch(attn_dkdv_f32_kernel<128>, grid, kWarps * 32, 0, st, p);
  }
  return check_launch("attn_dkdv_f32");
}

}  // namespace fxb
