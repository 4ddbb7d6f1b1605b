// Flash attention forward / backward on tcgen05 tensor cores (sm_100a).
//
// Semantics follow the reference FA2 kernels (ml/fxlm/kernels/attention.hip):
//   forward  :104-224  o = softmax(q k^T * scale [causal: key <= query]) v,
//                      lse = max + log(sum) of the scaled scores, natural log
//                      (:210-223), written (B,H,T) fp32;
//   bwd prep :229-251  delta = rowsum(dO * O);
//   bwd      :256-534  P = exp(s*scale - lse), dS = P * (dP - delta) * scale,
//                      dV = P^T dO, dK = dS^T Q, dQ = dS K.
// B200 design (new): 128x128 tiles; TMA (4-D maps over the strided (B,T,H,D)
// views, no copies, no multicast) feeds shared memory; one thread issues
// tcgen05.mma into tensor memory; softmax warps read scores with tcgen05.ld,
// several warps per TMEM lane quarter, each owning a slice of a tile's columns
// (forward at head dim 128: 16 warps, row maxima exchanged through shared
// memory once per tile; at head dim 64: two query tiles per CTA and one
// softmax thread per query row; both persistent, P written to and O
// accumulated in TMEM, lazily rescaled: details at the kernels). Backward
// works per key tile (at head dim 64 in persistent CTAs that walk (key tile,
// batch*head) items): S^T and dP^T land in TMEM, dV and dK accumulate in TMEM
// across query tiles, and each dQ partial is staged in shared memory and
// added into an fp32 workspace with asynchronous TMA reductions. Every wait
// is bounded (FXB_DERR_ATTN_WAIT); after an expired wait a thread keeps
// stepping through its loop without work, or leaves it, so that named
// barriers are always met by every participant.
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int TILE = 128;
constexpr int kFwdThreads = 576;  // forward: warps 0-15 softmax, 16 MMA, 17 TMA
constexpr int kBwdThreads = 576;  // backward: warps 0-15 softmax / dS, 16 MMA, 17 TMA
constexpr int kBwdWarpMma = 16, kBwdWarpTma = 17;
// head-dim-64 backward: warps 0-15 softmax / dS (four per TMEM lane quarter),
// 16-19 dQ flush (one per quarter), 20 MMA, 21 TMA for Q / dO, 22 TMA for
// K / V; the register cap comes from 768 threads (6 warps x 80 registers per
// sub-partition)
constexpr int kBwd64Threads = 736;
constexpr int kBwd64WarpFlush = 16, kBwd64WarpMma = 20, kBwd64WarpTma = 21, kBwd64WarpKV = 22;
constexpr int kBwdQS = 3;  // head-dim-64 backward: Q / dO ring stages
constexpr int kFwdWarpMma = 16, kFwdWarpTma = 17;
// Forward pipeline depths: K/V ring stages and Q buffers (shared memory:
// (QN + 2 KS) DH-wide tiles + exchange) and P buffers (tensor memory)
template <int DH> constexpr int fwd_kv_stages() { return DH <= 64 ? 5 : 2; }
template <int DH> constexpr int fwd_q_bufs() { return 2; }
template <int DH> constexpr int fwd_p_bufs() { return 2; }
constexpr int kFwdXchBytes = 6144;  // softmax row-statistics exchange area

struct FwdParams {
  int B, T, H, nqt, nkt, causal;
  float scale_log2;
  void* o;
  int64_t o_sb, o_st, o_sh;
  float* lse;
  int* err;
};

struct BwdParams {
  int B, T, H, nqt, nkt, causal;
  float scale_log2;  // scale * log2(e)
  float scale;
  const float* lse;
  const float* delta;
  float* dq_acc;  // (B*H, T, D) fp32
  void* dk;
  int64_t dk_sb, dk_st, dk_sh;
  void* dv;
  int64_t dv_sb, dv_st, dv_sh;
  int* err;
};

// byte offset of 16-byte chunk `chunk` (0..15 across two 64-column blocks) of
// row `r` in a [128 rows][128 cols] 16-bit tile stored as two 128B-swizzled
// column blocks of 16 KB
FXB_DEV uint32_t sw128_offset(int r, int chunk) {
  const int blk = chunk >> 3, c = chunk & 7;
  return (uint32_t)(blk * 16384 + r * 128 + ((c ^ (r & 7)) << 4));
}

// K-major operand tile [128 rows][D] stored as D/64 swizzled column blocks:
// descriptor of the tile and the byte offset of its K slice kk (16 elements)
FXB_DEV uint64_t kmajor_desc0(uint32_t base) { return umma_desc_sw128(base, 16, 1024); }
__host__ __device__ constexpr uint32_t kmajor_off(int kk) { return (kk >> 2) * 16384 + (kk & 3) * 32; }
FXB_DEV uint64_t kmajor_desc(uint32_t base, int kk) { return desc_add(kmajor_desc0(base), kmajor_off(kk)); }
// MN-major view of the same storage: MN along the columns, K along the rows
FXB_DEV uint64_t mnmajor_desc0(uint32_t base) { return umma_desc_sw128(base, 16384, 1024); }
__host__ __device__ constexpr uint32_t mnmajor_off(int kk) { return kk * 2048; }
FXB_DEV uint64_t mnmajor_desc(uint32_t base, int kk) { return desc_add(mnmajor_desc0(base), mnmajor_off(kk)); }

// ============================================================ forward
FXB_DEV float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Persistent kernel: each CTA walks work items (query tile, batch*head) in
// rounds of gridDim.x items (CTA order in even rounds, reverse order in odd
// ones); items are numbered heaviest first for causal attention (the last
// query tiles see the most key tiles). Tensor
// memory, barriers and tensor maps are set up once per CTA, Q is
// double-buffered (Dh 64) and the K/V ring, S buffers and P buffers run on
// counters that continue across items, so the next item's loads and first
// S = Q K^T overlap the current item's tail.
//
// O accumulates in tensor memory across the key tiles of an item (P.V with
// accumulate). The softmax keeps a reference maximum per row and computes P
// against it; only when a tile's row maximum exceeds the reference by more
// than 2^8 (P values stay <= 256) is the row's O rescaled in tensor memory
// (tcgen05.ld / st by the owning warp, after that row's previous P.V has
// completed) and the reference raised. P goes to tensor memory (tcgen05.st,
// 16-bit pairs) and is double-buffered there: the P.V MMA reads its A operand
// straight from tensor memory (only V comes from shared memory), and the
// softmax of tile j does not wait for P.V of tile j-1.
//
// Warp roles (576 threads): warps 0-15 softmax (warp w owns TMEM lane quarter
// w & 3, i.e. 32 query rows, and column part w >> 2 of every S tile: 32 of the
// 128 keys, and DH/4 of the O columns; four warps share each row's maximum and
// sum through shared memory), warp 16 MMA issuer, warp 17 TMA.
constexpr float kRescaleLog2 = 8.f;  // lazy-rescale threshold (log2 units)

template <int DH, int FMT>
__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  constexpr int QB = TILE * DH * 2;  // bytes of one [128][DH] tile
  constexpr int NBOX = DH / 64;
  constexpr int OC = DH / 4;         // O columns per softmax warp
  constexpr int KS = fwd_kv_stages<DH>();
  constexpr int QN = fwd_q_bufs<DH>();
  constexpr int PN = fwd_p_bufs<DH>();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;             // QN buffers
  const uint32_t sK = sQ + QN * QB;     // KS stages
  const uint32_t sV = sK + KS * QB;     // KS stages
  // row-statistics exchange: maxima [2 buf][4 part][128] fp32, then the row
  // sums [4 part][128] fp32 (6 KB)
  const uint32_t sX = sV + KS * QB;
  float* xch = reinterpret_cast<float*>(gbase + (sX - base));
  const uint32_t bars = sX + kFwdXchBytes;
  auto q_full = [&](int s) { return bars + 8u * s; };
  auto q_empty = [&](int s) { return bars + 8u * (2 + s); };
  auto k_full = [&](int s) { return bars + 8u * (4 + s); };
  auto v_full = [&](int s) { return bars + 8u * (4 + KS + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (4 + 2 * KS + s); };
  auto s_full = [&](int s) { return bars + 8u * (4 + 3 * KS + s); };
  auto s_empty = [&](int s) { return bars + 8u * (6 + 3 * KS + s); };
  auto p_full = [&](int s) { return bars + 8u * (8 + 3 * KS + s); };
  auto p_empty = [&](int s) { return bars + 8u * (10 + 3 * KS + s); };  // = P.V of that buffer done
  const uint32_t final_bar = bars + 8u * (12 + 3 * KS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (13 + 3 * KS));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int n_items = p.nqt * BH;
  // item -> (query tile, batch*head), heaviest query tiles first when causal
  auto item_coords = [&](int w, int& qt, int& bh, int& n_kv) {
    const int t = w / BH;
    bh = w - t * BH;
    qt = p.causal ? (p.nqt - 1 - t) : t;
    n_kv = p.causal ? min(qt + 1, p.nkt) : p.nkt;
  };
  // the k-th item of this CTA: rounds of gridDim.x items, taken in CTA order
  // in even rounds and in reverse order in odd ones, so that with items
  // numbered heaviest first the CTAs' totals even out (once an index passes
  // the end, every later round's does too)
  auto item_of = [&](int k) {
    const int r = k * (int)gridDim.x;
    return (k & 1) ? r + (int)gridDim.x - 1 - (int)blockIdx.x : r + (int)blockIdx.x;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1);
      mbar_init(s_full(s), 1);
      mbar_init(s_empty(s), 512);  // every softmax thread
      mbar_init(p_full(s), 512);
      mbar_init(p_empty(s), 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    mbar_init(final_bar, 1);
    fence_mbar_init();
  }
  if (warp == kFwdWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // q / k / v come from earlier kernels on the stream
  const uint32_t tS = tmem;        // S buffers (fp32) at columns 0 and 128
  const uint32_t tP = tmem + 256;  // P buffers (16-bit, two per column): 64 columns each
  const uint32_t tO = tmem + 384;  // O accumulator, DH columns

  // The TMA and MMA warps run their loops in lane 0 alone (the MMA issue is on
  // the softmax's critical path: no warp-wide handshakes there).
  if (warp == kFwdWarpTma) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int t = 0;   // K/V tiles issued (all items)
      int it = 0;  // items of this CTA
      int q_armed = 0;
      for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k), ++it) {
        int qt, bh, n_kv;
        item_coords(w, qt, bh, n_kv);
        const int b = bh / p.H, h = bh - b * p.H;
        const int qb = it % QN;
        if (!mbar_wait(q_empty(qb), ((it / QN) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        {
          mbar_expect_tx(q_full(qb), QB);
  #pragma unroll
          for (int c = 0; c < NBOX; ++c)
            tma_load_4d(sQ + qb * QB + c * 16384, &tmQ, q_full(qb), 64 * c, qt * TILE, h, b);
        }
        q_armed = it + 1;
        for (int j = 0; j < n_kv; ++j, ++t) {
          const int st = t % KS;
          if (!mbar_wait(kv_empty(st), ((t / KS) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          {
            mbar_expect_tx(k_full(st), QB);
  #pragma unroll
            for (int c = 0; c < NBOX; ++c)
              tma_load_4d(sK + st * QB + c * 16384, &tmK, k_full(st), 64 * c, j * TILE, h, b);
            mbar_expect_tx(v_full(st), QB);
  #pragma unroll
            for (int c = 0; c < NBOX; ++c)
              tma_load_4d(sV + st * QB + c * 16384, &tmV, v_full(st), 64 * c, j * TILE, h, b);
          }
          }
      }
      // drain: every copy issued has landed before shared memory goes away
      for (int i = (q_armed > QN ? q_armed - QN : 0); i < q_armed; ++i)
        mbar_wait(q_full(i % QN), (i / QN) & 1, p.err, FXB_DERR_ATTN_WAIT);
      for (int u = (t > KS ? t - KS : 0); u < t; ++u) {
        mbar_wait(k_full(u % KS), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT);
        mbar_wait(v_full(u % KS), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT);
      }
    }
    __syncwarp();
  } else if (warp == kFwdWarpMma) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IS = umma_idesc_f16(FMT, 0, 0, TILE, TILE);
      constexpr uint32_t IPV = umma_idesc_f16(FMT, 0, 1, TILE, DH);
      bool ok = true;
      int ts = 0;  // S tiles issued (all items)
      int tp = 0;  // P.V products issued (all items)
      int it = 0;
      // S = Q K^T of the next tile (global tile ts) into S buffer ts & 1
      auto issue_s = [&](uint32_t q_s) -> bool {
        const int st = ts % KS, sb = ts & 1;
        if (!mbar_wait(k_full(st), (ts / KS) & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        if (!mbar_wait(s_empty(sb), ((ts >> 1) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint64_t qd = kmajor_desc0(q_s), kd = kmajor_desc0(sK + st * QB);
        {
  #pragma unroll
          for (int kk = 0; kk < DH / 16; ++kk)
            umma_f16(tS + sb * TILE, desc_add(qd, kmajor_off(kk)), desc_add(kd, kmajor_off(kk)), IS,
                     kk > 0);
          umma_commit(s_full(sb));
        }
        ++ts;
        return true;
      };
      for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k), ++it) {
        int qt, bh, n_kv;
        item_coords(w, qt, bh, n_kv);
        const int qb = it % QN;
        const uint32_t q_s = sQ + qb * QB;
        if (!mbar_wait(q_full(qb), (it / QN) & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        if (!issue_s(q_s)) { ok = false; break; }
        for (int j = 0; j < n_kv && ok; ++j, ++tp) {
          if (j + 1 < n_kv && !issue_s(q_s)) { ok = false; break; }
          const int st = tp % KS, pb = tp % PN;
          if (!mbar_wait(p_full(pb), (tp / PN) & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          if (!mbar_wait(v_full(st), (tp / KS) & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint64_t vd = mnmajor_desc0(sV + st * QB);
          {
            if (j + 1 == n_kv) umma_commit(q_empty(qb));  // the item's last S has read Q
  #pragma unroll
            for (int kk = 0; kk < TILE / 16; ++kk)  // A = P from tensor memory, 16 keys = 8 columns
              umma_f16_ta(tO, tP + pb * 64 + kk * 8, desc_add(vd, mnmajor_off(kk)), IPV,
                          (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(p_empty(pb));
            umma_commit(kv_empty(st));
          }
          }
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax warps 0..15
    const int quarter = warp & 3, part = warp >> 2;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int col0 = part * 32;         // this thread's key columns within a tile
    const uint32_t tOw = tO + lane_off + part * OC;  // this warp's O columns
    bool ok = true;
    int t = 0;  // tiles consumed (all items)
    // Waits are made warp-uniform: the tensor-memory accesses that follow are
    // warp-collective.
    auto uwait = [&](uint32_t bar, uint32_t parity) -> bool {
      const bool r = mbar_wait(bar, parity, p.err, FXB_DERR_ATTN_WAIT);
      return __all_sync(0xffffffffu, r);
    };
    // wait until P.V of global tile u has completed (its P buffer is free and
    // its contribution is in O)
    auto wait_pv = [&](int u) -> bool { return uwait(p_empty(u % PN), (u / PN) & 1); };
    // this warp's O columns: 16 at a time through registers
    auto o_scale = [&](float alpha) {
#pragma unroll
      for (int c = 0; c < OC / 16; ++c) {
        uint32_t orr[16];
        tmem_ld16(tOw + c * 16, orr);
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < 16; ++d) orr[d] = __float_as_uint(__uint_as_float(orr[d]) * alpha);
        tmem_st16(tOw + c * 16, orr);
      }
      tmem_wait_st();
    };
    // After a failed (timed-out) wait a thread keeps stepping through the
    // tiles without waiting or computing, so that the four warps of a row
    // quarter always meet at the same named barriers.
    for (int k = 0, w = item_of(0); w < n_items; w = item_of(++k)) {
      int qt, bh, n_kv;
      item_coords(w, qt, bh, n_kv);
      const int q0 = qt * TILE;
      const int q = q0 + r;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kv; ++j, ++t) {
        const int sb = t & 1;
        if (ok && !uwait(s_full(sb), (t >> 1) & 1)) ok = false;
        const int kv0 = j * TILE + col0;
        float sv[32];
        float mx = -INFINITY;
        if (ok) {
          tc_fence_after();
          uint32_t sr[32];
          tmem_ld32(tS + sb * TILE + lane_off + col0, sr);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(s_empty(sb));  // the scores are in registers
          const bool need_mask = (kv0 + 32 > p.T) || (p.causal && kv0 + 32 > q0);
          // eight independent running maxima (short dependency chains)
          float mv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mv[i] = -INFINITY;
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = kv0 + i;
              sv[i] = (col >= p.T || (p.causal && col > q)) ? -INFINITY : __uint_as_float(sr[i]);
              mv[i & 7] = fmaxf(mv[i & 7], sv[i]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              sv[i] = __uint_as_float(sr[i]);
              mv[i & 7] = fmaxf(mv[i & 7], sv[i]);
            }
          }
          mx = fmaxf(fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3])),
                     fmaxf(fmaxf(mv[4], mv[5]), fmaxf(mv[6], mv[7])));
        }
        // exchange the partial row maxima among the four warps of this row
        // quarter (double-buffered by tile parity)
        float* xb = xch + (t & 1) * 512;
        xb[part * 128 + r] = mx;
        named_bar_sync(1 + quarter, 128);
        mx = fmaxf(fmaxf(xb[r], xb[128 + r]), fmaxf(xb[256 + r], xb[384 + r]));
        if (!ok) continue;
        const float m_new = fmaxf(m_ref, mx * p.scale_log2);
        if (j == 0) {
          m_ref = m_new;  // O is overwritten by this item's first P.V
        } else {
          // lazy rescale: raise the reference only when P would exceed 2^8
          const bool need = m_new > m_ref + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            if (!wait_pv(t - 1)) { ok = false; continue; }
            tc_fence_after();
            const float alpha = need ? ex2_ftz(m_ref - m_new) : 1.f;
            o_scale(alpha);
            l *= alpha;
            if (need) m_ref = m_new;
          }
        }
        const float m_off = (m_ref == -INFINITY) ? 0.f : m_ref;  // fully masked rows: P = 0
        // P buffer t % PN is free once P.V of tile t - PN has completed
        const int pb = t % PN;
        if (t >= PN && !wait_pv(t - PN)) { ok = false; continue; }
        // probabilities -> P (16-bit pairs) in tensor memory: this thread's 32
        // keys are the 16 columns part*16.. of P buffer pb in its lane; the
        // row sum uses eight partial sums (short dependency chains)
        float rsv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rsv[i] = 0.f;
        uint32_t pw[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float pv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            pv[i] = ex2_ftz(fmaf(sv[8 * u + i], p.scale_log2, -m_off));
            rsv[i] += pv[i];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) pw[4 * u + i] = pack2<T16>(pv[2 * i], pv[2 * i + 1]);
        }
        tmem_st16(tP + pb * 64 + lane_off + part * 16, pw);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full(pb));
        l += ((rsv[0] + rsv[1]) + (rsv[2] + rsv[3])) + ((rsv[4] + rsv[5]) + (rsv[6] + rsv[7]));
      }
      const bool done = ok && wait_pv(t - 1);
      if (!done) ok = false;
      // combine the four partial row sums (every softmax thread reaches this barrier)
      float* xs = xch + 1024;
      xs[part * 128 + r] = l;
      named_bar_sync(1 + quarter, 128);
      l = (xs[r] + xs[128 + r]) + (xs[256 + r] + xs[384 + r]);
      if (done) {
        tc_fence_after();
        const int b = bh / p.H, h = bh - b * p.H;
        const float inv = 1.f / l;
        T16* orow = static_cast<T16*>(p.o) + b * p.o_sb + (int64_t)q * p.o_st + h * p.o_sh + part * OC;
#pragma unroll
        for (int c = 0; c < OC / 16; ++c) {
          uint32_t orr[16];
          tmem_ld16(tOw + c * 16, orr);  // warp-collective: every lane loads
          tmem_wait_ld();
          if (q < p.T) {
#pragma unroll
            for (int d = 0; d < 16; d += 8) {
              float f[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(orr[d + i]) * inv;
              *reinterpret_cast<uint4*>(orow + c * 16 + d) = pack8<T16>(f);
            }
          }
        }
        if (part == 0 && q < p.T) p.lse[(int64_t)bh * p.T + q] = (m_ref + log2f(l)) * kLn2;
        tc_fence_before();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFwdWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ forward, head dim 64: two query tiles per CTA
// One work item is a pair of query tiles (256 query rows) of one batch*head;
// persistent CTAs walk the items heaviest first (causal: the last pairs see
// the most key tiles). Both tiles share one K/V stream (each K/V tile is
// loaded once for 256 rows).
//
// Warp roles (352 threads): warps 0-3 softmax group 0 (query tile 2i),
// warps 4-7 softmax group 1 (query tile 2i+1), warps 8 and 9 the MMA issuers
// of groups 0 and 1 (one issuing thread per group, so that neither group's
// products wait for the other group's softmax), warp 10 TMA.
// A softmax thread owns one query row: TMEM lane quarter (warp & 3) gives it
// row quarter*32 + lane of its group's S, so the row maximum and sum need no
// exchange between threads. Tensor memory (512 columns):
//   S0 [0,128)  S1 [128,256)   fp32 scores of the current key tile
//   P0 [256,320) P1 [320,384)  probabilities, 16-bit pairs (A operand of P.V)
//   O0 [384,448) O1 [448,512)  fp32 output accumulators
// A softmax thread loads its whole row of S from tensor memory once (four
// 32-column loads, one wait); with S and P in separate columns the group's
// next S = Q K^T is issued as soon as the row is in registers, while the
// exponentials run, the P columns are written and P.V runs. The MMA issue order per key tile j is S0(j+1), P0 V(j),
// S1(j+1), P1 V(j): the two groups drift half a tile apart and keep the
// tensor core and the exponential units busy in turn. O uses the same lazy
// rescaling as attn_fwd_kernel (only when a row maximum grows by more than
// 2^8), done by the owning thread after the group's previous P.V completed.
constexpr int kFwd2Threads = 352;
constexpr int kFwd2WarpMma = 8, kFwd2WarpTma = 10;  // warps 8, 9: MMA issuers of groups 0, 1
constexpr int kFwd2KS = 4;                // K/V ring stages
constexpr int kFwd2Tile = TILE * 64 * 2;  // one [128][64] 16-bit tile (16 KB)

template <int FMT>
__global__ void __launch_bounds__(kFwd2Threads, 1)
attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  constexpr int KS = kFwd2KS;
  constexpr int QB = kFwd2Tile;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;            // [group][buffer] Q tiles
  const uint32_t sK = sQ + 4 * QB;     // KS stages
  const uint32_t sV = sK + KS * QB;    // KS stages
  const uint32_t bars = sV + KS * QB;
  auto q_full = [&](int g, int b) { return bars + 8u * (g * 2 + b); };
  auto q_empty = [&](int g, int b) { return bars + 8u * (4 + g * 2 + b); };
  auto k_full = [&](int s) { return bars + 8u * (8 + s); };
  auto v_full = [&](int s) { return bars + 8u * (8 + KS + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (8 + 2 * KS + s); };
  auto s_full = [&](int g) { return bars + 8u * (8 + 3 * KS + g); };
  auto s_empty = [&](int g) { return bars + 8u * (10 + 3 * KS + g); };
  auto p_full = [&](int g) { return bars + 8u * (12 + 3 * KS + g); };
  auto p_empty = [&](int g) { return bars + 8u * (14 + 3 * KS + g); };  // = that group's P.V done
  const uint32_t final_bar = bars + 8u * (16 + 3 * KS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (17 + 3 * KS));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int npairs = (p.nqt + 1) / 2;
  const int n_items = npairs * BH;
  // item -> (pair, batch*head) and the key-tile counts of its two query tiles
  // (0 for a tile past the end of the sequence)
  auto item_coords = [&](int w, int& pi, int& bh, int* n_kv) {
    const int t = w / BH;
    bh = w - t * BH;
    pi = p.causal ? (npairs - 1 - t) : t;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int qt = 2 * pi + g;
      n_kv[g] = qt >= p.nqt ? 0 : (p.causal ? min(qt + 1, p.nkt) : p.nkt);
    }
  };
  // the k-th item of this CTA: rounds of gridDim.x items, taken in CTA order
  // in even rounds and in reverse order in odd ones, so that with items
  // numbered heaviest first the CTAs' totals even out (once an index passes
  // the end, every later round's does too)
  auto item_of = [&](int k) {
    const int r = k * (int)gridDim.x;
    return (k & 1) ? r + (int)gridDim.x - 1 - (int)blockIdx.x : r + (int)blockIdx.x;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(bars + 8u * i, 1);        // q_full
      mbar_init(bars + 8u * (4 + i), 1);  // q_empty
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 2);  // both groups' issuers
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full(g), 1);
      mbar_init(s_empty(g), 128);  // the group's softmax threads
      mbar_init(p_full(g), 128);
      mbar_init(p_empty(g), 1);
    }
    mbar_init(final_bar, 2);
    fence_mbar_init();
  }
  if (warp == kFwd2WarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // q / k / v come from earlier kernels on the stream

  if (warp == kFwd2WarpTma) {
    // ------------------------------------------------ TMA producer (lane 0)
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int t = 0;               // K/V tiles issued (all items)
      int cq[2] = {0, 0};      // Q tiles loaded per group
      for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k)) {
        int pi, bh, n_kv[2];
        item_coords(w, pi, bh, n_kv);
        const int b = bh / p.H, h = bh - b * p.H;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!n_kv[g]) continue;
          const int qb = cq[g] & 1;
          if (!mbar_wait(q_empty(g, qb), ((cq[g] >> 1) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          mbar_expect_tx(q_full(g, qb), QB);
          tma_load_4d(sQ + (g * 2 + qb) * QB, &tmQ, q_full(g, qb), 0, (2 * pi + g) * TILE, h, b);
          ++cq[g];
        }
        const int nk = max(n_kv[0], n_kv[1]);
        for (int j = 0; j < nk && ok; ++j, ++t) {
          const int st = t % KS;
          if (!mbar_wait(kv_empty(st), ((t / KS) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          mbar_expect_tx(k_full(st), QB);
          tma_load_4d(sK + st * QB, &tmK, k_full(st), 0, j * TILE, h, b);
          mbar_expect_tx(v_full(st), QB);
          tma_load_4d(sV + st * QB, &tmV, v_full(st), 0, j * TILE, h, b);
        }
      }
      // drain: every copy issued has landed before shared memory goes away
      for (int g = 0; g < 2; ++g)
        for (int i = (cq[g] > 2 ? cq[g] - 2 : 0); i < cq[g]; ++i)
          mbar_wait(q_full(g, i & 1), (i >> 1) & 1, p.err, FXB_DERR_ATTN_WAIT);
      for (int u = (t > KS ? t - KS : 0); u < t; ++u) {
        mbar_wait(k_full(u % KS), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT);
        mbar_wait(v_full(u % KS), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT);
      }
    }
    __syncwarp();
  } else if (warp == kFwd2WarpMma || warp == kFwd2WarpMma + 1) {
    // ------------------------------------------------ MMA issuer of group g (lane 0)
    if (lane == 0) {
      const int g = warp - kFwd2WarpMma;
      constexpr uint32_t IS = umma_idesc_f16(FMT, 0, 0, TILE, TILE);
      constexpr uint32_t IPV = umma_idesc_f16(FMT, 0, 1, TILE, 64);
      const uint32_t tSg = tmem + g * 128, tPg = tmem + 256 + g * 64, tOg = tmem + 384 + g * 64;
      bool ok = true;
      int t = 0;                    // K/V tiles of the stream (all items)
      int cq = 0, cs = 0, cp = 0;   // this group's Q tiles, S products, P.V products
      for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k)) {
        int pi, bh, n_kv[2];
        item_coords(w, pi, bh, n_kv);
        const int nk = max(n_kv[0], n_kv[1]);
        const int ng = n_kv[g];
        const int qb = cq & 1;
        if (ng && !mbar_wait(q_full(g, qb), (cq >> 1) & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        const int t0 = t;
        const uint64_t qd = kmajor_desc0(sQ + (g * 2 + qb) * QB);
        // S = Q K_j^T into the group's S columns
        auto issue_s = [&](int j) -> bool {
          const int u = t0 + j, st = u % KS;
          if (!mbar_wait(k_full(st), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
          if (!mbar_wait(s_empty(g), (cs & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
          tc_fence_after();
          const uint64_t kd = kmajor_desc0(sK + st * QB);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tSg, desc_add(qd, kmajor_off(kk)), desc_add(kd, kmajor_off(kk)), IS, kk > 0);
          umma_commit(s_full(g));
          if (j + 1 == ng) umma_commit(q_empty(g, qb));  // the group's last S has read Q
          ++cs;
          return true;
        };
        // O (+)= P V_j, A = P from tensor memory (16 keys = 8 columns per MMA)
        auto issue_pv = [&](int j) -> bool {
          const int u = t0 + j, st = u % KS;
          if (!mbar_wait(p_full(g), cp & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
          if (!mbar_wait(v_full(st), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
          tc_fence_after();
          const uint64_t vd = mnmajor_desc0(sV + st * QB);
#pragma unroll
          for (int kk = 0; kk < TILE / 16; ++kk)
            umma_f16_ta(tOg, tPg + kk * 8, desc_add(vd, mnmajor_off(kk)), IPV, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(p_empty(g));
          ++cp;
          return true;
        };
        if (ng && !issue_s(0)) { ok = false; break; }
        for (int j = 0; j < nk && ok; ++j) {
          if (j + 1 < ng && !issue_s(j + 1)) { ok = false; break; }
          if (j < ng && !issue_pv(j)) { ok = false; break; }
          // this group is done with K/V tile j. A group that does not use the
          // tile first waits for it to land: the stage's previous release has
          // then completed, so the arrival counts toward this use of the stage
          const int u = t0 + j, st = u % KS;
          if (j < ng) {
            umma_commit(kv_empty(st));
          } else {
            if (!mbar_wait(k_full(st), (u / KS) & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
            mbar_arrive(kv_empty(st));
          }
        }
        t += nk;
        if (ng) ++cq;
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax: warps 0-3 group 0, 4-7 group 1
    const int g = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the group's tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + g * 128 + lane_off;
    const uint32_t tP = tmem + 256 + g * 64 + lane_off;
    const uint32_t tO = tmem + 384 + g * 64 + lane_off;
    bool ok = true;
    int cs = 0;  // tiles this group consumed (all items)
    auto uwait = [&](uint32_t bar, uint32_t parity) -> bool {
      const bool rr = mbar_wait(bar, parity, p.err, FXB_DERR_ATTN_WAIT);
      return __all_sync(0xffffffffu, rr);
    };
    for (int k = 0, w = item_of(0); w < n_items; w = item_of(++k)) {
      int pi, bh, n_kv[2];
      item_coords(w, pi, bh, n_kv);
      const int nkv = n_kv[g];
      if (!nkv || !ok) { cs += ok ? nkv : 0; continue; }
      const int q0 = (2 * pi + g) * TILE;
      const int q = q0 + r;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv; ++j, ++cs) {
        if (!uwait(s_full(g), cs & 1)) { ok = false; break; }
        tc_fence_after();
        const int kv0 = j * TILE;
        const bool need_mask = (kv0 + TILE > p.T) || (p.causal && kv0 + TILE > q0 + 1);  // warp-uniform
        // valid keys of this row in the tile: columns < lim (key < T, key <= q when causal)
        const int lim = min(p.T, p.causal ? q + 1 : p.T) - kv0;
        // masked scores read as -inf (64 columns from column c0)
        auto mask64 = [&](uint32_t* v, int c0) {
          if (need_mask) {
            const int l64 = lim - c0;
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i >= l64) v[i] = __float_as_uint(-INFINITY);
          }
        };
        // the whole row of S in registers (one round trip to tensor memory)
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, v + 32 * c);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(s_empty(g));  // S is in registers: the next S may overwrite it
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= lim) v[i] = __float_as_uint(-INFINITY);
        }
        float mv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mv[i] = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; ++i) mv[i & 7] = fmaxf(mv[i & 7], __uint_as_float(v[i]));
        const float mx = fmaxf(fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3])),
                               fmaxf(fmaxf(mv[4], mv[5]), fmaxf(mv[6], mv[7])));
        const float m_new = fmaxf(m_ref, mx * p.scale_log2);
        bool resc = false;
        float alpha = 1.f;
        if (j == 0) {
          m_ref = m_new;  // O is overwritten by this item's first P.V
        } else {
          const bool need = m_new > m_ref + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            resc = true;
            if (need) {
              alpha = ex2_ftz(m_ref - m_new);
              m_ref = m_new;
            }
          }
        }
        const float m_off = (m_ref == -INFINITY) ? 0.f : m_ref;
        // probabilities, packed in place (word i: keys 2i, 2i+1)
        float rs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs[i] = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float e0 = ex2_ftz(fmaf(__uint_as_float(v[2 * i]), p.scale_log2, -m_off));
          const float e1 = ex2_ftz(fmaf(__uint_as_float(v[2 * i + 1]), p.scale_log2, -m_off));
          rs[(2 * i) & 7] += e0;
          rs[(2 * i + 1) & 7] += e1;
          v[i] = pack2<T16>(e0, e1);
        }
        // the group's previous P.V has completed: its P columns are free and O
        // is stable for a rescale
        if (j > 0 && !uwait(p_empty(g), (cs - 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_st16(tP + c * 16, v + 16 * c);
        if (resc) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t orr[16];
            tmem_ld16(tO + c * 16, orr);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 16; ++d) orr[d] = __float_as_uint(__uint_as_float(orr[d]) * alpha);
            tmem_st16(tO + c * 16, orr);
          }
          l *= alpha;
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full(g));
        l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      }
      if (!ok) continue;
      // the item's last P.V has completed: O is final
      if (!uwait(p_empty(g), (cs - 1) & 1)) { ok = false; continue; }
      tc_fence_after();
      const int b = bh / p.H, h = bh - b * p.H;
      const float inv = 1.f / l;
      T16* orow = static_cast<T16*>(p.o) + b * p.o_sb + (int64_t)q * p.o_st + h * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t orr[16];
        tmem_ld16(tO + c * 16, orr);  // warp-collective: every lane loads
        tmem_wait_ld();
        if (q < p.T) {
#pragma unroll
          for (int d = 0; d < 16; d += 8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(orr[d + i]) * inv;
            *reinterpret_cast<uint4*>(orow + c * 16 + d) = pack8<T16>(f);
          }
        }
      }
      if (q < p.T) p.lse[(int64_t)bh * p.T + q] = (m_ref + log2f(l)) * kLn2;
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFwd2WarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ backward
// delta[bh, t] = sum_d dO*O ; zero the dQ accumulator
template <typename T16, int DH>
__global__ void attn_bwd_prep_kernel(const T16* __restrict__ o, int64_t o_sb, int64_t o_st,
                                     int64_t o_sh, const T16* __restrict__ dout, int64_t do_sb,
                                     int64_t do_st, int64_t do_sh, float* __restrict__ delta,
                                     float* __restrict__ dq_acc, int B, int T, int H) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  // DH/8 lanes per row (8 bf16 each): coalesced 128-byte row reads
  constexpr int LPR = DH / 8;
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gtid / LPR;  // (b*H + h)*T + t
  const int sub = (int)(gtid % LPR);
  const bool ok = row < (int64_t)B * H * T;
  float s = 0.f;
  if (ok) {
    const int t = (int)(row % T);
    const int bh = (int)(row / T);
    const int b = bh / H, h = bh - b * H;
    const T16* orow = o + b * o_sb + (int64_t)t * o_st + h * o_sh + sub * 8;
    const T16* grow = dout + b * do_sb + (int64_t)t * do_st + h * do_sh + sub * 8;
    float a[8], g[8];
    unpack8<T16>(*reinterpret_cast<const uint4*>(orow), a);
    unpack8<T16>(*reinterpret_cast<const uint4*>(grow), g);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += a[i] * g[i];
  }
#pragma unroll
  for (int off = LPR / 2; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (!ok) return;
  if (sub == 0) delta[row] = s;
  if (!dq_acc) return;  // head dim 128: the transposed accumulator is cleared separately
  float4* z = reinterpret_cast<float4*>(dq_acc + row * DH + sub * 8);
  z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// dq = dq_acc * scale in the caller's layout
template <typename T16, int DH>
__global__ void attn_bwd_post_kernel(const float* __restrict__ dq_acc, T16* __restrict__ dq,
                                     int64_t dq_sb, int64_t dq_st, int64_t dq_sh, float scale,
                                     int B, int T, int H) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel on the stream
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // row*DH/8 + chunk
  const int64_t rows = (int64_t)B * H * T;
  if (idx >= rows * (DH / 8)) return;
  const int64_t row = idx / (DH / 8);
  const int d = (int)(idx % (DH / 8)) * 8;
  const int t = (int)(row % T);
  const int bh = (int)(row / T);
  const int b = bh / H, h = bh - b * H;
  const float4* src = reinterpret_cast<const float4*>(dq_acc + row * DH + d);
  float4 u = src[0], w = src[1];
  float f[8] = {u.x * scale, u.y * scale, u.z * scale, u.w * scale,
                w.x * scale, w.y * scale, w.z * scale, w.w * scale};
  *reinterpret_cast<uint4*>(dq + b * dq_sb + (int64_t)t * dq_st + h * dq_sh + d) = pack8<T16>(f);
}


// Persistent: one CTA per SM walks work items (key tile, batch*head) in rounds
// of gridDim.x items (CTA order in even rounds, reverse order in odd ones);
// items are numbered key tile major, so with a causal mask (key tile kt meets
// nqt - kt query tiles) they come heaviest first and the CTAs' totals even
// out. Per item the CTA walks the query tiles that see its key tile. Tensor
// memory stays allocated across items and every ring and barrier runs on
// across them (phases from the running tile count u and item count k), so
// one item's last tiles, its dK / dV epilogue and the next item's K / V load
// overlap instead of each CTA filling and draining the pipeline alone:
//  - the next item's K / V are prefetched into L2 when an item starts and
//    loaded once every MMA of the item has completed (kv_empty);
//  - the next item's first dV / dK MMAs wait until the softmax warps have
//    read the finished dK / dV out of tensor memory (acc_empty).
template <int FMT>
__global__ void __launch_bounds__(768, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  constexpr int DH = 64;
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  constexpr int QB = TILE * DH * 2;  // 16 KB
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  constexpr int QS = kBwdQS;         // Q / dO / LSE / delta ring stages
  const uint32_t sK = base;
  const uint32_t sV = sK + QB;
  const uint32_t sQ = sV + QB;        // QS stages
  const uint32_t sDO = sQ + QS * QB;  // QS stages
  const uint32_t sDS = sDO + QS * QB; // 2 buffers of dS^T [128 kv][128 q] 16-bit
  const uint32_t sDQ = sDS + 65536;   // dQ staging: 4 flush warps x 2 x [32 rows][16 fp32], 64B-swizzled
  const uint32_t sStat = sDQ + 16384; // lse2[QS][128], delta[QS][128] fp32
  float* lse_s = reinterpret_cast<float*>(gbase + (sStat - base));
  float* del_s = lse_s + QS * 128;
  const uint32_t bars = sStat + QS * 1024;
  const uint32_t kv_full = bars;
  auto qdo_full = [&](int s) { return bars + 8u * (1 + s); };
  auto qdo_empty = [&](int s) { return bars + 8u * (1 + QS + s); };
  const uint32_t s_full = bars + 8u * (1 + 2 * QS);
  const uint32_t s_empty = s_full + 8u;
  const uint32_t ds_full = s_full + 16u;
  const uint32_t dq_full = s_full + 24u;
  const uint32_t dq_empty = s_full + 32u;
  const uint32_t acc_full = s_full + 40u;
  const uint32_t pt_free = s_full + 48u;   // dV of the tile has read P^T from tensor memory
  const uint32_t kv_empty = s_full + 56u;  // every MMA of the item has completed: K / V free
  const uint32_t acc_empty = s_full + 64u; // the softmax warps have read the item's dK / dV
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (acc_empty + 8u - base));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int n_items = p.nkt * BH;
  auto item_of = [&](int k) {
    const int r = k * (int)gridDim.x;
    return (k & 1) ? r + (int)gridDim.x - 1 - (int)blockIdx.x : r + (int)blockIdx.x;
  };
  // item w -> key tile, batch*head and its query tiles [i0, nqt)
  struct Item { int kv0, bh, b, h, i0, n_it; };
  auto item = [&](int w) {
    Item t;
    const int kt = w / BH;
    t.bh = w - kt * BH;
    t.b = t.bh / p.H;
    t.h = t.bh - t.b * p.H;
    t.kv0 = kt * TILE;
    t.i0 = p.causal ? kt : 0;
    t.n_it = p.nqt - t.i0;
    return t;
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < QS; ++s) {
      mbar_init(qdo_full(s), 1 + 32);  // TMA bytes + the producer warp's LSE / delta stores
      mbar_init(qdo_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 512);  // every softmax thread
    mbar_init(ds_full, 512);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);  // every dQ flush thread
    mbar_init(acc_full, 1);
    mbar_init(pt_free, 1);
    mbar_init(kv_empty, 1);
    mbar_init(acc_empty, 512);  // every softmax thread
    fence_mbar_init();
  }
  if (warp == kBwd64WarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // q / k / v (and dO, lse) come from earlier kernels on the stream
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384;
  const uint32_t tPT = tmem + 448;  // P^T, 16-bit pairs (128 queries in 64 columns)

  if (warp == kBwd64WarpTma) {
    // ------------------------------------------------ producer: TMA (lane 0)
    // plus each query tile's LSE (log2 units) and delta, four queries per
    // lane, into the same ring stage as its Q / dO
    if (lane == 0) {
      tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV); tma_prefetch_desc(&tmDO);
    }
    __syncwarp();
    bool ok = true;
    int u = 0;  // query tiles issued (all items)
    // LSE / delta of a query tile are read from global memory one tile ahead
    // into registers, so that their latency passes while the producer waits
    // for the stage to be freed instead of after it
    float nl[4], nd[4];
    auto prefetch = [&](int bh, int qt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = qt * TILE + lane * 4 + i;
        const bool v = q < p.T;
        nl[i] = v ? p.lse[(int64_t)bh * p.T + q] * kLog2e : INFINITY;
        nd[i] = v ? p.delta[(int64_t)bh * p.T + q] : 0.f;
      }
    };
    if (item_of(0) < n_items) {
      const Item t0 = item(item_of(0));
      prefetch(t0.bh, t0.i0);
    }
    for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k)) {
      const Item t = item(w);
      const int wn = item_of(k + 1);
      for (int it = 0; it < t.n_it && ok; ++it, ++u) {
        const int st = u % QS;
        const int qq0 = (t.i0 + it) * TILE;
        if (!mbar_wait_warp(qdo_empty(st), ((u / QS) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        if (lane == 0) {
          mbar_expect_tx(qdo_full(st), 2 * QB);
          tma_load_4d(sQ + st * QB, &tmQ, qdo_full(st), 0, qq0, t.h, t.b);
          tma_load_4d(sDO + st * QB, &tmDO, qdo_full(st), 0, qq0, t.h, t.b);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lse_s[st * 128 + lane * 4 + i] = nl[i];
          del_s[st * 128 + lane * 4 + i] = nd[i];
        }
        mbar_arrive(qdo_full(st));
        if (it + 1 < t.n_it) {
          prefetch(t.bh, t.i0 + it + 1);
        } else if (wn < n_items) {
          const Item tn = item(wn);
          prefetch(tn.bh, tn.i0);
        }
      }
    }
    if (lane == 0) {
      // every copy issued has landed before shared memory goes away
      for (int v = (u > QS ? u - QS : 0); v < u; ++v)
        mbar_wait(qdo_full(v % QS), (v / QS) & 1, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else if (warp == kBwd64WarpKV) {
    // ------------------------------------------------ K / V loads (lane 0)
    // each item's K / V, once every MMA of the previous item has completed;
    // a warp of its own, so that neither the Q / dO ring nor the LSE / delta
    // reads delay it. The next item's K / V and first query tiles are
    // prefetched into L2 meanwhile.
    if (lane == 0) {
      int k = 0;
      for (int w = item_of(0); w < n_items; w = item_of(++k)) {
        const Item t = item(w);
        if (!mbar_wait(kv_empty, (k & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) break;
        mbar_expect_tx(kv_full, 2 * QB);
        tma_load_4d(sK, &tmK, kv_full, 0, t.kv0, t.h, t.b);
        tma_load_4d(sV, &tmV, kv_full, 0, t.kv0, t.h, t.b);
        const int wn = item_of(k + 1);
        if (wn < n_items) {
          const Item tn = item(wn);
          tma_prefetch_l2_4d(&tmK, 0, tn.kv0, tn.h, tn.b);
          tma_prefetch_l2_4d(&tmV, 0, tn.kv0, tn.h, tn.b);
          for (int j = 0; j < QS - 1 && j < tn.n_it; ++j) {
            tma_prefetch_l2_4d(&tmQ, 0, (tn.i0 + j) * TILE, tn.h, tn.b);
            tma_prefetch_l2_4d(&tmDO, 0, (tn.i0 + j) * TILE, tn.h, tn.b);
          }
        }
      }
      // the last load issued has landed before shared memory goes away
      if (k > 0) mbar_wait(kv_full, (k - 1) & 1, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else if (warp == kBwd64WarpMma) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t I_SS = umma_idesc_f16(FMT, 0, 0, TILE, TILE);  // S^T, dP^T
      constexpr uint32_t I_KV = umma_idesc_f16(FMT, 0, 1, TILE, DH);    // dV, dK
      constexpr uint32_t I_Q = umma_idesc_f16(FMT, 1, 1, TILE, DH);     // dQ
      bool ok = true;
      int u = 0;  // query tiles of all items so far
      int k = 0;
      // S^T and dP^T of the running tile v (once its Q / dO have landed and
      // the previous S^T / dP^T have been read out of tensor memory)
      auto issue_s = [&](int v) -> bool {
        const int st = v % QS;
        const uint32_t q_s = sQ + st * QB, do_s = sDO + st * QB;
        if (!mbar_wait(qdo_full(st), (v / QS) & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        if (!mbar_wait(s_empty, (v & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint64_t kd = kmajor_desc0(sK), qd = kmajor_desc0(q_s);
        const uint64_t vd = kmajor_desc0(sV), dod = kmajor_desc0(do_s);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk)
          umma_f16(tST, desc_add(kd, kmajor_off(kk)), desc_add(qd, kmajor_off(kk)), I_SS, kk > 0);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk)
          umma_f16(tDPT, desc_add(vd, kmajor_off(kk)), desc_add(dod, kmajor_off(kk)), I_SS, kk > 0);
        umma_commit(s_full);
        return true;
      };
      for (int w = item_of(0); w < n_items && ok; w = item_of(++k)) {
        const Item t = item(w);
        if (!mbar_wait(kv_full, k & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        const int u0 = u;
        if (t.n_it > 0 && !issue_s(u0)) { ok = false; break; }
        for (int it = 0; it < t.n_it && ok; ++it, ++u) {
          // the next tile's scores run on the tensor core while the softmax
          // warps turn this tile's scores into P^T and dS^T
          if (it + 1 < t.n_it && !issue_s(u + 1)) { ok = false; break; }
          const int st = u % QS;
          const uint32_t q_s = sQ + st * QB, do_s = sDO + st * QB;
          if (!mbar_wait(ds_full, u & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          // the previous item's dK / dV have left tensor memory
          if (it == 0 && !mbar_wait(acc_empty, (k & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ds_s = sDS + (uint32_t)(u & 1) * 32768u;
          const uint64_t dsd = kmajor_desc0(ds_s);
          const uint64_t dom = mnmajor_desc0(do_s), qm = mnmajor_desc0(q_s);
#pragma unroll
          for (int kk = 0; kk < TILE / 16; ++kk)  // A = P^T from tensor memory, 16 queries = 8 columns
            umma_f16_ta(tDV, tPT + kk * 8, desc_add(dom, mnmajor_off(kk)), I_KV, (it > 0 || kk > 0));
          // completes when dV has read P^T and every earlier MMA (the previous
          // tile's dQ, the last reader of the other dS^T buffer) is done
          umma_commit(pt_free);
#pragma unroll
          for (int kk = 0; kk < TILE / 16; ++kk)
            umma_f16(tDK, desc_add(dsd, kmajor_off(kk)), desc_add(qm, mnmajor_off(kk)), I_KV,
                     (it > 0 || kk > 0));
          // Q / dO of this tile have no readers after dK (dQ reads dS and K): the
          // producer may load tile u + QS into the stage now
          umma_commit(qdo_empty(st));
          if (!mbar_wait(dq_empty, (u & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint64_t dsm = mnmajor_desc0(ds_s), km = mnmajor_desc0(sK);
#pragma unroll
          for (int kk = 0; kk < TILE / 16; ++kk)
            umma_f16(tDQ, desc_add(dsm, mnmajor_off(kk)), desc_add(km, mnmajor_off(kk)), I_Q, kk > 0);
          umma_commit(dq_full);
        }
        if (!ok) break;
        umma_commit(acc_full);  // dK / dV of the item are final
        umma_commit(kv_empty);  // and K / V have no readers left
      }
      // every MMA issued has completed before tensor memory is freed
      if (k > 0) mbar_wait(acc_full, (k - 1) & 1, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else if (warp >= kBwd64WarpFlush) {
    // ------------------------------------------------ dQ flush warps 16..19
    // warp w: TMEM lane quarter w & 3 = query rows quarter*32.. of the tile's
    // dQ partial, all 64 head dims in two rounds of 32: tensor memory ->
    // registers -> this warp's 4 KB staging (two 64B-swizzled [32 rows][16
    // fp32] boxes) -> fp32 TMA add-reductions into the dQ accumulator (rows
    // past T are clipped by the tensor map). The accumulator is released for
    // the next tile's dQ MMA once both rounds have left tensor memory. The
    // softmax warps never wait on this path.
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t stg = sDQ + (uint32_t)quarter * 4096u;
    const int sw = (lane >> 1) & 3;
    bool ok = true;
    int u = 0;
    for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k)) {
      const Item t = item(w);
      for (int it = 0; it < t.n_it; ++it, ++u) {
        if (!__all_sync(0xffffffffu, mbar_wait(dq_full, u & 1, p.err, FXB_DERR_ATTN_WAIT))) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int rd = 0; rd < 2; ++rd) {
          uint32_t rr[32];
          tmem_ld16(tDQ + lane_off + rd * 32, rr);
          tmem_ld16(tDQ + lane_off + rd * 32 + 16, rr + 16);
          tmem_wait_ld();
          if (rd == 1) {
            tc_fence_before();
            mbar_arrive(dq_empty);  // the dQ partial has left tensor memory
          }
          if (lane == 0) bulk_wait_read0();  // the previous round's reductions have read the staging
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t row = stg + (uint32_t)c * 2048u + (uint32_t)lane * 64u;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_shared_v4(row + (uint32_t)((j ^ sw) << 4),
                           make_uint4(rr[16 * c + 4 * j], rr[16 * c + 4 * j + 1], rr[16 * c + 4 * j + 2],
                                      rr[16 * c + 4 * j + 3]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_reduce_add_3d(&tmDQ, stg + (uint32_t)c * 2048u, rd * 32 + c * 16,
                                (t.i0 + it) * TILE + quarter * 32, t.bh);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all0();  // dQ reductions complete before the kernel ends
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax / dS warps 0..15
    // warp w: TMEM lane quarter w & 3 (32 key rows of S^T / dP^T / dK / dV),
    // column part w >> 2 (32 of the 128 queries of S^T / dP^T, 16 of the 64
    // head dims of dK / dV): four warps per sub-partition keep its pipes busy
    // through the tensor-memory and barrier latencies of the chain
    const int quarter = warp & 3, part = warp >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int qc0 = part * 32;
    bool ok = true;
    int u = 0;
    // P^T / dS^T of tile u are computed while the dV / dK / dQ MMAs of tile
    // u-1 run, 16 queries at a time, each half stored as soon as it is done
    // (P^T to tensor memory, dS^T to shared buffer u & 1) once the previous
    // tile's dV has read P^T (pt_free, which also covers the dQ of tile u-2,
    // the last reader of this dS^T buffer).
    // The query tile's LSE / delta were written to the ring stage by the
    // producer warp before it arrived on qdo_full; waiting on that barrier here
    // makes them visible.
    for (int k = 0, w = item_of(0); w < n_items && ok; w = item_of(++k)) {
      const Item t = item(w);
      const int kv = t.kv0 + r;
      for (int it = 0; it < t.n_it; ++it, ++u) {
        const int q0 = (t.i0 + it) * TILE;
        const int sb = u % QS;
        // waits are made warp-uniform: the tensor-memory loads that follow are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait(qdo_full(sb), (u / QS) & 1, p.err, FXB_DERR_ATTN_WAIT)) ||
            !__all_sync(0xffffffffu, mbar_wait(s_full, u & 1, p.err, FXB_DERR_ATTN_WAIT))) { ok = false; break; }
        tc_fence_after();
        const bool diag = p.causal && (q0 < t.kv0 + TILE);
        // tile-uniform: every (key, query) pair of the tile is kept (queries past
        // T carry LSE = +inf, so their P and dS are zero without a mask)
        const bool full = !diag && t.kv0 + TILE <= p.T;
        uint8_t* ds = gbase + (sDS - base) + (u & 1) * 32768;
#pragma unroll
        for (int hq = 0; hq < 2; ++hq) {
          uint32_t sr[16], dr[16];
          tmem_ld16(tST + lane_off + qc0 + hq * 16, sr);
          tmem_ld16(tDPT + lane_off + qc0 + hq * 16, dr);
          tmem_wait_ld();
          if (hq == 1) {
            tc_fence_before();
            mbar_arrive(s_empty);  // S^T / dP^T are in registers: the next tile's may overwrite them
          }
          // the 16 queries' LSE (log2 units) and delta: 16-byte shared loads
          float ls[16], dl[16];
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const float4 a = *reinterpret_cast<const float4*>(lse_s + sb * 128 + qc0 + hq * 16 + 4 * v4);
            const float4 c = *reinterpret_cast<const float4*>(del_s + sb * 128 + qc0 + hq * 16 + 4 * v4);
            ls[4 * v4] = a.x; ls[4 * v4 + 1] = a.y; ls[4 * v4 + 2] = a.z; ls[4 * v4 + 3] = a.w;
            dl[4 * v4] = c.x; dl[4 * v4 + 1] = c.y; dl[4 * v4 + 2] = c.z; dl[4 * v4 + 3] = c.w;
          }
          uint32_t pw[8], dw[8];  // P^T and dS^T of 16 queries, 16-bit pairs
          if (full) {
            // no causal or key-row mask in this tile: exp2, subtract, multiply, pack
#pragma unroll
            for (int qc = 0; qc < 16; qc += 2) {
              const float e0 = ex2_ftz(fmaf(__uint_as_float(sr[qc]), p.scale_log2, -ls[qc]));
              const float e1 = ex2_ftz(fmaf(__uint_as_float(sr[qc + 1]), p.scale_log2, -ls[qc + 1]));
              pw[qc >> 1] = pack2<T16>(e0, e1);
              dw[qc >> 1] = pack2<T16>(e0 * (__uint_as_float(dr[qc]) - dl[qc]),
                                       e1 * (__uint_as_float(dr[qc + 1]) - dl[qc + 1]));
            }
          } else {
#pragma unroll
            for (int qc = 0; qc < 16; qc += 2) {
              float pp[2], dd[2];
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                float e = ex2_ftz(fmaf(__uint_as_float(sr[qc + i]), p.scale_log2, -ls[qc + i]));
                if (kv >= p.T || (diag && q0 + qc0 + hq * 16 + qc + i < kv)) e = 0.f;
                pp[i] = e;
                dd[i] = e * (__uint_as_float(dr[qc + i]) - dl[qc + i]);
              }
              pw[qc >> 1] = pack2<T16>(pp[0], pp[1]);
              dw[qc >> 1] = pack2<T16>(dd[0], dd[1]);
            }
          }
          if (hq == 0 && u > 0 &&
              !__all_sync(0xffffffffu, mbar_wait(pt_free, (u - 1) & 1, p.err, FXB_DERR_ATTN_WAIT))) {
            ok = false;
            break;
          }
          if (hq == 0) tc_fence_after();
          tmem_st8(tPT + lane_off + part * 16 + hq * 8, pw);
#pragma unroll
          for (int v2 = 0; v2 < 2; ++v2)
            *reinterpret_cast<uint4*>(ds + sw128_offset(r, part * 4 + hq * 2 + v2)) =
                make_uint4(dw[4 * v2], dw[4 * v2 + 1], dw[4 * v2 + 2], dw[4 * v2 + 3]);
        }
        if (!ok) break;
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_full);
      }
      if (!ok) break;
      // the item's final dK (scaled) and dV for key row kv, head dims part*16..+16
      if (!__all_sync(0xffffffffu, mbar_wait(acc_full, k & 1, p.err, FXB_DERR_ATTN_WAIT))) { ok = false; break; }
      tc_fence_after();
      uint32_t rk[16], rv[16];
      tmem_ld16(tDK + lane_off + part * 16, rk);
      tmem_ld16(tDV + lane_off + part * 16, rv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(acc_empty);  // the next item's first dV / dK MMAs may overwrite them
      if (kv < p.T) {
        T16* krow = static_cast<T16*>(p.dk) + t.b * p.dk_sb + (int64_t)kv * p.dk_st + t.h * p.dk_sh + part * 16;
        T16* vrow = static_cast<T16*>(p.dv) + t.b * p.dv_sb + (int64_t)kv * p.dv_st + t.h * p.dv_sh + part * 16;
#pragma unroll
        for (int v2 = 0; v2 < 2; ++v2) {
          float fk[8], fv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            fk[i] = __uint_as_float(rk[8 * v2 + i]) * p.scale;
            fv[i] = __uint_as_float(rv[8 * v2 + i]);
          }
          *reinterpret_cast<uint4*>(krow + 8 * v2) = pack8<T16>(fk);
          *reinterpret_cast<uint4*>(vrow + 8 * v2) = pack8<T16>(fv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBwd64WarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ backward, head dim 128
// Same schedule as attn_bwd_kernel (one CTA per key tile of 128 keys and
// batch*head, walking the query tiles that see it, the next tile's scores
// computed while the current tile's dV / dK / dQ MMAs run), with the query
// tile halved to 64 rows so that every accumulator fits the 512 tensor-memory
// columns at head dim 128:
//   S^T, dP^T  [128 keys][64 queries]       fp32   64 + 64 columns
//   dV, dK     [128 keys][128 head dims]    fp32  128 + 128 columns
//   dQ^T       [128 head dims][64 queries]  fp32   64 columns
//   P^T        [128 keys][64 queries]       16-bit pairs, 32 columns
// dQ is produced transposed (dQ^T = K^T dS^T, M = head dims): its rows are
// head dims, so the partial for a query tile leaves as fp32 TMA
// add-reductions into a transposed accumulator (B*H, 128, Tp), Tp = T
// rounded up to 64, which the post kernel reads back in the caller's layout.
// Shared memory: K, V (32 KB each), Q and dO double-buffered (16 KB tiles),
// dS^T double-buffered (16 KB), dQ staging (16 warps x 2 KB), LSE / delta.
// Warp roles: warps 0-15 softmax / dS (warp w:
// key rows (w & 3)*32.., query columns (w >> 2)*16..; for dQ^T head-dim rows
// (w & 3)*32.. and the same query columns; for the final dK / dV head dims
// (w >> 2)*32..), warp 16 MMA issuer, warp 17 TMA producer.
constexpr int QT128 = 64;  // query rows per tile at head dim 128
constexpr int kB128Tile = TILE * 128 * 2;   // K / V tile bytes (32 KB)
constexpr int kB128QTile = QT128 * 128 * 2; // Q / dO tile bytes (16 KB)
__host__ __device__ constexpr int t_pad128(int T) { return (T + QT128 - 1) / QT128 * QT128; }

template <int FMT>
__global__ void __launch_bounds__(kBwdThreads, 1)
attn_bwd128_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  constexpr int DH = 128;
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sK = base;                     // [128 keys][128] as two 16 KB column blocks
  const uint32_t sV = sK + kB128Tile;
  const uint32_t sQ = sV + kB128Tile;           // 2 stages of [64][128] (two 8 KB blocks)
  const uint32_t sDO = sQ + 2 * kB128QTile;     // 2 stages
  const uint32_t sDS = sDO + 2 * kB128QTile;    // 2 buffers of dS^T [128 keys][64 q] (16 KB)
  const uint32_t sDQ = sDS + 2 * 16384;         // dQ^T staging: 16 warps x [32 rows][16 fp32]
  const uint32_t sStat = sDQ + 32768;           // lse2[2][64], delta[2][64] fp32
  float* lse_s = reinterpret_cast<float*>(gbase + (sStat - base));
  float* del_s = lse_s + 2 * QT128;
  const uint32_t bars = sStat + 1024;
  const uint32_t kv_full = bars;
  auto qdo_full = [&](int s) { return bars + 8u * (1 + s); };
  auto qdo_empty = [&](int s) { return bars + 8u * (3 + s); };
  const uint32_t s_full = bars + 8u * 5;
  const uint32_t s_empty = bars + 8u * 6;
  const uint32_t ds_full = bars + 8u * 7;
  const uint32_t dq_full = bars + 8u * 8;
  const uint32_t dq_empty = bars + 8u * 9;
  const uint32_t acc_full = bars + 8u * 10;
  const uint32_t pt_free = bars + 8u * 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int kt = (int)(blockIdx.x / BH);
  const int bh = (int)(blockIdx.x - kt * BH);
  const int b = bh / p.H, h = bh - b * p.H;
  const int kv0 = kt * TILE;
  const int nq64 = (p.T + QT128 - 1) / QT128;
  const int i0 = p.causal ? kt * (TILE / QT128) : 0;  // first query tile that sees this key tile
  const int n_it = nq64 - i0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(qdo_full(s), 1 + 32);  // TMA bytes + the producer warp's LSE / delta stores
      mbar_init(qdo_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 512);
    mbar_init(ds_full, 512);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 512);
    mbar_init(acc_full, 1);
    mbar_init(pt_free, 1);
    fence_mbar_init();
  }
  if (warp == kBwdWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // q / k / v (and dO, lse, delta) come from earlier kernels on the stream
  const uint32_t tST = tmem, tDPT = tmem + 64, tDV = tmem + 128, tDK = tmem + 256;
  const uint32_t tDQ = tmem + 384, tPT = tmem + 448;

  if (warp == kBwdWarpTma) {
    // ------------------------------------------------ producer (lane 0 issues TMA)
    if (lane == 0) {
      tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV); tma_prefetch_desc(&tmDO);
      mbar_expect_tx(kv_full, 2 * kB128Tile);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_4d(sK + c * 16384, &tmK, kv_full, 64 * c, kv0, h, b);
        tma_load_4d(sV + c * 16384, &tmV, kv_full, 64 * c, kv0, h, b);
      }
    }
    __syncwarp();
    int armed = 0;
    for (int it = 0; it < n_it; ++it) {
      const int st = it & 1;
      const int qq0 = (i0 + it) * QT128;
      if (!mbar_wait_warp(qdo_empty(st), ((it >> 1) & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) break;
      if (lane == 0) {
        mbar_expect_tx(qdo_full(st), 2 * kB128QTile);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(sQ + st * kB128QTile + c * 8192, &tmQ, qdo_full(st), 64 * c, qq0, h, b);
          tma_load_4d(sDO + st * kB128QTile + c * 8192, &tmDO, qdo_full(st), 64 * c, qq0, h, b);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int qi = lane * 2 + i;
        const int q = qq0 + qi;
        const bool v = q < p.T;
        lse_s[st * QT128 + qi] = v ? p.lse[(int64_t)bh * p.T + q] * kLog2e : INFINITY;
        del_s[st * QT128 + qi] = v ? p.delta[(int64_t)bh * p.T + q] : 0.f;
      }
      mbar_arrive(qdo_full(st));
      armed = it + 1;
    }
    if (lane == 0) {
      mbar_wait(kv_full, 0, p.err, FXB_DERR_ATTN_WAIT);
      for (int it = (armed > 2 ? armed - 2 : 0); it < armed; ++it)
        mbar_wait(qdo_full(it & 1), (it >> 1) & 1, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else if (warp == kBwdWarpMma) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t I_SS = umma_idesc_f16(FMT, 0, 0, TILE, QT128);  // S^T, dP^T
      constexpr uint32_t I_KV = umma_idesc_f16(FMT, 0, 1, TILE, DH);     // dV, dK
      constexpr uint32_t I_QT = umma_idesc_f16(FMT, 1, 1, DH, QT128);    // dQ^T
      bool ok = mbar_wait(kv_full, 0, p.err, FXB_DERR_ATTN_WAIT);
      const uint64_t kd = kmajor_desc0(sK), vd = kmajor_desc0(sV);
      const uint64_t km = mnmajor_desc0(sK);  // K^T: head dims (M) contiguous
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        const uint32_t q_s = sQ + st * kB128QTile, do_s = sDO + st * kB128QTile;
        if (!mbar_wait(qdo_full(st), (it >> 1) & 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        if (!mbar_wait(s_empty, (it & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint64_t qd = umma_desc_sw128(q_s, 16, 1024), dod = umma_desc_sw128(do_s, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {  // K slices of 16 head dims; 64-row B tiles: 8 KB blocks
          const uint32_t offb = (kk >> 2) * 8192 + (kk & 3) * 32;
          umma_f16(tST, desc_add(kd, kmajor_off(kk)), desc_add(qd, offb), I_SS, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t offb = (kk >> 2) * 8192 + (kk & 3) * 32;
          umma_f16(tDPT, desc_add(vd, kmajor_off(kk)), desc_add(dod, offb), I_SS, kk > 0);
        }
        umma_commit(s_full);
        return true;
      };
      if (ok && n_it > 0) ok = issue_s(0);
      for (int it = 0; it < n_it && ok; ++it) {
        if (it + 1 < n_it && !issue_s(it + 1)) { ok = false; break; }
        const int st = it & 1;
        const uint32_t q_s = sQ + st * kB128QTile, do_s = sDO + st * kB128QTile;
        if (!mbar_wait(ds_full, it & 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ds_s = sDS + (uint32_t)st * 16384u;
        const uint64_t dsk = kmajor_desc0(ds_s);         // dS^T as A (K = queries, one block)
        const uint64_t dsm = mnmajor_desc0(ds_s);        // dS^T as B (N = queries, MN-major)
        const uint64_t dom = umma_desc_sw128(do_s, 8192, 1024);  // dO as B: N = head dims
        const uint64_t qm = umma_desc_sw128(q_s, 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < QT128 / 16; ++kk)  // dV += P^T dO, A = P^T from tensor memory
          umma_f16_ta(tDV, tPT + kk * 8, desc_add(dom, mnmajor_off(kk)), I_KV, (it > 0 || kk > 0));
        umma_commit(pt_free);
#pragma unroll
        for (int kk = 0; kk < QT128 / 16; ++kk)  // dK += dS^T Q
          umma_f16(tDK, desc_add(dsk, kmajor_off(kk)), desc_add(qm, mnmajor_off(kk)), I_KV,
                   (it > 0 || kk > 0));
        umma_commit(qdo_empty(st));
        if (!mbar_wait(dq_empty, (it & 1) ^ 1, p.err, FXB_DERR_ATTN_WAIT)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk)  // dQ^T = K^T dS^T over the 128 keys
          umma_f16(tDQ, desc_add(km, mnmajor_off(kk)), desc_add(dsm, mnmajor_off(kk)), I_QT, kk > 0);
        umma_commit(dq_full);
      }
      umma_commit(acc_full);
      mbar_wait(acc_full, 0, p.err, FXB_DERR_ATTN_WAIT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax / dS warps 0..15
    const int quarter = warp & 3, part = warp >> 2;
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dK, dV) / head-dim row (dQ^T)
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int qc0 = part * 16;          // this thread's 16 query columns
    bool ok = true;
    auto flush_dq = [&](int it) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full, it & 1, p.err, FXB_DERR_ATTN_WAIT))) return false;
      tc_fence_after();
      const uint32_t stg = sDQ + (uint32_t)warp * 2048u;
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
      const uint32_t row = stg + (uint32_t)lane * 64u;
      uint32_t rr[16];
      tmem_ld16(tDQ + lane_off + qc0, rr);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(row + (uint32_t)((c ^ ((lane >> 1) & 3)) << 4),
                     make_uint4(rr[4 * c], rr[4 * c + 1], rr[4 * c + 2], rr[4 * c + 3]));
      tc_fence_before();
      mbar_arrive(dq_empty);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_3d(&tmDQ, stg, (i0 + it) * QT128 + qc0, quarter * 32, bh);
        bulk_commit();
      }
      return true;
    };
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (i0 + it) * QT128;
      const int sb = it & 1;
      if (!ok) continue;
      if (!__all_sync(0xffffffffu, mbar_wait(qdo_full(sb), (it >> 1) & 1, p.err, FXB_DERR_ATTN_WAIT)) ||
          !__all_sync(0xffffffffu, mbar_wait(s_full, it & 1, p.err, FXB_DERR_ATTN_WAIT))) { ok = false; continue; }
      tc_fence_after();
      const bool diag = p.causal && (q0 < kv0 + TILE);
      uint32_t pw[8], dw[8];
      {
        uint32_t sr[16], dr[16];
        tmem_ld16(tST + lane_off + qc0, sr);
        tmem_ld16(tDPT + lane_off + qc0, dr);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(s_empty);
        const float* ls = lse_s + sb * QT128 + qc0;
        const float* dl = del_s + sb * QT128 + qc0;
#pragma unroll
        for (int qc = 0; qc < 16; qc += 2) {
          float pp[2], dd[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            float e = ex2_ftz(fmaf(__uint_as_float(sr[qc + i]), p.scale_log2, -ls[qc + i]));
            if (kv >= p.T || (diag && q0 + qc0 + qc + i < kv)) e = 0.f;
            pp[i] = e;
            dd[i] = e * (__uint_as_float(dr[qc + i]) - dl[qc + i]);
          }
          pw[qc >> 1] = pack2<T16>(pp[0], pp[1]);
          dw[qc >> 1] = pack2<T16>(dd[0], dd[1]);
        }
      }
      if (it > 0 && !__all_sync(0xffffffffu, mbar_wait(pt_free, (it - 1) & 1, p.err, FXB_DERR_ATTN_WAIT))) {
        ok = false;
        continue;
      }
      tc_fence_after();
      tmem_st8(tPT + lane_off + part * 8, pw);
      uint8_t* ds = gbase + (sDS - base) + (it & 1) * 16384;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int chunk = part * 2 + u;
        *reinterpret_cast<uint4*>(ds + r * 128 + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      if (it > 0 && !flush_dq(it - 1)) { ok = false; continue; }
    }
    if (ok && n_it > 0 && !flush_dq(n_it - 1)) ok = false;
    if (lane == 0) bulk_wait_all0();
    __syncwarp();
    // final dK (scaled) and dV of key row kv, head dims part*32..+32
    if (__all_sync(0xffffffffu, ok && mbar_wait(acc_full, 0, p.err, FXB_DERR_ATTN_WAIT))) {
      tc_fence_after();
      uint32_t rk[32], rv[32];
      tmem_ld32(tDK + lane_off + part * 32, rk);
      tmem_ld32(tDV + lane_off + part * 32, rv);
      tmem_wait_ld();
      if (kv < p.T) {
        T16* krow = static_cast<T16*>(p.dk) + b * p.dk_sb + (int64_t)kv * p.dk_st + h * p.dk_sh + part * 32;
        T16* vrow = static_cast<T16*>(p.dv) + b * p.dv_sb + (int64_t)kv * p.dv_st + h * p.dv_sh + part * 32;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float fk[8], fv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            fk[i] = __uint_as_float(rk[8 * u + i]) * p.scale;
            fv[i] = __uint_as_float(rv[8 * u + i]);
          }
          *reinterpret_cast<uint4*>(krow + 8 * u) = pack8<T16>(fk);
          *reinterpret_cast<uint4*>(vrow + 8 * u) = pack8<T16>(fv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBwdWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq = dq_acc^T * scale in the caller's layout (head dim 128): thread per
// (batch*head, 8-wide head-dim chunk, query), queries fastest so that each of
// the eight strided reads is coalesced across the warp
template <typename T16>
__global__ void attn_bwd128_post_kernel(const float* __restrict__ dqt, T16* __restrict__ dq,
                                        int64_t dq_sb, int64_t dq_st, int64_t dq_sh, float scale,
                                        int B, int T, int H, int Tp) {
  pdl_trigger();
  pdl_wait();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = (int64_t)B * H * 16 * T;
  if (idx >= n) return;
  const int t = (int)(idx % T);
  const int64_t rest = idx / T;
  const int dc = (int)(rest % 16);
  const int bh = (int)(rest / 16);
  const int b = bh / H, h = bh - b * H;
  const float* src = dqt + ((int64_t)bh * 128 + dc * 8) * Tp + t;
  float f[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = src[(int64_t)j * Tp] * scale;
  *reinterpret_cast<uint4*>(dq + b * dq_sb + (int64_t)t * dq_st + h * dq_sh + dc * 8) = pack8<T16>(f);
}

// ============================================================ host side
// Each CTA allocates all 512 TMEM columns, so at most one CTA may be resident
// per SM: the dynamic shared memory request is padded above half of the SM's
// 228 KB so a second CTA of any TMEM-using kernel can never be co-scheduled.
constexpr int kOneCtaPerSm = 120 * 1024;
template <int DH> constexpr int fwd_smem_raw() {
  return (fwd_q_bufs<DH>() + 2 * fwd_kv_stages<DH>()) * TILE * DH * 2 + kFwdXchBytes + 1024 + 256;
}
template <int DH> constexpr int fwd_smem() {
  return fwd_smem_raw<DH>() > kOneCtaPerSm ? fwd_smem_raw<DH>() : kOneCtaPerSm;
}
static_assert(fwd_smem<64>() <= 232448 && fwd_smem<128>() <= 232448, "forward shared memory");
// K, V, QS stages of Q and dO, 2 x dS^T, dQ staging, LSE / delta, align, barriers
constexpr int bwd_smem() { return (2 + 2 * kBwdQS) * TILE * 64 * 2 + 2 * 32768 + 16384 + kBwdQS * 1024 + 1024 + 256; }
static_assert(bwd_smem() <= 232448, "head-dim-64 backward shared memory");
// K, V, Q x2, dO x2, dS^T x2, dQ^T staging, LSE / delta, barriers, alignment
constexpr int bwd128_smem() { return 2 * kB128Tile + 4 * kB128QTile + 2 * 16384 + 32768 + 1024 + 256 + 1024; }
static_assert(bwd128_smem() <= 232448 && bwd128_smem() > kOneCtaPerSm, "head-dim-128 backward shared memory");

int make_map4(CUtensorMap* map, int dtype, const void* ptr, int D, int T, int H, int B,
              int64_t sb, int64_t st, int64_t sh, int box_rows = TILE) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)T, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)st * 2, (uint64_t)sh * 2, (uint64_t)sb * 2};
  uint32_t box[4] = {64, (uint32_t)box_rows, 1, 1};
  CUtensorMapDataType dt =
      dtype == FXB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fxb::encode_tiled(map, dt, 4, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// fp32 dQ accumulator (B*H, T, D) for the backward's TMA add-reductions:
// boxes of 32 rows x 16 columns (64 bytes, 64B swizzle)
int make_map_dq(CUtensorMap* map, float* dq_acc, int D, int T, int BH) {
  uint64_t dims[3] = {(uint64_t)D, (uint64_t)T, (uint64_t)BH};
  uint64_t strides[2] = {(uint64_t)D * 4, (uint64_t)T * D * 4};
  uint32_t box[3] = {16, 32, 1};
  return fxb::encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_acc, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
}

// transposed fp32 dQ accumulator (B*H, 128, Tp) of the head-dim-128
// backward: boxes of 16 queries x 32 head dims (64 bytes, 64B swizzle)
int make_map_dqt(CUtensorMap* map, float* dqt, int Tp, int BH) {
  uint64_t dims[3] = {(uint64_t)Tp, 128, (uint64_t)BH};
  uint64_t strides[2] = {(uint64_t)Tp * 4, (uint64_t)128 * Tp * 4};
  uint32_t box[3] = {16, 32, 1};
  return fxb::encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dqt, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
}

bool strides_ok(int64_t sb, int64_t st, int64_t sh) {
  return sb % 8 == 0 && st % 8 == 0 && sh % 8 == 0 && sb > 0 && st > 0 && sh > 0;
}

int check_args(const fxb_attn_args* a, bool bwd) {
  if (!a) return fxb::set_error(FXB_EINVAL, "attn: args is NULL");
  if (a->dtype != FXB_DTYPE_BF16 && a->dtype != FXB_DTYPE_F16)
    return fxb::set_error(FXB_EINVAL, "attn: dtype %d (bf16, f16 or f32)", a->dtype);
  if (a->D != 64 && a->D != 128)
    return fxb::set_error(FXB_EINVAL, "attn: head_dim %d not supported (64 or 128)", a->D);
  if (a->B < 1 || a->T < 1 || a->H < 1)
    return fxb::set_error(FXB_EINVAL, "attn: bad shape B=%d T=%d H=%d", a->B, a->T, a->H);
  // 1-D grids (the backward launches one CTA per key tile and batch*head)
  if ((int64_t)a->B * a->H * ((a->T + TILE - 1) / TILE) >= (int64_t(1) << 31))
    return fxb::set_error(FXB_EINVAL, "attn: B*H*ceil(T/128) >= 2^31");
  const void* ptrs[4] = {a->q, a->k, a->v, a->o};
  for (const void* q : ptrs)
    if (!q || !fxb::aligned16(q)) return fxb::set_error(FXB_EINVAL, "attn: q/k/v/o must be 16-byte aligned");
  if (!strides_ok(a->q_sb, a->q_st, a->q_sh) || !strides_ok(a->k_sb, a->k_st, a->k_sh) ||
      !strides_ok(a->v_sb, a->v_st, a->v_sh) || !strides_ok(a->o_sb, a->o_st, a->o_sh))
    return fxb::set_error(FXB_EINVAL, "attn: strides must be positive multiples of 8 elements");
  if (!a->lse) return fxb::set_error(FXB_EINVAL, "attn: lse is NULL");
  if (bwd) {
    const void* g[4] = {a->dout, a->dq, a->dk, a->dv};
    for (const void* q : g)
      if (!q || !fxb::aligned16(q)) return fxb::set_error(FXB_EINVAL, "attn bwd: dout/dq/dk/dv alignment");
    if (!strides_ok(a->do_sb, a->do_st, a->do_sh) || !strides_ok(a->dq_sb, a->dq_st, a->dq_sh) ||
        !strides_ok(a->dk_sb, a->dk_st, a->dk_sh) || !strides_ok(a->dv_sb, a->dv_st, a->dv_sh))
      return fxb::set_error(FXB_EINVAL, "attn bwd: strides must be positive multiples of 8");
    if (!a->workspace || !fxb::aligned16(a->workspace))
      return fxb::set_error(FXB_EINVAL, "attn bwd: workspace NULL or misaligned");
  }
  return FXB_OK;
}

// FXB_ATTN_FWD=1 selects the one-tile forward at head dim 64 (A/B tests)
bool fwd_one_tile() {
  static const bool v = [] {
    const char* e = getenv("FXB_ATTN_FWD");
    return e && e[0] == '1';
  }();
  return v;
}

template <typename K> int set_smem(K k, int bytes) {
  return fxb::check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                         "attn smem attribute");
}

constexpr int fwd2_smem() { return (4 + 2 * kFwd2KS) * kFwd2Tile + 1024 + 512; }
static_assert(fwd2_smem() <= 232448 && fwd2_smem() > kOneCtaPerSm, "two-tile forward shared memory");

template <int DH, int FMT>
int launch_fwd(const fxb_attn_args* a, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  int r;
  if ((r = make_map4(&mq, a->dtype, a->q, DH, a->T, a->H, a->B, a->q_sb, a->q_st, a->q_sh))) return r;
  if ((r = make_map4(&mk, a->dtype, a->k, DH, a->T, a->H, a->B, a->k_sb, a->k_st, a->k_sh))) return r;
  if ((r = make_map4(&mv, a->dtype, a->v, DH, a->T, a->H, a->B, a->v_sb, a->v_st, a->v_sh))) return r;
  FwdParams p;
  p.B = a->B; p.T = a->T; p.H = a->H;
  p.nqt = (a->T + TILE - 1) / TILE;
  p.nkt = p.nqt;
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->scale * kLog2e;
  p.o = a->o; p.o_sb = a->o_sb; p.o_st = a->o_st; p.o_sh = a->o_sh;
  p.lse = a->lse;
  p.err = fxb::dev_error_ptr();
  if (!p.err) return FXB_ECUDA;
  int dev = 0;
  cudaGetDevice(&dev);
  if (DH == 64 && !fwd_one_tile()) {
    // two query tiles per CTA (attn_fwd2_kernel)
    auto k2 = attn_fwd2_kernel<FMT>;
    static bool once2[64] = {false};
    if (!once2[dev & 63]) {
      if ((r = set_smem(k2, fwd2_smem()))) return r;
      once2[dev & 63] = true;
    }
    const int64_t items = (int64_t)((p.nqt + 1) / 2) * a->B * a->H;
    const int grid = (int)(items < fxb::num_sms() ? items : fxb::num_sms());
    fxb::pdl_launch(k2, grid, kFwd2Threads, fwd2_smem(), st, mq, mk, mv, p);
    return fxb::check_launch("attn_fwd2");
  }
  auto k = attn_fwd_kernel<DH, FMT>;
  static bool once[64] = {false};
  if (!once[dev & 63]) {
    if ((r = set_smem(k, fwd_smem<DH>()))) return r;
    once[dev & 63] = true;
  }
  const int64_t items = (int64_t)p.nqt * a->B * a->H;
  const int grid = (int)(items < fxb::num_sms() ? items : fxb::num_sms());
  fxb::pdl_launch(k, grid, kFwdThreads, fwd_smem<DH>(), st, mq, mk, mv, p);
  return fxb::check_launch("attn_fwd");
}

template <int FMT>
int launch_bwd128(const fxb_attn_args* a, cudaStream_t st) {
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  constexpr int DH = 128;
  const int64_t rows = (int64_t)a->B * a->H * a->T;
  const int Tp = t_pad128(a->T);
  float* delta = a->workspace;
  float* dqt = a->workspace + ((rows + 3) / 4) * 4;
  int r = fxb::check_cuda(cudaMemsetAsync(dqt, 0, (size_t)a->B * a->H * DH * Tp * sizeof(float), st),
                          "attn bwd: clear dQ accumulator");
  if (r) return r;
  fxb::pdl_launch(attn_bwd_prep_kernel<T16, DH>, (unsigned)((rows * (DH / 8) + 255) / 256), 256, 0, st,
      static_cast<const T16*>(a->o), a->o_sb, a->o_st, a->o_sh, static_cast<const T16*>(a->dout),
      a->do_sb, a->do_st, a->do_sh, delta, static_cast<float*>(nullptr), a->B, a->T, a->H);
  if ((r = fxb::check_launch("attn_bwd_prep"))) return r;
  CUtensorMap mq, mk, mv, mdo, mdq;
  if ((r = make_map4(&mq, a->dtype, a->q, DH, a->T, a->H, a->B, a->q_sb, a->q_st, a->q_sh, QT128))) return r;
  if ((r = make_map4(&mk, a->dtype, a->k, DH, a->T, a->H, a->B, a->k_sb, a->k_st, a->k_sh))) return r;
  if ((r = make_map4(&mv, a->dtype, a->v, DH, a->T, a->H, a->B, a->v_sb, a->v_st, a->v_sh))) return r;
  if ((r = make_map4(&mdo, a->dtype, a->dout, DH, a->T, a->H, a->B, a->do_sb, a->do_st, a->do_sh, QT128)))
    return r;
  if ((r = make_map_dqt(&mdq, dqt, Tp, a->B * a->H))) return r;
  BwdParams p;
  p.B = a->B; p.T = a->T; p.H = a->H;
  p.nqt = (a->T + TILE - 1) / TILE;
  p.nkt = p.nqt;
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->scale * kLog2e;
  p.scale = a->scale;
  p.lse = a->lse;
  p.delta = delta;
  p.dq_acc = dqt;
  p.dk = a->dk; p.dk_sb = a->dk_sb; p.dk_st = a->dk_st; p.dk_sh = a->dk_sh;
  p.dv = a->dv; p.dv_sb = a->dv_sb; p.dv_st = a->dv_st; p.dv_sh = a->dv_sh;
  p.err = fxb::dev_error_ptr();
  if (!p.err) return FXB_ECUDA;
  auto k = attn_bwd128_kernel<FMT>;
  static bool once[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!once[dev & 63]) {
    if ((r = set_smem(k, bwd128_smem()))) return r;
    once[dev & 63] = true;
  }
  fxb::pdl_launch(k, dim3((unsigned)(p.nkt * a->B * a->H)), kBwdThreads, bwd128_smem(), st, mq, mk, mv,
                  mdo, mdq, p);
  if ((r = fxb::check_launch("attn_bwd128"))) return r;
  const int64_t n = (int64_t)a->B * a->H * 16 * a->T;
  fxb::pdl_launch(attn_bwd128_post_kernel<T16>, (unsigned)((n + 255) / 256), 256, 0, st, dqt,
                  static_cast<T16*>(a->dq), a->dq_sb, a->dq_st, a->dq_sh, a->scale, a->B, a->T, a->H, Tp);
  return fxb::check_launch("attn_bwd128_post");
}

template <int FMT>
int launch_bwd(const fxb_attn_args* a, cudaStream_t st) {
  using T16 = typename std::conditional<FMT == 1, __nv_bfloat16, __half>::type;
  constexpr int DH = 64;
  const int64_t rows = (int64_t)a->B * a->H * a->T;
  float* delta = a->workspace;
  float* dq_acc = a->workspace + ((rows + 3) / 4) * 4;
  fxb::pdl_launch(attn_bwd_prep_kernel<T16, DH>, (unsigned)((rows * (DH / 8) + 255) / 256), 256, 0, st, 
      static_cast<const T16*>(a->o), a->o_sb, a->o_st, a->o_sh, static_cast<const T16*>(a->dout),
      a->do_sb, a->do_st, a->do_sh, delta, dq_acc, a->B, a->T, a->H);
  int r = fxb::check_launch("attn_bwd_prep");
  if (r) return r;
  CUtensorMap mq, mk, mv, mdo;
  if ((r = make_map4(&mq, a->dtype, a->q, DH, a->T, a->H, a->B, a->q_sb, a->q_st, a->q_sh))) return r;
  if ((r = make_map4(&mk, a->dtype, a->k, DH, a->T, a->H, a->B, a->k_sb, a->k_st, a->k_sh))) return r;
  if ((r = make_map4(&mv, a->dtype, a->v, DH, a->T, a->H, a->B, a->v_sb, a->v_st, a->v_sh))) return r;
  if ((r = make_map4(&mdo, a->dtype, a->dout, DH, a->T, a->H, a->B, a->do_sb, a->do_st, a->do_sh))) return r;
  CUtensorMap mdq;
  if ((r = make_map_dq(&mdq, dq_acc, DH, a->T, a->B * a->H))) return r;
  BwdParams p;
  p.B = a->B; p.T = a->T; p.H = a->H;
  p.nqt = (a->T + TILE - 1) / TILE;
  p.nkt = p.nqt;
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->scale * kLog2e;
  p.scale = a->scale;
  p.lse = a->lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = a->dk; p.dk_sb = a->dk_sb; p.dk_st = a->dk_st; p.dk_sh = a->dk_sh;
  p.dv = a->dv; p.dv_sb = a->dv_sb; p.dv_st = a->dv_st; p.dv_sh = a->dv_sh;
  p.err = fxb::dev_error_ptr();
  if (!p.err) return FXB_ECUDA;
  auto k = attn_bwd_kernel<FMT>;
  static bool once[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!once[dev & 63]) {
    if ((r = set_smem(k, bwd_smem()))) return r;
    once[dev & 63] = true;
  }
  const int items = p.nkt * a->B * a->H;
  dim3 grid((unsigned)(items < fxb::num_sms() ? items : fxb::num_sms()));  // persistent
  fxb::pdl_launch(k, grid, kBwd64Threads, bwd_smem(), st, mq, mk, mv, mdo, mdq, p);
  if ((r = fxb::check_launch("attn_bwd"))) return r;
  const int64_t n = rows * (DH / 8);
  fxb::pdl_launch(attn_bwd_post_kernel<T16, DH>, (unsigned)((n + 255) / 256), 256, 0, st, 
      dq_acc, static_cast<T16*>(a->dq), a->dq_sb, a->dq_st, a->dq_sh, a->scale, a->B, a->T, a->H);
  return fxb::check_launch("attn_bwd_post");
}

}  // namespace

namespace fxb {
int attn_fwd_f32(const fxb_attn_args* a, cudaStream_t st);  // csrc/attn_f32.cu
int attn_bwd_f32(const fxb_attn_args* a, cudaStream_t st);
}

extern "C" {

int fxb_attn_fwd(const fxb_attn_args* a, void* stream) {
  if (a && a->dtype == FXB_DTYPE_F32) return fxb::attn_fwd_f32(a, fxb::as_stream(stream));
  int r = check_args(a, false);
  if (r) return r;
  cudaStream_t st = fxb::as_stream(stream);
  if (a->dtype == FXB_DTYPE_BF16)
    return a->D == 64 ? launch_fwd<64, 1>(a, st) : launch_fwd<128, 1>(a, st);
  return a->D == 64 ? launch_fwd<64, 0>(a, st) : launch_fwd<128, 0>(a, st);
}

size_t fxb_attn_bwd_workspace(int32_t B, int32_t T, int32_t H, int32_t D) {
  if (B < 1 || T < 1 || H < 1 || D < 1) return 0;
  const int64_t rows = (int64_t)B * H * T;
  // delta, then the fp32 dQ accumulator: (B*H, T, D), or at head dim 128 the
  // transposed (B*H, 128, T rounded up to 64)
  const int64_t acc = D == 128 ? (int64_t)B * H * 128 * t_pad128(T) : rows * D;
  return (size_t)(((rows + 3) / 4) * 4 + acc) * sizeof(float);
}

int fxb_attn_bwd(const fxb_attn_args* a, void* stream) {
  if (a && a->dtype == FXB_DTYPE_F32) return fxb::attn_bwd_f32(a, fxb::as_stream(stream));
  int r = check_args(a, true);
  if (r) return r;
  cudaStream_t st = fxb::as_stream(stream);
  if (a->D == 128) return a->dtype == FXB_DTYPE_BF16 ? launch_bwd128<1>(a, st) : launch_bwd128<0>(a, st);
  return a->dtype == FXB_DTYPE_BF16 ? launch_bwd<1>(a, st) : launch_bwd<0>(a, st);
}

}  // extern "C"
