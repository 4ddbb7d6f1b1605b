// tcgen05 / TMEM GEMM for sm_100a with TMA-fed operands and fused epilogues.
//
//   C[m, n] = epilogue( sum_k A[m, k] * B[n, k] )
//
// Replaces the rocBLAS matmuls of the reference hot path (nn.Linear in
// ml/fxlm/model.py:48-51, torch.mm in ml/fxlm/cross_entropy.py:131-135 and
// ml/fxgpu/fused_linear.py:94). Design (B200-first, no reference analogue):
//   - persistent CTAs (one per SM), static tile schedule grouped along M for
//     L2 reuse; optional split-K for skinny outputs (dW), reduced with fp32
//     TMA add-reductions into the destination;
//   - warp 0: TMA producer (128B-swizzled boxes, no multicast), warp 1: MMA
//     issuer (one thread, tcgen05.mma cta_group::1 M=128 N=BN K=16) and TMEM
//     owner, warps 2-9: epilogue (tcgen05.ld 32x32b -> fused op -> 64B-swizzled
//     staging in shared memory -> TMA store / add-reduction, so global writes
//     are whole coalesced boxes issued asynchronously);
//   - STAGES-deep smem ring (full/empty mbarriers), two TMEM accumulators so
//     the epilogue of tile i overlaps the mainloop of tile i+1;
//   - operands K-major or MN-major (transposed) so forward, dX and dW GEMMs
//     all read their operands in place.
// Every mbarrier wait is bounded (common.cuh); on expiry the kernel records
// FXB_DERR_GEMM_WAIT, drains what it issued and frees its tensor memory.
#include <cstdlib>
#include "common.cuh"
#include "internal.h"

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
// Per-epilogue-warp output staging: two 2 KB buffers after the operand ring;
// the warp's lane 0 issues the TMA stores (or fp32 add-reductions) and owns
// their bulk groups.
constexpr int kEpiWarpBytes = 4096;
constexpr int kEpiBytes = 8 * kEpiWarpBytes;

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, num_kb;
  int epi;
  int c_dtype;
  float alpha;
  void* C;
  int64_t ldc;
  const void* R;
  int64_t ldr;
  void* Z;
  int64_t ldz;
  const void* bias;
  int* err;
};

template <int BN> struct Cfg {
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + kEpiBytes + 1024 /*align*/ + 256 /*barriers*/;
};

FXB_DEV void tile_coords(int unit, const GemmParams& p, int& tm, int& tn, int& split) {
  const int tiles = p.tiles_m * p.tiles_n;
  split = unit / tiles;
  int t = unit - split * tiles;
  constexpr int G = 8;  // group of M tiles sharing B tiles in L2
  const int per_group = G * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * G;
  int gs = p.tiles_m - first_m;
  if (gs > G) gs = G;
  const int r = t - g * per_group;
  tm = first_m + r % gs;
  tn = r / gs;
}

// ---------------------------------------------------------------- epilogue helpers
// The epilogue works on 16-column pieces of one row per lane: v[16] holds the
// accumulator values, n8 (0..2) counts the piece's valid groups of 8 columns
// (N % 8 == 0).
FXB_DEV float silu_f(float x) { return x / (1.f + __expf(-x)); }

// 16 values of row p (first n8 groups of 8; the rest zero)
template <typename T> FXB_DEV void load16_part(const T* p, float* f, int n8) {
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = 0.f;
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (q < 2 * n8) {
        float4 u = reinterpret_cast<const float4*>(p)[q];
        f[4 * q] = u.x; f[4 * q + 1] = u.y; f[4 * q + 2] = u.z; f[4 * q + 3] = u.w;
      }
  } else {
#pragma unroll
    for (int q = 0; q < 2; ++q)
      if (q < n8) unpack8<T>(reinterpret_cast<const uint4*>(p)[q], f + 8 * q);
  }
}

// epilogues that read a second (m, n) input from R
FXB_DEV bool epi_reads_r(int epi) {
  return epi == FXB_EPI_RESIDUAL || epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU;
}
// epilogues that also write the rounded pre-activation to Z (when Z is given)
FXB_DEV bool epi_writes_z(const GemmParams& p) {
  return p.Z && (p.epi == FXB_EPI_GELU || p.epi == FXB_EPI_BIAS_GELU || p.epi == FXB_EPI_BIAS_SILU);
}

// Issue the loads of one 32-column chunk of R (16-bit) into registers; called
// before the accumulator is ready so that their latency overlaps the mainloop.
FXB_DEV void prefetch_r16(const GemmParams& p, int m, int n0, uint4* pre) {
  const int n8 = min(4, (p.N - n0) >> 3);
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.R) +
                                                    (int64_t)m * p.ldr + n0);
#pragma unroll
  for (int q = 0; q < 4; ++q) pre[q] = (q < n8) ? src[q] : make_uint4(0, 0, 0, 0);
}

// R values of one 16-column piece: from the prefetched registers (16-bit C),
// loaded now (fp32 C), or zero for rows past M (their results are clipped by
// the store)
template <typename CT>
FXB_DEV void piece_r(const GemmParams& p, int m, int n0, int n8, bool use_pre, const uint4* pre2,
                     float* r) {
  if constexpr (sizeof(CT) == 2) {
    if (use_pre) {
      unpack8<CT>(pre2[0], r);
      unpack8<CT>(pre2[1], r + 8);
      return;
    }
  }
  if (m < p.M) {
    load16_part<CT>(static_cast<const CT*>(p.R) + (int64_t)m * p.ldr + n0, r, n8);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = 0.f;
  }
}

// Epilogue arithmetic of one 16-column piece of row m, in place on v: the
// value written to C (or added to it, FXB_EPI_ACCUM_F32). z receives the
// rounded pre-activation of the epilogues that also write Z.
template <typename CT>
FXB_DEV void epilogue_math(const GemmParams& p, int m, int n0, int n8, float* v, float* z,
                           bool use_pre, const uint4* pre2) {
  if constexpr (sizeof(CT) == 4) {
    // fp32 C: store, accumulate, residual and bias only (the host rejects the
    // activation epilogues), which keeps this instantiation small
    if (p.epi == FXB_EPI_RESIDUAL) {
      piece_r<CT>(p, m, n0, n8, false, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = v[i] * p.alpha + z[i];
    } else if (p.epi == FXB_EPI_BIAS) {
      load16_part<CT>(static_cast<const CT*>(p.bias) + n0, z, n8);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += z[i];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= p.alpha;
    }
    return;
  }
  switch (p.epi) {
    case FXB_EPI_RESIDUAL: {
      piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = v[i] * p.alpha + z[i];
      break;
    }
    case FXB_EPI_GELU:
    case FXB_EPI_BIAS_GELU:
    case FXB_EPI_BIAS_SILU:
    case FXB_EPI_BIAS: {
      if (p.epi != FXB_EPI_GELU) {
        load16_part<CT>(static_cast<const CT*>(p.bias) + n0, z, n8);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] += z[i];
      }
      if (p.epi == FXB_EPI_BIAS) break;
      // round the pre-activation once; the activation is computed from the
      // stored value so that backward (which reads Z) sees the same input
      if constexpr (sizeof(CT) == 2) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {  // paired conversions
          const float2 f = unpack2<CT>(pack2<CT>(v[i], v[i + 1]));
          z[i] = f.x;
          z[i + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) z[i] = v[i];
      }
      if (p.epi == FXB_EPI_BIAS_SILU) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = silu_f(z[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = gelu_tanh(z[i]);
      }
      break;
    }
    case FXB_EPI_DGELU: {
      piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= gelu_tanh_grad(z[i]);
      break;
    }
    case FXB_EPI_DSILU: {
      piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float s = 1.f / (1.f + __expf(-z[i]));
        v[i] *= s * (1.f + z[i] * (1.f - s));
      }
      break;
    }
    default: {  // FXB_EPI_STORE, FXB_EPI_ACCUM_F32
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= p.alpha;
    }
  }
}

// Staging buffers: 32 rows x 64 bytes (one row per lane) in the layout of a
// 64-byte-swizzled TMA box: 16-byte chunk q of row r sits at q ^ ((r >> 1) & 3),
// which also keeps each quarter-warp's 16-byte stores on distinct banks.
// stage_piece writes 16 values of row `lane`: 16-byte chunks 2h, 2h+1 of the
// row for 16-bit types, the whole 64-byte row for fp32 (h unused).
template <typename CT> FXB_DEV void stage_piece(uint32_t buf, int lane, int h, const float* f) {
  const uint32_t row = buf + (uint32_t)lane * 64u;
  const int sw = (lane >> 1) & 3;
  if constexpr (sizeof(CT) == 4) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      st_shared_v4(row + (uint32_t)((q ^ sw) << 4),
                   make_uint4(__float_as_uint(f[4 * q]), __float_as_uint(f[4 * q + 1]),
                              __float_as_uint(f[4 * q + 2]), __float_as_uint(f[4 * q + 3])));
  } else {
#pragma unroll
    for (int q = 0; q < 2; ++q)
      st_shared_v4(row + (uint32_t)(((2 * h + q) ^ sw) << 4), pack8<CT>(f + 8 * q));
  }
}

// before writing a staging buffer: the group that last used it has been read
// (all groups when both buffers are rewritten, else all but the newest)
FXB_DEV void stage_begin(int lane, bool both) {
  if (lane == 0) {
    if (both) bulk_wait_read0();
    else bulk_wait_read1();
  }
  __syncwarp();
}

// Issue the staged pieces (rows y..y+31): buffer 0 to map0 at column x0 and,
// when map1 is given, buffer 1 to map1 at x1. TMA clips rows >= M and
// columns >= N.
FXB_DEV void stage_issue(const CUtensorMap* map0, int x0, const CUtensorMap* map1, int x1, int y,
                         bool reduce, uint32_t sbuf, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) {
      tma_reduce_add_2d(map0, sbuf, x0, y);
      if (map1) tma_reduce_add_2d(map1, sbuf + 2048, x1, y);
    } else {
      tma_store_2d(map0, sbuf, x0, y);
      if (map1) tma_store_2d(map1, sbuf + 2048, x1, y);
    }
    bulk_commit();
  }
}

// One epilogue warp's share of an accumulator tile. The warp reads TMEM lanes
// of its quarter (row m for this lane; rows m0..m0+31 for the warp) and the
// columns [half*BN/2, (half+1)*BN/2) of the tile, i.e. NCH = BN/64 chunks of
// 32 columns, and writes them through its staging buffers.
template <int BN>
struct EpiWarp {
  static constexpr int NCH = BN / 64;
  // R (16-bit) of two chunks in flight, as a ring that runs across tiles:
  // chunk c of a tile sits in slot c & 1; once chunk c is done its slot is
  // refilled with chunk c + 2, or with chunk c + 2 - NCH of the warp's next
  // tile (NCH is even), so the next tile's first chunks load during this one.
  uint4 pre[2][4];
  bool pre_ok[2];  // slot holds R of a row inside M (16-bit C, R-reading epilogue)

  FXB_DEV void fill(const GemmParams& p, int slot, int m, int n0) {
    pre_ok[slot] = epi_reads_r(p.epi) && p.c_dtype != FXB_DTYPE_F32 && m < p.M;
    if (pre_ok[slot] && n0 < p.N) prefetch_r16(p, m, n0, pre[slot]);
  }
  // chunks 0 and 1 of the warp's first tile
  FXB_DEV void prefetch(const GemmParams& p, int m, int ntile0, int half) {
#pragma unroll
    for (int c = 0; c < 2; ++c) fill(p, c, m, ntile0 + (half * NCH + c) * 32);
  }

  // one 16-column piece: accumulator values (already loaded from tensor
  // memory) -> epilogue math
  template <typename CT>
  FXB_DEV int piece(const GemmParams& p, int m, int n0, const uint32_t* r, int slot,
                    const uint4* pre2, float* v, float* z) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
    const int n8 = max(0, min(2, (p.N - n0) >> 3));
    epilogue_math<CT>(p, m, n0, n8, v, z, sizeof(CT) == 2 && pre_ok[slot], pre2);
    return n8;
  }

  // Staging: an epilogue that writes only C alternates between the warp's two
  // 2 KB buffers (one bulk group per piece, so a piece waits only for the
  // group before last to have been read); one that also writes Z uses both
  // buffers for every piece and waits for the previous group.
  template <typename CT>
  FXB_DEV void chunk(const GemmParams& p, const CUtensorMap* tmC, const CUtensorMap* tmZ, int m,
                     int m0, int n0, uint32_t taddr, int cc, uint32_t sbuf, int lane,
                     uint32_t& cnt) {
    const bool wz = epi_writes_z(p);
    float v[16], z[16];
    uint32_t acc[32];  // the chunk's 32 accumulator columns: one tensor-memory load
    tmem_ld32(taddr, acc);
    tmem_wait_ld();
    if constexpr (sizeof(CT) == 2) {
      const uint32_t b = wz ? sbuf : sbuf + (cnt & 1u) * 2048u;
      stage_begin(lane, wz);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        piece<CT>(p, m, n0 + 16 * h, acc + 16 * h, cc & 1, &pre[cc & 1][2 * h], v, z);
        stage_piece<CT>(b, lane, h, v);
        if (wz) stage_piece<CT>(sbuf + 2048, lane, h, z);
      }
      stage_issue(tmC, n0, wz ? tmZ : nullptr, n0, m0, false, b, lane);
      ++cnt;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n8 = piece<CT>(p, m, n0 + 16 * h, acc + 16 * h, cc & 1, &pre[cc & 1][2 * h], v, z);
        if (n8 == 0) continue;  // warp-uniform
        const uint32_t b = wz ? sbuf : sbuf + (cnt & 1u) * 2048u;
        stage_begin(lane, wz);
        stage_piece<CT>(b, lane, 0, v);
        if (wz) stage_piece<CT>(sbuf + 2048, lane, 0, z);
        stage_issue(tmC, n0 + 16 * h, wz ? tmZ : nullptr, n0 + 16 * h, m0,
                    p.epi == FXB_EPI_ACCUM_F32, b, lane);
        ++cnt;
      }
    }
  }

  // m_next / ntile0_next: this warp's row and first column in its next tile
  // (has_next false when there is none)
  FXB_DEV void run(const GemmParams& p, const CUtensorMap* tmC, const CUtensorMap* tmZ, int m,
                   int m0, int ntile0, int half, uint32_t tbase, uint32_t sbuf, int lane,
                   uint32_t& cnt, bool has_next, int m_next, int ntile0_next) {
    // unrolled by the prefetch ring's period (two chunks) only: the chunk
    // body is large, and the instruction cache is shared with the MMA warp
#pragma unroll 1
    for (int cp = 0; cp < NCH; cp += 2)
#pragma unroll
    for (int ci = 0; ci < 2; ++ci) {
      const int cc = cp + ci;
      const int c = half * NCH + cc;
      const int n0 = ntile0 + c * 32;
      if (n0 < p.N) {  // warp-uniform
        const uint32_t taddr = tbase + c * 32;
        switch (p.c_dtype) {
          case FXB_DTYPE_BF16: chunk<__nv_bfloat16>(p, tmC, tmZ, m, m0, n0, taddr, ci, sbuf, lane, cnt); break;
          case FXB_DTYPE_F16: chunk<__half>(p, tmC, tmZ, m, m0, n0, taddr, ci, sbuf, lane, cnt); break;
          default: chunk<float>(p, tmC, tmZ, m, m0, n0, taddr, ci, sbuf, lane, cnt); break;
        }
      }
      if (cc + 2 < NCH) fill(p, ci, m, n0 + 64);
      else if (has_next) fill(p, ci, m_next, ntile0_next + (half * NCH + cc + 2 - NCH) * 32);
    }
  }
};

// ---------------------------------------------------------------- kernel
template <int BN, bool A_MN, bool B_MN, int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmZ,
               const GemmParams p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 1024B aligned for 128B swizzle
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;  // output staging
  const uint32_t bar0 = epi0 + kEpiBytes;
  // barrier layout: full[S], empty[S], tfull[2], tempty[2], final, then tmem slot
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * C::STAGES + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * C::STAGES + 2 + b); };
  const uint32_t final_bar = bar0 + 8u * (2 * C::STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bar0 - base) + 8 * (2 * C::STAGES + 5));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 8);  // one arrival per epilogue warp
    }
    mbar_init(final_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // operands come from the previous kernel on the stream

  const int total_units = p.tiles_m * p.tiles_n * p.splits;
  constexpr uint32_t IDESC = umma_idesc_f16(AB_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, BM, BN);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;          // bit s: stage s armed at least once
      uint32_t armed_parity = 0;   // bit s: parity of the last arming of stage s
      bool ok = true;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x) {
        int tm, tn, split;
        tile_coords(unit, p, tm, tn, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
          const uint32_t sa = base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          mbar_expect_tx(full_bar(stage), C::STAGE_BYTES);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_2d(sa, &tmA, full_bar(stage), tm * BM, k0);
            tma_load_2d(sa + 8192, &tmA, full_bar(stage), tm * BM + 64, k0);
          } else {
            tma_load_2d(sa, &tmA, full_bar(stage), k0, tm * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192, &tmB, full_bar(stage), tn * BN + 64 * j, k0);
          } else {
            tma_load_2d(sb, &tmB, full_bar(stage), k0, tn * BN);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every copy this thread issued has landed before smem goes away
      for (int s = 0; s < C::STAGES; ++s)
        if (armed & (1u << s)) mbar_wait(full_bar(s), (armed_parity >> s) & 1u, p.err, FXB_DERR_GEMM_WAIT);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x) {
        int tm, tn, split;
        tile_coords(unit, p, tm, tn, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        if (!mbar_wait(tempty_bar(abuf), aphase ^ 1, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + abuf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const uint64_t ad0 = A_MN ? umma_desc_sw128(sa, 8192, 1024) : umma_desc_sw128(sa, 16, 1024);
          const uint64_t bd0 = B_MN ? umma_desc_sw128(sb, 8192, 1024) : umma_desc_sw128(sb, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16(dcol, desc_add(ad0, A_MN ? kk * 2048 : kk * 32),
                     desc_add(bd0, B_MN ? kk * 2048 : kk * 32), IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit(empty_bar(stage));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull_bar(abuf));
        if (++abuf == 2) { abuf = 0; aphase ^= 1; }
      }
      // all MMAs issued by this thread complete before TMEM is released
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, p.err, FXB_DERR_GEMM_WAIT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2..9)
    // two warps per TMEM lane quarter, each taking half of the tile's columns
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t sbuf = epi0 + (uint32_t)(warp - 2) * kEpiWarpBytes;
    uint32_t ecnt = 0;  // staging pieces issued by this warp (buffer alternation)
    int abuf = 0;
    uint32_t aphase = 0;
    EpiWarp<BN> ew;
    if ((int)blockIdx.x < total_units) {
      int tm, tn, split;
      tile_coords(blockIdx.x, p, tm, tn, split);
      ew.prefetch(p, tm * BM + row_in_tile, tn * BN, half);
    }
    for (int unit = blockIdx.x; unit < total_units; unit += gridDim.x) {
      int tm, tn, split;
      tile_coords(unit, p, tm, tn, split);
      const int m = tm * BM + row_in_tile;
      const int next = unit + gridDim.x;
      int ntm = 0, ntn = 0, nsplit;
      if (next < total_units) tile_coords(next, p, ntm, ntn, nsplit);
      if (!mbar_wait(tfull_bar(abuf), aphase, p.err, FXB_DERR_GEMM_WAIT)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN;
      ew.run(p, &tmC, &tmZ, m, tm * BM + quarter * 32, tn * BN, half, tbase, sbuf, lane, ecnt,
             next < total_units, ntm * BM + row_in_tile, ntn * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(abuf));
      if (++abuf == 2) { abuf = 0; aphase ^= 1; }
    }
    if (lane == 0) bulk_wait_all0();  // stores done before the staging smem goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- 2-SM kernel
// CTA pair (cluster of 2) computing 256 x BN tiles with tcgen05.mma
// cta_group::2: each CTA loads its own 128 rows of A and its half (BN/2 rows)
// of B with plain (non-multicast) TMA whose completion is counted on the
// leader CTA's full barrier; the leader's single MMA thread reads both CTAs'
// shared memory and writes both CTAs' tensor memory, and commits to the
// barriers of both CTAs (tcgen05.commit multicast). Shared-memory operand
// traffic per SM is half of the 1-SM kernel's for the same tile width, which
// is what lets the tensor pipe run at full rate.
template <int BN> struct Cfg2 {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + kEpiBytes + 1024 + 256;
};

FXB_DEV void tile_coords2(int unit, const GemmParams& p, int& tm, int& tn, int& split) {
  tile_coords(unit, p, tm, tn, split);  // tm counts 256-row tiles here
}

template <int BN, bool A_MN, bool B_MN, int AB_FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmZ,
                const GemmParams p) {
  using C = Cfg2<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;  // output staging
  const uint32_t bar0 = epi0 + kEpiBytes;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * C::STAGES + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * C::STAGES + 2 + b); };
  const uint32_t final_bar = bar0 + 8u * (2 * C::STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bar0 - base) + 8 * (2 * C::STAGES + 5));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader (issues the MMAs)
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 16);  // 8 epilogue warps x 2 CTAs
    }
    mbar_init(final_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and tensor memory allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // operands come from the previous kernel on the stream

  const int total_units = p.tiles_m * p.tiles_n * p.splits;
  constexpr uint32_t IDESC = umma_idesc_f16(AB_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, 256, BN);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      bool ok = true;
      for (int unit = pair; unit < total_units && ok; unit += npairs) {
        int tm, tn, split;
        tile_coords2(unit, p, tm, tn, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int arow = tm * 256 + (int)rank * 128;
        const int brow = tn * BN + (int)rank * (BN / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
          const uint32_t sa = base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t fb = mapa_shared(full_bar(stage), 0);
          if (rank == 0) {
            mbar_expect_tx(full_bar(stage), 2 * C::STAGE_BYTES);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_2d_pair(sa, &tmA, fb, arow, k0);
            tma_load_2d_pair(sa + 8192, &tmA, fb, arow + 64, k0);
          } else {
            tma_load_2d_pair(sa, &tmA, fb, k0, arow);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d_pair(sb + j * 8192, &tmB, fb, brow + 64 * j, k0);
          } else {
            tma_load_2d_pair(sb, &tmB, fb, k0, brow);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // the leader's full barriers count both CTAs' bytes: draining them
      // means every copy of the pair has landed
      if (rank == 0)
        for (int s = 0; s < C::STAGES; ++s)
          if (armed & (1u << s)) mbar_wait(full_bar(s), (armed_parity >> s) & 1u, p.err, FXB_DERR_GEMM_WAIT);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0) {
      if (rank == 0) {
        int stage = 0;
        uint32_t phase = 0;
        int abuf = 0;
        uint32_t aphase = 0;
        bool ok = true;
        for (int unit = pair; unit < total_units && ok; unit += npairs) {
          int tm, tn, split;
          tile_coords2(unit, p, tm, tn, split);
          const int kb0 = split * p.kb_per_split;
          const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
          if (!mbar_wait(tempty_bar(abuf), aphase ^ 1, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dcol = tmem_base + abuf * BN;
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(full_bar(stage), phase, p.err, FXB_DERR_GEMM_WAIT)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = base + stage * C::STAGE_BYTES;
            const uint32_t sb = sa + C::A_BYTES;
            const uint64_t ad0 = A_MN ? umma_desc_sw128(sa, 8192, 1024) : umma_desc_sw128(sa, 16, 1024);
            const uint64_t bd0 = B_MN ? umma_desc_sw128(sb, 8192, 1024) : umma_desc_sw128(sb, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_f16_pair(dcol, desc_add(ad0, A_MN ? kk * 2048 : kk * 32),
                            desc_add(bd0, B_MN ? kk * 2048 : kk * 32), IDESC,
                            (kb > kb0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(empty_bar(stage), 0x3);
            if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          umma_commit_pair(tfull_bar(abuf), 0x3);
          if (++abuf == 2) { abuf = 0; aphase ^= 1; }
        }
        // completes (in both CTAs) once every MMA of the pair is done
        umma_commit_pair(final_bar, 0x3);
      }
      mbar_wait(final_bar, 0, p.err, FXB_DERR_GEMM_WAIT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2..9, both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = (int)rank * 128 + quarter * 32 + lane;
    const uint32_t sbuf = epi0 + (uint32_t)(warp - 2) * kEpiWarpBytes;
    uint32_t ecnt = 0;  // staging pieces issued by this warp (buffer alternation)
    int abuf = 0;
    uint32_t aphase = 0;
    EpiWarp<BN> ew;
    if (pair < total_units) {
      int tm, tn, split;
      tile_coords2(pair, p, tm, tn, split);
      ew.prefetch(p, tm * 256 + row_in_tile, tn * BN, half);
    }
    for (int unit = pair; unit < total_units; unit += npairs) {
      int tm, tn, split;
      tile_coords2(unit, p, tm, tn, split);
      const int m = tm * 256 + row_in_tile;
      const int next = unit + npairs;
      int ntm = 0, ntn = 0, nsplit;
      if (next < total_units) tile_coords2(next, p, ntm, ntn, nsplit);
      if (!mbar_wait(tfull_bar(abuf), aphase, p.err, FXB_DERR_GEMM_WAIT)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN;
      ew.run(p, &tmC, &tmZ, m, tm * 256 + (int)rank * 128 + quarter * 32, tn * BN, half, tbase,
             sbuf, lane, ecnt, next < total_units, ntm * 256 + row_in_tile, ntn * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(abuf), 0));
      if (++abuf == 2) { abuf = 0; aphase ^= 1; }
    }
    if (lane == 0) bulk_wait_all0();  // stores done before the staging smem goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's smem / tensor memory are no longer in use
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
constexpr int FXB_EPI_ATOMIC_F32 = FXB_EPI_ACCUM_F32;

struct Maps {
  CUtensorMap a, b, c, z;  // operands, output C, pre-activation Z (= c when unused)
};

template <int BN, bool A_MN, bool B_MN, int AB_FMT, bool PAIR>
int launch_one(const Maps& mp, const GemmParams& p, int grid, cudaStream_t st) {
  void (*k)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
            const GemmParams) =
      PAIR ? gemm_tc2_kernel<BN, A_MN, B_MN, AB_FMT> : gemm_tc_kernel<BN, A_MN, B_MN, AB_FMT>;
  constexpr int smem = PAIR ? Cfg2<BN>::SMEM : Cfg<BN>::SMEM;
  static_assert(smem <= 232448, "shared memory budget");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    int r = fxb::check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                            "gemm smem attribute");
    if (r) return r;
    attr_set[dev] = true;
  }
  fxb::pdl_launch(k, grid, kThreads, smem, st, mp.a, mp.b, mp.c, mp.z, p);
  return fxb::check_launch(PAIR ? "gemm_tc2" : "gemm_tc");
}

template <int BN, int AB_FMT, bool PAIR>
int launch_layout(bool amn, bool bmn, const Maps& mp, const GemmParams& p, int grid,
                  cudaStream_t st) {
  if (!amn && !bmn) return launch_one<BN, false, false, AB_FMT, PAIR>(mp, p, grid, st);
  if (!amn && bmn) return launch_one<BN, false, true, AB_FMT, PAIR>(mp, p, grid, st);
  if (amn && bmn) return launch_one<BN, true, true, AB_FMT, PAIR>(mp, p, grid, st);
  return launch_one<BN, true, false, AB_FMT, PAIR>(mp, p, grid, st);
}

struct Plan {
  bool pair;   // 2-SM (cta_group::2, 256-row tiles) or 1-SM (128-row tiles)
  int BN;      // tile width
  int splits;  // split-K factor (fp32 accumulate epilogue only)
};

// Choose tile shape and split-K by a cost model of the persistent schedule:
// waves x per-unit time, where a unit's k-block time is bounded by the
// shared-memory traffic of its MMA operands plus the TMA writes (128 B/clk
// per SM) and the epilogue of a tile overlaps the next tile's mainloop.
// Per-SM cycles per 64-deep k-block: 1-SM 128x128: 512, 1-SM 128x256: 768,
// 2-SM 256x128: 384, 2-SM 256x256: 512 (the last one is tensor-bound).
// `mode` (FXB_GEMM_FORCE=1sm|2sm, tests) restricts the choice.
Plan plan(int M, int N, int K, bool allow_split, int sms, int mode) {
  const int nkb = (K + BK - 1) / BK;
  double best = 1e30;
  Plan out{false, 128, 1};
  for (int pair = 1; pair >= 0; --pair) {
    if ((mode == 1 && pair) || (mode == 2 && !pair)) continue;
    const int rows = pair ? 256 : 128;
    const int slots = pair ? sms / 2 : sms;
    const int tm = (M + rows - 1) / rows;
    for (int bn : {256, 128}) {
      const int tn = (N + bn - 1) / bn;
      const double t_kb = pair ? (bn == 256 ? 512.0 : 384.0) : (bn == 256 ? 768.0 : 512.0);
      for (int s = 1; s <= (allow_split ? 16 : 1); s *= 2) {
        if (s > 1 && nkb / s < 4) break;  // keep >= 4 k-blocks per split
        const int kbs = (nkb + s - 1) / s;
        const long units = (long)tm * tn * s;
        const long waves = (units + slots - 1) / slots;
        const double mainloop = kbs * t_kb + 600.0;  // + pipeline fill
        const double epi = bn * 6.0;                  // TMEM -> registers -> global per tile
        const double cost = (double)waves * (mainloop > epi ? mainloop : epi) + (s > 1 ? 0.5 * units : 0);
        if (cost < best - 1e-9) { best = cost; out = Plan{pair != 0, bn, s}; }
      }
    }
  }
  return out;
}

int force_mode() {
  const char* e = getenv("FXB_GEMM_FORCE");
  if (!e) return 0;
  if (e[0] == '1') return 1;
  if (e[0] == '2') return 2;
  return 0;
}

int make_map(CUtensorMap* map, int ab_dtype, const void* ptr, uint64_t inner, uint64_t outer,
             int64_t ld, uint32_t box_inner, uint32_t box_outer) {
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {(uint64_t)ld * 2};
  uint32_t box[2] = {box_inner, box_outer};
  CUtensorMapDataType dt = ab_dtype == FXB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fxb::encode_tiled(map, dt, 2, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Output map (C or Z): 32 rows x 64 bytes per box (32 16-bit or 16 fp32
// columns), 64-byte swizzle to match the epilogue's staging layout.
int make_out_map(CUtensorMap* map, int c_dtype, const void* ptr, uint64_t cols, uint64_t rows,
                 int64_t ld) {
  const int esz = fxb::dtype_size(c_dtype);
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {(uint64_t)ld * esz};
  uint32_t box[2] = {(uint32_t)(64 / esz), 32};
  CUtensorMapDataType dt = c_dtype == FXB_DTYPE_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : c_dtype == FXB_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  return fxb::encode_tiled(map, dt, 2, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

}  // namespace

namespace fxb {
// Internal entry (also used by the fxgpu gather path): epi may be the internal
// FXB_EPI_ATOMIC_F32 value 7; force_splits > 0 overrides the planner.
int gemm_launch(const fxb_gemm_args* a, int epi, int force_splits, cudaStream_t st) {
  const int M = a->M, N = a->N, K = a->K;
  if (a->dtype != FXB_DTYPE_BF16 && a->dtype != FXB_DTYPE_F16)
    return set_error(FXB_EUNSUPPORTED, "gemm: A/B dtype %d (bf16 or f16 only)", a->dtype);
  if (dtype_size(a->c_dtype) == 0) return set_error(FXB_EINVAL, "gemm: bad c_dtype");
  if (M < 0 || N < 0 || K < 0) return set_error(FXB_EINVAL, "gemm: negative size");
  if (N % 8) return set_error(FXB_EINVAL, "gemm: N=%d must be a multiple of 8", N);
  if (!a->A || !a->B || !a->C) return set_error(FXB_EINVAL, "gemm: NULL operand");
  if (!aligned16(a->A) || !aligned16(a->B) || !aligned16(a->C))
    return set_error(FXB_EINVAL, "gemm: operands must be 16-byte aligned");
  const int csz = dtype_size(a->c_dtype);
  if ((a->ldc * csz) % 16) return set_error(FXB_EINVAL, "gemm: ldc*esize must be a multiple of 16");
  if (a->a_trans ? (M % 8 || a->lda < M) : (K % 8 || a->lda < K))
    return set_error(FXB_EINVAL, "gemm: A needs 16-byte rows (M or K %% 8) and lda >= row");
  if (a->b_trans ? (a->ldb < N) : (K % 8 || a->ldb < K))
    return set_error(FXB_EINVAL, "gemm: B needs 16-byte rows and ldb >= row");
  if ((a->lda % 8) || (a->ldb % 8)) return set_error(FXB_EINVAL, "gemm: lda/ldb must be multiples of 8");
  if (a->ldc < N) return set_error(FXB_EINVAL, "gemm: ldc < N");
  const bool needs_r = (epi == FXB_EPI_RESIDUAL || epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU);
  if (needs_r && (!a->R || !aligned16(a->R) || (a->ldr * csz) % 16))
    return set_error(FXB_EINVAL, "gemm: epilogue needs an aligned R");
  const bool has_bias = (epi == FXB_EPI_BIAS || epi == FXB_EPI_BIAS_GELU || epi == FXB_EPI_BIAS_SILU);
  if (has_bias && (!a->bias || !aligned16(a->bias)))
    return set_error(FXB_EINVAL, "gemm: epilogue needs an aligned bias");
  if (a->Z && (!aligned16(a->Z) || (a->ldz * csz) % 16))
    return set_error(FXB_EINVAL, "gemm: Z misaligned");
  if (epi == FXB_EPI_ATOMIC_F32 && a->c_dtype != FXB_DTYPE_F32)
    return set_error(FXB_EINVAL, "gemm: accumulate epilogue needs fp32 C");
  if (a->c_dtype == FXB_DTYPE_F32 && epi != FXB_EPI_STORE && epi != FXB_EPI_RESIDUAL &&
      epi != FXB_EPI_BIAS && epi != FXB_EPI_ATOMIC_F32)
    return set_error(FXB_EUNSUPPORTED, "gemm: epilogue %d with fp32 C (16-bit C only)", epi);
  if (epi < 0 || epi > FXB_EPI_DSILU) return set_error(FXB_EINVAL, "gemm: bad epilogue %d", epi);
  if (M == 0 || N == 0) return FXB_OK;
  if (K == 0) return set_error(FXB_EUNSUPPORTED, "gemm: K == 0");

  int* err = dev_error_ptr();
  if (!err) return FXB_ECUDA;
  const int sms = num_sms();
  Plan pl = plan(M, N, K, epi == FXB_EPI_ATOMIC_F32, sms, force_mode());
  const int BN = pl.BN;
  int splits = pl.splits;
  if (force_splits > 0 && epi == FXB_EPI_ATOMIC_F32) splits = force_splits;
  const int rows = pl.pair ? 256 : 128;

  Maps mp;
  int r;
  if (a->a_trans) r = make_map(&mp.a, a->dtype, a->A, (uint64_t)M, (uint64_t)K, a->lda, 64, 64);
  else r = make_map(&mp.a, a->dtype, a->A, (uint64_t)K, (uint64_t)M, a->lda, 64, 128);
  if (r) return r;
  if (a->b_trans) r = make_map(&mp.b, a->dtype, a->B, (uint64_t)N, (uint64_t)K, a->ldb, 64, 64);
  else r = make_map(&mp.b, a->dtype, a->B, (uint64_t)K, (uint64_t)N, a->ldb, 64,
                    (uint32_t)(pl.pair ? BN / 2 : BN));
  if (r) return r;
  r = make_out_map(&mp.c, a->c_dtype, a->C, (uint64_t)N, (uint64_t)M, a->ldc);
  if (r) return r;
  if (a->Z) {
    r = make_out_map(&mp.z, a->c_dtype, a->Z, (uint64_t)N, (uint64_t)M, a->ldz);
    if (r) return r;
  } else {
    mp.z = mp.c;
  }

  GemmParams p;
  p.M = M; p.N = N; p.K = K;
  p.tiles_m = (M + rows - 1) / rows;
  p.tiles_n = (N + BN - 1) / BN;
  p.num_kb = (K + BK - 1) / BK;
  p.splits = splits;
  p.kb_per_split = (p.num_kb + splits - 1) / splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;  // no empty splits
  p.epi = epi;
  p.c_dtype = a->c_dtype;
  p.alpha = a->alpha;
  p.C = a->C; p.ldc = a->ldc;
  p.R = a->R; p.ldr = a->ldr;
  p.Z = a->Z; p.ldz = a->ldz;
  p.bias = a->bias;
  p.err = err;
  const long units = (long)p.tiles_m * p.tiles_n * p.splits;
  const bool amn = a->a_trans != 0, bmn = a->b_trans != 0;
  if (pl.pair) {
    const long pairs = units < sms / 2 ? units : sms / 2;
    const int grid = (int)(2 * pairs);
    if (a->dtype == FXB_DTYPE_BF16)
      return BN == 256 ? launch_layout<256, 1, true>(amn, bmn, mp, p, grid, st)
                       : launch_layout<128, 1, true>(amn, bmn, mp, p, grid, st);
    return BN == 256 ? launch_layout<256, 0, true>(amn, bmn, mp, p, grid, st)
                     : launch_layout<128, 0, true>(amn, bmn, mp, p, grid, st);
  }
  const int grid = (int)(units < sms ? units : sms);
  if (a->dtype == FXB_DTYPE_BF16)
    return BN == 256 ? launch_layout<256, 1, false>(amn, bmn, mp, p, grid, st)
                     : launch_layout<128, 1, false>(amn, bmn, mp, p, grid, st);
  return BN == 256 ? launch_layout<256, 0, false>(amn, bmn, mp, p, grid, st)
                   : launch_layout<128, 0, false>(amn, bmn, mp, p, grid, st);
}
}  // namespace fxb

extern "C" int fxb_gemm(const fxb_gemm_args* args, void* stream) {
  if (!args) return fxb::set_error(FXB_EINVAL, "gemm: args is NULL");
  return fxb::gemm_launch(args, args->epilogue, 0, fxb::as_stream(stream));
}

extern "C" int fxb_gemm_plan(int32_t M, int32_t N, int32_t K, int32_t epilogue, int32_t* pair,
                             int32_t* bn, int32_t* splits) {
  if (!pair || !bn || !splits || M < 0 || N < 0 || K < 0)
    return fxb::set_error(FXB_EINVAL, "gemm_plan: bad arguments");
  Plan pl = plan(M, N, K, epilogue == FXB_EPI_ACCUM_F32, fxb::num_sms(), force_mode());
  *pair = pl.pair ? 1 : 0;
  *bn = pl.BN;
  *splits = pl.splits;
  return FXB_OK;
}
