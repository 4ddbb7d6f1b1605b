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
//   - tail split: when the tiles do not fill the last wave, the leftover tiles
//     are cut along K into pieces run side by side; piece 0 of a tile waits
//     (bounded) for the others' fp32 partial tiles, adds them and runs the
//     epilogue, so the last wave is as short as a piece instead of a tile.
// Every wait is bounded (common.cuh); on expiry the kernel records
// FXB_DERR_GEMM_WAIT, drains what it issued and frees its tensor memory.
//
// This header holds the device side (kernels, epilogues, launch templates);
// gemm.cu holds the planner and the C entry, and gemm_k0..3.cu instantiate
// one epilogue kind each (they compile in parallel).
#pragma once
#include "common.cuh"
#include "internal.h"

namespace fxb {
namespace gk {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
// Per-epilogue-warp output staging after the operand ring: two 2 KB
// buffers, or for the epilogue kind that writes C and Z (EK_ACT16) two pairs
// of them, so that a chunk's stores of C and Z drain while the next chunk is
// computed; the warp's lane 0 issues the TMA stores (or fp32 add-reductions)
// and owns their bulk groups.
constexpr int kSmemBudget = 232448;

// Epilogue kinds: each kernel instantiation carries one, so that its
// epilogue holds only the arithmetic of that kind (a runtime switch over every
// epilogue made the per-chunk code several times larger than the path taken).
constexpr int EK_LIN16 = 0;   // 16-bit C: store / residual / bias / multiply
constexpr int EK_ACT16 = 1;   // 16-bit C: GELU / bias+GELU / bias+SiLU / GELU+derivative (+ Z)
constexpr int EK_DACT16 = 2;  // 16-bit C: dGELU / dSiLU (reads R)
constexpr int EK_F32 = 3;     // fp32 C: store / residual / bias / accumulate
constexpr int EK_CESTAT = 4;  // no C: per-row softmax statistics of the tile (loss-only linear-CE)

// C element type of a kernel: fp32 for EK_F32, else the operand type
template <int EK, int AB_FMT> struct CType { using T = __nv_bfloat16; };
template <> struct CType<EK_LIN16, 0> { using T = __half; };
template <> struct CType<EK_ACT16, 0> { using T = __half; };
template <> struct CType<EK_DACT16, 0> { using T = __half; };
template <int AB_FMT> struct CType<EK_F32, AB_FMT> { using T = float; };
template <int AB_FMT> struct CType<EK_CESTAT, AB_FMT> { using T = float; };

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, num_kb;
  // units = full_units whole tiles (or split-K (tile, split) pairs), then
  // tail_splits pieces of tail_kb k-blocks for each remaining tile
  int total_units, full_units, tail_splits, tail_kb;
  float* ws;         // tail pieces' fp32 partial tiles
  unsigned* ws_cnt;  // per (tail tile, CTA) arrival counters, zero between launches
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
  // EK_CESTAT: per (row, 64- or 128-column half tile) the pair (max, sum of
  // exp(acc - max)) in ce_stats[row * ce_nstat + tile_n * 2 + half], and the
  // accumulator at column ce_target[row] in ce_tlogit[row]
  float2* ce_stats;
  int ce_nstat;
  const int64_t* ce_target;
  float* ce_tlogit;
};

template <int EK> struct Epi {
  static constexpr int WARP_BYTES = (EK == EK_ACT16) ? 8192 : 4096;
  static constexpr int BYTES = 8 * WARP_BYTES;
};

template <int BN, int EK> struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int RING_MAX = (kSmemBudget - Epi<EK>::BYTES - 1024 - 256) / STAGE_BYTES;
  static constexpr int STAGES = RING_MAX > 6 ? 6 : RING_MAX;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + Epi<EK>::BYTES + 1024 /*align*/ + 256 /*barriers*/;
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

// What a unit of the persistent schedule covers: tile (tm, tn), k-blocks
// [kb0, kb1), and for a tail piece its tail tile index and piece number
// (piece -1 for whole tiles).
struct UnitInfo {
  int tm, tn, kb0, kb1, tail, piece;
};
FXB_DEV UnitInfo unit_info(int unit, const GemmParams& p) {
  UnitInfo u;
  int split;
  if (unit < p.full_units) {
    tile_coords(unit, p, u.tm, u.tn, split);
    u.kb0 = split * p.kb_per_split;
    u.kb1 = min(p.num_kb, u.kb0 + p.kb_per_split);
    u.tail = -1;
    u.piece = -1;
  } else {
    const int v = unit - p.full_units;
    u.tail = v / p.tail_splits;
    u.piece = v - u.tail * p.tail_splits;
    tile_coords(p.full_units + u.tail, p, u.tm, u.tn, split);
    u.kb0 = u.piece * p.tail_kb;
    u.kb1 = min(p.num_kb, u.kb0 + p.tail_kb);
  }
  return u;
}

// The k-th unit of persistent slot `slot` (a CTA, or a CTA pair), -1 past its
// last: its whole tiles slot, slot + nslots, ... and its tail piece (tail
// unit v goes to slot v). A contributor runs its piece first, so its partial
// tile is written while the owner is still on its whole tiles; the owner runs
// its piece last. The owner's wait therefore depends only on units that wait
// for nothing.
FXB_DEV int unit_of(int slot, int k, const GemmParams& p, int nslots) {
  const int npieces = p.total_units - p.full_units;
  const bool has_piece = slot < npieces;
  const bool contrib = has_piece && (slot % p.tail_splits) != 0;
  if (contrib) {
    if (k == 0) return p.full_units + slot;
    --k;
  }
  const int nfull = slot < p.full_units ? (p.full_units - slot + nslots - 1) / nslots : 0;
  if (k < nfull) return slot + k * nslots;
  if (has_piece && !contrib && k == nfull) return p.full_units + slot;
  return -1;
}

// Partial-tile exchange of a tail tile. A contributor (piece > 0) writes its
// fp32 accumulator tile to the workspace and counts its epilogue warps in; the
// owner (piece 0) waits for all of them and adds their tiles, in piece order,
// to its own accumulator before the epilogue. Workspace layout per CTA tile:
// float4 index ((chunk * 4 + quarter) * 8 + j) * 32 + lane holds values
// 4j..4j+3 of the lane's 32-column chunk, so every warp access is one
// contiguous 512-byte span.
struct Red {
  float4* out;       // contributor: this lane's slot in its partial tile
  const float4* in;  // owner: this lane's slot in the first contributor's tile
  int nin;           // owner: contributor tiles to add
  int64_t stride4;   // float4 distance between consecutive contributors' tiles
};
template <int BN>
FXB_DEV Red tail_red(const GemmParams& p, const UnitInfo& u, int cta, int nctas, int quarter,
                     int lane) {
  Red r{nullptr, nullptr, 0, 0};
  if (u.piece < 0) return r;
  constexpr int64_t kTile4 = 32 * BN;  // float4s per 128-row CTA tile
  const int nc = p.tail_splits - 1;
  float4* ws4 = reinterpret_cast<float4*>(p.ws);
  const int64_t lane_off = (int64_t)quarter * 256 + lane;
  if (u.piece > 0) {
    r.out = ws4 + ((int64_t)(u.tail * nc + u.piece - 1) * nctas + cta) * kTile4 + lane_off;
  } else {
    r.in = ws4 + ((int64_t)u.tail * nc * nctas + cta) * kTile4 + lane_off;
    r.nin = nc;
    r.stride4 = (int64_t)nctas * kTile4;
  }
  return r;
}
// owner: wait (bounded) until every contributor warp of this CTA's tile is in
FXB_DEV void tail_wait(const GemmParams& p, const UnitInfo& u, int cta, int nctas, int lane) {
  if (u.piece != 0) return;
  if (lane == 0)
    spin_until_geq(p.ws_cnt + u.tail * nctas + cta, 8u * (unsigned)(p.tail_splits - 1), p.err,
                   FXB_DERR_GEMM_WAIT);
  __syncwarp();
  __threadfence();
}
// after the warp's epilogue: a contributor publishes its partial; the owner's
// last warp resets the counter for the next launch
FXB_DEV void tail_done(const GemmParams& p, const UnitInfo& u, int cta, int nctas, int lane) {
  if (u.piece < 0) return;
  unsigned* c = p.ws_cnt + u.tail * nctas + cta;
  if (u.piece > 0) {
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(c, 1u);
  } else if (lane == 0) {
    const unsigned expect = 8u * (unsigned)(p.tail_splits - 1);
    if (atomicAdd(c, 1u) == expect + 7u) atomicExch(c, 0u);
  }
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
template <int EK> FXB_DEV bool epi_reads_r(const GemmParams& p) {
  if constexpr (EK == EK_DACT16) return true;
  else if constexpr (EK == EK_ACT16) return false;
  else return p.epi == FXB_EPI_RESIDUAL || p.epi == FXB_EPI_MUL;
}
// epilogues that also write the rounded pre-activation to Z (when Z is given)
template <int EK> FXB_DEV bool epi_writes_z(const GemmParams& p) {
  if constexpr (EK == EK_ACT16) return p.Z != nullptr;
  else return false;
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
template <typename CT, int EK>
FXB_DEV void epilogue_math(const GemmParams& p, int m, int n0, int n8, float* v, float* z,
                           bool use_pre, const uint4* pre2) {
  if constexpr (EK == EK_LIN16 || EK == EK_F32) {
    if (p.epi == FXB_EPI_RESIDUAL) {
      piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = v[i] * p.alpha + z[i];
    } else if (EK == EK_LIN16 && p.epi == FXB_EPI_MUL) {
      piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = v[i] * p.alpha * z[i];
    } else if (p.epi == FXB_EPI_BIAS) {
      load16_part<CT>(static_cast<const CT*>(p.bias) + n0, z, n8);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += z[i];
    } else {  // FXB_EPI_STORE, FXB_EPI_ACCUM_F32
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= p.alpha;
    }
  } else if constexpr (EK == EK_ACT16) {
    if (p.epi == FXB_EPI_BIAS_GELU || p.epi == FXB_EPI_BIAS_SILU) {
      load16_part<CT>(static_cast<const CT*>(p.bias) + n0, z, n8);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += z[i];
    }
    // round the pre-activation once; the activation is computed from the
    // stored value so that backward (which reads Z) sees the same input
#pragma unroll
    for (int i = 0; i < 16; i += 2) {  // paired conversions
      const float2 f = unpack2<CT>(pack2<CT>(v[i], v[i + 1]));
      z[i] = f.x;
      z[i + 1] = f.y;
    }
    if (p.epi == FXB_EPI_BIAS_SILU) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = silu_f(z[i]);
    } else if (p.epi == FXB_EPI_GELU_DERIV) {
#pragma unroll
      for (int i = 0; i < 16; ++i) gelu_tanh_and_grad(z[i], &v[i], &z[i]);  // Z = gelu'
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = gelu_tanh(z[i]);
    }
  } else {  // EK_DACT16
    piece_r<CT>(p, m, n0, n8, use_pre, pre2, z);
    if (p.epi == FXB_EPI_DSILU) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float s = 1.f / (1.f + __expf(-z[i]));
        v[i] *= s * (1.f + z[i] * (1.f - s));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= gelu_tanh_grad(z[i]);
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
template <int BN, typename CT, int EK>
struct EpiWarp {
  static constexpr int NCH = BN / 64;
  // R (16-bit) of two chunks in flight, as a ring that runs across tiles:
  // chunk c of a tile sits in slot c & 1; once chunk c is done its slot is
  // refilled with chunk c + 2, or with chunk c + 2 - NCH of the warp's next
  // tile (NCH is even), so the next tile's first chunks load during this one.
  uint4 pre[2][4];
  bool pre_ok[2];  // slot holds R of a row inside M (16-bit C, R-reading epilogue)

  FXB_DEV void fill(const GemmParams& p, int slot, int m, int n0) {
    pre_ok[slot] = sizeof(CT) == 2 && epi_reads_r<EK>(p) && m < p.M;
    if (pre_ok[slot] && n0 < p.N) prefetch_r16(p, m, n0, pre[slot]);
  }
  // chunks 0 and 1 of the warp's first tile
  FXB_DEV void prefetch(const GemmParams& p, int m, int ntile0, int half) {
#pragma unroll
    for (int c = 0; c < 2; ++c) fill(p, c, m, ntile0 + (half * NCH + c) * 32);
  }

  // one 16-column piece: accumulator values (already loaded from tensor
  // memory) -> epilogue math
  FXB_DEV int piece(const GemmParams& p, int m, int n0, const uint32_t* r, int slot,
                    const uint4* pre2, float* v, float* z) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
    const int n8 = max(0, min(2, (p.N - n0) >> 3));
    epilogue_math<CT, EK>(p, m, n0, n8, v, z, sizeof(CT) == 2 && pre_ok[slot], pre2);
    return n8;
  }

  // Staging: each 32-column chunk is one bulk group (C, plus Z in the next
  // 2 KB for the epilogues that write it), and consecutive chunks alternate
  // between two buffer sets, so a chunk waits only for the group before last
  // to have been read.
  FXB_DEV void chunk(const GemmParams& p, const CUtensorMap* tmC, const CUtensorMap* tmZ, int m,
                     int m0, int n0, uint32_t taddr, int cc, uint32_t sbuf, int lane,
                     uint32_t& cnt) {
    const bool wz = epi_writes_z<EK>(p);
    float v[16], z[16];
    uint32_t acc[32];  // the chunk's 32 accumulator columns: one tensor-memory load
    tmem_ld32(taddr, acc);
    tmem_wait_ld();
    if constexpr (sizeof(CT) == 2) {
      // C (and Z, in the next 2 KB) alternate between two buffer sets: the
      // group before last has been read once the newest is the only one left
      const uint32_t b = sbuf + (cnt & 1u) * (EK == EK_ACT16 ? 4096u : 2048u);
      stage_begin(lane, false);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        piece(p, m, n0 + 16 * h, acc + 16 * h, cc & 1, &pre[cc & 1][2 * h], v, z);
        stage_piece<CT>(b, lane, h, v);
        if (wz) stage_piece<CT>(b + 2048, lane, h, z);
      }
      stage_issue(tmC, n0, wz ? tmZ : nullptr, n0, m0, false, b, lane);
      ++cnt;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n8 = piece(p, m, n0 + 16 * h, acc + 16 * h, cc & 1, &pre[cc & 1][2 * h], v, z);
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

  // Tail pieces (see Red). A contributor copies its accumulator columns to
  // its partial tile; the owner adds the contributors' tiles into tensor
  // memory before run(), so the epilogue's chunk loop is the same code for
  // every unit.
  FXB_DEV void write_partial(const GemmParams& p, int ntile0, int half, uint32_t tbase,
                             const Red& rd) {
#pragma unroll 1
    for (int cc = 0; cc < NCH; ++cc) {
      const int c = half * NCH + cc;
      if (ntile0 + c * 32 >= p.N) break;  // warp-uniform
      uint32_t acc[32];
      tmem_ld32(tbase + c * 32, acc);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        rd.out[c * 1024 + j * 32] =
            make_float4(__uint_as_float(acc[4 * j]), __uint_as_float(acc[4 * j + 1]),
                        __uint_as_float(acc[4 * j + 2]), __uint_as_float(acc[4 * j + 3]));
    }
  }
  FXB_DEV void fold_partials(const GemmParams& p, int ntile0, int half, uint32_t tbase,
                             const Red& rd) {
#pragma unroll 1
    for (int cc = 0; cc < NCH; ++cc) {
      const int c = half * NCH + cc;
      if (ntile0 + c * 32 >= p.N) break;  // warp-uniform
      uint32_t acc[32];
      tmem_ld32(tbase + c * 32, acc);
      tmem_wait_ld();
#pragma unroll 1
      for (int q = 0; q < rd.nin; q += 2) {  // two contributors' loads in flight
        const float4* src = rd.in + q * rd.stride4 + c * 1024;
        const bool two = q + 1 < rd.nin;
        float4 x[2][8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[0][j] = __ldcg(src + j * 32);
          x[1][j] = two ? __ldcg(src + rd.stride4 + j * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)  // in contributor order
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc[4 * j] = __float_as_uint(__uint_as_float(acc[4 * j]) + x[h][j].x);
            acc[4 * j + 1] = __float_as_uint(__uint_as_float(acc[4 * j + 1]) + x[h][j].y);
            acc[4 * j + 2] = __float_as_uint(__uint_as_float(acc[4 * j + 2]) + x[h][j].z);
            acc[4 * j + 3] = __float_as_uint(__uint_as_float(acc[4 * j + 3]) + x[h][j].w);
          }
      }
      tmem_st32(tbase + c * 32, acc);
    }
    tmem_wait_st();
  }

  // m_next / ntile0_next: this warp's row and first column in its next tile
  // (has_next false when there is none)
  // EK_CESTAT: the warp's columns of the tile reduced to (max, sum of exp) per
  // row with an online merge across its 32-column chunks, plus the target
  // column's value when it falls in them; no C is written
  FXB_DEV void run_stats(const GemmParams& p, int m, int ntile0, int half, uint32_t tbase) {
    constexpr float kL2e = 1.4426950408889634f;
    const int64_t tgt = (m < p.M) ? p.ce_target[m] : -1;
    float rm = -INFINITY, rsum = 0.f;
#pragma unroll 1
    for (int cc = 0; cc < NCH; ++cc) {
      const int c = half * NCH + cc;
      const int n0 = ntile0 + c * 32;
      if (n0 >= p.N) break;  // warp-uniform
      uint32_t acc[32];
      tmem_ld32(tbase + c * 32, acc);
      tmem_wait_ld();
      const int nv = min(32, p.N - n0);
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) cm = fmaxf(cm, __uint_as_float(acc[i]));
      const float nm = fmaxf(rm, cm);
      const float nml = nm * kL2e;
      float cs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) cs[i & 3] += exp2f(fmaf(__uint_as_float(acc[i]), kL2e, -nml));
      rsum = rsum * exp2f((rm - nm) * kL2e) + ((cs[0] + cs[1]) + (cs[2] + cs[3]));
      rm = nm;
      if (tgt >= n0 && tgt < n0 + nv) {
        float tv = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (tgt - n0 == i) tv = __uint_as_float(acc[i]);
        p.ce_tlogit[m] = tv;
      }
    }
    if (m < p.M)
      p.ce_stats[(int64_t)m * p.ce_nstat + (ntile0 / BN) * 2 + half] = make_float2(rm, rsum);
  }

  FXB_DEV void run(const GemmParams& p, const CUtensorMap* tmC, const CUtensorMap* tmZ, int m,
                   int m0, int ntile0, int half, uint32_t tbase, uint32_t sbuf, int lane,
                   uint32_t& cnt, bool has_next, int m_next, int ntile0_next) {
    if constexpr (EK == EK_CESTAT) {
      run_stats(p, m, ntile0, half, tbase);
      return;
    }
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
        chunk(p, tmC, tmZ, m, m0, n0, taddr, ci, sbuf, lane, cnt);
      }
      if (cc + 2 < NCH) fill(p, ci, m, n0 + 64);
      else if (has_next) fill(p, ci, m_next, ntile0_next + (half * NCH + cc + 2 - NCH) * 32);
    }
  }
};

// ---------------------------------------------------------------- kernel
template <int BN, bool A_MN, bool B_MN, int AB_FMT, int EK>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmZ,
               const GemmParams p) {
  using C = Cfg<BN, EK>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 1024B aligned for 128B swizzle
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;  // output staging
  const uint32_t bar0 = epi0 + Epi<EK>::BYTES;
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


  constexpr uint32_t IDESC = umma_idesc_f16(AB_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, BM, BN);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;          // bit s: stage s armed at least once
      uint32_t armed_parity = 0;   // bit s: parity of the last arming of stage s
      bool ok = true;
      for (int k = 0, unit; ok && (unit = unit_of(blockIdx.x, k, p, gridDim.x)) >= 0; ++k) {
        const UnitInfo u = unit_info(unit, p);
        const int tm = u.tm, tn = u.tn;
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
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
      for (int k = 0, unit; ok && (unit = unit_of(blockIdx.x, k, p, gridDim.x)) >= 0; ++k) {
        const UnitInfo u = unit_info(unit, p);
        const int kb0 = u.kb0, kb1 = u.kb1;
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
    const uint32_t sbuf = epi0 + (uint32_t)(warp - 2) * Epi<EK>::WARP_BYTES;
    uint32_t ecnt = 0;  // staging pieces issued by this warp (buffer alternation)
    int abuf = 0;
    uint32_t aphase = 0;
    EpiWarp<BN, typename CType<EK, AB_FMT>::T, EK> ew;
    if (unit_of(blockIdx.x, 0, p, gridDim.x) >= 0) {
      const UnitInfo u = unit_info(unit_of(blockIdx.x, 0, p, gridDim.x), p);
      ew.prefetch(p, u.tm * BM + row_in_tile, u.tn * BN, half);
    }
    for (int k = 0, unit; (unit = unit_of(blockIdx.x, k, p, gridDim.x)) >= 0; ++k) {
      const UnitInfo u = unit_info(unit, p);
      const int tm = u.tm, tn = u.tn;
      const int m = tm * BM + row_in_tile;
      const int next = unit_of(blockIdx.x, k + 1, p, gridDim.x);
      int ntm = 0, ntn = 0;
      if (next >= 0) {
        const UnitInfo nu = unit_info(next, p);
        ntm = nu.tm;
        ntn = nu.tn;
      }
      if (!mbar_wait(tfull_bar(abuf), aphase, p.err, FXB_DERR_GEMM_WAIT)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN;
      if (u.piece > 0) {
        ew.write_partial(p, tn * BN, half, tbase, tail_red<BN>(p, u, 0, 1, quarter, lane));
        // the R prefetched for this unit is unused: load the next unit's
        if (next >= 0) ew.prefetch(p, ntm * BM + row_in_tile, ntn * BN, half);
      } else {
        if (u.piece == 0) {
          tail_wait(p, u, 0, 1, lane);
          ew.fold_partials(p, tn * BN, half, tbase, tail_red<BN>(p, u, 0, 1, quarter, lane));
        }
        ew.run(p, &tmC, &tmZ, m, tm * BM + quarter * 32, tn * BN, half, tbase, sbuf, lane, ecnt,
               next >= 0, ntm * BM + row_in_tile, ntn * BN);
      }
      tail_done(p, u, 0, 1, lane);
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
template <int BN, int EK> struct Cfg2 {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int RING_MAX = (kSmemBudget - Epi<EK>::BYTES - 1024 - 256) / STAGE_BYTES;
  static constexpr int STAGES = RING_MAX > 8 ? 8 : RING_MAX;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + Epi<EK>::BYTES + 1024 + 256;
};

template <int BN, bool A_MN, bool B_MN, int AB_FMT, int EK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmZ,
                const GemmParams p) {
  using C = Cfg2<BN, EK>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;  // output staging
  const uint32_t bar0 = epi0 + Epi<EK>::BYTES;
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


  constexpr uint32_t IDESC = umma_idesc_f16(AB_FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, 256, BN);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      bool ok = true;
      for (int k = 0, unit; ok && (unit = unit_of(pair, k, p, npairs)) >= 0; ++k) {
        const UnitInfo u = unit_info(unit, p);  // tm counts 256-row tiles here
        const int tm = u.tm, tn = u.tn, kb0 = u.kb0, kb1 = u.kb1;
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
        for (int k = 0, unit; ok && (unit = unit_of(pair, k, p, npairs)) >= 0; ++k) {
          const UnitInfo u = unit_info(unit, p);
          const int kb0 = u.kb0, kb1 = u.kb1;
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
    const uint32_t sbuf = epi0 + (uint32_t)(warp - 2) * Epi<EK>::WARP_BYTES;
    uint32_t ecnt = 0;  // staging pieces issued by this warp (buffer alternation)
    int abuf = 0;
    uint32_t aphase = 0;
    EpiWarp<BN, typename CType<EK, AB_FMT>::T, EK> ew;
    if (unit_of(pair, 0, p, npairs) >= 0) {
      const UnitInfo u = unit_info(unit_of(pair, 0, p, npairs), p);
      ew.prefetch(p, u.tm * 256 + row_in_tile, u.tn * BN, half);
    }
    for (int k = 0, unit; (unit = unit_of(pair, k, p, npairs)) >= 0; ++k) {
      const UnitInfo u = unit_info(unit, p);
      const int tm = u.tm, tn = u.tn;
      const int m = tm * 256 + row_in_tile;
      const int next = unit_of(pair, k + 1, p, npairs);
      int ntm = 0, ntn = 0;
      if (next >= 0) {
        const UnitInfo nu = unit_info(next, p);
        ntm = nu.tm;
        ntn = nu.tn;
      }
      if (!mbar_wait(tfull_bar(abuf), aphase, p.err, FXB_DERR_GEMM_WAIT)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN;
      if (u.piece > 0) {
        ew.write_partial(p, tn * BN, half, tbase, tail_red<BN>(p, u, (int)rank, 2, quarter, lane));
        // the R prefetched for this unit is unused: load the next unit's
        if (next >= 0) ew.prefetch(p, ntm * 256 + row_in_tile, ntn * BN, half);
      } else {
        if (u.piece == 0) {
          tail_wait(p, u, (int)rank, 2, lane);
          ew.fold_partials(p, tn * BN, half, tbase, tail_red<BN>(p, u, (int)rank, 2, quarter, lane));
        }
        ew.run(p, &tmC, &tmZ, m, tm * 256 + (int)rank * 128 + quarter * 32, tn * BN, half, tbase,
               sbuf, lane, ecnt, next >= 0, ntm * 256 + row_in_tile, ntn * BN);
      }
      tail_done(p, u, (int)rank, 2, lane);
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

template <int BN, bool A_MN, bool B_MN, int AB_FMT, bool PAIR, int EK>
int launch_one(const Maps& mp, const GemmParams& p, int grid, cudaStream_t st) {
  void (*k)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
            const GemmParams) =
      PAIR ? gemm_tc2_kernel<BN, A_MN, B_MN, AB_FMT, EK> : gemm_tc_kernel<BN, A_MN, B_MN, AB_FMT, EK>;
  constexpr int smem = PAIR ? Cfg2<BN, EK>::SMEM : Cfg<BN, EK>::SMEM;
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

template <int BN, int AB_FMT, bool PAIR, int EK>
int launch_layout(bool amn, bool bmn, const Maps& mp, const GemmParams& p, int grid,
                  cudaStream_t st) {
  if (!amn && !bmn) return launch_one<BN, false, false, AB_FMT, PAIR, EK>(mp, p, grid, st);
  if (!amn && bmn) return launch_one<BN, false, true, AB_FMT, PAIR, EK>(mp, p, grid, st);
  if (amn && bmn) return launch_one<BN, true, true, AB_FMT, PAIR, EK>(mp, p, grid, st);
  return launch_one<BN, true, false, AB_FMT, PAIR, EK>(mp, p, grid, st);
}

// Launch the kernel of epilogue kind EK for (pair, BN, operand type, layouts).
// Each kind is instantiated in its own translation unit (gemm_k<EK>.cu).
template <int EK>
int gemm_dispatch(bool pair, int BN, int ab_fmt, bool amn, bool bmn, const Maps& mp,
                  const GemmParams& p, int grid, cudaStream_t st) {
  if (pair) {
    if (ab_fmt == 1)
      return BN == 256 ? launch_layout<256, 1, true, EK>(amn, bmn, mp, p, grid, st)
                       : launch_layout<128, 1, true, EK>(amn, bmn, mp, p, grid, st);
    return BN == 256 ? launch_layout<256, 0, true, EK>(amn, bmn, mp, p, grid, st)
                     : launch_layout<128, 0, true, EK>(amn, bmn, mp, p, grid, st);
  }
  if (ab_fmt == 1)
    return BN == 256 ? launch_layout<256, 1, false, EK>(amn, bmn, mp, p, grid, st)
                     : launch_layout<128, 1, false, EK>(amn, bmn, mp, p, grid, st);
  return BN == 256 ? launch_layout<256, 0, false, EK>(amn, bmn, mp, p, grid, st)
                   : launch_layout<128, 0, false, EK>(amn, bmn, mp, p, grid, st);
}

}  // namespace gk
}  // namespace fxb
