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
#include "gemm_kernel.cuh"

namespace fxb {
namespace gk {
// instantiated in gemm_k0.cu .. gemm_k3.cu
extern template int gemm_dispatch<EK_LIN16>(bool, int, int, bool, bool, const Maps&,
                                            const GemmParams&, int, cudaStream_t);
extern template int gemm_dispatch<EK_ACT16>(bool, int, int, bool, bool, const Maps&,
                                            const GemmParams&, int, cudaStream_t);
extern template int gemm_dispatch<EK_DACT16>(bool, int, int, bool, bool, const Maps&,
                                             const GemmParams&, int, cudaStream_t);
extern template int gemm_dispatch<EK_F32>(bool, int, int, bool, bool, const Maps&,
                                          const GemmParams&, int, cudaStream_t);
extern template int gemm_dispatch<EK_CESTAT>(bool, int, int, bool, bool, const Maps&,
                                             const GemmParams&, int, cudaStream_t);
}  // namespace gk
}  // namespace fxb

namespace {
using namespace fxb::gk;

struct Plan {
  bool pair;        // 2-SM (cta_group::2, 256-row tiles) or 1-SM (128-row tiles)
  int BN;           // tile width
  int splits;       // split-K factor (fp32 accumulate epilogue only)
  int tail_splits;  // K pieces per tail tile (1: no tail split)
};

// Workspace of the tail split: arrival counters, then the contributors' fp32
// partial tiles (at most one 128 x 256 tile per SM: tail tiles x (pieces - 1)
// never exceed the slots of one wave).
constexpr size_t kWsCounterBytes = 4096;
size_t workspace_bytes(int sms) { return kWsCounterBytes + (size_t)sms * 128 * 256 * 4; }

// Choose tile shape, split-K and tail split by a cost model of the persistent
// schedule: waves x per-unit time, where a unit's k-block time is bounded by
// the shared-memory traffic of its MMA operands plus the TMA writes (128 B/clk
// per SM) and the epilogue of a tile overlaps the next tile's mainloop.
// Per-SM cycles per 64-deep k-block: 1-SM 128x128: 512, 1-SM 128x256: 768,
// 2-SM 256x128: 384, 2-SM 256x256: 512 (the last one is tensor-bound).
// Epilogue per 128-row CTA tile (measured): ~18 cycles per column to store,
// +10 when it reads R, +12 when it also writes Z. A tail split replaces the
// last, partly filled wave of whole tiles by one wave of K pieces plus the
// partial-tile exchange (~8 cycles per column per piece at ~64 B/clk of L2
// traffic per SM). `mode` (FXB_GEMM_FORCE=1sm|2sm, tests) restricts the choice.
Plan plan(int M, int N, int K, int epi, bool tail_ok, int sms, int mode) {
  const bool allow_split = epi == FXB_EPI_ACCUM_F32;
  const bool reads_r = epi == FXB_EPI_RESIDUAL || epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU ||
                       epi == FXB_EPI_MUL;
  const bool writes_z = epi == FXB_EPI_GELU || epi == FXB_EPI_BIAS_GELU || epi == FXB_EPI_BIAS_SILU ||
                        epi == FXB_EPI_GELU_DERIV;
  const double epi_col = 18.0 + (reads_r ? 10.0 : 0.0) + (writes_z ? 12.0 : 0.0);
  const int nkb = (K + BK - 1) / BK;
  double best = 1e30;
  Plan out{false, 128, 1, 1};
  for (int pair = 1; pair >= 0; --pair) {
    if ((mode == 1 && pair) || (mode == 2 && !pair)) continue;
    const int rows = pair ? 256 : 128;
    const int slots = pair ? sms / 2 : sms;
    const int tm = (M + rows - 1) / rows;
    for (int bn : {256, 128}) {
      const int tn = (N + bn - 1) / bn;
      const double t_kb = pair ? (bn == 256 ? 512.0 : 384.0) : (bn == 256 ? 768.0 : 512.0);
      const double epi_t = bn * epi_col;
      for (int s = 1; s <= (allow_split ? 16 : 1); s *= 2) {
        if (s > 1 && nkb / s < 4) break;  // keep >= 4 k-blocks per split
        const int kbs = (nkb + s - 1) / s;
        const long units = (long)tm * tn * s;
        const long waves = (units + slots - 1) / slots;
        const double mainloop = kbs * t_kb + 600.0;  // + pipeline fill
        const double cost = (double)waves * (mainloop > epi_t ? mainloop : epi_t) + (s > 1 ? 0.5 * units : 0);
        if (cost < best - 1e-9) { best = cost; out = Plan{pair != 0, bn, s, 1}; }
      }
      if (allow_split || !tail_ok) continue;
      const long tiles = (long)tm * tn;
      const long full_waves = tiles / slots, tail = tiles % slots;
      if (tail == 0) continue;
      int S = (int)(slots / tail);
      if (S > 8) S = 8;
      if (S > nkb / 2) S = nkb / 2;
      if (S < 2) continue;
      const double main_full = nkb * t_kb + 600.0;
      const double main_piece = ((nkb + S - 1) / S) * t_kb + 600.0;
      const double cost = (double)full_waves * (main_full > epi_t ? main_full : epi_t) +
                          (main_piece > epi_t ? main_piece : epi_t) + 8.0 * bn * S;
      if (cost < best - 1e-9) { best = cost; out = Plan{pair != 0, bn, 1, S}; }
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
  const bool needs_r = (epi == FXB_EPI_RESIDUAL || epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU ||
                        epi == FXB_EPI_MUL);
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
  if (a->c_dtype != FXB_DTYPE_F32 && a->c_dtype != a->dtype)
    return set_error(FXB_EUNSUPPORTED, "gemm: C dtype %d must be fp32 or the A/B dtype", a->c_dtype);
  if (epi < 0 || epi > FXB_EPI_MUL) return set_error(FXB_EINVAL, "gemm: bad epilogue %d", epi);
  const int kind = a->c_dtype == FXB_DTYPE_F32 ? EK_F32
                   : (epi == FXB_EPI_GELU || epi == FXB_EPI_BIAS_GELU || epi == FXB_EPI_BIAS_SILU ||
                      epi == FXB_EPI_GELU_DERIV)
                       ? EK_ACT16
                   : (epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU) ? EK_DACT16
                                                                      : EK_LIN16;
  if (M == 0 || N == 0) return FXB_OK;
  if (K == 0) return set_error(FXB_EUNSUPPORTED, "gemm: K == 0");

  int* err = dev_error_ptr();
  if (!err) return FXB_ECUDA;
  const int sms = num_sms();
  const bool tail_ok = a->workspace && aligned16(a->workspace) &&
                       a->workspace_bytes >= (int64_t)workspace_bytes(sms);
  Plan pl = plan(M, N, K, epi, tail_ok, sms, force_mode());
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
  const long slots = pl.pair ? sms / 2 : sms;
  const long tiles = (long)p.tiles_m * p.tiles_n;
  p.tail_splits = pl.tail_splits;
  p.tail_kb = (p.num_kb + pl.tail_splits - 1) / pl.tail_splits;
  if (pl.tail_splits > 1) {
    p.tail_splits = (p.num_kb + p.tail_kb - 1) / p.tail_kb;  // no empty pieces
    p.full_units = (int)((tiles / slots) * slots);
    p.total_units = p.full_units + (int)(tiles - p.full_units) * p.tail_splits;
  } else {
    p.full_units = (int)(tiles * p.splits);
    p.total_units = p.full_units;
  }
  p.ws_cnt = static_cast<unsigned*>(a->workspace);
  p.ws = tail_ok ? reinterpret_cast<float*>(static_cast<char*>(a->workspace) + kWsCounterBytes)
                 : nullptr;
  p.epi = epi;
  p.c_dtype = a->c_dtype;
  p.alpha = a->alpha;
  p.C = a->C; p.ldc = a->ldc;
  p.R = a->R; p.ldr = a->ldr;
  p.Z = a->Z; p.ldz = a->ldz;
  p.bias = a->bias;
  p.err = err;
  const long units = p.total_units;
  const bool amn = a->a_trans != 0, bmn = a->b_trans != 0;
  const long used = units < slots ? units : slots;
  const int grid = (int)(pl.pair ? 2 * used : used);
  const int fmt = a->dtype == FXB_DTYPE_BF16 ? 1 : 0;
  switch (kind) {
    case EK_LIN16: return gemm_dispatch<EK_LIN16>(pl.pair, BN, fmt, amn, bmn, mp, p, grid, st);
    case EK_ACT16: return gemm_dispatch<EK_ACT16>(pl.pair, BN, fmt, amn, bmn, mp, p, grid, st);
    case EK_DACT16: return gemm_dispatch<EK_DACT16>(pl.pair, BN, fmt, amn, bmn, mp, p, grid, st);
    default: return gemm_dispatch<EK_F32>(pl.pair, BN, fmt, amn, bmn, mp, p, grid, st);
  }
}
}  // namespace fxb

namespace fxb {
int gemm_f32(const fxb_gemm_args* a, cudaStream_t st);  // csrc/gemm_f32.cu
}

// ---------------------------------------------------------------- loss-only linear CE
namespace {
// statistics pairs per row: two per tile of the narrowest tile width (128)
int64_t ce_nstat(int V) { return 2 * (((int64_t)V + 127) / 128); }

// row_loss[r] = logsumexp over the row's (max, sum) pairs - target logit, or
// 0 for an ignored / out-of-range target. One warp per row; the pairs are
// merged around the row maximum (fixed order: deterministic).
__global__ void ce_stats_merge_kernel(const float2* __restrict__ stats, int nstat,
                                      const float* __restrict__ tlogit,
                                      const int64_t* __restrict__ target, float* __restrict__ row_loss,
                                      int64_t rows, int V, int64_t ignore_index) {
  pdl_trigger();
  pdl_wait();  // statistics come from the GEMM before it on the stream
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  const float2* sr = stats + r * nstat;
  float mx = -INFINITY;  // over the pairs that hold columns (sum > 0)
  for (int i = lane; i < nstat; i += 32)
    if (sr[i].y > 0.f) mx = fmaxf(mx, sr[i].x);
  mx = warp_max(mx);
  float s = 0.f;
  for (int i = lane; i < nstat; i += 32) {
    const float2 v = sr[i];
    if (v.y > 0.f) s += v.y * expf(v.x - mx);
  }
  s = warp_sum(s);
  if (lane == 0) {
    const int64_t t = target[r];
    const bool valid = t != ignore_index && t >= 0 && t < V;
    row_loss[r] = valid ? (mx + logf(s)) - tlogit[r] : 0.f;
  }
}
}  // namespace

extern "C" size_t fxb_linear_ce_loss_workspace(int64_t N, int32_t V) {
  if (N < 0 || V < 1) return 0;
  return (size_t)(N * ce_nstat(V) * sizeof(float2) + ((N + 3) / 4) * 4 * sizeof(float));
}

extern "C" int fxb_linear_ce_loss(int32_t dtype, const void* x, int64_t ldx, const void* w,
                                  int64_t ldw, const int64_t* target, float* row_loss,
                                  void* workspace, int64_t N, int32_t D, int32_t V,
                                  int64_t ignore_index, void* stream) {
  using namespace fxb;
  using namespace fxb::gk;
  if (dtype != FXB_DTYPE_BF16 && dtype != FXB_DTYPE_F16)
    return set_error(FXB_EUNSUPPORTED, "linear_ce_loss: dtype %d (bf16 or f16)", dtype);
  if (N < 0 || D <= 0 || V <= 0 || D % 8 || V % 8 || N > INT32_MAX)
    return set_error(FXB_EINVAL, "linear_ce_loss: bad shape N=%lld D=%d V=%d (D, V multiples of 8)",
                     (long long)N, D, V);
  if (!x || !w || !target || !row_loss || !workspace)
    return set_error(FXB_EINVAL, "linear_ce_loss: NULL argument");
  if (!aligned16(x) || !aligned16(w) || !aligned16(workspace) || ldx < D || ldw < D || ldx % 8 || ldw % 8)
    return set_error(FXB_EINVAL, "linear_ce_loss: x / w / workspace alignment or leading dimensions");
  if (N == 0) return FXB_OK;
  cudaStream_t st = as_stream(stream);
  int* err = dev_error_ptr();
  if (!err) return FXB_ECUDA;
  const int sms = num_sms();
  const int M = (int)N, NN = V, K = D;
  Plan pl = plan(M, NN, K, FXB_EPI_STORE, false, sms, force_mode());
  const int BN = pl.BN;
  const int rows = pl.pair ? 256 : 128;
  const int nstat = (int)ce_nstat(V);
  float2* stats = static_cast<float2*>(workspace);
  float* tlogit = reinterpret_cast<float*>(stats + (int64_t)N * nstat);
  Maps mp;
  int r = make_map(&mp.a, dtype, x, (uint64_t)K, (uint64_t)M, ldx, 64, 128);
  if (r) return r;
  r = make_map(&mp.b, dtype, w, (uint64_t)K, (uint64_t)NN, ldw, 64, (uint32_t)(pl.pair ? BN / 2 : BN));
  if (r) return r;
  // no output is stored; the descriptor slots point at the statistics buffer
  r = make_out_map(&mp.c, FXB_DTYPE_F32, stats, 16, (uint64_t)N, 16);
  if (r) return r;
  mp.z = mp.c;
  GemmParams p{};
  p.M = M; p.N = NN; p.K = K;
  p.tiles_m = (M + rows - 1) / rows;
  p.tiles_n = (NN + BN - 1) / BN;
  p.num_kb = (K + BK - 1) / BK;
  p.splits = 1;
  p.kb_per_split = p.num_kb;
  p.tail_splits = 1;
  p.tail_kb = p.num_kb;
  p.full_units = p.tiles_m * p.tiles_n;
  p.total_units = p.full_units;
  p.epi = FXB_EPI_STORE;
  p.c_dtype = FXB_DTYPE_F32;
  p.alpha = 1.f;
  p.err = err;
  p.ce_stats = stats;
  p.ce_nstat = nstat;
  p.ce_target = target;
  p.ce_tlogit = tlogit;
  // pairs of tiles past the vocabulary end (nstat counts 128-column tiles)
  // and rows whose target is not in range are never written by the GEMM
  r = check_cuda(cudaMemsetAsync(stats, 0, (size_t)N * nstat * sizeof(float2), st), "linear_ce_loss: clear");
  if (r) return r;
  const long slots = pl.pair ? sms / 2 : sms;
  const long used = p.total_units < slots ? p.total_units : slots;
  const int grid = (int)(pl.pair ? 2 * used : used);
  const int fmt = dtype == FXB_DTYPE_BF16 ? 1 : 0;
  r = gemm_dispatch<EK_CESTAT>(pl.pair, BN, fmt, false, false, mp, p, grid, st);
  if (r) return r;
  const int64_t threads = N * 32;
  pdl_launch(ce_stats_merge_kernel, (unsigned)((threads + 255) / 256), 256, 0, st,
             static_cast<const float2*>(stats), nstat, static_cast<const float*>(tlogit), target,
             row_loss, (int64_t)N, V, ignore_index);
  return check_launch("ce_stats_merge");
}

// fp32 operands (the parity mode): validated here, computed by the SIMT kernel
static int gemm_f32_entry(const fxb_gemm_args* a, cudaStream_t st) {
  using namespace fxb;
  const int M = a->M, N = a->N, K = a->K, epi = a->epilogue;
  if (M < 0 || N < 0 || K < 0) return set_error(FXB_EINVAL, "gemm: negative size");
  if (!a->A || !a->B || !a->C) return set_error(FXB_EINVAL, "gemm: NULL operand");
  if (epi < 0 || epi > FXB_EPI_MUL) return set_error(FXB_EINVAL, "gemm: bad epilogue %d", epi);
  if (a->lda < (a->a_trans ? M : K) || a->ldb < (a->b_trans ? N : K) || a->ldc < N)
    return set_error(FXB_EINVAL, "gemm: leading dimension shorter than a row");
  const bool needs_r = (epi == FXB_EPI_RESIDUAL || epi == FXB_EPI_DGELU || epi == FXB_EPI_DSILU ||
                        epi == FXB_EPI_MUL);
  if (needs_r && (!a->R || a->ldr < N)) return set_error(FXB_EINVAL, "gemm: epilogue needs R");
  const bool needs_z = (epi == FXB_EPI_GELU || epi == FXB_EPI_BIAS_GELU || epi == FXB_EPI_BIAS_SILU ||
                        epi == FXB_EPI_GELU_DERIV);
  if (needs_z && (!a->Z || a->ldz < N)) return set_error(FXB_EINVAL, "gemm: epilogue needs Z");
  const bool has_bias = (epi == FXB_EPI_BIAS || epi == FXB_EPI_BIAS_GELU || epi == FXB_EPI_BIAS_SILU);
  if (has_bias && !a->bias) return set_error(FXB_EINVAL, "gemm: epilogue needs bias");
  if (M == 0 || N == 0) return FXB_OK;
  if (K == 0) return set_error(FXB_EUNSUPPORTED, "gemm: K == 0");
  return gemm_f32(a, st);
}

extern "C" int fxb_gemm(const fxb_gemm_args* args, void* stream) {
  if (!args) return fxb::set_error(FXB_EINVAL, "gemm: args is NULL");
  if (args->dtype == FXB_DTYPE_F32) return gemm_f32_entry(args, fxb::as_stream(stream));
  return fxb::gemm_launch(args, args->epilogue, 0, fxb::as_stream(stream));
}

extern "C" size_t fxb_gemm_workspace_size(void) { return workspace_bytes(fxb::num_sms()); }

extern "C" int fxb_gemm_plan(int32_t M, int32_t N, int32_t K, int32_t epilogue, int32_t* pair,
                             int32_t* bn, int32_t* splits) {
  if (!pair || !bn || !splits || M < 0 || N < 0 || K < 0)
    return fxb::set_error(FXB_EINVAL, "gemm_plan: bad arguments");
  Plan pl = plan(M, N, K, epilogue, true, fxb::num_sms(), force_mode());
  *pair = pl.pair ? 1 : 0;
  *bn = pl.BN;
  *splits = epilogue == FXB_EPI_ACCUM_F32 ? pl.splits : pl.tail_splits;
  return FXB_OK;
}
