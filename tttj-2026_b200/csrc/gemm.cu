// Instantiations and launcher of the K1 tcgen05 GEMM (gemm_tc.cuh).
#include "launch.h"
#include "gemm_tc.cuh"

namespace tttj {

namespace {

constexpr int STAGES_BN64 = 8;   // 8 x 24 KB ring (+32 KB output staging)
constexpr int STAGES_BN128 = 6;  // 6 x 32 KB ring (+32 KB output staging)
constexpr int STAGES_BN256 = 4;  // 4 x 48 KB ring (+32 KB output staging)
// CTA pairs hold half of B per CTA: the same shared memory buys deeper rings.
constexpr int STAGES_PAIR_BN128 = 8;  // 8 x 24 KB
constexpr int STAGES_PAIR_BN256 = 6;  // 6 x 32 KB
// With two TMA-fed residual staging blocks per epilogue warp (64 KB), the rings that
// still fit: 5 x 32 KB or 6 x 24 KB.  (Measured on C5 out_proj: two blocks and five
// stages 149 us, three blocks and four stages 150 us at a higher clock, one block
// prefetched through registers with six stages 173 us.)
constexpr int RBUF = 2;
constexpr int STAGES_RB_PAIR_BN256 = 5;
constexpr int STAGES_RB_PAIR_BN128 = 6;
constexpr int STAGES_RB_BN128 = 5;
constexpr int STAGES_RB_BN64 = 6;

template <int BN, int EPI, int STAGES, bool PAIR, int RB = 0, int EPIW = GEMM_EPI_WARPS>
cudaError_t launch_t(const GemmLaunch& g, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, EPI, STAGES, PAIR, RB, EPIW>;
  constexpr int smem = GemmSmem<BN, STAGES, PAIR, RB, EPIW>::TOTAL;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  static_assert(smem <= 232448, "GEMM shared memory exceeds the 227 KB per-CTA limit");
  if (PAIR)
    return launch_pdl_cluster(kern, dim3(g.grid), dim3(gemm_threads(EPIW)), smem, stream, 2,
                              g.tmA, g.tmB, g.tmC, g.p);
  return launch_pdl(kern, dim3(g.grid), dim3(gemm_threads(EPIW)), smem, stream, g.tmA, g.tmB,
                    g.tmC, g.p);
}

template <int BN, int STAGES, bool PAIR>
cudaError_t launch_bn(const GemmLaunch& g, cudaStream_t stream) {
  switch (g.epi) {
    case EPI_BIAS:
      return launch_t<BN, EPI_BIAS, STAGES, PAIR>(g, stream);
    case EPI_BIAS_GELU:
      return launch_t<BN, EPI_BIAS_GELU, STAGES, PAIR>(g, stream);
    case EPI_BIAS_RESIDUAL:
      return launch_t<BN, EPI_BIAS_RESIDUAL, STAGES, PAIR>(g, stream);
    case EPI_BIAS_RESIDUAL_F32:
      return launch_t<BN, EPI_BIAS_RESIDUAL_F32, STAGES, PAIR>(g, stream);
    case EPI_RESIDUAL_F32_STATS:
      return launch_t<BN, EPI_RESIDUAL_F32_STATS, STAGES, PAIR>(g, stream);
    case EPI_LN_FOLD:
      return launch_t<BN, EPI_LN_FOLD, STAGES, PAIR>(g, stream);
    case EPI_LN_FOLD_GELU:
      return launch_t<BN, EPI_LN_FOLD_GELU, STAGES, PAIR>(g, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

// The erf-GELU epilogues of 256-wide tiles with twelve epilogue warps.
template <int STAGES, bool PAIR>
cudaError_t launch_wide(const GemmLaunch& g, cudaStream_t stream) {
  constexpr int W = GEMM_EPI_WARPS_WIDE;
  switch (g.epi) {
    case EPI_BIAS_GELU:
      return launch_t<256, EPI_BIAS_GELU, STAGES, PAIR, 0, W>(g, stream);
    case EPI_LN_FOLD_GELU:
      return launch_t<256, EPI_LN_FOLD_GELU, STAGES, PAIR, 0, W>(g, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

// The in-place fp32 residual epilogues with TMA-fed residual staging.
template <int BN, int STAGES, bool PAIR>
cudaError_t launch_rbuf(const GemmLaunch& g, cudaStream_t stream) {
  switch (g.epi) {
    case EPI_BIAS_RESIDUAL_F32:
      return launch_t<BN, EPI_BIAS_RESIDUAL_F32, STAGES, PAIR, RBUF>(g, stream);
    case EPI_RESIDUAL_F32_STATS:
      return launch_t<BN, EPI_RESIDUAL_F32_STATS, STAGES, PAIR, RBUF>(g, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace

// The residual epilogue (fp32 residual in and out, fp16 copy, statistics) moves ~10 bytes
// per output element against 2 K FLOPs; at short K it, not the MMA, sets the pace, and
// with the residual prefetched only one 32-column chunk ahead through registers each
// chunk waits for its load (measured: C5 out_proj, K = 1024, at half the DRAM
// bandwidth, long-scoreboard stalls first).  TMA-fed staging blocks let the residual
// loads run ahead without registers; they cost a ring stage, which long-K GEMMs can
// spare as well (measured with and without at K = 2048-4096: ffn_out C5 355 -> 350-354
// us, C4 116-120 -> 114 us, C2 forward 0.428 -> 0.426 ms, same box).
int gemm_choose_rbuf(int bn, int pair, int k, int epi, bool in_place) {
  (void)k;
  const bool residual = epi == EPI_BIAS_RESIDUAL_F32 || epi == EPI_RESIDUAL_F32_STATS;
  if (!residual || !in_place) return 0;
  if (bn == 256 && !pair) return 0;  // a 48 KB stage: too few would fit
  return RBUF;
}

int gemm_choose_bn(int rows, int n, int num_sms) {
  // The widest column tile whose tile count (128-row tiles) still fills >= 90% of the
  // SMs: wider tiles re-read A less and amortise the epilogue over a longer MMA, but a
  // tile count below the SM count leaves SMs idle.  (Measured on B200 over the
  // projection shapes of the benchmark configurations: BN 256 wins every large GEMM by
  // up to 1.4x over BN 128; the narrow tiles win only when 256-wide tiles cannot fill
  // the machine.)
  const long m_tiles = (rows + GEMM_BM - 1) / GEMM_BM;
  const long need = (long)num_sms * 9 / 10;
  for (int bn : {256, 128}) {
    if (n % bn == 0 && m_tiles * (n / bn) >= need) return bn;
  }
  return 64;
}

// Long-K residual GEMMs (ffn_out: fp32 residual epilogue, K >= 2048): the tile shape
// with the shortest estimated main loop plus epilogue tail.  Per k-block of 64, a CTA's
// shared memory takes the TMA writes of its A and B boxes and the MMA's reads of the
// same bytes at ~128 B/clock, and the tensor core needs 2 * (columns it computes)
// clocks: a 128 x 128 single-CTA tile is held to half the tensor rate by shared memory,
// a 128 x 256 one to two thirds, a CTA pair's 256 x 256 tile runs at the full rate (each
// CTA holds half of B).  The epilogue of the last tile (fp32 residual in and out, fp16
// copy, statistics) is not hidden behind any MMA: ~50 clocks per output column of the
// CTA's 128 rows.  (Measured on B200 with per-k-block clock stamps, C2 ffn_out:
// 128 x 128 tiles 21 us, 128 x 256 18 us, pair 256 x 256 17.8 us.)  Only shapes whose
// tiles occupy at least three quarters of the SMs compete: with fewer, the busy SMs'
// own feed, not shared memory, sets the pace (measured: C2 at 1024-2048 rows runs
// faster on 64-wide single-CTA tiles than on half-empty pairs).  Returns false when no
// shape qualifies.
static bool choose_long_k_residual(int rows, int n, int k, int num_sms, int* bn, int* pair) {
  double best = 0.0;
  for (int cand_pair = 0; cand_pair <= 1; ++cand_pair) {
    for (int cand_bn : {128, 256}) {
      if (n % cand_bn) continue;
      const long rows_per_tile = cand_pair ? 2 * GEMM_BM : GEMM_BM;
      const long tiles = (rows + rows_per_tile - 1) / rows_per_tile * (n / cand_bn);
      const long units = cand_pair ? num_sms / 2 : num_sms;
      if (tiles * 4 < units * 3) continue;
      const long waves = (tiles + units - 1) / units;
      const double b_bytes = (cand_pair ? cand_bn / 2 : cand_bn) * GEMM_BK * 2.0;
      const double smem_clk = 2.0 * (GEMM_BM * GEMM_BK * 2.0 + b_bytes) / 128.0;
      const double kblock_clk = smem_clk > 2.0 * cand_bn ? smem_clk : 2.0 * cand_bn;
      const double est = (double)waves * ((k + GEMM_BK - 1) / GEMM_BK) * kblock_clk + 50.0 * cand_bn;
      if (best == 0.0 || est < best) {
        best = est;
        *bn = cand_bn;
        *pair = cand_pair;
      }
    }
  }
  return best != 0.0;
}

void gemm_choose(int rows, int n, int k, int epi, int num_sms, int* bn, int* pair) {
  const bool residual = epi == EPI_BIAS_RESIDUAL_F32 || epi == EPI_RESIDUAL_F32_STATS;
  if (residual && k >= 2048 && n % 128 == 0 && num_sms >= 2 &&
      choose_long_k_residual(rows, n, k, num_sms, bn, pair))
    return;
  *bn = gemm_choose_bn(rows, n, num_sms);
  // CTA pairs (256-row tiles) cut each SM's operand traffic by a third and deepen the
  // ring, which pays where the main loop dominates: long K, and enough tiles that the
  // doubled tile size does not cost a partial wave.  They lose (measured) on short-K /
  // few-wave GEMMs where the pair's coupling and ramp-up outweigh the feed.  (The
  // erf-GELU GEMMs at K = 1024 lost with eight epilogue warps and win with twelve:
  // C5 ffn_in 397-407 -> 382-383 us, same box.)
  *pair = 0;
  if (*bn == 128 || *bn == 256) {
    const double units = (double)(num_sms / 2);
    const double waves = (double)((rows + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * (n / *bn) / units;
    if ((k >= 2048 && waves >= 3.0) || (k >= 1024 && waves >= 6.0)) *pair = 1;
  }
}

// Epilogue warps: twelve for the erf-GELU epilogues of 256-wide tiles, whose per-element
// arithmetic makes the epilogue as long as or longer than the main loop at K <= 1024
// (per-tile clock stamps: C5 ffn_in ~9.5k epilogue vs ~8.7k MMA clocks per tile, C2
// ~9k vs ~4k); eight otherwise.  Measured same box: ffn_in C5 403 -> 381 us, C2 35.3 ->
// 33.9 us; the LayerNorm fold alone (QKV) measured 1-3% slower with twelve.
int gemm_choose_epiw(int bn, int epi, int rbuf) {
  const bool gelu = epi == EPI_BIAS_GELU || epi == EPI_LN_FOLD_GELU;
  return (gelu && bn == 256 && rbuf == 0) ? GEMM_EPI_WARPS_WIDE : GEMM_EPI_WARPS;
}

cudaError_t gemm_launch(const GemmLaunch& g, cudaStream_t stream) {
  if (g.epiw == GEMM_EPI_WARPS_WIDE) {
    if (g.bn != 256) return cudaErrorInvalidValue;
    if (g.pair) return launch_wide<STAGES_PAIR_BN256, true>(g, stream);
    return launch_wide<STAGES_BN256, false>(g, stream);
  }
  if (g.rbuf) {
    if (g.rbuf != RBUF) return cudaErrorInvalidValue;
    if (g.pair && g.bn == 256) return launch_rbuf<256, STAGES_RB_PAIR_BN256, true>(g, stream);
    if (g.pair && g.bn == 128) return launch_rbuf<128, STAGES_RB_PAIR_BN128, true>(g, stream);
    if (!g.pair && g.bn == 128) return launch_rbuf<128, STAGES_RB_BN128, false>(g, stream);
    if (!g.pair && g.bn == 64) return launch_rbuf<64, STAGES_RB_BN64, false>(g, stream);
    return cudaErrorInvalidValue;
  }
  if (g.pair) {
    if (g.bn == 256) return launch_bn<256, STAGES_PAIR_BN256, true>(g, stream);
    if (g.bn == 128) return launch_bn<128, STAGES_PAIR_BN128, true>(g, stream);
    return cudaErrorInvalidValue;
  }
  if (g.bn == 256) return launch_bn<256, STAGES_BN256, false>(g, stream);
  if (g.bn == 128) return launch_bn<128, STAGES_BN128, false>(g, stream);
  if (g.bn == 64) return launch_bn<64, STAGES_BN64, false>(g, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tttj
