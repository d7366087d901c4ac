// K1: persistent, warp-specialised tcgen05 GEMM with fused epilogues.
//
//   out[m, n] = epilogue( sum_k A[m, k] * W[n, k] + bias[n] )
//
// A is a token-major activation [rows, K] fp16, W an nn.Linear weight [N, K] fp16
// (both K-major).  This replaces the reference's cuBLAS `F.linear` calls and its
// Triton linear-epilogue kernels (kernels/case13_linear.py:149-259,
// kernels/layerwise_hybrid.py:188-192,307,324-327) for the four projections of
// BaselineTransformerBlock (benchmarks/torch_transformer_benchmark.py:72-75,131-132).
//
// CTA = 10 warps: warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
// warp 1 owns TMEM and issues tcgen05.mma (M=128, N=BN, K=16; one elected lane), warps 2-9
// drain the double-buffered TMEM accumulator (tcgen05.ld 32x32b) through the
// epilogue while the next tile's MMAs run.  Two epilogue warps share each TMEM lane
// quadrant and split the tile's columns.  Each epilogue warp stages a 32x32 output
// block in shared memory (swizzled to match the store's tensor map) and writes it
// with one TMA tile store; only the tile that straddles the last valid row falls back
// to row-masked stores.  One CTA per SM; tiles are walked persistently, N-tile
// fastest, so the CTAs in flight share A row-blocks in L2.
// Large GEMMs run on CTA pairs (PAIR, a cluster of 2): the even CTA issues M=256
// tcgen05.mma.cta_group::2 over both CTAs' shared memory, each CTA loads its 128 rows
// of A and half of the tile's B columns (its loads complete on the leader's barrier),
// and each drains its own 128 x BN accumulator.  Per SM that is two thirds of the
// operand bytes of a 128 x BN tile, and the freed shared memory deepens the ring.
// The number of valid rows is read from device memory, so one launch shape serves
// every valid-token count (no host synchronisation on the mask).
#pragma once
#include "common.cuh"
#include "params.h"

namespace tttj {

// PAIR: the tile is 256 x BN, computed by a CTA pair (cluster of 2) with cta_group::2
// MMAs; each CTA holds 128 rows of A and BN/2 rows of B per stage and drains its own
// 128 x BN accumulator.
// RBUF (fp32 residual epilogues updating the residual in place): each epilogue warp
// owns RBUF 32 x 32 fp32 staging blocks into which TMA loads the residual chunks
// RBUF - 1 chunks ahead of the one being drained (0: one staging block, the residual
// prefetched one chunk ahead through registers).
// EPIW: epilogue warps (GEMM_EPI_WARPS, or GEMM_EPI_WARPS_WIDE for fp16 outputs).
template <int BN, int STAGES, bool PAIR = false, int RBUF = 0, int EPIW = GEMM_EPI_WARPS>
struct GemmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int OUT_BUFS = RBUF > 0 ? RBUF : 1;
  // Staging block per epilogue warp: 32 x 32 fp32, or 32 x 32 fp16 for the wide variant.
  static constexpr int BLK_BYTES = EPIW == GEMM_EPI_WARPS ? GEMM_STAGE_OUT_BYTES : GEMM_STAGE_OUT_BYTES / 2;
  static constexpr int OUT_BYTES = EPIW * BLK_BYTES * OUT_BUFS;
  // full / empty per stage, 2 + 2 accumulator barriers, drain, TMEM slot + abort flag,
  // one residual-load barrier per staging block.
  static constexpr int BAR_BYTES = (2 * STAGES + 6 + EPIW * RBUF) * 8 + 16;
  // +1024 so the tile ring can be aligned to the 1024-byte swizzle atom.
  static constexpr int TOTAL = TILE_BYTES + OUT_BYTES + BAR_BYTES + 1024;
};

template <int BN, int EPI, int STAGES, bool PAIR, int RBUF = 0, int EPIW = GEMM_EPI_WARPS>
__global__ void __launch_bounds__(gemm_threads(EPIW), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using L = GemmSmem<BN, STAGES, PAIR, RBUF, EPIW>;
  static_assert(EPIW == GEMM_EPI_WARPS ||
                    (EPIW == GEMM_EPI_WARPS_WIDE && BN == 256 && RBUF == 0 &&
                     EPI != EPI_BIAS_RESIDUAL && EPI != EPI_BIAS_RESIDUAL_F32 &&
                     EPI != EPI_RESIDUAL_F32_STATS),
                "12 epilogue warps serve the fp16-output epilogues of 256-wide tiles");
  static_assert(RBUF == 0 || RBUF >= 2, "residual staging: one block, or at least two");
  static_assert(RBUF == 0 || EPI == EPI_BIAS_RESIDUAL_F32 || EPI == EPI_RESIDUAL_F32_STATS,
                "TMA residual loads serve the in-place fp32 residual epilogues");
  constexpr int CTAS = PAIR ? 2 : 1;
  constexpr int TM = GEMM_BM * CTAS;  // rows of a tile
  // Scheduling unit: the CTA, or the CTA pair (CTAs 2c and 2c+1 form cluster c).
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * L::A_BYTES;
  const uint32_t sOut = sA + L::TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::TILE_BYTES + L::OUT_BYTES);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_accf = bar_empty + 8 * STAGES;
  const uint32_t bar_acce = bar_accf + 16;
  const uint32_t bar_drain = bar_acce + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar_res = smem_u32(bars + 2 * STAGES + 6);  // [GEMM_EPI_WARPS][RBUF]

  const int warp = warp_id();
  const int lane = lane_id();

  const int n_tiles = p.n / BN + ((p.n % BN) ? 1 : 0);
  const int k_iters = (p.k + GEMM_BK - 1) / GEMM_BK;  // columns past k are zero-filled by TMA
  const uint64_t limit = p.wait_limit_ns;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8 * b, 1);
      // One arrival per epilogue warp of each CTA (a pair's leader counts both CTAs).
      mbar_init(bar_acce + 8 * b, EPIW * CTAS);
    }
    mbar_init(bar_drain, 1);
    for (int i = 0; i < EPIW * RBUF; ++i) mbar_init(bar_res + 8 * i, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), 2 * BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), 2 * BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // A pair's barriers receive arrivals from the peer CTA: both must be initialised first.
  if (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The weights do not depend on the previous kernel: while this CTA waits for it
  // (programmatic dependent launch starts it early), ask L2 for the B boxes of the
  // CTA's first tile.
  if (warp == 0 && lane == 0) {
    const int n_blk0 = unit % n_tiles;
    const int b_row0 = n_blk0 * BN + (int)rank * (BN / CTAS);
    for (int kk = 0; kk < k_iters; ++kk) tma_prefetch_l2_2d(&tmB, kk * GEMM_BK, b_row0);
  }
  griddep_wait();
  griddep_launch();
  const int rows = p.rows_dev ? min(*p.rows_dev, p.rows_max) : p.rows_max;
  const int m_tiles = (rows + TM - 1) / TM;
  const int num_tiles = m_tiles * n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      for (int tile = unit; tile < num_tiles && ok; tile += n_units) {
        const int m_blk = tile / n_tiles;
        const int n_blk = tile - m_blk * n_tiles;
        const int a_row = m_blk * TM + (int)rank * GEMM_BM;
        const int b_row = n_blk * BN + (int)rank * (BN / CTAS);
        for (int kk = 0; kk < k_iters; ++kk) {
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, limit)) {
            ok = false;
            break;
          }
          if (PAIR) {
            // Both CTAs' loads complete on the leader's full barrier, which the leader
            // arms for the bytes of both.
            const uint32_t full_leader = map_to_cta(bar_full + 8 * stage, 0);
            if (rank == 0) mbar_arrive_expect_tx(bar_full + 8 * stage, 2 * L::STAGE_BYTES);
            tma_load_2d_pair(sA + stage * L::A_BYTES, &tmA, full_leader, kk * GEMM_BK, a_row);
            tma_load_2d_pair(sB + stage * L::B_BYTES, &tmB, full_leader, kk * GEMM_BK, b_row);
          } else {
            mbar_arrive_expect_tx(bar_full + 8 * stage, L::STAGE_BYTES);
            tma_load_2d(sA + stage * L::A_BYTES, &tmA, bar_full + 8 * stage, kk * GEMM_BK, a_row);
            tma_load_2d(sB + stage * L::B_BYTES, &tmB, bar_full + 8 * stage, kk * GEMM_BK, b_row);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_PRODUCER);
        // Let the loads already issued land before the CTA can exit.  (A pair's
        // follower cannot observe its loads, which complete on the leader's barrier;
        // both CTAs meet at the final cluster barrier, after every other role has given
        // up waiting, by which time they have landed.)
        if (!PAIR || rank == 0) {
          for (long j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j) {
            mbar_wait(bar_full + 8 * (int)(j % STAGES), (uint32_t)((j / STAGES) & 1), nullptr,
                      limit);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop (waits combined with a vote, so the stage
    // descriptors stay warp-uniform) and one elected lane issues each MMA / commit:
    // issued from a one-lane branch, every MMA would first move its operands into
    // uniform registers.  A pair's MMAs are issued by its leader only.
    constexpr unsigned FULL = 0xffffffffu;
    if (!PAIR || rank == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(TM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = unit; tile < num_tiles && ok; tile += n_units) {
        if (!__all_sync(FULL, mbar_wait(bar_acce + 8 * acc, acc_phase ^ 1u, abort_flag, limit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kk = 0; kk < k_iters; ++kk) {
          if (!__all_sync(FULL, mbar_wait(bar_full + 8 * stage, phase, abort_flag, limit))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(sA + stage * L::A_BYTES);
          const uint64_t bdesc = desc_kmajor_sw128(sB + stage * L::B_BYTES);
#pragma unroll
          for (int j = 0; j < GEMM_BK / 16; ++j) {
            // Advance 16 fp16 (32 B) along K inside the 128-byte swizzle atom.
            if (PAIR)
              mma_f16_ss_pair_warp(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j),
                                   idesc, (kk | j) != 0 ? 1u : 0u);
            else
              mma_f16_ss_warp(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), idesc,
                              (kk | j) != 0 ? 1u : 0u);
          }
          issued_any = true;
          // Frees the stage in both CTAs of a pair.
          if (PAIR)
            mma_commit_pair_mc_warp(bar_empty + 8 * stage, 0x3);
          else
            mma_commit_warp(bar_empty + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR)
          mma_commit_pair_mc_warp(bar_accf + 8 * acc, 0x3);
        else
          mma_commit_warp(bar_accf + 8 * acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        if (lane == 0) {
          *abort_flag = 1;
          report_status(p.status, TTTJ_DEV_TIMEOUT_MMA);
        }
        if (issued_any) {
          // Wait for the MMAs already issued before TMEM is released.
          if (PAIR)
            mma_commit_pair_warp(bar_drain);
          else
            mma_commit_warp(bar_drain);
          mbar_wait(bar_drain, 0, nullptr, limit);
        }
      }
    }
  } else {
    // ---------------- epilogue: warps 2..9 ----------------
    constexpr bool RES_F32 = EPI == EPI_BIAS_RESIDUAL_F32 || EPI == EPI_RESIDUAL_F32_STATS;
    constexpr bool OUT_F32 = RES_F32;
    constexpr bool FOLD = EPI == EPI_LN_FOLD || EPI == EPI_LN_FOLD_GELU;
    const int quad = warp & 3;                  // TMEM lane quadrant this warp may access
    const int col_half = (warp - 2) >> 2;       // which share of the tile's columns
    const int row_in_tile = quad * 32 + lane;
    const uint32_t stage_out = sOut + (uint32_t)((warp - 2) * L::BLK_BYTES);
    int acc = 0;
    uint32_t acc_phase = 0;
    // fp16-output staging halves per warp block (32 x 32 x 2 B each), and the TMA stores
    // this warp issued from them.
    constexpr int NSB16 = OUT_F32 ? 1 : (L::BLK_BYTES / 2048 >= 2 ? 2 : 1);
    uint32_t out_seq = 0;
    // Eight epilogue warps: this warp's columns of a tile are one contiguous run of
    // BN/2, chunks col_half*(BN/64) .. +BN/64-1 of 32 columns each.  Twelve: every third
    // chunk, starting at chunk col_half (3, 3 and 2 chunks of a 256-wide tile).
    constexpr int NPART = EPIW / 4;
    constexpr int CHUNKS = EPIW == GEMM_EPI_WARPS ? BN / 64 : (BN / 32 + NPART - 1) / NPART;
    // Residual reads are the epilogue's long-latency operand.  Each warp asks L2 for
    // its rows' segment of the NEXT tile while the current one is drained, loads the
    // first chunk of the current tile before the accumulator is ready, and loads chunk
    // c + 1 as soon as chunk c's values are consumed.
    auto prefetch_residual = [&](int t) {
      // (RBUF > 0: the TMA loads run ahead already.)
      if (!(RES_F32 || EPI == EPI_BIAS_RESIDUAL) || RBUF > 0 || t >= num_tiles) return;
      const int mb = t / n_tiles;
      const int c0 = (t - mb * n_tiles) * BN + col_half * (BN / 2);
      const int r = mb * TM + (int)rank * GEMM_BM + row_in_tile;
      const int esize = RES_F32 ? 4 : 2;
      const uint32_t bytes = (uint32_t)(min(BN / 2, p.n - c0) * esize) & ~15u;
      if (r < rows && c0 < p.n && bytes > 0)
        bulk_prefetch_l2(static_cast<const uint8_t*>(p.residual) +
                             ((size_t)r * p.ldr + c0) * esize, bytes);
    };
    // Residual of the chunk being drained, in one of two register layouts.  Full tiles
    // of the fp32 epilogues use the "coalesced" one: element q of lane l is row
    // 4q + l/8 of the warp's 32 rows, columns 4(l%8)..+3, so each load instruction
    // reads four whole 128-byte row segments; the values reach their row's lane through
    // the staging block.  Otherwise lane l holds row l's 32 columns ("by row").
    float4 rc[8];
    auto load_res = [&](bool coalesced, int row0, int row, int col0) {
      if (RES_F32 && coalesced) {
        const float* base = static_cast<const float*>(p.residual) +
                            (size_t)(row0 + (lane >> 3)) * p.ldr + col0 + 4 * (lane & 7);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          rc[q] = *reinterpret_cast<const float4*>(base + (size_t)(4 * q) * p.ldr);
      } else if (RES_F32) {
        const float4* rs = reinterpret_cast<const float4*>(
            static_cast<const float*>(p.residual) + (size_t)row * p.ldr + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q) rc[q] = rs[q];
      } else if (EPI == EPI_BIAS_RESIDUAL) {
        const uint4* rs = reinterpret_cast<const uint4*>(
            static_cast<const __half*>(p.residual) + (size_t)row * p.ldr + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 x = rs[q];
          const float2 a = unpack_half2(x.x), b = unpack_half2(x.y);
          const float2 c = unpack_half2(x.z), d = unpack_half2(x.w);
          rc[2 * q] = make_float4(a.x, a.y, b.x, b.y);
          rc[2 * q + 1] = make_float4(c.x, c.y, d.x, d.y);
        }
      }
    };
    // RBUF > 0: the residual chunks of full tiles come by TMA (from tmC: the residual is
    // updated in place) into this warp's staging blocks, in the order the warp drains
    // them, RBUF - 1 chunks ahead.  Load j goes to block j % RBUF and completes on its
    // barrier's phase (j / RBUF) & 1; block j % RBUF is refilled (load j + RBUF - 1)
    // once the TMA store of chunk j - 1, which read it, has finished reading.  Every lane
    // walks the same cursor; lane 0 issues.
    const uint32_t res_buf0 = sOut + (uint32_t)((warp - 2) * RBUF * GEMM_STAGE_OUT_BYTES);
    const uint32_t res_bar0 = bar_res + (uint32_t)(8 * (warp - 2) * RBUF);
    int ld_k = 0, ld_cc = 0;        // load cursor: k-th tile of this unit, chunk in the tile
    long ld_issued = 0, ld_used = 0;
    auto issue_next_load = [&]() {
      if constexpr (RBUF > 0) {
        while (true) {
          const int t = unit + ld_k * n_units;
          if (t >= num_tiles) return;
          const int cc = ld_cc;
          if (++ld_cc == CHUNKS) {
            ld_cc = 0;
            ++ld_k;
          }
          const int mb = t / n_tiles;
          const int cta_r0 = mb * TM + (int)rank * GEMM_BM;
          const int c0 = (t - mb * n_tiles) * BN + (col_half * CHUNKS + cc) * 32;
          if (cta_r0 + GEMM_BM > rows || c0 >= p.n) continue;  // drained without TMA
          const int b = (int)(ld_issued % RBUF);
          if (lane == 0) {
            mbar_arrive_expect_tx(res_bar0 + 8 * b, GEMM_STAGE_OUT_BYTES);
            tma_load_2d(res_buf0 + (uint32_t)(b * GEMM_STAGE_OUT_BYTES), &tmC, res_bar0 + 8 * b,
                        c0, cta_r0 + quad * 32);
          }
          ++ld_issued;
          return;
        }
      }
    };
    if constexpr (RBUF > 0) {
      for (int i = 0; i < RBUF - 1; ++i) issue_next_load();
    }
    // Row statistics of the LayerNorm this epilogue applies (FOLD), or whose mean
    // pivots the statistics it writes (EPI_RESIDUAL_F32_STATS), are loaded one tile
    // ahead: the loads for tile t + n_units issue when tile t starts and land while
    // its chunks drain.  (Loaded at the start of their own tile they cost each tile
    // several thousand clocks, measured with per-tile clock stamps.)  Counts above
    // MAXP partials are loaded in place.
    constexpr int MAXP = 16;
    constexpr bool ROWSTATS = FOLD || EPI == EPI_RESIDUAL_F32_STATS;
    const float2* st_src = FOLD ? p.stats_in : p.stats_prev;
    const int st_parts = FOLD ? p.stats_parts : p.stats_prev_parts;
    const bool st_ahead = ROWSTATS && st_parts <= MAXP;
    float2 pst[ROWSTATS ? MAXP : 1];
    float ppiv = 0.f;
    auto fetch_row_stats = [&](int t) {
      if constexpr (ROWSTATS) {
        if (!st_ahead || t >= num_tiles) return;
        const int r = (t / n_tiles) * TM + (int)rank * GEMM_BM + row_in_tile;
        if (r >= rows) return;
        const float2* st = st_src + (size_t)r * st_parts;
        if ((st_parts & 1) == 0) {
          // Two partials per 16-byte load (even counts: a row starts 16-byte aligned).
          const float4* st4 = reinterpret_cast<const float4*>(st);
#pragma unroll
          for (int j = 0; j < MAXP / 2; ++j) {
            if (2 * j < st_parts) {
              const float4 v = __ldg(st4 + j);
              pst[2 * j] = make_float2(v.x, v.y);
              pst[2 * j + 1] = make_float2(v.z, v.w);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < MAXP; ++j)
            if (j < st_parts) pst[j] = __ldg(st + j);
        }
        if (EPI == EPI_RESIDUAL_F32_STATS) ppiv = __ldg(p.pivot_prev + r);
      }
    };
    fetch_row_stats(unit);
    prefetch_residual(unit);
    for (int tile = unit; tile < num_tiles; tile += n_units) {
      const int m_blk = tile / n_tiles;
      const int n_blk = tile - m_blk * n_tiles;
      prefetch_residual(tile + n_units);
      const int cta_row0 = m_blk * TM + (int)rank * GEMM_BM;  // this CTA's 128 rows
      const int row0 = cta_row0 + quad * 32;  // first of this warp's 32 rows
      const int row = row0 + lane;
      const bool row_ok = row < rows;
      // Every row of the CTA's tile is valid: stage + TMA store.  Otherwise masked stores.
      const bool full_tile = cta_row0 + GEMM_BM <= rows;
      const bool staged_res = RES_F32 && full_tile;
      // Everything that does not depend on the accumulator is fetched before waiting
      // for it: the LayerNorm statistics of this row and the first residual chunk.
      float ln_mean = 0.f, ln_rstd = 0.f;
      // EPI_RESIDUAL_F32_STATS: the pivot of this row's new statistics is the mean of
      // the residual before the add (the previous LayerNorm's statistics).
      float shift = 0.f;
      if (ROWSTATS && row_ok) {
        // Partials summed in a fixed order: deterministic, and every CTA of a row
        // agrees on the result.
        float ssum = 0.f, ssq = 0.f, piv = 0.f;
        if (st_ahead) {
#pragma unroll
          for (int j = 0; j < MAXP; ++j) {
            if (j < st_parts) {
              ssum += pst[j].x;
              ssq += pst[j].y;
            }
          }
          piv = ppiv;
        } else {
          const float2* st = st_src + (size_t)row * st_parts;
          for (int j = 0; j < st_parts; ++j) {
            const float2 v2 = st[j];
            ssum += v2.x;
            ssq += v2.y;
          }
          if (EPI == EPI_RESIDUAL_F32_STATS) piv = p.pivot_prev[row];
        }
        if (FOLD) {
          // Partials are of x - pivot, so ln_mean is small against the spread of the
          // row and the variance does not cancel.
          const float inv_k = 1.0f / (float)p.k;
          ln_mean = ssum * inv_k;
          const float var = fmaxf(ssq * inv_k - ln_mean * ln_mean, 0.f);
          ln_rstd = rsqrtf(var + p.ln_eps);
        } else {
          shift = piv + ssum * (1.0f / (float)p.n);
        }
      }
      fetch_row_stats(tile + n_units);
      const int seg0 = n_blk * BN + col_half * (BN / 2);
      if (seg0 < p.n && ((staged_res && RBUF == 0) || (!staged_res && row_ok)))
        load_res(staged_res, row0, row, seg0);
      if (!mbar_wait(bar_accf + 8 * acc, acc_phase, abort_flag, limit)) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      bool res_failed = false;            // a residual load did not arrive in time
      float row_sum = 0.f, row_sq = 0.f;  // EPI_RESIDUAL_F32_STATS
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int cc = 0; cc < CHUNKS; ++cc) {
        const int c = EPIW == GEMM_EPI_WARPS ? col_half * CHUNKS + cc : col_half + NPART * cc;
        if (EPIW != GEMM_EPI_WARPS && c >= BN / 32) break;  // warp-uniform
        const int col0 = n_blk * BN + c * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
        if (col0 >= p.n) {  // warp-uniform
          tmem_wait_ld();
          continue;
        }
        // Per-column operands, loaded while the TMEM read is in flight.
        float4 bb[8], cs[8];
        const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q) bb[q] = __ldg(b4 + q);
        if (FOLD) {
          const float4* c4 = reinterpret_cast<const float4*>(p.colsum + col0);
#pragma unroll
          for (int q = 0; q < 8; ++q) cs[q] = __ldg(c4 + q);
        }
        tmem_wait_ld();
        float v[32];
        if (FOLD) {
          // v = rstd (acc - mean c) + b', in f32x2 pairs.
          const unsigned long long nm2 = pk2(-ln_mean, -ln_mean), rs2 = pk2(ln_rstd, ln_rstd);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float2 lo = upk2(fma2p(fma2p(nm2, pk2(cs[q].x, cs[q].y),
                                               pk2(__uint_as_float(r[4 * q + 0]), __uint_as_float(r[4 * q + 1]))),
                                         rs2, pk2(bb[q].x, bb[q].y)));
            const float2 hi = upk2(fma2p(fma2p(nm2, pk2(cs[q].z, cs[q].w),
                                               pk2(__uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))),
                                         rs2, pk2(bb[q].z, bb[q].w)));
            v[4 * q + 0] = lo.x;
            v[4 * q + 1] = lo.y;
            v[4 * q + 2] = hi.x;
            v[4 * q + 3] = hi.y;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[4 * q + 0] = __uint_as_float(r[4 * q + 0]) + bb[q].x;
            v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + bb[q].y;
            v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + bb[q].z;
            v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + bb[q].w;
          }
        }
        if (EPI == EPI_BIAS_GELU || EPI == EPI_LN_FOLD_GELU) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 g = gelu_erf2(v[i], v[i + 1]);
            v[i] = g.x;
            v[i + 1] = g.y;
          }
        }
        const bool more = cc + 1 < CHUNKS && col0 + 32 < p.n;
        if (staged_res) {
          // 32 rows x 128 B, 128-byte swizzle: 16-byte chunk j of row r at j ^ (r % 8).
          uint32_t blk = stage_out;
          if constexpr (RBUF > 0) {
            // The residual chunk was loaded into block ld_used % RBUF by TMA.
            const int b = (int)(ld_used % RBUF);
            blk = res_buf0 + (uint32_t)(b * GEMM_STAGE_OUT_BYTES);
            if (!__all_sync(0xffffffffu, mbar_wait(res_bar0 + 8 * b, (uint32_t)((ld_used / RBUF) & 1),
                                                   abort_flag, limit))) {
              res_failed = true;
              break;
            }
          } else {
            // The previous TMA store from this warp's staging block must have read it.
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {  // residual in, transposed by position
              const int rr = 4 * q + (lane >> 3), j = lane & 7;
              const uint32_t dst = blk + (uint32_t)(rr * 128 + ((j ^ (rr & 7)) << 4));
              asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(rc[q].x),
                           "f"(rc[q].y), "f"(rc[q].z), "f"(rc[q].w)
                           : "memory");
            }
            __syncwarp();
          }
          const uint32_t rbase = blk + (uint32_t)(lane * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // this row's residual; the sum goes to the same slot
            const uint32_t a = rbase + (uint32_t)(((j ^ (lane & 7)) & 7) << 4);
            float4 x;
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                         : "r"(a)
                         : "memory");
            v[4 * j + 0] += x.x;
            v[4 * j + 1] += x.y;
            v[4 * j + 2] += x.z;
            v[4 * j + 3] += x.w;
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v[4 * j + 0]),
                         "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                         : "memory");
          }
          if (RBUF == 0 && more) load_res(true, row0, row, col0 + 32);
          if (EPI == EPI_RESIDUAL_F32_STATS) {
            float s4[4] = {0.f, 0.f, 0.f, 0.f}, q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = v[i] - shift;
              s4[i & 3] += d;
              q4[i & 3] = fmaf(d, d, q4[i & 3]);
            }
            row_sum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
            row_sq += (q4[0] + q4[1]) + (q4[2] + q4[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, blk, col0, row0);
            bulk_commit();
          }
          if (EPI == EPI_RESIDUAL_F32_STATS) {
            // fp16 copy of the new residual minus its row's pivot (the next
            // LayerNorm-folded GEMM's A operand), read back from the staging block four
            // whole rows per instruction; row rr's pivot comes from lane rr.
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int rr = 4 * q + (lane >> 3), j = lane & 7;
              const float sh = __shfl_sync(0xffffffffu, shift, rr);
              const uint32_t a = blk + (uint32_t)(rr * 128 + ((j ^ (rr & 7)) << 4));
              float4 x;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                           : "r"(a)
                           : "memory");
              *reinterpret_cast<uint2*>(p.out16 + (size_t)(row0 + rr) * p.ld16 + col0 + 4 * j) =
                  make_uint2(pack_half2(x.x - sh, x.y - sh), pack_half2(x.z - sh, x.w - sh));
            }
          }
          if constexpr (RBUF > 0) {
            // Refill the block of the previous chunk (load ld_used + RBUF - 1) once its TMA
            // store has read it; order this warp's generic reads of that block before the
            // async-proxy write.
            ++ld_used;
            if (lane == 0) bulk_wait_read_1();
            __syncwarp();
            fence_proxy_async_smem();
            issue_next_load();
          }
          continue;
        }
        if ((RES_F32 || EPI == EPI_BIAS_RESIDUAL) && row_ok) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[4 * q + 0] += rc[q].x;
            v[4 * q + 1] += rc[q].y;
            v[4 * q + 2] += rc[q].z;
            v[4 * q + 3] += rc[q].w;
          }
          if (more) load_res(false, row0, row, col0 + 32);
        }
        if (EPI == EPI_RESIDUAL_F32_STATS && row_ok) {
          float d[32];
          float s4[4] = {0.f, 0.f, 0.f, 0.f}, q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            d[i] = v[i] - shift;
            s4[i & 3] += d[i];
            q4[i & 3] = fmaf(d[i], d[i], q4[i & 3]);
          }
          row_sum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
          row_sq += (q4[0] + q4[1]) + (q4[2] + q4[3]);
          uint4* d16 = reinterpret_cast<uint4*>(p.out16 + (size_t)row * p.ld16 + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d16[q] = make_uint4(pack_half2(d[8 * q + 0], d[8 * q + 1]),
                                pack_half2(d[8 * q + 2], d[8 * q + 3]),
                                pack_half2(d[8 * q + 4], d[8 * q + 5]),
                                pack_half2(d[8 * q + 6], d[8 * q + 7]));
        }
        if (full_tile) {
          // fp16 outputs take 2 KB of the warp's staging block per chunk: with a 4 KB
          // block the chunks alternate between its halves, and a half is rewritten once
          // the store before last (which read it) is done reading.  Otherwise the
          // previous TMA store from the block must have read it.
          const uint32_t sbuf =
              OUT_F32 ? stage_out : stage_out + (uint32_t)((out_seq % NSB16) * 2048);
          if (lane == 0) {
            if (NSB16 > 1)
              bulk_wait_read_1();
            else
              bulk_wait_read_all();
          }
          __syncwarp();
          if (OUT_F32) {
            // 32 rows x 128 B, 128-byte swizzle: 16-byte chunk j of row r at j ^ (r % 8).
            const uint32_t rbase = stage_out + (uint32_t)(lane * 128);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t dst = rbase + (uint32_t)(((j ^ (lane & 7)) & 7) << 4);
              asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                           "f"(v[4 * j + 0]), "f"(v[4 * j + 1]), "f"(v[4 * j + 2]),
                           "f"(v[4 * j + 3])
                           : "memory");
            }
          } else {
            // 32 rows x 64 B, 64-byte swizzle: 16-byte chunk j of row r at j ^ ((r / 2) % 4).
            const uint32_t rbase = sbuf + (uint32_t)(lane * 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t dst = rbase + (uint32_t)(((j ^ ((lane >> 1) & 3)) & 3) << 4);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                           "r"(pack_half2(v[8 * j + 0], v[8 * j + 1])),
                           "r"(pack_half2(v[8 * j + 2], v[8 * j + 3])),
                           "r"(pack_half2(v[8 * j + 4], v[8 * j + 5])),
                           "r"(pack_half2(v[8 * j + 6], v[8 * j + 7]))
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, sbuf, col0, row0);
            bulk_commit();
          }
          ++out_seq;
        } else if (row_ok) {
          if (OUT_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) +
                                                    (size_t)row * p.ldo + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[q] = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) +
                                                  (size_t)row * p.ldo + col0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              dst[q] = make_uint4(pack_half2(v[8 * q + 0], v[8 * q + 1]),
                                  pack_half2(v[8 * q + 2], v[8 * q + 3]),
                                  pack_half2(v[8 * q + 4], v[8 * q + 5]),
                                  pack_half2(v[8 * q + 6], v[8 * q + 7]));
            }
          }
        }
      }
      if (res_failed) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_EPILOGUE);
        break;
      }
      // The warp's TMEM reads are complete (tcgen05.wait::ld in every lane): release
      // the accumulator to the (leader's) MMA thread.  The arrival orders nothing else
      // (a release would first wait for this thread's global stores).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster_relaxed(map_to_cta(bar_acce + 8 * acc, 0));
        else
          mbar_arrive_relaxed(bar_acce + 8 * acc);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if (EPI == EPI_RESIDUAL_F32_STATS && row_ok) {
        p.stats_out[(size_t)row * p.stats_parts + 2 * n_blk + col_half] =
            make_float2(row_sum, row_sq);
        if (n_blk == 0 && col_half == 0) p.pivot_out[row] = shift;
      }
    }
    // Residual loads still in flight (only after a timeout) land before the CTA exits,
    // and so do the stores issued by this warp.
    if constexpr (RBUF > 0) {
      for (long j = ld_used; j < ld_issued; ++j)
        mbar_wait(res_bar0 + 8 * (int)(j % RBUF), (uint32_t)((j / RBUF) & 1), nullptr, limit);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  // A pair's CTAs leave together: the leader's MMAs write the follower's TMEM, and the
  // follower's loads and arrivals target the leader's barriers.
  if (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, 2 * BN);
    else
      tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace tttj
