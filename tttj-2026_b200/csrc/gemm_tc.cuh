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
// warp 1 owns TMEM and one thread issues tcgen05.mma (M=128, N=BN, K=16), warps 2-9
// drain the double-buffered TMEM accumulator (tcgen05.ld 32x32b) through the
// epilogue while the next tile's MMAs run.  Two epilogue warps share each TMEM lane
// quadrant and split the tile's columns.  Each epilogue warp stages a 32x32 output
// block in shared memory (swizzled to match the store's tensor map) and writes it
// with one TMA tile store; only the tile that straddles the last valid row falls back
// to row-masked stores.  One CTA per SM; tiles are walked persistently, N-tile
// fastest, so the CTAs in flight share A row-blocks in L2.
// The number of valid rows is read from device memory, so one launch shape serves
// every valid-token count (no host synchronisation on the mask).
#pragma once
#include "common.cuh"
#include "params.h"

namespace tttj {

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int OUT_BYTES = GEMM_EPI_WARPS * GEMM_STAGE_OUT_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 4 + 1) * 8 + 16;
  // +1024 so the tile ring can be aligned to the 1024-byte swizzle atom.
  static constexpr int TOTAL = TILE_BYTES + OUT_BYTES + BAR_BYTES + 1024;
};

template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
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

  const int warp = warp_id();
  const int lane = lane_id();

  const int n_tiles = p.n / BN + ((p.n % BN) ? 1 : 0);
  const int k_iters = p.k / GEMM_BK;
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
      mbar_init(bar_acce + 8 * b, GEMM_EPI_WARPS * 32);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  griddep_wait();
  griddep_launch();
  const int rows = p.rows_dev ? min(*p.rows_dev, p.rows_max) : p.rows_max;
  const int m_tiles = (rows + GEMM_BM - 1) / GEMM_BM;
  const int num_tiles = m_tiles * n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / n_tiles;
        const int n_blk = tile - m_blk * n_tiles;
        for (int kk = 0; kk < k_iters; ++kk) {
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_full + 8 * stage, L::STAGE_BYTES);
          tma_load_2d(sA + stage * L::A_BYTES, &tmA, bar_full + 8 * stage, kk * GEMM_BK,
                      m_blk * GEMM_BM);
          tma_load_2d(sB + stage * L::B_BYTES, &tmB, bar_full + 8 * stage, kk * GEMM_BK,
                      n_blk * BN);
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
        // Let the loads already issued land before the CTA can exit.
        for (long j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j) {
          mbar_wait(bar_full + 8 * (int)(j % STAGES), (uint32_t)((j / STAGES) & 1), nullptr,
                    limit);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(GEMM_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(bar_acce + 8 * acc, acc_phase ^ 1u, abort_flag, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kk = 0; kk < k_iters; ++kk) {
          if (!mbar_wait(bar_full + 8 * stage, phase, abort_flag, limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(sA + stage * L::A_BYTES);
          const uint64_t bdesc = desc_kmajor_sw128(sB + stage * L::B_BYTES);
#pragma unroll
          for (int j = 0; j < GEMM_BK / 16; ++j) {
            // Advance 16 fp16 (32 B) along K inside the 128-byte swizzle atom.
            mma_f16_ss(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), idesc,
                       (kk | j) != 0 ? 1u : 0u);
          }
          issued_any = true;
          mma_commit(bar_empty + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(bar_accf + 8 * acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_MMA);
        if (issued_any) {
          // Wait for the MMAs already issued before TMEM is released.
          mma_commit(bar_drain);
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
    const int col_half = (warp - 2) >> 2;       // which half of the tile's columns
    const int row_in_tile = quad * 32 + lane;
    const uint32_t stage_out = sOut + (uint32_t)((warp - 2) * GEMM_STAGE_OUT_BYTES);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile / n_tiles;
      const int n_blk = tile - m_blk * n_tiles;
      if (!mbar_wait(bar_accf + 8 * acc, acc_phase, abort_flag, limit)) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      const int row = m_blk * GEMM_BM + row_in_tile;
      const bool row_ok = row < rows;
      float ln_mean = 0.f, ln_rstd = 0.f;
      if (FOLD && row_ok) {
        float ssum = 0.f, ssq = 0.f;
        const float2* st = p.stats_in + (size_t)row * p.stats_parts;
        for (int j = 0; j < p.stats_parts; ++j) {  // fixed order: deterministic
          const float2 v2 = st[j];
          ssum += v2.x;
          ssq += v2.y;
        }
        const float inv_k = 1.0f / (float)p.k;
        ln_mean = ssum * inv_k;
        const float var = fmaxf(ssq * inv_k - ln_mean * ln_mean, 0.f);
        ln_rstd = rsqrtf(var + p.ln_eps);
      }
      float row_sum = 0.f, row_sq = 0.f;  // EPI_RESIDUAL_F32_STATS
      // Every row of the tile is valid: stage + TMA store.  Otherwise masked stores.
      const bool full_tile = (m_blk + 1) * GEMM_BM <= rows;
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int cc = 0; cc < BN / 64; ++cc) {
        const int c = col_half * (BN / 64) + cc;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
        tmem_wait_ld();
        const int col0 = n_blk * BN + c * 32;
        if (col0 >= p.n) continue;  // warp-uniform
        const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
        float v[32];
        if (FOLD) {
          const float4* c4 = reinterpret_cast<const float4*>(p.colsum + col0);
          const float nm = -ln_mean;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            const float4 cs = __ldg(c4 + q);
            v[4 * q + 0] = fmaf(fmaf(nm, cs.x, __uint_as_float(r[4 * q + 0])), ln_rstd, bb.x);
            v[4 * q + 1] = fmaf(fmaf(nm, cs.y, __uint_as_float(r[4 * q + 1])), ln_rstd, bb.y);
            v[4 * q + 2] = fmaf(fmaf(nm, cs.z, __uint_as_float(r[4 * q + 2])), ln_rstd, bb.z);
            v[4 * q + 3] = fmaf(fmaf(nm, cs.w, __uint_as_float(r[4 * q + 3])), ln_rstd, bb.w);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            v[4 * q + 0] = __uint_as_float(r[4 * q + 0]) + bb.x;
            v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + bb.y;
            v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + bb.z;
            v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + bb.w;
          }
        }
        if (EPI == EPI_BIAS_GELU || EPI == EPI_LN_FOLD_GELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
        }
        if (row_ok) {
          if (RES_F32) {
            const float4* rs = reinterpret_cast<const float4*>(
                static_cast<const float*>(p.residual) + (size_t)row * p.ldr + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 rv = rs[q];
              v[4 * q + 0] += rv.x;
              v[4 * q + 1] += rv.y;
              v[4 * q + 2] += rv.z;
              v[4 * q + 3] += rv.w;
            }
          } else if (EPI == EPI_BIAS_RESIDUAL) {
            const uint4* rs = reinterpret_cast<const uint4*>(
                static_cast<const __half*>(p.residual) + (size_t)row * p.ldr + col0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 rv = rs[q];
              const uint32_t rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 res = unpack_half2(rr[e]);
                v[8 * q + 2 * e + 0] += res.x;
                v[8 * q + 2 * e + 1] += res.y;
              }
            }
          }
        }
        if (EPI == EPI_RESIDUAL_F32_STATS && row_ok) {
          float s4[4] = {0.f, 0.f, 0.f, 0.f}, q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s4[i & 3] += v[i];
            q4[i & 3] = fmaf(v[i], v[i], q4[i & 3]);
          }
          row_sum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
          row_sq += (q4[0] + q4[1]) + (q4[2] + q4[3]);
          // fp16 copy of the new residual: the next (LayerNorm-folded) GEMM's A operand.
          uint4* d16 = reinterpret_cast<uint4*>(p.out16 + (size_t)row * p.ld16 + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d16[q] = make_uint4(pack_half2(v[8 * q + 0], v[8 * q + 1]),
                                pack_half2(v[8 * q + 2], v[8 * q + 3]),
                                pack_half2(v[8 * q + 4], v[8 * q + 5]),
                                pack_half2(v[8 * q + 6], v[8 * q + 7]));
        }
        if (full_tile) {
          // The previous TMA store from this warp's staging block must have read it.
          if (lane == 0) bulk_wait_read_all();
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
            const uint32_t rbase = stage_out + (uint32_t)(lane * 64);
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
            tma_store_2d(&tmC, stage_out, col0, m_blk * GEMM_BM + quad * 32);
            bulk_commit();
          }
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
      tc_fence_before();
      mbar_arrive(bar_acce + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if (EPI == EPI_RESIDUAL_F32_STATS && row_ok)
        p.stats_out[(size_t)row * p.stats_parts + 2 * n_blk + col_half] =
            make_float2(row_sum, row_sq);
    }
    // Stores issued by this warp must complete before the CTA exits.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace tttj
