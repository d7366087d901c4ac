// Kernel parameter blocks and tile constants shared between the kernels and the
// host-side launch code.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef TTTJ_WAIT_LIMIT_NS
// A device-side wait that has not completed after this many nanoseconds is treated
// as a hang: the waiting role records an error code and the kernel winds down.
#define TTTJ_WAIT_LIMIT_NS 2000000000ull
#endif

// Status codes written into the caller-visible device status word.
enum TttjDeviceStatus : int {
  TTTJ_DEV_OK = 0,
  TTTJ_DEV_TIMEOUT_PRODUCER = 0x101,
  TTTJ_DEV_TIMEOUT_MMA = 0x102,
  TTTJ_DEV_TIMEOUT_EPILOGUE = 0x103,
  TTTJ_DEV_TIMEOUT_SELFTEST = 0x1ff,
  TTTJ_DEV_TIMEOUT_ATTN = 0x201,
  TTTJ_DEV_TIMEOUT_RESIDENT = 0x301,
};


namespace tttj {

enum GemmEpilogue : int {
  EPI_BIAS = 0,           // out = fp16(acc + bias)
  EPI_BIAS_GELU = 1,      // out = fp16(gelu_erf(acc + bias))
  EPI_BIAS_RESIDUAL = 2,  // out = fp16(residual + acc + bias), out may alias residual
  EPI_BIAS_RESIDUAL_F32 = 3,  // fp32 out = fp32 residual + acc + bias (the residual stream)
  // EPI_BIAS_RESIDUAL_F32 that also prepares the next LayerNorm, relative to a per-row
  // pivot c = the row mean of the residual before this add (from stats_prev /
  // pivot_prev): out16 = fp16(out - c), stats_out[row] = (sum, sum of squares) of
  // out - c over this tile's columns, pivot_out[row] = c.  Shifting by a value close to
  // the row mean keeps the variance and the fp16 copy exact for rows whose mean is
  // large against their spread (no sum-of-squares cancellation).
  EPI_RESIDUAL_F32_STATS = 4,
  // LayerNorm folded into the GEMM: A = fp16(x - c), W = W * gamma (per K column), and
  // out = fp16(rstd * (acc - m * colsum[n]) + bias[n]) with m = mean(x - c) and rstd
  // of each row from stats_in[row] = (sum, sum of squares) of x - c over K,
  // bias = b + W beta.  (x - c - m = x - mean(x), whatever the pivot c.)
  EPI_LN_FOLD = 5,
  EPI_LN_FOLD_GELU = 6,  // the same followed by exact erf-GELU
};

struct GemmParams {
  const int* rows_dev;  // device count of valid rows (nullable: use rows_max)
  int rows_max;         // rows allocated in A / out
  int n;                // output columns (multiple of 32)
  int k;                // reduction length (multiple of 8; the last block is zero-filled)
  const float* bias;    // [n] fp32
  void* out;            // [rows, ldo], fp16 (fp32 for EPI_BIAS_RESIDUAL_F32)
  int ldo;
  const void* residual;  // [rows, ldr], same type as out (residual epilogues)
  int ldr;
  int* status;          // device status word (nullable)
  unsigned long long wait_limit_ns;
  // EPI_RESIDUAL_F32_STATS
  __half* out16;        // [rows, ld16] fp16 copy of out - pivot
  int ld16;
  float2* stats_out;    // [rows][stats_parts] (sum, sum of squares) partials of out - pivot
  float* pivot_out;     // [rows] pivot of stats_out / out16
  const float2* stats_prev;  // [rows][stats_prev_parts] partials of the residual before the add
  const float* pivot_prev;   // [rows] their pivot
  int stats_prev_parts;
  // EPI_LN_FOLD*
  const float2* stats_in;  // [rows][stats_parts] partials of the LayerNorm input rows
  int stats_parts;
  const float* colsum;     // [n] sum over K of the folded weight row
  float ln_eps;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_EPI_WARPS = 8;  // two per TMEM lane quadrant, each owning half the columns
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;
constexpr int GEMM_STAGE_OUT_BYTES = 32 * 32 * 4;  // per-warp staging: 32 rows x 32 fp32
// fp16-output epilogues on 256-wide tiles may run 12 epilogue warps (three per TMEM lane
// quadrant, every third 32-column chunk each), staging 32 rows x 32 fp16 per warp.
constexpr int GEMM_EPI_WARPS_WIDE = 12;
constexpr int gemm_threads(int epi_warps) { return 64 + 32 * epi_warps; }

// tcgen05 attention: work items of 2 query tiles x 128 rows (one tile at head_dim 256),
// 128-key KV tiles.
struct AtcParams {
  const int* seq_off;     // [B+1] first packed row of each sequence
  const int2* items;      // work list: {b, (query pair << 8) | h}
  const int* item_count;  // number of valid items
  int* work_counter;      // zeroed before the launch; CTAs take items with atomicAdd
  __half* ctx;            // [rows_max, qkv_width]
  int rows_max;           // rows allocated in qkv / ctx (stores past it are dropped)
  int qkv_width;          // columns of each of the q | k | v blocks = ctx row stride
  float scale_log2;       // hd^-0.5 * log2(e)
  int* status;            // device status word (nullable)
  unsigned long long wait_limit_ns;
};
constexpr int ATC_BM = 128;         // query rows per tile = TMEM lanes
constexpr int ATC_BN = 128;         // keys per KV tile
// Query rows per work item for a head-dim layout: two tiles, one at head_dim 256.
constexpr int atc_item_rows(int layout_hd) { return layout_hd == 256 ? 128 : 256; }
// warps 0-3 / 4-7 softmax tile 0 / 1, warp 8 TMA, warps 9 / 10 MMA for tile 0 / 1
constexpr int ATC_THREADS = 352;

struct TokenPlan {
  int* seq_len;     // [B]
  int* seq_off;     // [B+1]; seq_off[B] = number of valid tokens
  int* packed_src;  // [B*S] packed row -> b*S + s
  int* dst_map;     // [B*S] b*S + s -> packed row, or -1
  int2* items;      // [B*H*ceil(S/128)] attention work list (bound for every item size)
  int* item_count;  // [1]
  int* counters;    // [PLAN_COUNTERS] dynamic work counters, zeroed by the plan and gather kernels
};

// K3 resident stack: one CTA runs every layer of one sequence of <= 128 tokens.
constexpr int RES_ROWS = 128;            // rows of a sequence = TMEM lanes
constexpr int RES_STAGE_BYTES = 16384;   // one weight box: <= 128 rows x 64 fp16 (minimum stage)
constexpr int RES_MAX_STAGES = 12;
constexpr int RES_WORKERS = 256;         // warps 2-9: two per TMEM lane quadrant
constexpr int RES_THREADS = 64 + RES_WORKERS;
constexpr int RES_MISC_BYTES = 6144;     // barriers, row statistics, row maps
constexpr int RES_SMEM_LIMIT = 232448;   // 227 KB per CTA

struct ResParams {
  const void* x;          // [B, S, D] fp16 or fp32 input
  const uint8_t* mask;    // [B, S] valid_token_mask bytes, or null (all valid)
  void* out;              // [B, S, D] output, same dtype as x
  int x_f32;              // 1: x and out are fp32
  int B, S, D, H, F, L, causal;
  int hp;                 // layout head dim (32, 64, 128)
  int gh;                 // heads per attention step (2: head pairs, hp 32, even H)
  int Q;                  // H * hp: width of each of the q | k | v weight blocks
  float scale_log2;       // hd^-0.5 * log2(e)
  float eps;
  // Per-layer fp32 vectors: layer l at base + l * stride bytes.  Each layer's are
  // copied into shared memory (one block, see ResLayout) before the layer starts.
  const float* bqkv;      // LayerNorm-folded [3Q]
  const float* cqkv;      // column sums of the folded Wqkv [3Q]
  const float* b1;        // folded [F]
  const float* c1;        // [F]
  size_t fold_stride;
  const float* bo;        // [D]
  const float* b2;        // [D]
  size_t layer_stride;
  const float* lnf_w;     // [D]
  const float* lnf_b;     // [D]
  int* status;
  int* status_host;       // pinned host mirror of the status word (nullable)
  unsigned long long wait_limit_ns;
};

// Shared-memory layout of the resident kernel for (D, F, hp, Q); the same on host and
// device.  Regions start on 1024-byte boundaries (128-byte swizzle atoms).
struct ResLayout {
  int Dp;     // D rounded up to 64 (columns of the fp16 residual copy)
  int FC;     // FFN columns per chunk (min(F, 128))
  int FCp;    // FC rounded up to 64
  int NB;     // output columns per residual MMA group (min(D, 128))
  int NH;     // residual column groups (D / NB)
  int KC;     // 64-column K chunks of D
  int NF;     // FFN chunks
  int tile;   // bytes of one [128 x hp] operand tile
  int gh;     // heads per attention step: 2 ("head pairs", hp 32 only) or 1
  // One layer's vectors, in floats: bqkv [3Q] cqkv [3Q] bo [D] b1 [F] c1 [F] b2 [D].
  int v_bq, v_cq, v_bo, v_b1, v_c1, v_b2, v_floats;
  int vec_bytes;  // one layer's block (two are kept: layer l in buffer l & 1)
  // hp <= 64: a head's q, k and v weight boxes of one K chunk share a stage (stacked
  // rows), so one MMA group with N = 3 hp computes all three.
  int qkv_merged;
  int stage_bytes;
  int stages;     // weight ring stages that fit
  int xa, qkvh, vec, ring, misc, total;
};

__host__ __device__ inline ResLayout res_layout(int D, int F, int hp, int Q, int gh) {
  ResLayout y;
  y.Dp = (D + 63) / 64 * 64;
  y.FC = F < 128 ? F : 128;
  y.FCp = (y.FC + 63) / 64 * 64;
  y.NB = D < 128 ? D : 128;
  y.NH = D / y.NB;
  y.KC = y.Dp / 64;
  y.NF = (F + y.FC - 1) / y.FC;
  y.tile = RES_ROWS * hp * 2;
  y.gh = gh;
  y.v_bq = 0;
  y.v_cq = 3 * Q;
  y.v_bo = 6 * Q;
  y.v_b1 = 6 * Q + D;
  y.v_c1 = 6 * Q + D + F;
  y.v_b2 = 6 * Q + D + 2 * F;
  y.v_floats = 6 * Q + 2 * D + 2 * F;
  y.vec_bytes = y.v_floats * 4;
  const int qkv = 3 * gh * y.tile, hbuf = RES_ROWS * y.FCp * 2;
  y.xa = 0;
  y.qkvh = y.xa + RES_ROWS * y.Dp * 2;
  y.vec = y.qkvh + (qkv > hbuf ? qkv : hbuf);
  y.ring = y.vec + (2 * y.vec_bytes + 1023) / 1024 * 1024;
  y.qkv_merged = hp <= 64;
  y.stage_bytes = RES_STAGE_BYTES;
  if (y.qkv_merged && 3 * gh * hp * 128 > y.stage_bytes) y.stage_bytes = 3 * gh * hp * 128;
  const int room = RES_SMEM_LIMIT - 1024 - RES_MISC_BYTES - y.ring;
  y.stages = room / y.stage_bytes;
  if (y.stages > RES_MAX_STAGES) y.stages = RES_MAX_STAGES;
  y.misc = y.ring + y.stages * y.stage_bytes;
  y.total = y.misc + RES_MISC_BYTES + 1024;  // + alignment slack
  return y;
}

constexpr int PLAN_COUNTERS = 256;  // one per attention launch of a forward (layers)

constexpr int PLAN_THREADS = 1024;

}  // namespace tttj
