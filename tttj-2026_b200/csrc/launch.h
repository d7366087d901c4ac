// Internal host-side launch interface shared by the .cu translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "params.h"

namespace tttj {

// Launch `kern` with programmatic stream serialization (see griddep_wait in
// common.cuh): the kernel may begin its set-up while the previous kernel of the stream
// finishes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// launch_pdl for a kernel launched in clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

struct GemmLaunch {
  CUtensorMap tmA;
  CUtensorMap tmB;
  CUtensorMap tmC;  // output, 32x32 boxes (TMA tile stores)
  GemmParams p;
  int bn;    // 64, 128 or 256
  int pair;  // 1: 256 x bn tiles on CTA pairs (cta_group::2), 0: 128 x bn tiles per CTA
  int epi;   // GemmEpilogue
  int grid;  // persistent CTAs (even for pairs)
  int rbuf;  // fp32 residual staging blocks per epilogue warp fed by TMA (0: none)
  int epiw;  // epilogue warps (GEMM_EPI_WARPS or GEMM_EPI_WARPS_WIDE)
};

// Tile shape for a GEMM of `rows` x `n` x `k` with epilogue `epi` on `num_sms` SMs:
// column width (a function of rows and n only, so every GEMM with the same output
// shape uses the same width) and whether CTA pairs compute it (see gemm.cu).
int gemm_choose_bn(int rows, int n, int num_sms);
void gemm_choose(int rows, int n, int k, int epi, int num_sms, int* bn, int* pair);
// Residual staging blocks (gemm_tc.cuh RBUF) for a GEMM with that tile shape: 2 for the
// in-place fp32 residual epilogues with short K, else 0.
int gemm_choose_rbuf(int bn, int pair, int k, int epi, bool in_place);
// Epilogue warps for a GEMM with that tile width, epilogue and residual staging.
int gemm_choose_epiw(int bn, int epi, int rbuf);
cudaError_t gemm_launch(const GemmLaunch& g, cudaStream_t stream);

// tcgen05 attention for a head-dim layout of 32, 64, 128 or 256 (plan with q_block
// atc_item_rows(head_dim), kv_block ATC_BN).  tmQKV: fp16 [rows, 3 * qkv_width] map, box
// {min(head_dim, 64), 128}, swizzle 64 B (head_dim 32) / 128 B.  max_seq_len: the
// longest sequence the launch may see (it picks the kernel's item buffering).
cudaError_t attention_tc_launch(const CUtensorMap& tmQKV, const AtcParams& p, int head_dim,
                                int causal, int grid, int max_seq_len, cudaStream_t stream);

// K3 resident stack (resident.cuh): weights as 3-D TMA maps over the layers
// ({columns, rows, layer}, one box per MMA unit).
struct ResLaunch {
  CUtensorMap tmWqkv;  // folded Wqkv [3Q, D] per layer, box {64, hp}
  CUtensorMap tmWo;    // out_proj [D, Q] per layer, box {min(hp, 64), min(D, 128)}
  CUtensorMap tmW1;    // folded W1 [F, D] per layer, box {64, min(F, 128)}
  CUtensorMap tmW2;    // W2 [D, F] per layer, box {64, min(D, 128)}
  ResParams p;
};
cudaError_t resident_launch(const ResLaunch& r, cudaStream_t stream);

// Items for the query blocks starting in [q_lo, q_hi) only (defaults: all).
cudaError_t plan_tokens_launch(const uint8_t* mask, int B, int S, int H, int causal, int q_block,
                               int kv_block, const TokenPlan& plan, cudaStream_t stream,
                               int q_lo = 0, int q_hi = 0x7fffffff);
cudaError_t ln_gather_launch(const void* x, int x_dtype, const int* packed_src, const int* rows_dev,
                             int rows_max, int D, float* resid, __half* x16, float2* stats,
                             float* pivot, int n_parts, int* counters, cudaStream_t stream);
// rows_out output rows; with hd < hp the input's rows are heads of hd rows placed at
// the start of output groups of hp rows, the rest zero (hd == hp: one row each).
cudaError_t fold_ln_launch(const __half* w, const float* b, const float* gamma, const float* beta,
                           int rows_out, int k, int hd, int hp, __half* w_out, float* b_out,
                           float* colsum, cudaStream_t stream);
// w [rows, cols] -> w_out [rows, (cols / hd) * hp]: column groups of hd widened to hp
// with zero columns.
cudaError_t pad_head_cols_launch(const __half* w, int rows, int cols, int hd, int hp,
                                 __half* w_out, cudaStream_t stream);
// in_dtype: 0 = fp16 rows, 1 = fp32 rows.
cudaError_t ln_rows_launch(const void* in, int in_dtype, const int* rows_dev, int rows_max, int D,
                           const float* gamma, const float* beta, float eps, __half* out,
                           cudaStream_t stream);
cudaError_t ln_final_launch(const float* resid, const int* dst_map, int tokens, int D,
                            const float* gamma, const float* beta, float eps, void* out,
                            int out_dtype, const int* status, int* status_host,
                            cudaStream_t stream);
// Per-stage capture kernels (debug.cu).
cudaError_t debug_gather_launch(const void* src, int src_f16, int ld, int col_base, int cols, int hd,
                                int hp, const int* dst_map, int b, int S, float* dst, cudaStream_t s);
cudaError_t debug_ln_launch(const float* x, const float* gamma, const float* beta, float eps, int S,
                            int D, const int* dst_map, int b, float* out, cudaStream_t s);
cudaError_t debug_scores_launch(const float* q, const float* k, const int* dst_map, int b, int S,
                                int H, int hd, int causal, float scale, float* scores, float* probs,
                                cudaStream_t s);
cudaError_t debug_diff_launch(const float* a, const float* b, long n, float* out, cudaStream_t s);

cudaError_t selftest_wait_launch(int* status, int* status_host, unsigned long long limit_ns,
                                 cudaStream_t stream);

}  // namespace tttj
