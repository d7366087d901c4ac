// Launchers of the token plan and the LayerNorm row kernels (rows.cuh).
#include "launch.h"
#include "rows.cuh"

namespace tttj {

namespace {
constexpr int ROWS_PER_CTA = 8;  // one warp per row, 256 threads

inline int ln_vpl(int D) { return (D + 255) / 256; }
}  // namespace

cudaError_t plan_tokens_launch(const uint8_t* mask, int B, int S, int H, int causal, int q_block,
                               int kv_block, const TokenPlan& plan, cudaStream_t stream, int q_lo,
                               int q_hi) {
  const int nkeys = (S + kv_block - 1) / kv_block + 1;
  const size_t ints = ((size_t)(2 * B + 1 + nkeys + 1) + 3) & ~(size_t)3;
  const size_t smem = sizeof(int) * ints + 512 * (PLAN_THREADS / 32);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(plan_tokens_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(plan_tokens_kernel, dim3(1), dim3(PLAN_THREADS), smem, stream, mask, B, S, H,
                    causal, q_block, kv_block, q_lo, q_hi, plan);
}

#define TTTJ_VPL_DISPATCH(VPL_EXPR, CALL) \
  switch (VPL_EXPR) {                     \
    case 1: { constexpr int V = 1; CALL; break; } \
    case 2: { constexpr int V = 2; CALL; break; } \
    case 3: { constexpr int V = 3; CALL; break; } \
    case 4: { constexpr int V = 4; CALL; break; } \
    case 5: case 6: { constexpr int V = 6; CALL; break; } \
    case 7: case 8: { constexpr int V = 8; CALL; break; } \
    default: return cudaErrorInvalidValue; \
  }

cudaError_t ln_gather_launch(const void* x, int x_dtype, const int* packed_src, const int* rows_dev,
                             int rows_max, int D, float* resid, __half* x16, float2* stats,
                             float* pivot, int n_parts, int* counters, cudaStream_t stream) {
  const int grid = (rows_max + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
  if (grid == 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (x_dtype == 0) {
    TTTJ_VPL_DISPATCH(ln_vpl(D), (e = launch_pdl(ln_gather_kernel<V, __half>, dim3(grid),
                                                 dim3(32 * ROWS_PER_CTA), 0, stream,
                                                 static_cast<const __half*>(x), packed_src,
                                                 rows_dev, D, resid, x16, stats, pivot, n_parts,
                                                 counters)));
  } else {
    TTTJ_VPL_DISPATCH(ln_vpl(D), (e = launch_pdl(ln_gather_kernel<V, float>, dim3(grid),
                                                 dim3(32 * ROWS_PER_CTA), 0, stream,
                                                 static_cast<const float*>(x), packed_src,
                                                 rows_dev, D, resid, x16, stats, pivot, n_parts,
                                                 counters)));
  }
  return e;
}

cudaError_t fold_ln_launch(const __half* w, const float* b, const float* gamma, const float* beta,
                           int rows_out, int k, int hd, int hp, __half* w_out, float* b_out,
                           float* colsum, cudaStream_t stream) {
  const int grid = (rows_out + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
  if (grid == 0) return cudaSuccess;
  fold_ln_kernel<<<grid, 32 * ROWS_PER_CTA, 0, stream>>>(w, b, gamma, beta, rows_out, k, hd, hp,
                                                          w_out, b_out, colsum);
  return cudaGetLastError();
}

cudaError_t pad_head_cols_launch(const __half* w, int rows, int cols, int hd, int hp,
                                 __half* w_out, cudaStream_t stream) {
  const long total = (long)rows * (cols / hd) * hp;
  const int grid = (int)((total + 255) / 256);
  if (grid == 0) return cudaSuccess;
  pad_head_cols_kernel<<<grid, 256, 0, stream>>>(w, rows, cols, hd, hp, w_out);
  return cudaGetLastError();
}

cudaError_t ln_rows_launch(const void* in, int in_dtype, const int* rows_dev, int rows_max, int D,
                           const float* gamma, const float* beta, float eps, __half* out,
                           cudaStream_t stream) {
  const int grid = (rows_max + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
  if (grid == 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (in_dtype == 0) {
    TTTJ_VPL_DISPATCH(ln_vpl(D), (e = launch_pdl(ln_rows_kernel<V, __half>, dim3(grid), dim3(32 * ROWS_PER_CTA), 0, stream,
                                      static_cast<const __half*>(in), rows_dev, rows_max, D, gamma,
                                      beta, eps, out)));
  } else {
    TTTJ_VPL_DISPATCH(ln_vpl(D), (e = launch_pdl(ln_rows_kernel<V, float>, dim3(grid), dim3(32 * ROWS_PER_CTA), 0, stream,
                                      static_cast<const float*>(in), rows_dev, rows_max, D, gamma,
                                      beta, eps, out)));
  }
  return e;
}

cudaError_t ln_final_launch(const float* resid, const int* dst_map, int tokens, int D,
                            const float* gamma, const float* beta, float eps, void* out,
                            int out_dtype, const int* status, int* status_host,
                            cudaStream_t stream) {
  const int grid = (tokens + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
  if (grid == 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (out_dtype == 0) {
    TTTJ_VPL_DISPATCH(ln_vpl(D),
                      (e = launch_pdl(ln_final_scatter_kernel<V, __half>, dim3(grid), dim3(32 * ROWS_PER_CTA), 0,
                                     stream, resid, dst_map, tokens, D, gamma, beta, eps,
                                     static_cast<__half*>(out), status, status_host)));
  } else {
    TTTJ_VPL_DISPATCH(ln_vpl(D),
                      (e = launch_pdl(ln_final_scatter_kernel<V, float>, dim3(grid), dim3(32 * ROWS_PER_CTA), 0,
                                     stream, resid, dst_map, tokens, D, gamma, beta, eps,
                                     static_cast<float*>(out), status, status_host)));
  }
  return e;
}

cudaError_t selftest_wait_launch(int* status, int* status_host, unsigned long long limit_ns,
                                 cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(status, status_host, limit_ns);
  return cudaGetLastError();
}

}  // namespace tttj
