// Instantiations and launcher of the K2 tcgen05 attention kernel (attention_tc.cuh).
#include "launch.h"
#include "attention_tc.cuh"

namespace tttj {

namespace {
template <int HD, bool CAUSAL, int QB = 2>
cudaError_t launch_tc(const CUtensorMap& tm, const AtcParams& p, int grid, cudaStream_t stream) {
  auto kern = attention_tc_kernel<HD, CAUSAL, QB>;
  constexpr int smem = AtcSmem<HD, QB>::TOTAL;
  static_assert(smem <= 232448, "attention shared memory exceeds the 227 KB per-CTA limit");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(ATC_THREADS), smem, stream, tm, p);
}
}  // namespace

cudaError_t attention_tc_launch(const CUtensorMap& tm, const AtcParams& p, int head_dim,
                                int causal, int grid, int max_seq_len, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  // Three Q buffers for sequences of 257-2048 tokens (C2: attention 26.7 -> 26.2 us);
  // longer ones keep the deeper K/V ring (C4 measured no better with three).
  if (head_dim == 64 && max_seq_len > 256 && max_seq_len <= 2048)
    return causal ? launch_tc<64, true, 3>(tm, p, grid, stream) : launch_tc<64, false, 3>(tm, p, grid, stream);
  if (head_dim == 64)
    return causal ? launch_tc<64, true>(tm, p, grid, stream) : launch_tc<64, false>(tm, p, grid, stream);
  if (head_dim == 32)
    return causal ? launch_tc<32, true>(tm, p, grid, stream) : launch_tc<32, false>(tm, p, grid, stream);
  if (head_dim == 128)
    return causal ? launch_tc<128, true>(tm, p, grid, stream) : launch_tc<128, false>(tm, p, grid, stream);
  if (head_dim == 256)
    return causal ? launch_tc<256, true>(tm, p, grid, stream) : launch_tc<256, false>(tm, p, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tttj
