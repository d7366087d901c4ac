// Instantiations and launcher of the K2 tcgen05 attention kernel (attention_tc.cuh).
#include "launch.h"
#include "attention_tc.cuh"

namespace tttj {

namespace {
template <int HD, bool CAUSAL>
cudaError_t launch_tc(const CUtensorMap& tm, const AtcParams& p, int grid, cudaStream_t stream) {
  auto kern = attention_tc_kernel<HD, CAUSAL>;
  constexpr int smem = AtcSmem<HD>::TOTAL;
  static_assert(smem <= 232448, "attention shared memory exceeds the 227 KB per-CTA limit");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(ATC_THREADS), smem, stream, tm, p);
}
}  // namespace

cudaError_t attention_tc_launch(const CUtensorMap& tm, const AtcParams& p, int head_dim,
                                int causal, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
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
