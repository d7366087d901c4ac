// Instantiations and launcher of the K2 attention kernel (attention_mma.cuh).
#include "launch.h"
#include "attention_mma.cuh"

namespace tttj {

namespace {
template <int HD, bool CAUSAL>
cudaError_t launch_t(const AttnParams& p, int grid, cudaStream_t stream) {
  auto kern = attention_mma_kernel<HD, CAUSAL>;
  constexpr int smem = AttnSmem<HD>::BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, ATT_THREADS, smem, stream>>>(p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t attention_launch(const AttnParams& p, int head_dim, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  if (head_dim == 64) return p.causal ? launch_t<64, true>(p, grid, stream)
                                      : launch_t<64, false>(p, grid, stream);
  if (head_dim == 32) return p.causal ? launch_t<32, true>(p, grid, stream)
                                      : launch_t<32, false>(p, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tttj
