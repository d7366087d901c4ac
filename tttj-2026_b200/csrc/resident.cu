// Instantiations and launcher of the K3 resident-stack kernel (resident.cuh).
#include "launch.h"
#include "resident.cuh"

namespace tttj {

namespace {
template <int HP, bool PAIR>
cudaError_t launch_res(const ResLaunch& r, cudaStream_t stream) {
  auto kern = resident_stack_kernel<HP, PAIR>;
  // At least half the SM's shared memory: one CTA per SM, so a CTA never waits for
  // another to release the 512 TMEM columns it allocates.
  int smem = res_layout(r.p.D, r.p.F, HP, r.p.Q, PAIR ? 2 : 1).total;
  if (smem < 116 * 1024) smem = 116 * 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(r.p.B), dim3(RES_THREADS), (size_t)smem, stream, r.tmWqkv, r.tmWo,
                    r.tmW1, r.tmW2, r.p);
}
}  // namespace

cudaError_t resident_launch(const ResLaunch& r, cudaStream_t stream) {
  if (r.p.B <= 0) return cudaSuccess;
  switch (r.p.hp) {
    case 32: return r.p.gh == 2 ? launch_res<32, true>(r, stream) : launch_res<32, false>(r, stream);
    case 64: return launch_res<64, false>(r, stream);
    case 128: return launch_res<128, false>(r, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tttj
