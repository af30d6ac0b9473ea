// token.cu — instantiates the persistent token kernel (token.cuh) for both
// variant sets and exposes its set-up and launch to the runtime.
#include <cuda_runtime.h>

#include "token.cuh"

namespace b2 {

cudaError_t tk_prepare(int vs, size_t smem, int* per_sm) {
    auto k = vs ? token_kernel<1> : token_kernel<0>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k, kTkThreads, smem);
}

cudaError_t tk_launch(int vs, const cudaLaunchConfig_t& cfg, const TkParams& P) {
    cudaLaunchConfig_t c = cfg;
    if (vs) return cudaLaunchKernelEx(&c, token_kernel<1>, P);
    return cudaLaunchKernelEx(&c, token_kernel<0>, P);
}

}  // namespace b2
