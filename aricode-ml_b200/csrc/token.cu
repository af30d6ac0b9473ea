// token.cu — instantiates the persistent token kernel (token.cuh) for both
// variant sets and exposes its set-up and launch to the runtime.
#include <cuda_runtime.h>

#include "token.cuh"

namespace b2 {

cudaError_t tk_prepare(int vs, bool tags, size_t smem, int* per_sm) {
    auto k = vs ? (tags ? token_kernel<1, true> : token_kernel<1, false>)
                : (tags ? token_kernel<0, true> : token_kernel<0, false>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k, kTkThreads, smem);
}

cudaError_t tk_launch(int vs, bool tags, const cudaLaunchConfig_t& cfg, const TkParams& P) {
    cudaLaunchConfig_t c = cfg;
    if (vs) return tags ? cudaLaunchKernelEx(&c, token_kernel<1, true>, P) : cudaLaunchKernelEx(&c, token_kernel<1, false>, P);
    return tags ? cudaLaunchKernelEx(&c, token_kernel<0, true>, P) : cudaLaunchKernelEx(&c, token_kernel<0, false>, P);
}

}  // namespace b2
