// launch.cu — the per-launch kernels' launchers (declared in kernels.cuh): the
// GEMV kernel templates, the attention kernel and the embedding kernel are
// instantiated here once for the runtime and the kernel-level C ABI.
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace b2 {

template <typename WT, int KMAX, int RS, bool PAIRED>
inline cudaError_t launch_gemv_t(GemvParams p, const GemvShape& sh, cudaStream_t s, bool pdl) {
    p.nstages = sh.nstages;
    p.stage_rows = sh.R;
    p.ring_offset = sh.ring_offset;
    auto k = gemv_kernel<WT, KMAX, RS, PAIRED>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem);
    if (e != cudaSuccess) return e;
    return launch_ex(k, dim3(sh.grid), dim3(kGemvThreads), sh.smem, s, pdl, p);
}

template <typename WT, int KMAX, bool PAIRED>
inline cudaError_t launch_gemv_r(const GemvParams& p, const GemvShape& sh, cudaStream_t s, bool pdl) {
    if constexpr (KMAX > 1) {               // rows over 4 KB: at most 4 rows fit a 32 KB stage
        if (sh.R == 1) return launch_gemv_t<WT, KMAX, 1, PAIRED>(p, sh, s, pdl);
        if (sh.R == 2) return launch_gemv_t<WT, KMAX, 2, PAIRED>(p, sh, s, pdl);
        if constexpr (!PAIRED)
            if (sh.R == 4) return launch_gemv_t<WT, KMAX, 4, PAIRED>(p, sh, s, pdl);
        return cudaErrorInvalidValue;
    } else {
    switch (sh.R) {
        case 1: return launch_gemv_t<WT, KMAX, 1, PAIRED>(p, sh, s, pdl);
        case 2: return launch_gemv_t<WT, KMAX, 2, PAIRED>(p, sh, s, pdl);
        case 4: return launch_gemv_t<WT, KMAX, 4, PAIRED>(p, sh, s, pdl);
        case 8: return launch_gemv_t<WT, KMAX, 8, PAIRED>(p, sh, s, pdl);
        default:
            if constexpr (PAIRED) return cudaErrorInvalidValue;
            else return launch_gemv_t<WT, KMAX, 16, PAIRED>(p, sh, s, pdl);
    }
    }
}

// weights int8 (w_i8) or f32; rows up to kGemvMaxK*256 16-byte blocks long
cudaError_t launch_gemv(const GemvParams& p, bool w_i8, cudaStream_t s, bool pdl, int grid_cap,
                        GemvShape* out_shape) {
    const GemvShape sh = gemv_shape(p, w_i8 ? 1 : 4, grid_cap);
    if (out_shape) *out_shape = sh;
    if (sh.K < 1 || sh.K > kGemvMaxK || sh.smem > 227 * 1024) return cudaErrorInvalidValue;
    if (w_i8) {
        if (sh.paired) {
            if (sh.K <= 1) return launch_gemv_r<int8_t, 1, true>(p, sh, s, pdl);
            if (sh.K <= 3) return launch_gemv_r<int8_t, 3, true>(p, sh, s, pdl);
            return launch_gemv_r<int8_t, kGemvMaxK, true>(p, sh, s, pdl);
        }
        if (sh.K <= 1) return launch_gemv_r<int8_t, 1, false>(p, sh, s, pdl);
        if (sh.K <= 3) return launch_gemv_r<int8_t, 3, false>(p, sh, s, pdl);
        return launch_gemv_r<int8_t, kGemvMaxK, false>(p, sh, s, pdl);
    }
    if (sh.paired) return cudaErrorInvalidValue;
    if (sh.K <= 1) return launch_gemv_r<float, 1, false>(p, sh, s, pdl);
    return launch_gemv_r<float, kGemvMaxK, false>(p, sh, s, pdl);
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t s, bool pdl) {
    const int G = p.H / p.KVH;
    const size_t smem = attn_smem_bytes(G, p.dh, p.nsplit_max);
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return launch_ex(attn_decode_kernel, dim3(p.nsplit_max, p.KVH), dim3(kAttnThreads), smem, s, pdl, p);
}

cudaError_t launch_gemv_i4(const GemvParams& p, cudaStream_t s, bool pdl, int grid_cap) {
    const GemvShape sh = gemv_shape(p, 1, grid_cap);
    // packed rows of up to 2 x 256 16-byte blocks = 16384 codes a thread pass covers
    if (sh.K < 1 || sh.K > 2 || sh.smem > 227 * 1024 || p.paired || p.rope) return cudaErrorInvalidValue;
    auto go = [&](auto kern) {
        GemvParams q = p;
        q.nstages = sh.nstages;
        q.stage_rows = sh.R;
        q.ring_offset = sh.ring_offset;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem);
        if (e != cudaSuccess) return e;
        return launch_ex(kern, dim3(sh.grid), dim3(kGemvThreads), sh.smem, s, pdl, q);
    };
    if (sh.K == 1) {
        switch (sh.R) {
            case 1: return go(gemv_i4_kernel<1, 1>);
            case 2: return go(gemv_i4_kernel<1, 2>);
            case 4: return go(gemv_i4_kernel<1, 4>);
            case 8: return go(gemv_i4_kernel<1, 8>);
            default: return go(gemv_i4_kernel<1, 16>);
        }
    }
    switch (sh.R) {
        case 1: return go(gemv_i4_kernel<2, 1>);
        case 2: return go(gemv_i4_kernel<2, 2>);
        case 4: return go(gemv_i4_kernel<2, 4>);
        default: return go(gemv_i4_kernel<2, 8>);
    }
}

cudaError_t launch_attn_batched(const AttnParams& p, int nseq, cudaStream_t s) {
    const int G = p.H / p.KVH;
    const size_t smem = attn_smem_bytes(G, p.dh, p.nsplit_max);
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return launch_ex(attn_decode_kernel, dim3(p.nsplit_max, p.KVH, nseq), dim3(kAttnThreads), smem, s, false, p);
}

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl) {
    return launch_ex(embed_kernel, dim3(1), dim3(256), 0, s, pdl, p);
}

}  // namespace b2
