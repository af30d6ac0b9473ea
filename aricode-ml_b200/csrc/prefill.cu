// prefill.cu — host side of the batched prefill kernels (prefill.cuh): TMA tensor
// maps (through the driver entry point, no libcuda link) and the launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "prefill.cuh"

namespace b2 {

namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// 2-D byte matrix [rows][cols] with row stride `stride` bytes; box = 128 bytes of
// a row x box_rows rows, 128-byte swizzle (the UMMA K-major SW128 layout);
// reads past cols or rows are zeros
bool byte_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t stride, uint32_t box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {(cuuint32_t)kPfKBlock, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// B2_PF_TRACE=<file>: every GEMM launch synchronises and appends its per-CTA
// timeline (u32 grid x, grid y, K; then u64 [CTA][8], see PfGemmParams::trace)
const char* trace_path() {
    static const char* p = std::getenv("B2_PF_TRACE");
    return (p && p[0]) ? p : nullptr;
}

template <int NM>
cudaError_t launch_nm(const void* A0, const void* A1, const unsigned char* planes, int ldp, const PfGemmParams& p,
                      cudaStream_t s) {
    using Sh = PfShape<NM>;
    CUtensorMap a0, a1, b;
    if (!byte_map(&a0, A0, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.K, kPfRows) ||
        !byte_map(&a1, NM == 2 ? A1 : A0, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.K, kPfRows) ||
        !byte_map(&b, planes, (uint64_t)p.K, 4ull * p.Tpad, (uint64_t)ldp, Sh::N))
        return cudaErrorInvalidValue;
    auto k = prefill_gemm_kernel<NM>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::SmemBytes);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((p.M + kPfRows - 1) / kPfRows), (unsigned)((p.T + Sh::N - 1) / Sh::N));
    // few tiles (few tokens, few rows): split K over up to 8 CTAs a tile so that most
    // SMs take part; the splits' integer dots add exactly in any order
    static int sms = 0;
    if (!sms && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0) != cudaSuccess) sms = 148;
    const int tiles = (int)(grid.x * grid.y);
    const int kb = (p.K + kPfKBlock - 1) / kPfKBlock;
    if (p.acc && p.cnt && tiles <= kPfSplitCounters && (long long)tiles * NM * Sh::N <= (long long)kPfSplitTiles * kPfSplitCols) {
        // one wave (a CTA per SM): a second wave of CTAs costs more than their shorter
        // K ranges save (measured: 86 tiles split 8 ways, 67 -> 93 us)
        grid.z = (unsigned)std::max(1, std::min({sms / tiles, kb / 4, 8}));
    }
    if (!trace_path()) {
        k<<<grid, kPfThreads, Sh::SmemBytes, s>>>(a0, a1, b, p);
        return cudaGetLastError();
    }
    PfGemmParams q = p;
    const size_t n = (size_t)grid.x * grid.y * grid.z * 8;
    if ((e = cudaMalloc(&q.trace, n * 8)) != cudaSuccess) return e;
    cudaMemsetAsync(q.trace, 0, n * 8, s);
    k<<<grid, kPfThreads, Sh::SmemBytes, s>>>(a0, a1, b, q);
    e = cudaStreamSynchronize(s);
    std::vector<unsigned long long> h(n);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), q.trace, n * 8, cudaMemcpyDeviceToHost);
    cudaFree(q.trace);
    if (FILE* f = std::fopen(trace_path(), "ab")) {
        const unsigned hdr[4] = {grid.x, grid.y, (unsigned)p.K, (unsigned)NM | (grid.z << 8)};
        std::fwrite(hdr, 4, 4, f);
        std::fwrite(h.data(), 8, n, f);
        std::fclose(f);
    }
    return e;
}

}  // namespace

cudaError_t launch_prefill_gemm(int nm, const void* A0, const void* A1, const unsigned char* planes, int ldp,
                                const PfGemmParams& p, cudaStream_t s) {
    // TMA rules: 16-byte aligned bases and row strides; every x coordinate is a
    // multiple of 128 bytes
    if ((reinterpret_cast<uintptr_t>(A0) & 15) || (nm == 2 && (reinterpret_cast<uintptr_t>(A1) & 15)) ||
        (reinterpret_cast<uintptr_t>(planes) & 15) || (p.K & 15) || (ldp & 15) || ldp < p.K || p.Tpad % 128)
        return cudaErrorInvalidValue;
    return nm == 2 ? launch_nm<2>(A0, A1, planes, ldp, p, s) : launch_nm<1>(A0, A1, planes, ldp, p, s);
}

cudaError_t launch_prefill_planes(const PfPlanesParams& p, int T, cudaStream_t s) {
    const size_t smem = (size_t)p.n * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(prefill_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    prefill_planes_kernel<<<T, 256, smem, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_attn(const PfAttnParams& p, cudaStream_t s) {
    const int G = p.H / p.KVH;
    const size_t smem = prefill_attn_smem(G, p.dh);
    const int kd = (p.dh + 31) / 32;
    auto k = kd <= 1 ? prefill_attn_part_kernel<1> : kd == 2 ? prefill_attn_part_kernel<2>
                                                 : kd <= 4 ? prefill_attn_part_kernel<4> : prefill_attn_part_kernel<8>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int nchunks = (p.pos0 + p.T + kAttnChunk - 1) / kAttnChunk;
    const dim3 grid((unsigned)p.KVH, (unsigned)nchunks, (unsigned)((p.T + kPfAttnGroup - 1) / kPfAttnGroup));
    k<<<grid, kPfAttnWarps * 32, smem, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long items = (long long)p.T * p.H;
    prefill_attn_combine_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_batch_attn(const AttnParams& a, int nseq, int ldo, cudaStream_t s) {
    const int kd = (a.dh + 31) / 32;
    auto k = kd <= 1 ? attn_batch_part_kernel<1> : kd == 2 ? attn_batch_part_kernel<2>
                                                  : kd <= 4 ? attn_batch_part_kernel<4> : attn_batch_part_kernel<8>;
    cudaError_t e;
    const dim3 grid((unsigned)nseq, (unsigned)a.KVH, (unsigned)((a.nsplit_max + kBtWarps - 1) / kBtWarps));
    k<<<grid, kBtWarps * 32, 0, s>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // merge: prefill_attn_combine_kernel with one "token" per sequence
    PfAttnParams c{};
    c.out = a.out; c.part = a.part; c.H = a.H; c.KVH = a.KVH; c.dh = a.dh; c.max_seq = a.max_seq;
    c.nsplit_max = a.nsplit_max; c.T = nseq; c.pos0 = 0; c.err = a.err; c.n_of = a.n_of;
    c.ldo = ldo; c.mir = a.mir;
    const long long items = (long long)nseq * a.H;
    prefill_attn_combine_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(c);
    return cudaGetLastError();
}

cudaError_t launch_batch_tail(const float* logits, int vocab, const BatchState& b, int B, cudaStream_t s) {
    batch_argmax_kernel<<<B, 1024, 0, s>>>(logits, vocab, b);
    batch_count_kernel<<<1, 1, 0, s>>>(b);
    return cudaGetLastError();
}

// One thread: the previous launches on this stream are complete, so their peer
// stores are performed; the flag exchange (system-scope release and acquire) then
// orders them before every rank's next launch. The epoch is a counter in this
// rank's memory (every rank takes the same barriers in the same order), so a
// captured graph that replays the launch takes a new epoch each time.
static __global__ void tp_sync_kernel(unsigned* flags, Mirror mir, int rank, int nranks, unsigned* epoch, int* err) {
    if (threadIdx.x != 0) return;
    const unsigned e = *epoch + 1u;
    *epoch = e;
    if (!tp_flag_exchange(flags, rank, nranks, mir, e)) set_err(err, B2_DEV_ERR_TIMEOUT);
}

cudaError_t launch_tp_sync(unsigned* flags, const Mirror& mir, int rank, int nranks, unsigned* epoch, int* err,
                           cudaStream_t s) {
    tp_sync_kernel<<<1, 32, 0, s>>>(flags, mir, rank, nranks, epoch, err);
    return cudaGetLastError();
}

cudaError_t launch_batch_check(const BatchState& b, int B, cudaStream_t s) {
    batch_check_kernel<<<(B + 127) / 128, 128, 0, s>>>(b, B);
    return cudaGetLastError();
}

cudaError_t launch_prefill_embed(const int8_t* emb, const float* emb_s, long long ld, const int* ids, int pos0,
                                 int vocab, int d, float* x, int T, int* err, cudaStream_t s) {
    prefill_embed_kernel<<<T, 256, 0, s>>>(emb, emb_s, ld, ids, pos0, vocab, d, x, err);
    return cudaGetLastError();
}

}  // namespace b2
