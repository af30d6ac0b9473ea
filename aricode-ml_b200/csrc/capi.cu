// capi.cu — kernel-level entry points of include/b2dec.h. Device pointers in and
// out, caller's stream, no allocation, no synchronisation. Each call runs the
// same kernels the model runtime uses (with trivial prologue/epilogue settings).
#include <cuda_runtime.h>

#include "../../include/b2dec.h"
#include "prefill.cuh"

using namespace b2;

namespace {

int sm_count_current() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

int status(cudaError_t e) { return e == cudaSuccess ? B2_OK : B2_E_CUDA; }

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int b2_gemv_i8_rowscale(const int8_t* W, int64_t ld, const float* scale, const float* x,
                        const float* bias, float* y, int m, int n, void* stream) {
    if (!W || !scale || !x || !y || m <= 0 || n <= 0 || ld < n || ld % 16 || !al16(W)) return B2_E_INVALID;
    if (n > kXfixMaxN) return B2_E_INVALID;          // the int32 plane sums would overflow
    GemvParams p{};
    p.W[0] = W; p.S[0] = scale; p.bias[0] = bias;
    p.rows[0] = m; p.nseg = 1; p.n = n; p.ld = (int)ld;
    p.x = x; p.norm = NORM_NONE; p.epi = EPI_STORE; p.y = y;
    return status(launch_gemv(p, true, static_cast<cudaStream_t>(stream), false, sm_count_current()));
}

size_t b2_gemm_i8_rowscale_workspace(int T, int64_t ld) {
    const size_t Tpad = ((size_t)T + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile;
    const size_t ldp = ((size_t)ld + 127) / 128 * 128;
    return ((4 * Tpad * ldp + 255) & ~(size_t)255) + (size_t)T * sizeof(int);
}

int b2_gemm_i8_rowscale(const int8_t* W, int64_t ld, const float* scale, const float* X, int64_t ldx,
                        const float* bias, float* Y, int64_t ldy, int m, int n, int T, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (!W || !scale || !X || !Y || !workspace || m <= 0 || n <= 0 || T <= 0 || ld < n || ld % 16 || !al16(W) ||
        ldx < n || ldy < m || n > kXfixMaxN || workspace_bytes < b2_gemm_i8_rowscale_workspace(T, ld) ||
        !al16(workspace))
        return B2_E_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int Tpad = (T + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile;
    const int ldp = (int)((ld + 127) / 128 * 128);
    unsigned char* planes = static_cast<unsigned char*>(workspace);
    int* S = reinterpret_cast<int*>(planes + ((4 * (size_t)Tpad * ldp + 255) & ~(size_t)255));
    PfPlanesParams pp{};
    pp.x = X; pp.ldx = (int)ldx; pp.n = n; pp.norm = NORM_NONE; pp.eps = 0.0f;
    pp.planes = planes; pp.ldp = ldp; pp.kp = ldp; pp.Tpad = Tpad; pp.S = S;
    cudaError_t e = launch_prefill_planes(pp, T, s);
    if (e != cudaSuccess) return B2_E_CUDA;
    PfGemmParams g{};
    g.M = m; g.K = (int)ld; g.T = T; g.Tpad = Tpad; g.epi = PF_STORE; g.S = S;
    g.scale[0] = scale; g.scale[1] = scale; g.bias = bias; g.out = Y; g.ldo = (int)ldy;
    return status(launch_prefill_gemm(1, W, nullptr, planes, ldp, g, s));
}

int b2_gemv_i4_rowscale(const uint8_t* W, int64_t ld, const float* scale, const float* x, const float* bias,
                        float* y, int m, int n, void* stream) {
    if (!W || !scale || !x || !y || m <= 0 || n <= 0 || n % 2 || ld * 2 < n || ld % 16 || !al16(W) ||
        n > kXfixMaxN)
        return B2_E_INVALID;
    GemvParams p{};
    p.W[0] = W; p.S[0] = scale; p.bias[0] = bias;
    p.rows[0] = m; p.nseg = 1; p.n = n; p.ld = (int)ld; p.i4 = 1;
    p.x = x; p.norm = NORM_NONE; p.epi = EPI_STORE; p.y = y;
    return status(launch_gemv_i4(p, static_cast<cudaStream_t>(stream), false, sm_count_current()));
}

int b2_gemv_f32(const float* W, int64_t ld, const float* x, const float* bias, float* y, int m, int n,
                void* stream) {
    if (!W || !x || !y || m <= 0 || n <= 0 || ld < n || ld % 4 || !al16(W)) return B2_E_INVALID;
    GemvParams p{};
    p.W[0] = W; p.bias[0] = bias;
    p.rows[0] = m; p.nseg = 1; p.n = n; p.ld = (int)ld;
    p.x = x; p.norm = NORM_NONE; p.epi = EPI_STORE; p.y = y;
    return status(launch_gemv(p, false, static_cast<cudaStream_t>(stream), false, sm_count_current()));
}

int b2_rmsnorm(const float* x, const float* g, float* y, int d, float eps, void* stream) {
    if (!x || !g || !y || d <= 0) return B2_E_INVALID;
    rmsnorm_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, g, y, d, eps);
    return status(cudaGetLastError());
}

int b2_layernorm(const float* x, const float* g, const float* b, float* y, int d, float eps, void* stream) {
    if (!x || !g || !b || !y || d <= 0) return B2_E_INVALID;
    layernorm_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, g, b, y, d, eps);
    return status(cudaGetLastError());
}

int b2_rope_apply(float* v, const float* table, int pos, int d_head, int n_vec, void* stream) {
    if (!v || !table || d_head <= 0 || d_head % 2 || n_vec <= 0 || pos < 0) return B2_E_INVALID;
    const int pairs = n_vec * d_head / 2;
    rope_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(v, table, pos, d_head, pairs);
    return status(cudaGetLastError());
}

size_t b2_attn_decode_workspace(int n_heads, int n_kv_heads, int d_head, int max_seq) {
    if (n_heads <= 0 || n_kv_heads <= 0 || d_head <= 0 || max_seq <= 0) return 0;
    return attn_scratch_bytes(n_heads, n_kv_heads, d_head, max_seq);
}

int b2_attn_decode(const float* q, const float* K, const float* V, float* out, int n_heads, int n_kv_heads,
                   int d_head, int n, int max_seq, void* workspace, size_t workspace_bytes, void* stream) {
    if (!q || !K || !V || !out || !workspace || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads ||
        d_head <= 0 || d_head > 256 || d_head % 4 || n <= 0 || n > max_seq ||
        (reinterpret_cast<uintptr_t>(K) & 15) || (reinterpret_cast<uintptr_t>(V) & 15))
        return B2_E_INVALID;
    if (workspace_bytes < attn_scratch_bytes(n_heads, n_kv_heads, d_head, max_seq)) return B2_E_INVALID;
    AttnParams a{};
    a.q = q; a.K = K; a.V = V; a.out = out;
    a.nsplit_max = (max_seq + kAttnChunk - 1) / kAttnChunk;
    const size_t part = (size_t)n_heads * a.nsplit_max * (d_head + 2) * sizeof(float);
    a.part = static_cast<float*>(workspace);
    a.counters = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + ((part + 255) & ~(size_t)255));
    a.H = n_heads; a.KVH = n_kv_heads; a.dh = d_head; a.max_seq = max_seq;
    a.st = nullptr; a.n_fixed = n;
    return status(launch_attn(a, static_cast<cudaStream_t>(stream), false));
}

int b2_argmax(const float* v, int64_t n, int32_t* out, void* stream) {
    if (!v || !out || n <= 0) return B2_E_INVALID;
    argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(v, (long long)n, out);
    return status(cudaGetLastError());
}

int b2_silu_mul(const float* g, const float* u, float* h, int n, void* stream) {
    if (!g || !u || !h || n <= 0) return B2_E_INVALID;
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(g, u, h, n);
    return status(cudaGetLastError());
}

int b2_gelu(const float* x, float* y, int n, void* stream) {
    if (!x || !y || n <= 0) return B2_E_INVALID;
    gelu_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return status(cudaGetLastError());
}

int b2_quantize_rows(const float* W, int64_t m, int64_t n, int8_t* q, int64_t ldq, float* scale, void* stream) {
    if (!W || !q || !scale || m <= 0 || n <= 0 || ldq < n) return B2_E_INVALID;
    quantize_rows_kernel<<<(unsigned)((m + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(W, m, n, q, ldq,
                                                                                                scale);
    return status(cudaGetLastError());
}

int b2_synth_quant_rows(uint64_t seed, uint64_t tensor_id, int64_t n, float stdv, int64_t r0, int64_t r1,
                        int64_t c0, int64_t c1, int8_t* q, int64_t ldq, float* scale, void* stream) {
    if (!q || !scale || n <= 0 || r0 < 0 || r1 <= r0 || c0 < 0 || c1 <= c0 || c1 > n || ldq < c1 - c0)
        return B2_E_INVALID;
    synth_quant_kernel<<<(unsigned)((r1 - r0 + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        seed, tensor_id, n, stdv, r0, r1, c0, c1, q, ldq, scale);
    return status(cudaGetLastError());
}

int b2_synth_fill_f32(uint64_t seed, uint64_t tensor_id, int64_t m, int64_t n, float stdv, float* out,
                      void* stream) {
    if (!out || m <= 0 || n <= 0) return B2_E_INVALID;
    const long long tot = (long long)m * n;
    synth_fill_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        seed, tensor_id, m, n, n, stdv, out);
    return status(cudaGetLastError());
}

}  // extern "C"
