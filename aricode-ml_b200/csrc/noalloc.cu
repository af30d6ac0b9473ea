// noalloc.cu — decode attention whose scratch lives in a fixed device array.
//
// Some hosts cannot hand this library device memory for scratch: a process whose
// device memory is owned by a host framework that reserves it up front and does
// not let libraries call cudaMalloc (cudaMalloc/cudaFree synchronise the device
// and can fail under memory pressure in the middle of serving), or a thin FFI
// binding that has no device allocator of its own. For them,
// b2_attn_decode_static runs the same split-KV attention kernel as
// b2_attn_decode, with its split partials and per-head counters in
// g_attn_scratch below instead of a caller-provided workspace.
//
// Rules of this entry point:
//   * the array holds at most B2_ATTN_STATIC_SCRATCH_BYTES (4 MiB); larger
//     problems are rejected with B2_E_INVALID and a message in
//     b2_last_error(NULL, ...);
//   * every GPU that loads the library keeps the 4 MiB until the process exits;
//   * the first call on a device looks up the array's device address there
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture. The address is cached per device for the life
//     of the process and never looked up again, so a host that resets a device
//     (cudaDeviceReset) must not call this entry point on it afterwards;
//   * all calls share the array and it keeps the last call's contents: the
//     per-head counters are cleared on the caller's stream at the start of every
//     call (the partials are always written before they are read), and calls
//     that overlap on the GPU (different streams, no ordering) race on it;
//   * nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/b2dec.h"
#include "kernels.cuh"

void b2_internal_set_error(const std::string& msg);   // runtime.cu

namespace {

using namespace b2;

constexpr size_t kStaticScratchBytes = B2_ATTN_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 128;

// Device-side scratch. In host code this name is only a stand-in for the symbol,
// not a device address: host code reaches the array through the pointer that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_scratch_on[kMaxDevices] = {};

// Per-device set-up, once: device address of g_attn_scratch on the current device.
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        b2_internal_set_error(std::string("b2_attn_decode_static: cudaGetDevice: ") + cudaGetErrorString(e));
        return B2_E_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        b2_internal_set_error("b2_attn_decode_static: device index out of range");
        return B2_E_INVALID;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_on[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p) {
            b2_internal_set_error(std::string("b2_attn_decode_static: cudaGetSymbolAddress: ") +
                                  cudaGetErrorString(e));
            return B2_E_CUDA;
        }
        g_scratch_on[dev] = p;
    }
    *out = g_scratch_on[dev];
    return B2_OK;
}

}  // namespace

extern "C" int b2_attn_decode_static(const float* q, const float* K, const float* V, float* out,
                                     int n_heads, int n_kv_heads, int d_head, int n, int max_seq,
                                     void* stream) {
    if (!q || !K || !V || !out || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads ||
        d_head <= 0 || d_head > 256 || d_head % 4 || n <= 0 || n > max_seq ||
        (reinterpret_cast<uintptr_t>(K) & 15) || (reinterpret_cast<uintptr_t>(V) & 15)) {
        b2_internal_set_error("b2_attn_decode_static: invalid arguments");
        return B2_E_INVALID;
    }
    const size_t need = attn_scratch_bytes(n_heads, n_kv_heads, d_head, max_seq);
    if (need > kStaticScratchBytes) {
        b2_internal_set_error("b2_attn_decode_static: needs " + std::to_string(need) +
                              " bytes of scratch, the static array holds " +
                              std::to_string(kStaticScratchBytes) +
                              " (n_heads * ceil(max_seq/64) * (d_head+2) * 4 + n_kv_heads * 4)");
        return B2_E_INVALID;
    }
    void* base = nullptr;
    const int rc = scratch_address(&base);
    if (rc != B2_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    AttnParams a{};
    a.q = q; a.K = K; a.V = V; a.out = out;
    a.nsplit_max = (max_seq + kAttnChunk - 1) / kAttnChunk;
    const size_t part = (size_t)n_heads * a.nsplit_max * (d_head + 2) * sizeof(float);
    a.part = static_cast<float*>(base);
    a.counters = reinterpret_cast<unsigned*>(static_cast<char*>(base) + ((part + 255) & ~(size_t)255));
    a.H = n_heads; a.KVH = n_kv_heads; a.dh = d_head; a.max_seq = max_seq;
    a.st = nullptr; a.n_fixed = n;
    // the counters must start at zero; clear them in stream order before the kernel
    cudaError_t e = cudaMemsetAsync(a.counters, 0, (size_t)n_kv_heads * sizeof(unsigned), s);
    if (e == cudaSuccess) e = launch_attn(a, s, false);
    if (e != cudaSuccess) {
        b2_internal_set_error(std::string("b2_attn_decode_static: ") + cudaGetErrorString(e));
        return B2_E_CUDA;
    }
    return B2_OK;
}
