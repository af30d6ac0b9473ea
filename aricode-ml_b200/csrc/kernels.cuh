// kernels.cuh — small kernels of the decode path and the launch helpers shared by
// the runtime (runtime.cu) and the kernel-level C ABI (capi.cu).
#pragma once
#include <cuda_runtime.h>

#include "attn.cuh"
#include "b2_common.cuh"
#include "gemv.cuh"

namespace b2 {

// ------------------------------------------------------------------ embedding
// Token selection + embedding row for one decode step (aricode_pack.py:2205-2284):
// tok = prompt[t] while t < prompt_len, else the previous step's argmax;
// x = f32(q[tok]) * scale[tok] (+ learned position row t).
struct EmbedParams {
    const void* emb;        // [vocab][ld] int8 or f32
    int emb_i8;             // 1 int8, 2 int4 (two codes a byte, even column low), 0 f32
    const float* emb_s;     // per-row scales (int8)
    long long ld;
    const float* pos_tab;   // [max_pos][d] or nullptr
    int max_pos;
    int d, vocab, max_seq;
    const int* prompt;      // device prompt ids
    StepState* st;
    float* x;               // residual stream [d]
    unsigned long long* tx; // token kernel: x as (value, tag) words instead
};

static __global__ void embed_kernel(const __grid_constant__ EmbedParams p) {
    __shared__ int s_tok, s_pos, s_ok;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) {
        StepState* st = p.st;
        int ok = 0;
        if (st->active) {
            const int t = st->step;
            if (t >= p.max_seq || (p.pos_tab && t >= p.max_pos)) {
                atomicCAS(&st->err, 0, (int)B2_DEV_ERR_KV_OVERFLOW);
                st->active = 0;
            } else {
                const int tok = t < st->prompt_len ? p.prompt[t] : st->next_tok;
                if (tok < 0 || tok >= p.vocab) {
                    atomicCAS(&st->err, 0, (int)B2_DEV_ERR_BAD_TOKEN);
                    st->active = 0;
                } else {
                    st->pos = t;
                    st->step = t + 1;
                    s_tok = tok;
                    s_pos = t;
                    ok = 1;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const int tok = s_tok, pos = s_pos;
    for (int i = threadIdx.x; i < p.d; i += blockDim.x) {
        float v;
        if (p.emb_i8 == 2) {
            const int b = reinterpret_cast<const unsigned char*>(p.emb)[(size_t)tok * p.ld + (i >> 1)];
            const int q = (((b >> ((i & 1) * 4)) & 15) ^ 8) - 8;
            v = fmul((float)q, p.emb_s[tok]);
        } else if (p.emb_i8) {
            const int8_t q = reinterpret_cast<const int8_t*>(p.emb)[(size_t)tok * p.ld + i];
            v = fmul((float)q, p.emb_s[tok]);
        } else {
            v = reinterpret_cast<const float*>(p.emb)[(size_t)tok * p.ld + i];
        }
        if (p.pos_tab) v = fadd(v, p.pos_tab[(size_t)pos * p.d + i]);
        p.x[i] = v;
    }
}

// (re)start a decode sequence on the device without a host round trip
static __global__ void set_state_kernel(StepState* st, int step, int prompt_len, int max_new,
                                        int next_tok, int eos) {
    pdl_wait();
    st->step = step;
    st->pos = step;
    st->prompt_len = prompt_len;
    st->max_new = max_new;
    st->next_tok = next_tok;
    st->n_out = 0;
    st->active = 1;
    st->eos = eos;
    st->err = 0;
}

// ------------------------------------------------------------------ sampling
// Sampling beyond greedy, one step (sampling_f32.ari:31-153 as the decoder loop
// calls it, aricode_pack.py:2291-2306; oracle b2o_sample): advance the step's
// LCG, optionally keep the top-k distinct logits, then temperature softmax and
// an inverse-CDF draw. Runs after the LM head (which wrote the logits and left
// the token choice to this kernel) as one CTA; the two f64 running sums are
// sequential on one thread, as in the reference (their rounding order is the
// result), with their inputs loaded in batches.
enum SampleMode : int { SAMPLE_GREEDY = 0, SAMPLE_TEMPERATURE = 1, SAMPLE_TOPK = 2 };
constexpr int kSampleThreads = 1024;

struct SampleParams {
    float* logits;          // [vocab], overwritten (filtered, then probabilities)
    double* e;              // [vocab] scratch: the unrounded f64 exponentials
    int vocab;
    int mode, top_k;
    double temperature;
    StepState* st;
    int* out_ids;
};

// first index of the maximum, NaN never wins, logits[0] NaN -> 0 (sample_greedy_f32)
__device__ __forceinline__ int sample_block_argmax(const float* l, int n, float* wv, int* wi) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = 0.0f;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += kSampleThreads) {
        const float v = l[i];
        if (bi == 0x7fffffff || amax_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    for (int s = 16; s >= 1; s >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || amax_better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { wv[warp] = bv; wi[warp] = bi; }
    __syncthreads();
    float cv = 0.0f;
    int ci = 0x7fffffff;
    for (int w = 0; w < kSampleThreads / 32; ++w)
        if (wi[w] != 0x7fffffff && (ci == 0x7fffffff || amax_better(wv[w], wi[w], cv, ci))) { cv = wv[w]; ci = wi[w]; }
    __syncthreads();
    const float v0 = l[0];
    return (v0 != v0 || ci == 0x7fffffff) ? 0 : ci;
}

// largest f64 value of the logits strictly below `below` (or -1e30): one top-k pass
__device__ __forceinline__ double sample_block_max_below(const float* l, int n, double below, double* wd) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double cur = -1.0e30;
    for (int i = tid; i < n; i += kSampleThreads) {
        const double v = (double)l[i];
        if (v < below && v > cur) cur = v;
    }
    for (int s = 16; s >= 1; s >>= 1) cur = fmax(cur, __shfl_xor_sync(0xffffffffu, cur, s));
    if (lane == 0) wd[warp] = cur;
    __syncthreads();
    double r = -1.0e30;
    for (int w = 0; w < kSampleThreads / 32; ++w) r = fmax(r, wd[w]);
    __syncthreads();
    return r;
}

static __global__ void __launch_bounds__(kSampleThreads) sample_kernel(const __grid_constant__ SampleParams p) {
    __shared__ float wv[kSampleThreads / 32];
    __shared__ int wi[kSampleThreads / 32];
    __shared__ double wd[kSampleThreads / 32];
    __shared__ double s_mx, s_inv;
    __shared__ int s_tok;
    StepState* st = p.st;
    if (!*(volatile int*)&st->active || *(volatile int*)&st->err) return;
    const int tid = threadIdx.x, n = p.vocab;
    float* l = p.logits;
    const unsigned rng = *(volatile unsigned*)&st->rng * 1103515245u + 12345u;
    const double unit = ddiv((double)(int)(rng & 65535u), 65536.0);
    if (p.mode == SAMPLE_TOPK && p.top_k < n) {
        if (p.top_k <= 0) {
            const int best = sample_block_argmax(l, n, wv, wi);
            for (int j = tid; j < n; j += kSampleThreads)
                if (j != best) l[j] = -1.0e6f;
        } else {
            double prev = 1.0e30, kth = 0.0;
            for (int pass = 0; pass < p.top_k; ++pass) {
                kth = sample_block_max_below(l, n, prev, wd);
                prev = kth;
            }
            for (int j = tid; j < n; j += kSampleThreads)
                if ((double)l[j] < kth) l[j] = -1.0e6f;
        }
        __syncthreads();
    }
    int tok;
    if (p.temperature <= 0.0) {
        tok = sample_block_argmax(l, n, wv, wi);
    } else {
        const double inv_t = ddiv(1.0, p.temperature);
        for (int i = tid; i < n; i += kSampleThreads) l[i] = __double2float_rn(dmul((double)l[i], inv_t));
        __syncthreads();
        // max with the reference's scan semantics: l[0] NaN stays NaN, later NaNs never win
        {
            double cur = -__longlong_as_double(0x7ff0000000000000ll);
            for (int i = tid; i < n; i += kSampleThreads) {
                const double v = (double)l[i];
                if (v > cur) cur = v;
            }
            for (int s = 16; s >= 1; s >>= 1) cur = fmax(cur, __shfl_xor_sync(0xffffffffu, cur, s));
            if ((tid & 31) == 0) wd[tid >> 5] = cur;
            __syncthreads();
            if (tid == 0) {
                double r = wd[0];
                for (int w = 1; w < kSampleThreads / 32; ++w) r = fmax(r, wd[w]);
                const double v0 = (double)l[0];
                s_mx = v0 != v0 ? v0 : r;
            }
            __syncthreads();
        }
        const double mx = s_mx;
        for (int i = tid; i < n; i += kSampleThreads) {
            const double e = exp_d(__dsub_rn((double)l[i], mx));
            p.e[i] = e;
            l[i] = __double2float_rn(e);
        }
        __syncthreads();
        if (tid == 0) {
            double sum = 0.0;
            int i = 0;
            for (; i + 16 <= n; i += 16) {
                double b[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) b[u] = p.e[i + u];
#pragma unroll
                for (int u = 0; u < 16; ++u) sum = dadd(sum, b[u]);
            }
            for (; i < n; ++i) sum = dadd(sum, p.e[i]);
            s_inv = ddiv(1.0, sum);
        }
        __syncthreads();
        const double inv_sum = s_inv;
        for (int i = tid; i < n; i += kSampleThreads) l[i] = __double2float_rn(dmul((double)l[i], inv_sum));
        __syncthreads();
        if (tid == 0) {
            double cum = 0.0;
            int found = n - 1;
            bool done = false;
            for (int i = 0; i < n && !done; i += 16) {
                float b[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) b[u] = i + u < n ? l[i + u] : 0.0f;
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    if (!done && i + u < n) {
                        cum = dadd(cum, (double)b[u]);
                        if (cum > unit) { found = i + u; done = true; }
                    }
                }
            }
            s_tok = found;
        }
        __syncthreads();
        tok = s_tok;
    }
    if (tid == 0) {
        st->rng = rng;
        st->next_tok = tok;
        if (st->pos >= st->prompt_len - 1) {
            if (st->eos >= 0 && tok == st->eos) {
                st->active = 0;                          // EOS is not emitted
            } else {
                p.out_ids[st->n_out] = tok;
                st->n_out += 1;
                if (st->n_out >= st->max_new) st->active = 0;
            }
        }
    }
}

// ------------------------------------------------------------------ standalone ops
// 256-thread block; same reduction pattern as the GEMV prologue / oracle reduce256
__device__ __forceinline__ float block_reduce256(float part, float* red) {
    const float w = butterfly32(part);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = w;
    __syncthreads();
    const float tot = fadd(fadd(fadd(red[0], red[1]), fadd(red[2], red[3])),
                           fadd(fadd(red[4], red[5]), fadd(red[6], red[7])));
    __syncthreads();
    return tot;
}

static __global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, const float* g, float* y,
                                                      int d, float eps) {
    __shared__ float red[8];
    float a = 0.0f;
    for (int i = threadIdx.x; i < d; i += 256) a = ffma(x[i], x[i], a);
    const float ms = fdiv(block_reduce256(a, red), (float)d);
    const float inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, eps)));
    for (int i = threadIdx.x; i < d; i += 256) y[i] = fmul(fmul(x[i], inv), g[i]);
}

static __global__ void __launch_bounds__(256) layernorm_kernel(const float* x, const float* g,
                                                        const float* b, float* y, int d,
                                                        float eps) {
    __shared__ float red[8];
    float a = 0.0f;
    for (int i = threadIdx.x; i < d; i += 256) a = fadd(a, x[i]);
    const float mean = fdiv(block_reduce256(a, red), (float)d);
    a = 0.0f;
    for (int i = threadIdx.x; i < d; i += 256) { const float dx = fsub(x[i], mean); a = ffma(dx, dx, a); }
    const float var = fdiv(block_reduce256(a, red), (float)d);
    const float inv = fdiv(1.0f, __fsqrt_rn(fadd(var, eps)));
    for (int i = threadIdx.x; i < d; i += 256) {
        const float t = fmul(fsub(x[i], mean), inv);
        y[i] = (float)dadd(dmul((double)t, (double)g[i]), (double)b[i]);
    }
}

static __global__ void rope_kernel(float* v, const float* table, int pos, int dh, int n_pairs) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const int vec = i / (dh / 2), pr = i % (dh / 2);
    float* pv = v + (size_t)vec * dh + 2 * pr;
    const float c = table[(size_t)pos * dh + 2 * pr], s = table[(size_t)pos * dh + 2 * pr + 1];
    const float x0 = pv[0], x1 = pv[1];
    pv[0] = fsub(fmul(x0, c), fmul(x1, s));
    pv[1] = fadd(fmul(x0, s), fmul(x1, c));
}

static __global__ void __launch_bounds__(1024) argmax_kernel(const float* v, long long n, int* out) {
    __shared__ float sv[32];
    __shared__ int si[32], sh[32];
    float bv = 0.0f; int bi = 0x7fffffff; bool have = false;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = v[i];
        if (!have || amax_better(x, (int)i, bv, bi)) { bv = x; bi = (int)i; have = true; }
    }
    for (int s = 16; s >= 1; s >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
        const int oh = __shfl_xor_sync(0xffffffffu, (int)have, s);
        if (oh && (!have || amax_better(ov, oi, bv, bi))) { bv = ov; bi = oi; have = true; }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv[w] = bv; si[w] = bi; sh[w] = have; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float cv = 0.0f; int ci = 0; bool ch = false;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k)
            if (sh[k] && (!ch || amax_better(sv[k], si[k], cv, ci))) { cv = sv[k]; ci = si[k]; ch = true; }
        const float v0 = v[0];
        out[0] = (v0 != v0 || !ch) ? 0 : ci;
    }
}

static __global__ void silu_mul_kernel(const float* g, const float* u, float* h, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = fmul(silu_f(g[i]), u[i]);
}

static __global__ void gelu_kernel(const float* x, float* y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = gelu_f(x[i]);
}

// per-row int8 quantiser, numpy float32 semantics (aricode_pack.py:3356-3379): warp per row
static __global__ void quantize_rows_kernel(const float* W, long long m, long long n, int8_t* q,
                                     long long ldq, float* scale) {
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= m) return;
    const float* w = W + row * n;
    float mx = 0.0f;
    for (long long c = lane; c < n; c += 32) mx = fmaxf(mx, fabsf(w[c]));
    for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    const float sc = fdiv(mx, 127.0f);
    const float safe = sc > 0.0f ? sc : 1.0f;
    int8_t* qr = q + row * ldq;
    for (long long c = lane; c < ldq; c += 32) {
        if (c < n) {
            float v = rintf(fdiv(w[c], safe));
            v = fminf(fmaxf(v, -128.0f), 127.0f);
            qr[c] = (int8_t)(int)v;
        } else {
            qr[c] = 0;
        }
    }
    if (lane == 0) scale[row] = sc;
}

// synthetic weights: splitmix64 key -> four 16-bit uniforms -> centred sum * std/std_sum
// (identical to oracle b2o_synth_value)
__device__ __forceinline__ float synth_value(unsigned long long seed, unsigned long long tid,
                                             unsigned long long idx, float stdv) {
    unsigned long long z = seed * 0xD1B54A32D192ED03ull + tid * 0xA0761D6478BD642Full + idx;
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z = z ^ (z >> 31);
    const int s = (int)(z & 0xFFFF) + (int)((z >> 16) & 0xFFFF) + (int)((z >> 32) & 0xFFFF) +
                  (int)(z >> 48) - 131070;
    const float c = fmul(stdv, 0x1.bb67aep-16f);
    return fmul((float)s, c);
}

static __global__ void synth_quant_kernel(unsigned long long seed, unsigned long long tid, long long n,
                                   float stdv, long long r0, long long r1, long long c0,
                                   long long c1, int8_t* q, long long ldq, float* scale) {
    const long long row = r0 + (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= r1) return;
    float mx = 0.0f;
    for (long long c = lane; c < n; c += 32)
        mx = fmaxf(mx, fabsf(synth_value(seed, tid, (unsigned long long)(row * n + c), stdv)));
    for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    const float sc = fdiv(mx, 127.0f);
    const float safe = sc > 0.0f ? sc : 1.0f;
    int8_t* qr = q + (row - r0) * ldq;
    const long long w = c1 - c0;
    for (long long c = lane; c < ldq; c += 32) {
        if (c < w) {
            float v = rintf(fdiv(synth_value(seed, tid, (unsigned long long)(row * n + c0 + c), stdv), safe));
            v = fminf(fmaxf(v, -128.0f), 127.0f);
            qr[c] = (int8_t)(int)v;
        } else {
            qr[c] = 0;
        }
    }
    if (lane == 0) scale[row - r0] = sc;
}

static __global__ void synth_fill_kernel(unsigned long long seed, unsigned long long tid, long long m,
                                  long long n, long long ld, float stdv, float* out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m * ld) return;
    const long long r = i / ld, c = i % ld;
    out[i] = c < n ? synth_value(seed, tid, (unsigned long long)(r * n + c), stdv) : 0.0f;
}

// Synthetic KV rows [0, count) of one attention sub-block: value of global
// element ((kv0 + kh) * max_seq + pos) * dh + i with unit std, written at the
// local head kh (oracle b2o_state_fill_kv; kv0 = this rank's first KV head)
static __global__ void synth_kv_kernel(unsigned long long seed, unsigned long long tid, float* cache, int kvh,
                                       int kv0, int max_seq, int dh, int count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long per = (long long)count * dh;
    if (i >= per * kvh) return;
    const int kh = (int)(i / per);
    const long long rem = i % per;
    const int pos = (int)(rem / dh), d = (int)(rem % dh);
    const unsigned long long at = ((unsigned long long)(kv0 + kh) * max_seq + pos) * dh + d;
    cache[((long long)kh * max_seq + pos) * dh + d] = synth_value(seed, tid, at, 1.0f);
}

static __global__ void fill_kernel(float* out, long long n, float v) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = v;
}

// ------------------------------------------------------------------ launch helpers
inline cudaLaunchAttribute pdl_attr(bool pdl) {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    return a;
}

template <typename K, typename P>
inline cudaError_t launch_ex(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             bool pdl, const P& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1] = {pdl_attr(pdl)};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

constexpr size_t kGemvSmemBudget = 200 * 1024;   // one 544-thread CTA per SM
constexpr size_t kGemvStageTarget = 32 * 1024;   // >= 16 KB: bulk copies stream at full rate
constexpr int kGemvMaxK = 4;                       // 16-byte blocks per thread per row

struct GemvShape {
    int K;          // 16-byte blocks per thread per row
    int R;          // rows per stage
    bool paired;
    int grid;
    int nstages;
    int ring_offset;
    size_t smem;
};

inline int host_total_rows(const GemvParams& p) {
    if (p.paired) return p.rows[0];
    int t = 0;
    for (int s = 0; s < p.nseg; ++s) t += p.rows[s];
    return t;
}

inline GemvShape gemv_shape(const GemvParams& p, int esz, int grid_cap) {
    GemvShape sh{};
    sh.paired = p.paired != 0;
    const int nm = sh.paired ? 2 : 1;
    const size_t row_bytes = (size_t)p.ld * esz;
    sh.K = (int)((row_bytes / 16 + 255) / 256);
    const int unit = p.rope ? 2 : 1;
    const int total = host_total_rows(p);
    const int units = (total + unit - 1) / unit;
    sh.grid = units < grid_cap ? units : grid_cap;
    if (sh.grid < 1) sh.grid = 1;
    // rows per stage: a power of two (<= 16, <= 8 when paired) keeping the stage <= 32 KB
    int R = sh.paired ? 8 : 16;
    while (R > 1 && (size_t)R * row_bytes * nm > kGemvStageTarget) R >>= 1;
    sh.R = R;
    const int rows_cta = ((units + sh.grid - 1) / sh.grid) * unit;
    const size_t part_bytes = (size_t)rows_cta * nm * 8 * sizeof(float);
    sh.ring_offset = (int)((1024 + part_bytes + 127) & ~(size_t)127);
    const size_t stage = (size_t)R * row_bytes * nm;
    size_t budget = kGemvSmemBudget;
    if (budget < sh.ring_offset + 2 * kGemvGroups * stage) budget = sh.ring_offset + 2 * kGemvGroups * stage;
    long long ns = (long long)((budget - sh.ring_offset) / stage);
    const long long stages_cta = (rows_cta + R - 1) / R + (p.paired ? 0 : p.nseg);
    if (ns > stages_cta) ns = stages_cta;
    ns = ns / kGemvGroups * kGemvGroups;               // each slot belongs to one group
    if (ns < 2 * kGemvGroups) ns = 2 * kGemvGroups;
    if (ns > kGemvMaxStages) ns = kGemvMaxStages;
    sh.nstages = (int)ns;
    sh.smem = sh.ring_offset + (size_t)ns * stage;
    return sh;
}

// Launchers (defined once, in launch.cu, so that the GEMV kernel templates are
// instantiated in one translation unit only).
// weights int8 (w_i8) or f32; rows up to kGemvMaxK*256 16-byte blocks long
cudaError_t launch_gemv(const GemvParams& p, bool w_i8, cudaStream_t s, bool pdl, int grid_cap,
                        GemvShape* out_shape = nullptr);
cudaError_t launch_attn(const AttnParams& p, cudaStream_t s, bool pdl);
// int4 rows (p.i4, p.ld = packed bytes per row)
cudaError_t launch_gemv_i4(const GemvParams& p, cudaStream_t s, bool pdl, int grid_cap);
// the same kernel over nseq sequences (grid z; AttnParams::n_of and the strides)
cudaError_t launch_attn_batched(const AttnParams& p, int nseq, cudaStream_t s);
cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl);

}  // namespace b2
