// attn.cuh — split-KV decode attention over the f32 KV cache (sm_100a).
//
// Restates one decode step of _gqa_score_head_i8 (attention_gqa_kv_i8.ari:97-117)
// and attn_kv_step_f32's scoring half (attention_kv_f32.ari:134-162) for every
// query head at once:
//     scores_j = Kc[j] . q          (q already rotated and pre-scaled by 1/sqrt(dh))
//     scores[n..max_seq) = -60      (the reference's inactive-tail sentinel)
//     p = softmax(scores over all max_seq)
//     out = sum_{j<n} p_j Vc[j]
// as a flash-decode: CTA (split s, kv head) handles keys [64s, 64s+64) for the
// query heads of its group, writes (m_s, l_s, o_s) to scratch, and the last CTA
// of each kv head combines the splits and the closed-form -60 tail
// ((max_seq - n) virtual logits). Arithmetic order = oracle/refdec.c attn_head().
#pragma once
#include "b2_common.cuh"

namespace b2 {

constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 256;

struct AttnParams {
    const float* q;        // [H * dh]
    const float* K;        // [KVH][max_seq][dh]
    const float* V;
    float* out;            // [H * dh]
    float* part;           // scratch [H][nsplit_max][dh + 2]: o_s[dh], m_s, l_s
    unsigned* counters;    // scratch [KVH], zero between launches
    int H, KVH, dh, max_seq, nsplit_max;
    StepState* st;         // nullptr: n = n_fixed
    int n_fixed;
    int* err;
    Mirror mir;            // token kernel, tensor parallelism: out also written to the peers
    // batched decode (grid z = sequence): sequence z reads q + z * sq, K/V + z * skv,
    // writes out + z * sq, uses part + z * spart and counters + z * KVH, and sees
    // n_of[z] + 1 keys (n_of: positions; nullptr for one sequence)
    const int* n_of;
    long long sq, skv, spart;
    // token kernel, (value, tag) words: q, this step's K / V rows [KVH * dh], the
    // split partials (same layout as part) and the output
    const unsigned long long* tq;
    const unsigned long long* tkn;
    const unsigned long long* tvn;
    unsigned long long* tpart;
    unsigned long long* tout;
};

// bytes of scratch one call needs
inline size_t attn_scratch_bytes(int H, int KVH, int dh, int max_seq) {
    const size_t ns = (size_t)(max_seq + kAttnChunk - 1) / kAttnChunk;
    const size_t part = (size_t)H * ns * (dh + 2) * sizeof(float);
    return ((part + 255) & ~(size_t)255) + (size_t)KVH * sizeof(unsigned);
}

inline size_t attn_smem_bytes(int G, int dh, int nsplit_max) {
    return 64 + 2 * (size_t)kAttnChunk * dh * sizeof(float) +
           ((size_t)G * dh + (size_t)G * kAttnChunk + 2 * (size_t)G + (size_t)G * nsplit_max +
            (size_t)G + 8) * sizeof(float);
}

// K/V rows of one split are contiguous ([kv_head][max_seq][dh] layout): two bulk
// copies bring the split's keys and values into shared memory (dh % 4 == 0).
static __global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(128) unsigned char asmem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(asmem);
    const int G = p.H / p.KVH, dh = p.dh;
    float* Ks = reinterpret_cast<float*>(asmem + 64);         // [64][dh]
    float* Vs = Ks + kAttnChunk * dh;                          // [64][dh]
    float* qs = Vs + kAttnChunk * dh;                          // [G][dh]
    float* sc = qs + G * dh;                                   // [G][64] scores, then exp
    float* mpart = sc + G * kAttnChunk;                        // [G]
    float* lpart = mpart + G;                                  // [G]
    float* wsm = lpart + G;                                    // [G][nsplit_max]
    float* Lsm = wsm + G * p.nsplit_max;                       // [G]
    __shared__ int last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) { mbar_init(bar, 1); fence_mbar_init(); }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    const bool active = p.st ? (*(volatile int*)&p.st->active != 0) : true;
    if (!active) return;
    const int z = blockIdx.z;
    const int n = p.n_of ? p.n_of[z] + 1 : (p.st ? *(volatile int*)&p.st->pos + 1 : p.n_fixed);
    const int s = blockIdx.x, kvh = blockIdx.y;
    // this sequence's inputs, cache, outputs and scratch (z = 0 for one sequence)
    const float* __restrict__ qz = p.q + z * p.sq;
    float* outz = p.out + z * p.sq;
    float* partz = p.part + z * p.spart;
    unsigned* cntz = p.counters + (size_t)z * p.KVH;
    const int nsplit = (n + kAttnChunk - 1) / kAttnChunk;
    if (s >= nsplit) return;
    const int j0 = s * kAttnChunk;
    const int len = min(kAttnChunk, n - j0);
    const float* Kh = p.K + z * p.skv + (size_t)kvh * p.max_seq * dh;
    const float* Vh = p.V + z * p.skv + (size_t)kvh * p.max_seq * dh;
    if (tid == 0) {
        const uint32_t bytes = (uint32_t)len * dh * 4;
        mbar_arrive_expect_tx(bar, 2 * bytes);
        bulk_g2s(Ks, Kh + (size_t)j0 * dh, bytes, bar);
        bulk_g2s(Vs, Vh + (size_t)j0 * dh, bytes, bar);
    }
    const int h0 = kvh * G;
    for (int i = tid; i < G * dh; i += kAttnThreads) qs[i] = qz[(size_t)h0 * dh + i];
    if (!mbar_wait_bounded(bar, 0)) {
        set_err(p.err, B2_DEV_ERR_TIMEOUT);
        mbar_wait_bounded(bar, 0);                 // last bounded wait for the copies in flight
        return;
    }
    __syncthreads();

    // scores: warp per key, 32-lane dot over dh (lane L: d = L, L+32, ...)
    for (int jj = warp; jj < len; jj += kAttnThreads / 32) {
        const float* kr = Ks + jj * dh;
        float kv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int d = lane + 32 * i;
            kv[i] = d < dh ? kr[d] : 0.0f;
        }
        for (int g = 0; g < G; ++g) {
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < dh) a = ffma(qs[g * dh + d], kv[i], a);
            }
            a = butterfly32(a);
            if (lane == 0) sc[g * kAttnChunk + jj] = a;
        }
    }
    __syncthreads();

    // per head: chunk max, exp, chunk sum
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -__int_as_float(0x7f800000);
        bool any = false;
        for (int jj = lane; jj < len; jj += 32) {
            const float v = sc[g * kAttnChunk + jj];
            m = any ? fmaxf(m, v) : v;
            any = true;
        }
        for (int o = 16; o >= 1; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, o);
            const int oa = __shfl_xor_sync(0xffffffffu, (int)any, o);
            if (oa) { m = any ? fmaxf(m, om) : om; any = true; }
        }
        float a = 0.0f;
        for (int jj = lane; jj < len; jj += 32) {
            const float e = exp_f(fsub(sc[g * kAttnChunk + jj], m));
            sc[g * kAttnChunk + jj] = e;
            a = fadd(a, e);
        }
        a = butterfly32(a);
        if (lane == 0) { mpart[g] = m; lpart[g] = a; }
    }
    __syncthreads();

    // o_s[d] = sum_j e_j V[j][d], j ascending
    const int stride = dh + 2;
    for (int it = tid; it < G * dh; it += kAttnThreads) {
        const int g = it / dh, d = it % dh;
        const float* e = sc + g * kAttnChunk;
        float a = 0.0f;
        for (int jj = 0; jj < len; ++jj) a = ffma(e[jj], Vs[jj * dh + d], a);
        float* pp = partz + ((size_t)(h0 + g) * p.nsplit_max + s) * stride;
        pp[d] = a;
        if (d == 0) { pp[dh] = mpart[g]; pp[dh + 1] = lpart[g]; }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = (atomicAdd(cntz + kvh, 1u) == (unsigned)(nsplit - 1));
    __syncthreads();
    if (!last) return;
    __threadfence();

    // combine the splits (and the -60 tail) for the G heads of this kv head
    for (int g = tid; g < G; g += kAttnThreads) {
        const float* base = partz + (size_t)(h0 + g) * p.nsplit_max * stride;
        float M = __ldcg(base + dh);
        for (int t = 1; t < nsplit; ++t) M = fmaxf(M, __ldcg(base + (size_t)t * stride + dh));
        if (n < p.max_seq) M = fmaxf(M, -60.0f);
        float l = 0.0f;
        for (int t = 0; t < nsplit; ++t) {
            const float w = exp_f(fsub(__ldcg(base + (size_t)t * stride + dh), M));
            wsm[g * p.nsplit_max + t] = w;
            l = ffma(__ldcg(base + (size_t)t * stride + dh + 1), w, l);
        }
        if (n < p.max_seq) l = ffma((float)(p.max_seq - n), exp_f(fsub(-60.0f, M)), l);
        Lsm[g] = l;
    }
    __syncthreads();
    for (int it = tid; it < G * dh; it += kAttnThreads) {
        const int g = it / dh, d = it % dh;
        const float* base = partz + (size_t)(h0 + g) * p.nsplit_max * stride;
        float o = 0.0f;
        for (int t = 0; t < nsplit; ++t)
            o = ffma(__ldcg(base + (size_t)t * stride + d), wsm[g * p.nsplit_max + t], o);
        outz[(size_t)(h0 + g) * dh + d] = fdiv(o, Lsm[g]);
    }
    if (tid == 0) cntz[kvh] = 0u;
}

}  // namespace b2
