// gemv.cuh — batch-1 weight-streaming GEMV for the decode path (sm_100a).
//
// Replaces the reference's arr_i8_matvec_f32_perrow / arr_f32_matvec builtins
// (call sites tools/aricode_pack.py:183, :1789-1808, attention_gqa_kv_i8.ari:149-151,
// :191, attention_kv_f32.ari:122-140) and fuses what runs around them:
//   prologue : input vector -> shared memory, optionally RMSNorm / LayerNorm
//              (rmsnorm_affine_f32 aricode_pack.py:585-607, layernorm_affine_f32 :503-521)
//   epilogue : per-row scale, bias (emit_linear :182-185), residual add (:2015-2018),
//              RoPE + 1/sqrt(d_head) + KV-cache append (attention_gqa_kv_i8.ari:154-182),
//              SiLU*up (silu_mul_f32 :626-632), GELU (gelu_f32 :539-572),
//              greedy argmax over the logits (sample_greedy_f32, sampling_f32.ari:10-24).
//
// Data movement: rows of W are contiguous in HBM, so a group of R rows is one
// contiguous block. One producer lane streams groups into a shared-memory ring
// with 1-D bulk async copies (TMA engine, mbarrier completion); 8 consumer warps
// each own whole groups: group j -> warp j % 8, slot j % NS with NS a multiple
// of 8, so every slot belongs to one warp and its barrier phases stay in order. The producer starts before griddepcontrol.wait, so under
// programmatic dependent launch the ring fills with this kernel's weights while
// the previous kernel is still running.
//
// Arithmetic order (identical to oracle/refdec.c b2o_dot_i8 / b2o_dot_f32): lane L
// owns 16-byte blocks L, L+32, ...; four accumulators take element t of a block
// into a[t & 3] by fused multiply-add; lane partial (a0+a1)+(a2+a3); XOR
// butterfly 16,8,4,2,1.
#pragma once
#include "b2_common.cuh"

namespace b2 {

enum EpiKind : int { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_GELU = 4,
                     EPI_ARGMAX = 5 };
enum NormKind : int { NORM_NONE = 0, NORM_RMS = 1, NORM_LN = 2 };

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvMaxStages = 32;     // multiple of kGemvConsumerWarps

struct GemvParams {
    const void* W[3];          // up to 3 segments sharing n and ld (Q, K, V)
    const float* S[3];         // per-row scales (int8 weights)
    const float* bias[3];      // optional per-row bias
    int rows[3];
    int nseg;
    int paired;                // 1: each group takes R rows of segment 0 and of segment 1
    int n;                     // logical input length
    int ld;                    // row stride in elements (16-byte multiple)
    int nstages;               // ring depth
    const float* x;            // input vector [n]
    int norm;
    const float* ng;
    const float* nb;
    float eps;
    int epi;
    float* y;                  // output (ARGMAX: logits, optional)
    const float* resid;        // EPI_RESID
    // EPI_QKV
    int rope;
    const float* rope_tab;     // [max_seq, dh]
    int dh;
    float qscale;
    float* qout;
    float* kcache;             // [kv_heads][max_seq][dh]
    float* vcache;
    int max_seq;
    // EPI_ARGMAX
    float* amax_val;           // [gridDim.x]
    int* amax_idx;             // [gridDim.x]
    int* amax_v0nan;           // 1 when logit 0 is NaN (sequential argmax returns 0 then)
    unsigned* amax_count;      // last-CTA ticket, zero between launches
    int* out_tok;              // argmax result
    int* out_ids;              // generation output ring (with st)
    // step state: position, active flag, error word (nullptr for kernel-level calls)
    StepState* st;
    int pos_fixed;             // position when st == nullptr
    int* err;
};

// ordering for greedy sampling: non-NaN beats NaN, larger wins, ties -> lower index
__device__ __forceinline__ bool amax_better(float va, int ia, float vb, int ib) {
    const bool na = va != va, nb = vb != vb;
    if (na != nb) return nb;                   // a wins iff b is NaN
    if (!na && va != vb) return va > vb;
    return ia < ib;
}

struct GroupInfo { int seg, row0, nrows; };

template <int R>
__device__ __forceinline__ GroupInfo group_info(const GemvParams& p, long long g) {
    GroupInfo gi{0, 0, 0};
    const int nseg = p.paired ? 1 : p.nseg;
    for (int s = 0; s < nseg; ++s) {
        const long long ng = (p.rows[s] + R - 1) / R;
        if (g < ng) {
            gi.seg = s;
            gi.row0 = (int)(g * R);
            gi.nrows = min(R, p.rows[s] - gi.row0);
            return gi;
        }
        g -= ng;
    }
    return gi;
}

template <int R>
__device__ __forceinline__ long long total_groups(const GemvParams& p) {
    long long t = 0;
    const int nseg = p.paired ? 1 : p.nseg;
    for (int s = 0; s < nseg; ++s) t += (p.rows[s] + R - 1) / R;
    return t;
}

// 4 int8 (xor 0x80 applied) x 4 floats into a[0..3]
__device__ __forceinline__ void fma_word(float* a, uint32_t u, const float4& xv) {
    a[0] = ffma(i8_to_f(u, 0), xv.x, a[0]);
    a[1] = ffma(i8_to_f(u, 1), xv.y, a[1]);
    a[2] = ffma(i8_to_f(u, 2), xv.z, a[2]);
    a[3] = ffma(i8_to_f(u, 3), xv.w, a[3]);
}

// Reduction over the consumer threads' 256 partials (thread t < 256 holds partial t):
// warp butterfly, then ((W0+W1)+(W2+W3)) + ((W4+W5)+(W6+W7)). Same as reduce256().
__device__ __forceinline__ float consumer_reduce256(float part, float* red, int tid) {
    const float w = butterfly32(part);
    if ((tid & 31) == 0 && tid < 256) red[tid >> 5] = w;
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
    const float tot = fadd(fadd(fadd(red[0], red[1]), fadd(red[2], red[3])),
                           fadd(fadd(red[4], red[5]), fadd(red[6], red[7])));
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
    return tot;
}

template <typename WT, int R, bool PAIRED>
__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_kernel(const __grid_constant__ GemvParams p) {
    constexpr int RT = PAIRED ? R * 2 : R;          // rows held per group
    constexpr int ESZ = (int)sizeof(WT);
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxStages;
    float* red = reinterpret_cast<float*>(empty + kGemvMaxStages);        // 64 floats
    float* xs = reinterpret_cast<float*>(smem + 1024);
    const int ld = p.ld;
    const int rows_per_stage = RT;
    const uint32_t seg_bytes = (uint32_t)R * ld * ESZ;
    const uint32_t stage_bytes = (uint32_t)rows_per_stage * ld * ESZ;
    unsigned char* ring = smem + 1024 + (((size_t)ld * 4 + 127) & ~(size_t)127);
    const int NS = p.nstages;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const long long G = total_groups<R>(p);
    const long long g0 = (long long)blockIdx.x * G / gridDim.x;
    const long long g1 = (long long)(blockIdx.x + 1) * G / gridDim.x;
    const int nloc = (int)(g1 - g0);

    if (NS <= 0 || NS > kGemvMaxStages || NS % kGemvConsumerWarps != 0) {   // uniform per grid
        if (tid == 0) set_err(p.err, B2_DEV_ERR_TIMEOUT);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemvConsumerWarps) {
        // ---------------- producer: stream this CTA's groups into the ring
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < nloc; ++j) {
                const int slot = j % NS;
                const int round = j / NS;
                if (round > 0 && !mbar_wait_bounded(&empty[slot], (uint32_t)((round - 1) & 1))) {
                    set_err(p.err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
                const GroupInfo gi = group_info<R>(p, g0 + j);
                const uint32_t bytes = (uint32_t)gi.nrows * ld * ESZ;
                unsigned char* dst = ring + (size_t)slot * stage_bytes;
                const unsigned char* src0 =
                    reinterpret_cast<const unsigned char*>(p.W[gi.seg]) + (size_t)gi.row0 * ld * ESZ;
                if constexpr (PAIRED) {
                    const unsigned char* src1 =
                        reinterpret_cast<const unsigned char*>(p.W[1]) + (size_t)gi.row0 * ld * ESZ;
                    mbar_arrive_expect_tx(&full[slot], 2 * bytes);
                    bulk_g2s(dst, src0, bytes, &full[slot]);
                    bulk_g2s(dst + seg_bytes, src1, bytes, &full[slot]);
                } else {
                    mbar_arrive_expect_tx(&full[slot], bytes);
                    bulk_g2s(dst, src0, bytes, &full[slot]);
                }
                ++issued;
            }
            // drain: no copy may still be in flight when the CTA exits
            for (int j = max(0, issued - NS); j < issued; ++j)
                if (!mbar_wait_bounded(&full[j % NS], (uint32_t)((j / NS) & 1))) {
                    set_err(p.err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    const bool active = p.st ? (*(volatile int*)&p.st->active != 0) : true;
    const int pos = p.st ? *(volatile int*)&p.st->pos : p.pos_fixed;
    const int n = p.n;

    // prologue: x (optionally normalised) into shared memory, zero-padded to ld
    if (p.norm == NORM_NONE) {
        for (int i = tid; i < ld; i += kGemvConsumerWarps * 32) xs[i] = i < n ? p.x[i] : 0.0f;
    } else if (p.norm == NORM_RMS) {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float v = p.x[i]; a = ffma(v, v, a); }
        const float tot = consumer_reduce256(a, red, tid);
        const float ms = fdiv(tot, (float)n);
        const float inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, p.eps)));
        for (int i = tid; i < ld; i += kGemvConsumerWarps * 32)
            xs[i] = i < n ? fmul(fmul(p.x[i], inv), p.ng[i]) : 0.0f;
    } else {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) a = fadd(a, p.x[i]);
        const float mean = fdiv(consumer_reduce256(a, red, tid), (float)n);
        a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float dx = fsub(p.x[i], mean); a = ffma(dx, dx, a); }
        const float var = fdiv(consumer_reduce256(a, red, tid), (float)n);
        const float inv = fdiv(1.0f, __fsqrt_rn(fadd(var, p.eps)));
        for (int i = tid; i < ld; i += kGemvConsumerWarps * 32) {
            if (i < n) {
                const float t = fmul(fsub(p.x[i], mean), inv);
                xs[i] = (float)dadd(dmul((double)t, (double)p.ng[i]), (double)p.nb[i]);
            } else {
                xs[i] = 0.0f;
            }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");

    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    bool have_best = false;
    bool ok = true;

    for (int j = warp; j < nloc; j += kGemvConsumerWarps) {
        const int slot = j % NS;
        if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / NS) & 1))) {
            set_err(p.err, B2_DEV_ERR_TIMEOUT);
            ok = false;
            break;
        }
        const GroupInfo gi = group_info<R>(p, g0 + j);
        const unsigned char* stage = ring + (size_t)slot * stage_bytes;
        float acc[RT][4];
#pragma unroll
        for (int r = 0; r < RT; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.0f;
        if (active) {
            if constexpr (ESZ == 1) {
                const int nblk = ld >> 4;
                for (int b = lane; b < nblk; b += 32) {
                    const float4 x0 = lds128f(xs + 16 * b);
                    const float4 x1 = lds128f(xs + 16 * b + 4);
                    const float4 x2 = lds128f(xs + 16 * b + 8);
                    const float4 x3 = lds128f(xs + 16 * b + 12);
#pragma unroll
                    for (int r = 0; r < RT; ++r) {
                        const uint4 w = lds128(stage + (size_t)r * ld + 16 * b);
                        fma_word(acc[r], w.x ^ 0x80808080u, x0);
                        fma_word(acc[r], w.y ^ 0x80808080u, x1);
                        fma_word(acc[r], w.z ^ 0x80808080u, x2);
                        fma_word(acc[r], w.w ^ 0x80808080u, x3);
                    }
                }
            } else {
                const int nblk = ld >> 2;
                for (int b = lane; b < nblk; b += 32) {
                    const float4 xv = lds128f(xs + 4 * b);
#pragma unroll
                    for (int r = 0; r < RT; ++r) {
                        const float4 w = lds128f(stage + ((size_t)r * ld + 4 * b) * 4);
                        acc[r][0] = ffma(w.x, xv.x, acc[r][0]);
                        acc[r][1] = ffma(w.y, xv.y, acc[r][1]);
                        acc[r][2] = ffma(w.z, xv.z, acc[r][2]);
                        acc[r][3] = ffma(w.w, xv.w, acc[r][3]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);       // stage consumed
        if (!active) continue;

        float dot[RT];
#pragma unroll
        for (int r = 0; r < RT; ++r)
            dot[r] = butterfly32(fadd(fadd(acc[r][0], acc[r][1]), fadd(acc[r][2], acc[r][3])));

        // lane r finishes row gi.row0 + r
        const int r = lane;
        float v = 0.0f, v2 = 0.0f;
#pragma unroll
        for (int k = 0; k < R; ++k)
            if (r == k) { v = dot[k]; if constexpr (PAIRED) v2 = dot[R + k]; }
        const bool live = r < gi.nrows;
        const int row = gi.row0 + r;
        const int seg = gi.seg;
        if constexpr (PAIRED) {       // EPI_SWIGLU
            if (live) {
                const float g = fmul(v, p.S[0][row]);
                const float u = fmul(v2, p.S[1][row]);
                p.y[row] = fmul(silu_f(g), u);
            }
            continue;
        }
        float val = v;
        if (live) {
            if constexpr (ESZ == 1) val = fmul(val, p.S[seg][row]);
            if (p.bias[seg]) val = fadd(val, p.bias[seg][row]);
            else if constexpr (ESZ == 4) val = fadd(val, 0.0f);
        }
        if (p.epi == EPI_QKV) {
            float out = val;
            if (p.rope && seg < 2) {
                const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
                const int hd = row % p.dh;
                const float* tr = p.rope_tab + (size_t)pos * p.dh + (hd & ~1);
                const float c = tr[0], s = tr[1];
                out = (hd & 1) ? fadd(fmul(partner, s), fmul(val, c))
                               : fsub(fmul(val, c), fmul(partner, s));
            }
            if (live) {
                if (seg == 0) {
                    p.qout[row] = fmul(out, p.qscale);
                } else if (pos < p.max_seq) {
                    const int kvh = row / p.dh, hd = row % p.dh;
                    float* cache = seg == 1 ? p.kcache : p.vcache;
                    cache[((size_t)kvh * p.max_seq + pos) * p.dh + hd] = out;
                } else {
                    set_err(p.err, B2_DEV_ERR_KV_OVERFLOW);
                }
            }
        } else if (p.epi == EPI_RESID) {
            if (live) p.y[row] = fadd(val, p.resid[row]);
        } else if (p.epi == EPI_GELU) {
            if (live) p.y[row] = gelu_f(val);
        } else if (p.epi == EPI_ARGMAX) {
            if (live) {
                if (p.y) p.y[row] = val;
                if (row == 0 && p.amax_v0nan) *p.amax_v0nan = (val != val) ? 1 : 0;
                if (!have_best || amax_better(val, row, best_v, best_i)) {
                    best_v = val; best_i = row; have_best = true;
                }
            }
        } else {
            if (live) p.y[row] = val;
        }
    }
    (void)ok;

    if (p.epi == EPI_ARGMAX && active) {
        // warp -> CTA -> grid argmax (the comparator is a total order, so the
        // result does not depend on the reduction shape)
        for (int s = 16; s >= 1; s >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, s);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, s);
            const int oh = __shfl_xor_sync(0xffffffffu, (int)have_best, s);
            if (oh && (!have_best || amax_better(ov, oi, best_v, best_i))) {
                best_v = ov; best_i = oi; have_best = true;
            }
        }
        __shared__ float wv[kGemvConsumerWarps];
        __shared__ int wi[kGemvConsumerWarps];
        __shared__ int wh[kGemvConsumerWarps];
        __shared__ int last;
        if (lane == 0) { wv[warp] = best_v; wi[warp] = best_i; wh[warp] = have_best; }
        asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
        if (tid == 0) {
            float cv = 0.0f; int ci = 0x7fffffff; bool ch = false;
            for (int w = 0; w < kGemvConsumerWarps; ++w)
                if (wh[w] && (!ch || amax_better(wv[w], wi[w], cv, ci))) { cv = wv[w]; ci = wi[w]; ch = true; }
            p.amax_val[blockIdx.x] = cv;
            p.amax_idx[blockIdx.x] = ch ? ci : 0x7fffffff;
            __threadfence();
            const unsigned t = atomicAdd(p.amax_count, 1u);
            last = (t == gridDim.x - 1);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
        if (last && tid == 0) {
            __threadfence();
            float cv = 0.0f; int ci = 0x7fffffff; bool ch = false;
            for (int c = 0; c < (int)gridDim.x; ++c) {
                const int ii = __ldcg(p.amax_idx + c);
                const float vv = __ldcg(p.amax_val + c);
                if (ii != 0x7fffffff && (!ch || amax_better(vv, ii, cv, ci))) { cv = vv; ci = ii; ch = true; }
            }
            int tok = ch ? ci : 0;
            if (p.amax_v0nan && __ldcg(p.amax_v0nan)) tok = 0;    // sequential scan keeps index 0
            if (p.out_tok) *p.out_tok = tok;
            if (p.st) {
                StepState* st = p.st;
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
            *p.amax_count = 0u;
            __threadfence();
        }
    }
}

}  // namespace b2
