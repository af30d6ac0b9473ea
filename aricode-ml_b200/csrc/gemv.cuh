// gemv.cuh — batch-1 weight-streaming GEMV for the decode path (sm_100a).
//
// Replaces the reference's arr_i8_matvec_f32_perrow / arr_f32_matvec builtins
// (call sites tools/aricode_pack.py:183, :1789-1808, attention_gqa_kv_i8.ari:149-151,
// :191, attention_kv_f32.ari:122-140) and fuses what runs around them:
//   prologue : input vector, optionally RMSNorm / LayerNorm
//              (rmsnorm_affine_f32 aricode_pack.py:585-607, layernorm_affine_f32 :503-521)
//   epilogue : per-row scale, bias (emit_linear :182-185), residual add (:2015-2018),
//              RoPE + 1/sqrt(d_head) + KV-cache append (attention_gqa_kv_i8.ari:154-182),
//              SiLU*up (silu_mul_f32 :626-632), GELU (gelu_f32 :539-572),
//              greedy argmax over the logits (sample_greedy_f32, sampling_f32.ari:10-24).
//
// Data movement: each CTA owns a balanced, contiguous range of rows. Consecutive
// rows are contiguous in HBM, so a stage of R whole rows (~16 KB) is ONE 1-D bulk
// async copy (TMA engine, mbarrier completion) into a shared-memory ring; a
// producer warp keeps the ring full. Its copies start before griddepcontrol.wait:
// under programmatic dependent launch the weights stream in while the previous
// kernel is still finishing.
//
// Compute: two groups of 8 consumer warps take alternate stages. Within a group
// the 256 threads split every row: thread s owns the 16-byte blocks s, s+256, ...
// (its slice of x lives in registers, normalised once), so a stage is read once
// from shared memory, conflict-free. Per row: four accumulators a[t & 3] updated
// by fused multiply-adds (issued as packed f32x2 pairs: two independent IEEE
// round-to-nearest operations, the same results as scalar ones), slot partial
// (a0+a1)+(a2+a3), warp butterfly, then the 8 warp sums
// ((W0+W1)+(W2+W3))+((W4+W5)+(W6+W7)) — oracle/refdec.c b2o_dot_i8 / b2o_dot_f32.
#pragma once
#include "b2_common.cuh"

namespace b2 {

enum EpiKind : int { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_GELU = 4,
                     EPI_ARGMAX = 5 };
enum NormKind : int { NORM_NONE = 0, NORM_RMS = 1, NORM_LN = 2 };

constexpr int kGemvGroupWarps = 8;                                 // warps per consumer group
constexpr int kGemvGroups = 2;                                     // groups on alternate stages
constexpr int kGemvConsumerWarps = kGemvGroupWarps * kGemvGroups;
constexpr int kGemvConsumerThreads = kGemvConsumerWarps * 32;
constexpr int kGemvThreads = kGemvConsumerThreads + 32;            // + producer warp
constexpr int kGemvMaxStages = 32;                                 // multiple of kGemvGroups

struct GemvParams {
    const void* W[3];          // up to 3 segments sharing n and ld (Q, K, V)
    const float* S[3];         // per-row scales (int8 weights)
    const float* bias[3];      // optional per-row bias
    int rows[3];
    int nseg;
    int paired;                // 1: every stage carries R rows of segment 0 and of segment 1
    int n;                     // logical input length
    int ld;                    // row stride in elements (16-byte multiple)
    int nstages;               // ring depth (multiple of kGemvGroups)
    int stage_rows;            // rows per stage (R)
    int ring_offset;           // byte offset of the ring in shared memory
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

// 4 int8 of u (xor 0x80 applied) against x: (a0,a1) += (w0,w1)*(x0,x1),
// (a2,a3) += (w2,w3)*(x2,x3); w = (2^23 + 128 + b) - (2^23 + 128), exact.
__device__ __forceinline__ void fma_word2(float2& a01, float2& a23, uint32_t u, float2 x01, float2 x23) {
    const float2 c = make_float2(-8388736.0f, -8388736.0f);
    float2 w01 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u)),
                             __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441u)));
    float2 w23 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442u)),
                             __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443u)));
    w01 = __fadd2_rn(w01, c);
    w23 = __fadd2_rn(w23, c);
    a01 = __ffma2_rn(w01, x01, a01);
    a23 = __ffma2_rn(w23, x23, a23);
}

__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerThreads) : "memory");
}

// Reduction over 256 partials held by consumer threads 0..255 (the others pass
// zeros and take part only in the barriers): warp butterfly, then
// ((W0+W1)+(W2+W3)) + ((W4+W5)+(W6+W7)). Same as the oracle's reduce256().
__device__ __forceinline__ float consumer_reduce256(float part, float* red, int tid) {
    const float w = butterfly32(part);
    if ((tid & 31) == 0 && tid < 256) red[tid >> 5] = w;
    consumer_bar();
    const float tot = fadd(fadd(fadd(red[0], red[1]), fadd(red[2], red[3])),
                           fadd(fadd(red[4], red[5]), fadd(red[6], red[7])));
    consumer_bar();
    return tot;
}

__device__ __forceinline__ float tree8(const float* w) {
    return fadd(fadd(fadd(w[0], w[1]), fadd(w[2], w[3])), fadd(fadd(w[4], w[5]), fadd(w[6], w[7])));
}

__device__ __forceinline__ void seg_of(const GemvParams& p, int row, int& seg, int& local) {
    seg = 0;
    local = row;
    while (seg < p.nseg - 1 && local >= p.rows[seg]) { local -= p.rows[seg]; ++seg; }
}

__device__ __forceinline__ int total_rows(const GemvParams& p) {
    if (p.paired) return p.rows[0];
    int t = 0;
    for (int s = 0; s < p.nseg; ++s) t += p.rows[s];
    return t;
}

// rows [r0, r1) of CTA b: balanced in units of `unit` rows (2 keeps RoPE pairs together)
__device__ __forceinline__ void cta_rows(int total, int unit, int& r0, int& r1) {
    const long long units = (total + unit - 1) / unit;
    const long long u0 = (long long)blockIdx.x * units / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * units / gridDim.x;
    r0 = (int)(u0 * unit);
    r1 = (int)(u1 * unit < (long long)total ? u1 * unit : (long long)total);
}

// Stage walk shared by producer and consumers: from logical row `cur`, the next
// stage takes up to R rows that stay inside one segment.
struct StageRows { int seg, local, nr; };
__device__ __forceinline__ StageRows next_stage(const GemvParams& p, int cur, int r1, int R) {
    StageRows st;
    if (p.paired) { st.seg = 0; st.local = cur; st.nr = min(R, r1 - cur); return st; }
    seg_of(p, cur, st.seg, st.local);
    st.nr = min(min(R, r1 - cur), p.rows[st.seg] - st.local);
    return st;
}

// Exchange butterfly over the 32 lanes for N row partials at once (N a power of
// two <= 32). At stride s the lane keeps half of its rows and trades the other
// half with lane ^ s; each kept sum is own + partner, exactly the operands the
// plain butterfly (v <- v + shfl_xor(v, s)) adds for that row, so the row totals
// are bit-identical to per-row butterflies while N rows cost about N + 4 shuffles.
// On return v[0] holds row (lane >> (5 - log2 N)); the 32/N lanes sharing those
// high bits hold the same total.
template <int N>
__device__ __forceinline__ void exchange_butterfly(float (&v)[N], int lane) {
    int cnt = N;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        if (cnt > 1) {
            const bool upper = (lane & s) != 0;
            const int h = cnt / 2;
#pragma unroll
            for (int i = 0; i < (N > 1 ? N / 2 : 1); ++i) {
                if (i < h) {
                    const float send = upper ? v[i] : v[h + i];
                    const float keep = upper ? v[h + i] : v[i];
                    v[i] = fadd(keep, __shfl_xor_sync(0xffffffffu, send, s));
                }
            }
            cnt = h;
        } else {
            v[0] = fadd(v[0], __shfl_xor_sync(0xffffffffu, v[0], s));
        }
    }
}

template <int N> struct Log2 { static constexpr int v = 1 + Log2<N / 2>::v; };
template <> struct Log2<1> { static constexpr int v = 0; };

template <typename WT, int KMAX, int RS, bool PAIRED>
__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_kernel(const __grid_constant__ GemvParams p) {
    constexpr int ESZ = (int)sizeof(WT);
    constexpr int EPB = 16 / ESZ;                                // elements per 16-byte block
    constexpr int NM = PAIRED ? 2 : 1;                           // matrices per stage
    constexpr int NR = RS * NM;                                  // rows reduced together
    constexpr int LG = Log2<NR>::v;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxStages;
    float* red = reinterpret_cast<float*>(empty + kGemvMaxStages);      // 8 floats
    float* part = reinterpret_cast<float*>(smem + 1024);                 // [rows_cta][NM][8]
    const int ld = p.ld;
    const uint32_t row_bytes = (uint32_t)ld * ESZ;
    const uint32_t stage_bytes = (uint32_t)RS * row_bytes * NM;
    unsigned char* ring = smem + p.ring_offset;
    const int NS = p.nstages;
    const int nblk = (int)(row_bytes >> 4);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    int r0, r1;
    cta_rows(total_rows(p), p.rope ? 2 : 1, r0, r1);

    if (NS < 2 * kGemvGroups || NS > kGemvMaxStages || NS % kGemvGroups || p.stage_rows != RS) {
        if (tid == 0) set_err(p.err, B2_DEV_ERR_TIMEOUT);     // uniform per grid
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGemvGroupWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemvConsumerWarps) {
        // ---------------- producer: one bulk copy (two when paired) per stage
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            int cur = r0;
            for (int j = 0; cur < r1; ++j) {
                const StageRows sr = next_stage(p, cur, r1, RS);
                const int slot = j % NS, round = j / NS;
                if (round > 0 && !mbar_wait_bounded(&empty[slot], (uint32_t)((round - 1) & 1))) {
                    ok = false;
                    break;
                }
                const uint32_t bytes = (uint32_t)sr.nr * row_bytes;
                unsigned char* dst = ring + (size_t)slot * stage_bytes;
                mbar_arrive_expect_tx(&full[slot], bytes * NM);
                bulk_g2s(dst, reinterpret_cast<const unsigned char*>(p.W[sr.seg]) +
                                  (size_t)sr.local * row_bytes, bytes, &full[slot]);
                if constexpr (PAIRED)
                    bulk_g2s(dst + (size_t)RS * row_bytes, reinterpret_cast<const unsigned char*>(p.W[1]) +
                                                               (size_t)sr.local * row_bytes, bytes, &full[slot]);
                ++issued;
                cur += sr.nr;
            }
            if (!ok) set_err(p.err, B2_DEV_ERR_TIMEOUT);
            // drain: no copy may still be in flight when the CTA exits
            for (int j = max(0, issued - NS); j < issued; ++j)
                if (!mbar_wait_bounded(&full[j % NS], (uint32_t)((j / NS) & 1))) {
                    set_err(p.err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }

    // ---------------- consumers: group g takes stages j with j % kGemvGroups == g
    const int group = warp / kGemvGroupWarps;
    const int gwarp = warp % kGemvGroupWarps;
    const int slotid = tid % 256;                                // this thread's block slot
    pdl_wait();
    const bool active = p.st ? (*(volatile int*)&p.st->active != 0) : true;
    const int pos = p.st ? *(volatile int*)&p.st->pos : p.pos_fixed;
    const int n = p.n;

    // prologue: this thread's slice of x (blocks slot, slot+256, ...), normalised
    float scale_a = 1.0f, shift_m = 0.0f;
    if (p.norm == NORM_RMS) {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float v = p.x[i]; a = ffma(v, v, a); }
        const float tot = consumer_reduce256(a, red, tid);
        const float ms = fdiv(tot, (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(ms, p.eps)));
    } else if (p.norm == NORM_LN) {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) a = fadd(a, p.x[i]);
        shift_m = fdiv(consumer_reduce256(a, red, tid), (float)n);
        a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float dx = fsub(p.x[i], shift_m); a = ffma(dx, dx, a); }
        const float var = fdiv(consumer_reduce256(a, red, tid), (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(var, p.eps)));
    }
    const int K = (nblk + 255) / 256;
    float2 xr[KMAX][EPB / 2];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        const int b = slotid + 256 * k;
#pragma unroll
        for (int t = 0; t < EPB; ++t) {
            const int i = b * EPB + t;
            float v = 0.0f;
            if (k < K && b < nblk && i < n) {
                const float xv = p.x[i];
                if (p.norm == NORM_RMS) v = fmul(fmul(xv, scale_a), p.ng[i]);
                else if (p.norm == NORM_LN)
                    v = (float)dadd(dmul((double)fmul(fsub(xv, shift_m), scale_a), (double)p.ng[i]),
                                    (double)p.nb[i]);
                else v = xv;
            }
            if (t & 1) xr[k][t / 2].y = v;
            else xr[k][t / 2].x = v;
        }
    }

    // stream the stages: all rows of a stage at once, then one exchange butterfly
    int cur = r0;
    for (int j = 0; cur < r1; ++j) {
        const StageRows sr = next_stage(p, cur, r1, RS);
        if (j % kGemvGroups == group) {
            const int slot = j % NS;
            if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / NS) & 1))) {
                set_err(p.err, B2_DEV_ERR_TIMEOUT);
                break;
            }
            const unsigned char* stage = ring + (size_t)slot * stage_bytes;
            if (active) {
                float2 a01[NR], a23[NR];
#pragma unroll
                for (int r = 0; r < NR; ++r) a01[r] = a23[r] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int k = 0; k < KMAX; ++k) {
                    const int b = slotid + 256 * k;
                    if (k < K && b < nblk) {
#pragma unroll
                        for (int r = 0; r < NR; ++r) {
                            // rows past sr.nr read stale (in-bounds) stage bytes; never stored
                            const unsigned char* row = stage + (size_t)r * row_bytes + 16 * b;
                            if constexpr (ESZ == 1) {
                                const uint4 w = lds128(row);
                                fma_word2(a01[r], a23[r], w.x ^ 0x80808080u, xr[k][0], xr[k][1]);
                                fma_word2(a01[r], a23[r], w.y ^ 0x80808080u, xr[k][2], xr[k][3]);
                                fma_word2(a01[r], a23[r], w.z ^ 0x80808080u, xr[k][4], xr[k][5]);
                                fma_word2(a01[r], a23[r], w.w ^ 0x80808080u, xr[k][6], xr[k][7]);
                            } else {
                                const float4 w = lds128f(row);
                                a01[r] = __ffma2_rn(make_float2(w.x, w.y), xr[k][0], a01[r]);
                                a23[r] = __ffma2_rn(make_float2(w.z, w.w), xr[k][1], a23[r]);
                            }
                        }
                    }
                }
                float v[NR];
#pragma unroll
                for (int r = 0; r < NR; ++r)
                    v[r] = fadd(fadd(a01[r].x, a01[r].y), fadd(a23[r].x, a23[r].y));
                exchange_butterfly<NR>(v, lane);
                if ((lane & ((32 >> LG) - 1)) == 0) {
                    const int rr = lane >> (5 - LG);             // stage row (m * RS + r)
                    const int m = rr / RS, r = rr % RS;
                    if (r < sr.nr) part[((cur - r0 + r) * NM + m) * 8 + gwarp] = v[0];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        cur += sr.nr;
    }
    consumer_bar();
    if (!active) return;

    // ---------------- epilogue: thread per row (per row pair with RoPE)
    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    bool have_best = false;
    const int nrows = r1 - r0;
    const int step = p.rope ? 2 : 1;
    for (int rl = tid * step; rl < nrows; rl += kGemvConsumerThreads * step) {
        const int lrow = r0 + rl;
        if constexpr (PAIRED) {                              // EPI_SWIGLU
            const float g = fmul(tree8(part + (rl * 2 + 0) * 8), p.S[0][lrow]);
            const float u = fmul(tree8(part + (rl * 2 + 1) * 8), p.S[1][lrow]);
            p.y[lrow] = fmul(silu_f(g), u);
            continue;
        }
        int seg, row;
        seg_of(p, lrow, seg, row);
        float val[2] = {0.0f, 0.0f};
        for (int e = 0; e < step; ++e) {
            float v = tree8(part + (rl + e) * 8);
            if constexpr (ESZ == 1) v = fmul(v, p.S[seg][row + e]);
            if (p.bias[seg]) v = fadd(v, p.bias[seg][row + e]);
            else if constexpr (ESZ == 4) v = fadd(v, 0.0f);
            val[e] = v;
        }
        if (p.epi == EPI_QKV) {
            float out[2] = {val[0], val[1]};
            if (p.rope && seg < 2) {
                // pair (2i, 2i+1): rows start even and segment sizes are even
                const int hd = row % p.dh;
                const float* tr = p.rope_tab + (size_t)pos * p.dh + hd;
                const float c = tr[0], sn = tr[1];
                out[0] = fsub(fmul(val[0], c), fmul(val[1], sn));
                out[1] = fadd(fmul(val[0], sn), fmul(val[1], c));
            }
            for (int e = 0; e < step; ++e) {
                const int rr = row + e;
                if (seg == 0) {
                    p.qout[rr] = fmul(out[e], p.qscale);
                } else if (pos < p.max_seq) {
                    const int kvh = rr / p.dh, hd = rr % p.dh;
                    float* cache = seg == 1 ? p.kcache : p.vcache;
                    cache[((size_t)kvh * p.max_seq + pos) * p.dh + hd] = out[e];
                } else {
                    set_err(p.err, B2_DEV_ERR_KV_OVERFLOW);
                }
            }
        } else if (p.epi == EPI_RESID) {
            p.y[row] = fadd(val[0], p.resid[row]);
        } else if (p.epi == EPI_GELU) {
            p.y[row] = gelu_f(val[0]);
        } else if (p.epi == EPI_ARGMAX) {
            if (p.y) p.y[row] = val[0];
            if (row == 0 && p.amax_v0nan) *p.amax_v0nan = (val[0] != val[0]) ? 1 : 0;
            if (!have_best || amax_better(val[0], row, best_v, best_i)) {
                best_v = val[0]; best_i = row; have_best = true;
            }
        } else {
            p.y[row] = val[0];
        }
    }

    if (p.epi == EPI_ARGMAX) {
        // thread -> warp -> CTA -> grid (the comparator is a total order, so the
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
        consumer_bar();
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
        consumer_bar();
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
