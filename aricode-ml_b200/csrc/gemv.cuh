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
// from shared memory, conflict-free.
//   int8 rows: an exact integer dot on a 32-bit fixed-point copy of x, four dp4a
//   per 4 codes (one per byte plane of x), plane sums reduced in any order and
//   rounded once (oracle/refdec.c b2o_xfix / b2o_dot_i8x; see gemv_stage_i8);
//   f32 rows: four accumulators a[t] updated by fused multiply-adds (packed f32x2
//   pairs: two independent IEEE round-to-nearest operations), slot partial
//   (a0+a1)+(a2+a3), warp butterfly, then the 8 warp sums
//   ((W0+W1)+(W2+W3))+((W4+W5)+(W6+W7)) — oracle/refdec.c b2o_dot_f32.
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
    // tensor parallelism (token kernel): output rows mirrored to the peers; row
    // ids of the argmax offset by row_base; each rank's best logit exchanged
    // through tp_cval / tp_cidx / tp_cnan / tp_aflag ([kMaxRanks] each, in the
    // rank's exchange buffer, mirrored like the outputs)
    Mirror mir;
    int row_base;
    int tp_rank, tp_size;
    const unsigned* tp_seq;    // token-kernel launches completed (the flags' epochs)
    int defer_tok;             // EPI_ARGMAX: a sampler kernel chooses the token (no step bookkeeping here)
    int i4;                    // int4 rows: two codes a byte (ld in bytes), gemv_i4_kernel
    float* tp_cval;
    int* tp_cidx;
    int* tp_cnan;
    unsigned* tp_aflag;
    // token kernel, (value, tag) words (nullptr: plain floats): tx the input vector
    // (read with tag checks), ty the output (y, or q for EPI_QKV), tresid the
    // residual, tkn / tvn this step's K and V rows [kv_heads * dh] (EPI_QKV)
    const unsigned long long* tx;
    unsigned long long* ty;
    const unsigned long long* tresid;
    unsigned long long* tkn;
    unsigned long long* tvn;
};

// ordering for greedy sampling: non-NaN beats NaN, larger wins, ties -> lower index
__device__ __forceinline__ bool amax_better(float va, int ia, float vb, int ib) {
    const bool na = va != va, nb = vb != vb;
    if (na != nb) return nb;                   // a wins iff b is NaN
    if (!na && va != vb) return va > vb;
    return ia < ib;
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

// rows [r0, r1) of CTA b of nb: balanced in units of `unit` rows (2 keeps RoPE pairs together)
__device__ __forceinline__ void cta_rows(int total, int unit, int b, int nb, int& r0, int& r1) {
    const long long units = (total + unit - 1) / unit;
    const long long u0 = (long long)b * units / nb;
    const long long u1 = (long long)(b + 1) * units / nb;
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

// The same exchange over integers (exact in any order: only the lane layout matters)
template <int N>
__device__ __forceinline__ void exchange_butterfly_i(int (&v)[N], int lane) {
    int cnt = N;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        if (cnt > 1) {
            const bool upper = (lane & s) != 0;
            const int h = cnt / 2;
#pragma unroll
            for (int i = 0; i < (N > 1 ? N / 2 : 1); ++i) {
                if (i < h) {
                    const int send = upper ? v[i] : v[h + i];
                    const int keep = upper ? v[h + i] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
                }
            }
            cnt = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], s);
        }
    }
}

// ---------------------------------------------------------------------------
// int8 rows: exact dot product on a fixed-point copy of x (oracle/refdec.c
// b2o_xfix / b2o_dot_i8x). With max|x| < 2^E, S = 31 - E and X_i = trunc(x_i 2^S)
// (|X_i| < 2^31), a row's dot is the exact integer D = sum_i w_i X_i rounded once,
// f32((double)D 2^-S). Integer sums are exact in any order, so the thread layout
// and the reduction tree do not change the bits. X is split into byte planes
// X = P0 + 2^8 P1 + 2^16 P2 + 2^24 P3 (P0..P2 unsigned, P3 signed); one dp4a
// takes four codes of a row against the same four elements of one plane. A
// plane sum of a row is at most 128 * 255 * n in magnitude, below 2^31 for rows
// of up to kXfixMaxN = 65536 codes (128 * 255 * 65536 = 2,139,095,040); longer
// rows would overflow the int32 sums, so every entry point refuses them.
// ---------------------------------------------------------------------------
constexpr int kXfixBad = -100000;                  // S when x holds a NaN or an infinity
constexpr int kXfixMaxN = 65536;

// S from the largest |x| bit pattern (non-negative floats order as their bits)
__device__ __forceinline__ int xfix_shift(uint32_t amax_bits) {
    if (amax_bits >= 0x7f800000u) return kXfixBad;
    if (amax_bits == 0u) return 0;
    const int e = (int)(amax_bits >> 23);
    const int E = e > 0 ? e - 126 : (32 - __clz((int)amax_bits)) - 149;   // frexp exponent
    return 31 - E;
}

__device__ __forceinline__ double pow2d(int k) { return __longlong_as_double((long long)(1023 + k) << 52); }

__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// trunc(x * 2^S) from the bits of x (integer operations only): x = man * 2^(e - 150)
// with the implicit bit in man (subnormals: e = 1, no implicit bit), so the
// magnitude is man shifted by k = e - 150 + S (k <= 7, as |x| 2^S < 2^31), and the
// shift right truncates toward zero like the conversion it replaces.
__device__ __forceinline__ uint32_t xfix_elem(float x, int S) {
    const uint32_t u = __float_as_uint(x);
    const int ex = (int)((u >> 23) & 0xffu);
    const uint32_t man = (u & 0x7fffffu) | (ex ? 0x800000u : 0u);
    const int k = (ex ? ex : 1) - 150 + S;
    const uint32_t mag = k >= 0 ? (man << k) : (k > -32 ? (man >> (-k)) : 0u);
    return (u >> 31) ? 0u - mag : mag;
}

// chunk swizzle of a block of planes in shared memory (xfix_smem)
__device__ __forceinline__ int xfix_swz(int b) { return (b >> 1) & 3; }

// four X values -> their four byte planes (element 0 in the low byte)
__device__ __forceinline__ void xfix_planes4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t (&pl)[4]) {
    const uint32_t lo01 = __byte_perm(x0, x1, 0x5140u), hi01 = __byte_perm(x0, x1, 0x7362u);
    const uint32_t lo23 = __byte_perm(x2, x3, 0x5140u), hi23 = __byte_perm(x2, x3, 0x7362u);
    pl[0] = __byte_perm(lo01, lo23, 0x5410u);
    pl[1] = __byte_perm(lo01, lo23, 0x7632u);
    pl[2] = __byte_perm(hi01, hi23, 0x5410u);
    pl[3] = __byte_perm(hi01, hi23, 0x7632u);
}

// Shared-memory x (L floats, L a multiple of 16) -> planes in place: block b's
// 16 words hold w[p * 4 + q] = byte p of elements 16b + 4q .. + 3, its four
// 16-byte chunks (plane p in chunk p) stored at chunk p ^ xfix_swz(b), so that
// eight threads reading consecutive blocks hit eight bank groups. A thread
// converts one group of 4 elements per pass (a warp covers 8 whole blocks, so
// every read of a block precedes its writes after __syncwarp). With S <= 127,
// x * 2^S is exact in f32 (|x| 2^S < 2^31; a product that underflows is below 1
// and truncates to 0 either way) and cvt.rzi gives trunc; otherwise the integer
// path. Every consumer thread calls it; it ends with the consumer barrier.
__device__ __forceinline__ void xfix_smem(float* xs, int L, int S, int tid) {
    const int nq = L / 4;
    const float p2 = S <= 127 ? __uint_as_float((uint32_t)(S + 127) << 23) : 0.0f;
    for (int q0 = tid - (tid & 31); q0 < nq; q0 += kGemvConsumerThreads) {
        const int qd = q0 + (tid & 31);
        uint32_t pl[4] = {0u, 0u, 0u, 0u};
        if (qd < nq && S != kXfixBad) {
            const float4 v = *reinterpret_cast<const float4*>(xs + 4 * qd);
            uint32_t X[4];
            if (S <= 127) {
                X[0] = (uint32_t)__float2int_rz(__fmul_rn(v.x, p2));
                X[1] = (uint32_t)__float2int_rz(__fmul_rn(v.y, p2));
                X[2] = (uint32_t)__float2int_rz(__fmul_rn(v.z, p2));
                X[3] = (uint32_t)__float2int_rz(__fmul_rn(v.w, p2));
            } else {
                X[0] = xfix_elem(v.x, S); X[1] = xfix_elem(v.y, S);
                X[2] = xfix_elem(v.z, S); X[3] = xfix_elem(v.w, S);
            }
            xfix_planes4(X[0], X[1], X[2], X[3], pl);
        }
        __syncwarp();
        if (qd < nq) {
            const int b = qd >> 2, f = xfix_swz(b);
            uint32_t* wb = reinterpret_cast<uint32_t*>(xs) + 16 * b + (qd & 3);
            wb[4 * (0 ^ f)] = pl[0]; wb[4 * (1 ^ f)] = pl[1]; wb[4 * (2 ^ f)] = pl[2]; wb[4 * (3 ^ f)] = pl[3];
        }
        __syncwarp();
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerThreads) : "memory");
}

// 16 consecutive elements of x -> their planes: w[p * 4 + q] holds byte p of
// elements 4q .. 4q + 3 (element 4q in the low byte)
__device__ __forceinline__ void xfix_block(const float (&x)[16], int S, uint32_t (&w)[16]) {
    if (S == kXfixBad) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0u;
        return;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t X[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            X[k] = S <= 127 ? (uint32_t)__float2int_rz(__fmul_rn(x[4 * q + k], __uint_as_float((uint32_t)(S + 127) << 23)))
                            : xfix_elem(x[4 * q + k], S);   // exact either way (see xfix_smem)
        const uint32_t lo01 = __byte_perm(X[0], X[1], 0x5140u), hi01 = __byte_perm(X[0], X[1], 0x7362u);
        const uint32_t lo23 = __byte_perm(X[2], X[3], 0x5140u), hi23 = __byte_perm(X[2], X[3], 0x7362u);
        w[0 * 4 + q] = __byte_perm(lo01, lo23, 0x5410u);
        w[1 * 4 + q] = __byte_perm(lo01, lo23, 0x7632u);
        w[2 * 4 + q] = __byte_perm(hi01, hi23, 0x5410u);
        w[3 * 4 + q] = __byte_perm(hi01, hi23, 0x7632u);
    }
}

// c + sum of 4 signed codes (a) times 4 unsigned / signed plane bytes (b)
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// the exact dot D from its four plane sums
__device__ __forceinline__ long long xfix_dot(int p0, int p1, int p2, int p3) {
    return (long long)p0 + (long long)p1 * 256ll + (long long)p2 * 65536ll + (long long)p3 * 16777216ll;
}
// one row's value from its exact dot: f32(D 2^-S), one rounding
__device__ __forceinline__ float xfix_value(long long D, int S) {
    if (S == kXfixBad) return __uint_as_float(0x7fc00000u);
    return __double2float_rn(__dmul_rn(__ll2double_rn(D), pow2d(-S)));
}
// one row's value from its four plane sums
__device__ __forceinline__ float xfix_row(const int* pl, int S) {
    return xfix_value(xfix_dot(pl[0], pl[1], pl[2], pl[3]), S);
}

// Block-wide S: every consumer thread passes the largest |x| bits it has seen;
// amx (shared, zero on entry) collects them. Ends with the consumer barrier.
__device__ __forceinline__ int xfix_shift_cta(uint32_t local, unsigned* amx) {
    local = __reduce_max_sync(0xffffffffu, local);
    if ((threadIdx.x & 31) == 0) atomicMax(amx, local);
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerThreads) : "memory");
    return xfix_shift(*(volatile unsigned*)amx);
}

// One int8 stage: nr (<= RS) rows of each of the NM matrices at `stage` (the
// second matrix starts RS rows in), x as planes in registers (KB 16-byte blocks a
// thread: s, s + 256, ...). Each row's four plane sums are added into
// part[((row * NM + m) * 4 + plane] (shared, zeroed before the first stage) for
// rows rl0 .. rl0 + nr - 1 of the CTA. Rows are reduced eight at a time.
template <int KB, int RS, int NM>
__device__ __forceinline__ void gemv_stage_i8(const unsigned char* stage, uint32_t row_bytes, int nblk, int slotid,
                                              int lane, const uint32_t (&xp)[KB][16], int* part, int rl0, int nr) {
    constexpr int NR = RS * NM;
    constexpr int NH = NR < 8 ? NR : 8;
    constexpr int NV = NH * 4;
    constexpr int LG = Log2<NV>::v;
#pragma unroll
    for (int h0 = 0; h0 < NR; h0 += NH) {
        int acc[NH][4];
#pragma unroll
        for (int r = 0; r < NH; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[r][q] = 0;
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int b = slotid + 256 * k;
            if (b < nblk) {
#pragma unroll
                for (int r = 0; r < NH; ++r) {
                    // rows past nr read stale (in-bounds) stage bytes; never stored
                    const uint4 w = lds128(stage + (size_t)(h0 + r) * row_bytes + 16 * b);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[r][0] = dp4a_su(ww[q], xp[k][0 * 4 + q], acc[r][0]);
                        acc[r][1] = dp4a_su(ww[q], xp[k][1 * 4 + q], acc[r][1]);
                        acc[r][2] = dp4a_su(ww[q], xp[k][2 * 4 + q], acc[r][2]);
                        acc[r][3] = dp4a_ss(ww[q], xp[k][3 * 4 + q], acc[r][3]);
                    }
                }
            }
        }
        int v[NV];
#pragma unroll
        for (int r = 0; r < NH; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) v[r * 4 + q] = acc[r][q];
        exchange_butterfly_i<NV>(v, lane);
        if ((lane & ((32 >> LG) - 1)) == 0) {
            const int vi = lane >> (5 - LG);
            const int rr = h0 + vi / 4, pl = vi % 4;       // stage row (m * RS + r), plane
            const int m = rr / RS, r = rr % RS;
            if (r < nr) atomicAdd(part + ((rl0 + r) * NM + m) * 4 + pl, v[0]);
        }
    }
}

// A thread's planes from the f32 slice gemv_load_x left in registers
template <int KMAX>
__device__ __forceinline__ void xfix_from_slice(const float2 (&xr)[KMAX][8], int S, uint32_t (&xp)[KMAX][16]) {
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        float t[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) { t[2 * i] = xr[k][i].x; t[2 * i + 1] = xr[k][i].y; }
        xfix_block(t, S, xp[k]);
    }
}


// ============================================================================
// Building blocks shared by the per-launch kernel below and the persistent
// token kernel (token.cuh): the same code, so both give identical bits.
// ============================================================================

template <typename WT> struct GemvElems { static constexpr int EPB = 16 / (int)sizeof(WT); };

// EPB consecutive floats from v[i0 ..] (zeros past n), as 16-byte vector loads
// when allowed; cg: through L2 (values written by other CTAs of the same kernel)
template <int EPB>
__device__ __forceinline__ void load_slice(const float* v, int i0, int n, bool vec, bool cg, float (&out)[EPB]) {
    if (vec) {
#pragma unroll
        for (int q = 0; q < EPB / 4; ++q) {
            const int i = i0 + 4 * q;
            float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < n)
                t = cg ? __ldcg(reinterpret_cast<const float4*>(v + i)) : __ldg(reinterpret_cast<const float4*>(v + i));
            out[4 * q] = t.x; out[4 * q + 1] = t.y; out[4 * q + 2] = t.z; out[4 * q + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int t = 0; t < EPB; ++t) {
            const int i = i0 + t;
            out[t] = i < n ? (cg ? __ldcg(v + i) : __ldg(v + i)) : 0.0f;
        }
    }
}

// Consumer prologue: this thread's slice of x (blocks slot, slot+256, ...), after
// RMSNorm / LayerNorm when p.norm asks for it. Every consumer thread calls it (the
// norm's reduction uses the consumer barrier). x was written by other CTAs of the
// same token kernel, so it is read through L2 (ld.global.cg). With one block per
// row, the slice and its norm gains are requested before the norm's own strided
// values, so the prologue costs about one L2 round trip.
template <typename WT, int KMAX, bool EARLY = (KMAX == 1)>
__device__ __forceinline__ void gemv_load_x(const GemvParams& p, float2 (&xr)[KMAX][GemvElems<WT>::EPB / 2],
                                            float* red, int tid) {
    constexpr int EPB = GemvElems<WT>::EPB;
    const int n = p.n;
    const float* x = p.x;
    const int slotid = tid % 256;
    const int nblk = (int)(((size_t)p.ld * sizeof(WT)) >> 4);
    const int K = (nblk + 255) / 256;
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const bool vec = (n % 4) == 0 && al16(x) && (!p.ng || al16(p.ng)) && (!p.nb || al16(p.nb));
    // 1. the slice (raw, into xr) and the norm gains of its first block; EARLY
    // requests them before the norm's loads (one round trip), otherwise after it
    // (fewer registers live during the norm)
    float gs[EPB], bs[EPB];
    auto load_raw = [&]() {
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            const int b = slotid + 256 * k;
            float t4[EPB];
            if (k < K && b < nblk) load_slice<EPB>(x, b * EPB, n, vec, true, t4);
            else {
#pragma unroll
                for (int t = 0; t < EPB; ++t) t4[t] = 0.0f;
            }
#pragma unroll
            for (int t = 0; t < EPB / 2; ++t) xr[k][t] = make_float2(t4[2 * t], t4[2 * t + 1]);
        }
        const bool have = K >= 1 && slotid < nblk;
        if (p.norm != NORM_NONE && have) load_slice<EPB>(p.ng, slotid * EPB, n, vec, false, gs);
        if (p.norm == NORM_LN && have) load_slice<EPB>(p.nb, slotid * EPB, n, vec, false, bs);
    };
    if constexpr (EARLY) load_raw();
    // 2. the norm: 256 partials (thread t: elements t, t + 256, ... in order)
    constexpr int NB = KMAX == 1 ? 16 : 4;           // loads in flight per batch (registers)
    float scale_a = 1.0f, shift_m = 0.0f;
    auto partial = [&](int kind, float mean) {       // 0: sum x^2, 1: sum x, 2: sum (x-mean)^2
        float a = 0.0f;
        if (tid < 256) {
            for (int base = tid; base < n; base += 256 * NB) {
                float v[NB];
#pragma unroll
                for (int u = 0; u < NB; ++u) { const int i = base + 256 * u; v[u] = i < n ? __ldcg(x + i) : 0.0f; }
#pragma unroll
                for (int u = 0; u < NB; ++u) {
                    if (base + 256 * u >= n) continue;
                    if (kind == 0) a = ffma(v[u], v[u], a);
                    else if (kind == 1) a = fadd(a, v[u]);
                    else { const float dx = fsub(v[u], mean); a = ffma(dx, dx, a); }
                }
            }
        }
        return a;
    };
    if (p.norm == NORM_RMS) {
        const float tot = consumer_reduce256(partial(0, 0.0f), red, tid);
        const float ms = fdiv(tot, (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(ms, p.eps)));
    } else if (p.norm == NORM_LN) {
        shift_m = fdiv(consumer_reduce256(partial(1, 0.0f), red, tid), (float)n);
        const float var = fdiv(consumer_reduce256(partial(2, shift_m), red, tid), (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(var, p.eps)));
    }
    if constexpr (!EARLY) load_raw();
    // 3. normalise the slice
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        const int b = slotid + 256 * k;
#pragma unroll
        for (int t = 0; t < EPB; ++t) {
            const int i = b * EPB + t;
            float v = 0.0f;
            if (k < K && b < nblk && i < n) {
                const float xv = (t & 1) ? xr[k][t / 2].y : xr[k][t / 2].x;
                float g = 0.0f, bb = 0.0f;
                if (p.norm != NORM_NONE) {
                    if (k == 0) { g = gs[t]; bb = bs[t]; }
                    else { g = p.ng[i]; if (p.norm == NORM_LN) bb = p.nb[i]; }
                }
                if (p.norm == NORM_RMS) v = fmul(fmul(xv, scale_a), g);
                else if (p.norm == NORM_LN)
                    v = (float)dadd(dmul((double)fmul(fsub(xv, shift_m), scale_a), (double)g), (double)bb);
                else v = xv;
            }
            if (t & 1) xr[k][t / 2].y = v;
            else xr[k][t / 2].x = v;
        }
    }
}

// ---------------------------------------------------------------------------
// x in shared memory (token kernel): the vector is staged once per CTA and phase
// at xs[0 .. L) (zeros past n, L = n rounded up to 16), its norm gains at gs[],
// bs[]. The prologue normalises it in place; the stages read one 16-byte block
// of x per row group from shared memory instead of holding the slice in
// registers. Same operations, in the same order, as gemv_load_x + the stages.
// ---------------------------------------------------------------------------
// Returns the largest |x| bit pattern among the values this thread normalised
// (or, without a norm, read): the int8 rows' fixed-point shift needs the CTA max.
__device__ __forceinline__ uint32_t gemv_norm_smem(const GemvParams& p, float* xs, const float* gs, const float* bs,
                                                   float* red, int tid) {
    const int n = p.n;
    uint32_t am = 0u;
    if (p.norm == NORM_NONE) {
        for (int i = tid; i < n; i += kGemvConsumerThreads) am = max(am, abs_bits(xs[i]));
        return am;
    }
    float scale_a = 1.0f, shift_m = 0.0f;
    if (p.norm == NORM_RMS) {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float v = xs[i]; a = ffma(v, v, a); }
        const float tot = consumer_reduce256(a, red, tid);
        const float ms = fdiv(tot, (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(ms, p.eps)));
    } else {
        float a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) a = fadd(a, xs[i]);
        shift_m = fdiv(consumer_reduce256(a, red, tid), (float)n);
        a = 0.0f;
        if (tid < 256)
            for (int i = tid; i < n; i += 256) { const float dx = fsub(xs[i], shift_m); a = ffma(dx, dx, a); }
        const float var = fdiv(consumer_reduce256(a, red, tid), (float)n);
        scale_a = fdiv(1.0f, __fsqrt_rn(fadd(var, p.eps)));
    }
    // every raw value has been read (the reduction's barriers); normalise in place
    for (int i = tid; i < n; i += kGemvConsumerThreads) {
        const float xv = xs[i];
        const float v = p.norm == NORM_RMS
                            ? fmul(fmul(xv, scale_a), gs[i])
                            : (float)dadd(dmul((double)fmul(fsub(xv, shift_m), scale_a), (double)gs[i]), (double)bs[i]);
        xs[i] = v;
        am = max(am, abs_bits(v));
    }
    return am;
}

// Compile-time shaped stage with x read from shared memory: RS rows per matrix,
// NM matrices, all NR = RS * NM rows reduced by one exchange butterfly; KB = most
// 16-byte blocks a thread owns in a row (the block loop is unrolled).
template <typename WT, int RS, int NM, int KB>
__device__ __forceinline__ void gemv_consume_stage_xt(const unsigned char* stage, uint32_t row_bytes, int nblk,
                                                      int slotid, int lane, int gwarp, const float* xs,
                                                      float* part, int rl0, int nr) {
    static_assert(sizeof(WT) == 4, "f32 rows (int8 rows: gemv_stage_i8)");
    constexpr int EPB = GemvElems<WT>::EPB;
    constexpr int NR = RS * NM;
    constexpr int LG = Log2<NR>::v;
    float2 a01[NR], a23[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) a01[r] = a23[r] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < KB; ++k) {
        const int b = slotid + 256 * k;
        if (b >= nblk) break;
        float2 xb[EPB / 2];
#pragma unroll
        for (int q = 0; q < EPB / 4; ++q) {
            const float4 x4 = lds128f(xs + b * EPB + 4 * q);
            xb[2 * q] = make_float2(x4.x, x4.y);
            xb[2 * q + 1] = make_float2(x4.z, x4.w);
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            // rows past nr read stale (in-bounds) stage bytes; never stored
            const unsigned char* row = stage + (size_t)r * row_bytes + 16 * b;
            const float4 w = lds128f(row);
            a01[r] = __ffma2_rn(make_float2(w.x, w.y), xb[0], a01[r]);
            a23[r] = __ffma2_rn(make_float2(w.z, w.w), xb[1], a23[r]);
        }
    }
    float v[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) v[r] = fadd(fadd(a01[r].x, a01[r].y), fadd(a23[r].x, a23[r].y));
    exchange_butterfly<NR>(v, lane);
    if ((lane & ((32 >> LG) - 1)) == 0) {
        const int rr = lane >> (5 - LG);
        const int m = rr / RS, r = rr % RS;
        if (r < nr) part[((rl0 + r) * NM + m) * 8 + gwarp] = v[0];
    }
}

// One stage: nr (<= RS) rows of each of the NM matrices at `stage` (row stride
// row_bytes; the second matrix starts RS rows in). Writes this warp's sums to
// part[(row * NM + m) * 8 + gwarp] for rows rl0 .. rl0 + nr - 1 of the CTA. Rows
// are reduced four at a time (each row's butterfly is the same either way).
template <typename WT, int KMAX, int RS, bool PAIRED>
__device__ __forceinline__ void gemv_consume_stage(const unsigned char* stage, uint32_t row_bytes, int nblk,
                                                   int slotid, int lane, int gwarp,
                                                   const float2 (&xr)[KMAX][GemvElems<WT>::EPB / 2],
                                                   float* part, int rl0, int nr) {
    static_assert(sizeof(WT) == 4, "f32 rows (int8 rows: gemv_stage_i8)");
    constexpr int NM = PAIRED ? 2 : 1;
    constexpr int NR = RS * NM;
    constexpr int NH = NR < 4 ? NR : 4;
    constexpr int LG = Log2<NH>::v;
    const int K = (nblk + 255) / 256;
#pragma unroll
    for (int h0 = 0; h0 < NR; h0 += NH) {
        float2 a01[NH], a23[NH];
#pragma unroll
        for (int r = 0; r < NH; ++r) a01[r] = a23[r] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            const int b = slotid + 256 * k;
            if (k < K && b < nblk) {
#pragma unroll
                for (int r = 0; r < NH; ++r) {
                    // rows past nr read stale (in-bounds) stage bytes; never stored
                    const unsigned char* row = stage + (size_t)(h0 + r) * row_bytes + 16 * b;
                    const float4 w = lds128f(row);
                    a01[r] = __ffma2_rn(make_float2(w.x, w.y), xr[k][0], a01[r]);
                    a23[r] = __ffma2_rn(make_float2(w.z, w.w), xr[k][1], a23[r]);
                }
            }
        }
        float v[NH];
#pragma unroll
        for (int r = 0; r < NH; ++r) v[r] = fadd(fadd(a01[r].x, a01[r].y), fadd(a23[r].x, a23[r].y));
        exchange_butterfly<NH>(v, lane);
        if ((lane & ((32 >> LG) - 1)) == 0) {
            const int rr = h0 + (lane >> (5 - LG));        // stage row (m * RS + r)
            const int m = rr / RS, r = rr % RS;
            if (r < nr) part[((rl0 + r) * NM + m) * 8 + gwarp] = v[0];
        }
    }
}

// Producer: issue the stages of rows [r0, r1) into the ring, one bulk copy per
// matrix per stage; j is the running stage index (slot j % NS, round j / NS).
// With inflight > 0 (< NS), at most that many copies are outstanding: stage
// j - inflight is complete before stage j is issued, which keeps the memory
// queues short for everyone else's loads. Returns false on a timed-out wait.
template <int NM>
__device__ __forceinline__ bool gemv_produce(const GemvParams& p, int r0, int r1, int RS, uint32_t row_bytes,
                                             unsigned char* ring, uint32_t slot_stride, int NS,
                                             uint64_t* full, uint64_t* empty, int& j, int inflight = 0,
                                             int rows = 0) {
    const int R = rows > 0 ? rows : RS;          // rows per stage (<= RS, the paired matrix offset)
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, R);
        const int slot = j % NS, round = j / NS;
        if (round > 0 && !mbar_wait_bounded(&empty[slot], (uint32_t)((round - 1) & 1))) return false;
        if (inflight > 0 && j >= inflight &&
            !mbar_wait_bounded(&full[(j - inflight) % NS], (uint32_t)(((j - inflight) / NS) & 1)))
            return false;
        const uint32_t bytes = (uint32_t)sr.nr * row_bytes;
        unsigned char* dst = ring + (size_t)slot * slot_stride;
        mbar_arrive_expect_tx(&full[slot], bytes * NM);
        bulk_g2s(dst, reinterpret_cast<const unsigned char*>(p.W[sr.seg]) + (size_t)sr.local * row_bytes, bytes,
                 &full[slot]);
        if constexpr (NM == 2)
            bulk_g2s(dst + (size_t)RS * row_bytes,
                     reinterpret_cast<const unsigned char*>(p.W[1]) + (size_t)sr.local * row_bytes, bytes,
                     &full[slot]);
        ++j;
        cur += sr.nr;
    }
    return true;
}

// Consumers: walk the same stages; group g takes stage j when (j % NS) % 2 == g
// (NS even, so every slot belongs to one group and its phases advance in order).
// compute = false only releases the slots. Returns false on a timed-out wait.
template <typename WT, int KMAX, int RS, bool PAIRED>
__device__ __forceinline__ bool gemv_consume(const GemvParams& p, int r0, int r1, const unsigned char* ring,
                                             uint32_t slot_stride, int NS, uint64_t* full, uint64_t* empty,
                                             int& j, int group, int gwarp, int lane, int slotid,
                                             const float2 (&xr)[KMAX][GemvElems<WT>::EPB / 2], float* part,
                                             bool compute, int rows = RS) {
    const uint32_t row_bytes = (uint32_t)p.ld * (uint32_t)sizeof(WT);
    const int nblk = (int)(row_bytes >> 4);
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, rows);
        const int slot = j % NS;
        if ((slot & 1) == group) {
            if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / NS) & 1))) return false;
            if (compute)
                gemv_consume_stage<WT, KMAX, RS, PAIRED>(ring + (size_t)slot * slot_stride, row_bytes, nblk, slotid,
                                                         lane, gwarp, xr, part, cur - r0, sr.nr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        ++j;
        cur += sr.nr;
    }
    return true;
}

// The same walk for int8 rows (x as planes, plane sums into part[] as int32)
template <int KMAX, int RS, int NM>
__device__ __forceinline__ bool gemv_consume_i8(const GemvParams& p, int r0, int r1, const unsigned char* ring,
                                                uint32_t slot_stride, int NS, uint64_t* full, uint64_t* empty,
                                                int& j, int group, int lane, int slotid,
                                                const uint32_t (&xp)[KMAX][16], int* part, bool compute) {
    const uint32_t row_bytes = (uint32_t)p.ld;
    const int nblk = (int)(row_bytes >> 4);
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, RS);
        const int slot = j % NS;
        if ((slot & 1) == group) {
            if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / NS) & 1))) return false;
            if (compute)
                gemv_stage_i8<KMAX, RS, NM>(ring + (size_t)slot * slot_stride, row_bytes, nblk, slotid, lane, xp, part,
                                            cur - r0, sr.nr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        ++j;
        cur += sr.nr;
    }
    return true;
}

// Per-row epilogue inputs for rows r0 .. r0 + 511 of the CTA, loaded during the
// prologue (their latency overlaps the x loads) and parked in shared memory as
// epi[rl * 4 + k]: k = 0 scale (gate scale when paired), 1 bias (up scale when
// paired), 2 RoPE cos or residual, 3 RoPE sin.
struct EpiRow { float v[4]; };

template <int ESZ, bool PAIRED>
__device__ __forceinline__ EpiRow gemv_epi_load(const GemvParams& p, int r0, int r1, int pos, int tid) {
    EpiRow e{{1.0f, 0.0f, 0.0f, 0.0f}};
    if (tid >= r1 - r0) return e;
    const int lrow = r0 + tid;
    if constexpr (PAIRED) {
        e.v[0] = p.S[0][lrow];
        e.v[1] = p.S[1][lrow];
    } else {
        int seg, row;
        seg_of(p, lrow, seg, row);
        if constexpr (ESZ == 1) e.v[0] = p.S[seg][row];
        if (p.bias[seg]) e.v[1] = p.bias[seg][row];
        if (p.epi == EPI_QKV && p.rope && seg < 2 && !(row & 1)) {
            const float* tr = p.rope_tab + (size_t)pos * p.dh + row % p.dh;
            e.v[2] = tr[0];
            e.v[3] = tr[1];
        } else if (p.epi == EPI_RESID) {
            e.v[2] = p.tresid ? tag_val(ld_tag(p.tresid + row)) : __ldcg(p.resid + row);
        }
    }
    return e;
}

__device__ __forceinline__ void gemv_epi_store(const EpiRow& e, int nrows, int tid, float* epi) {
    if (tid < nrows) *reinterpret_cast<float4*>(epi + tid * 4) = make_float4(e.v[0], e.v[1], e.v[2], e.v[3]);
}

// Epilogue: one consumer thread per row (per row pair with RoPE) finishes the rows
// [r0, r1) from the warp sums in part[]. CTA `cta` of `ncta` takes part in the
// grid-wide argmax (EPI_ARGMAX) through amax_* and the last-CTA ticket. epi, when
// given, holds the preloaded per-row inputs of the first 512 rows.
// otag: the tag written with each output when the outputs are (value, tag) words
template <int ESZ, bool PAIRED>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, int r0, int r1, const float* part, int pos,
                                              int tid, int cta, int ncta, const float* epi = nullptr, int S = 0,
                                              unsigned otag = 0u) {
    // int8: part holds int32 plane sums [row][NM][4]; f32: warp sums [row][NM][8]
    const int* parti = reinterpret_cast<const int*>(part);
    auto dotv = [&](int rl, int m) {
        if constexpr (ESZ == 1) return xfix_row(parti + (rl * (PAIRED ? 2 : 1) + m) * 4, S);
        else return tree8(part + (rl * (PAIRED ? 2 : 1) + m) * 8);
    };
    const int warp = tid >> 5, lane = tid & 31;
    auto pre = [&](int rl) { return epi && rl < kGemvConsumerThreads; };
    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    bool have_best = false;
    const int nrows = r1 - r0;
    const int step = p.rope ? 2 : 1;
    for (int rl = tid * step; rl < nrows; rl += kGemvConsumerThreads * step) {
        const int lrow = r0 + rl;
        if constexpr (PAIRED) {                              // EPI_SWIGLU
            const float sg = pre(rl) ? epi[rl * 4] : p.S[0][lrow];
            const float su = pre(rl) ? epi[rl * 4 + 1] : p.S[1][lrow];
            const float g = fmul(dotv(rl, 0), sg);
            const float u = fmul(dotv(rl, 1), su);
            if (p.ty) mirror_st_tag(p.mir, p.ty + lrow, fmul(silu_f(g), u), otag);
            else mirror_store(p.mir, p.y + lrow, fmul(silu_f(g), u));
            continue;
        }
        int seg, row;
        seg_of(p, lrow, seg, row);
        float val[2] = {0.0f, 0.0f};
        for (int e = 0; e < step; ++e) {
            float v = dotv(rl + e, 0);
            if constexpr (ESZ == 1) v = fmul(v, pre(rl + e) ? epi[(rl + e) * 4] : p.S[seg][row + e]);
            if (p.bias[seg]) v = fadd(v, pre(rl + e) ? epi[(rl + e) * 4 + 1] : p.bias[seg][row + e]);
            else if constexpr (ESZ == 4) v = fadd(v, 0.0f);
            val[e] = v;
        }
        if (p.epi == EPI_QKV) {
            float out[2] = {val[0], val[1]};
            if (p.rope && seg < 2) {
                // pair (2i, 2i+1): rows start even and segment sizes are even
                const int hd = row % p.dh;
                const float* tr = p.rope_tab + (size_t)pos * p.dh + hd;
                const float c = pre(rl) ? epi[rl * 4 + 2] : tr[0];
                const float sn = pre(rl) ? epi[rl * 4 + 3] : tr[1];
                out[0] = fsub(fmul(val[0], c), fmul(val[1], sn));
                out[1] = fadd(fmul(val[0], sn), fmul(val[1], c));
            }
            for (int e = 0; e < step; ++e) {
                const int rr = row + e;
                if (seg == 0) {
                    if (p.ty) st_tag(p.ty + rr, fmul(out[e], p.qscale), otag);
                    else p.qout[rr] = fmul(out[e], p.qscale);
                } else if (pos < p.max_seq) {
                    const int kvh = rr / p.dh, hd = rr % p.dh;
                    float* cache = seg == 1 ? p.kcache : p.vcache;
                    cache[((size_t)kvh * p.max_seq + pos) * p.dh + hd] = out[e];
                    if (p.tkn) st_tag((seg == 1 ? p.tkn : p.tvn) + rr, out[e], otag);
                } else {
                    set_err(p.err, B2_DEV_ERR_KV_OVERFLOW);
                }
            }
        } else if (p.epi == EPI_RESID) {
            const float r = pre(rl) ? epi[rl * 4 + 2]
                                    : (p.tresid ? tag_val(ld_tag(p.tresid + row)) : __ldcg(p.resid + row));
            if (p.ty) mirror_st_tag(p.mir, p.ty + row, fadd(val[0], r), otag);
            else mirror_store(p.mir, p.y + row, fadd(val[0], r));
        } else if (p.epi == EPI_GELU) {
            if (p.ty) mirror_st_tag(p.mir, p.ty + row, gelu_f(val[0]), otag);
            else mirror_store(p.mir, p.y + row, gelu_f(val[0]));
        } else if (p.epi == EPI_ARGMAX) {
            if (p.y) p.y[row] = val[0];
            if (row + p.row_base == 0 && p.amax_v0nan) *p.amax_v0nan = (val[0] != val[0]) ? 1 : 0;
            if (!have_best || amax_better(val[0], row + p.row_base, best_v, best_i)) {
                best_v = val[0]; best_i = row + p.row_base; have_best = true;
            }
        } else {
            if (p.ty) mirror_st_tag(p.mir, p.ty + row, val[0], otag);
            else mirror_store(p.mir, p.y + row, val[0]);
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
            p.amax_val[cta] = cv;
            p.amax_idx[cta] = ch ? ci : 0x7fffffff;
            __threadfence();
            const unsigned t = atomicAdd(p.amax_count, 1u);
            last = (t == (unsigned)ncta - 1);
        }
        consumer_bar();
        if (last && tid == 0) {
            __threadfence();
            float cv = 0.0f; int ci = 0x7fffffff; bool ch = false;
            for (int c = 0; c < ncta; ++c) {
                const int ii = __ldcg(p.amax_idx + c);
                const float vv = __ldcg(p.amax_val + c);
                if (ii != 0x7fffffff && (!ch || amax_better(vv, ii, cv, ci))) { cv = vv; ci = ii; ch = true; }
            }
            int tok = ch ? ci : 0;
            bool v0nan = p.amax_v0nan && __ldcg(p.amax_v0nan);
            if (p.tp_size > 1) {
                // every rank's best, slot tp_rank on every rank, then the flags; the
                // comparator is a total order, so all ranks reach the same token
                const int r = p.tp_rank;
                mirror_store(p.mir, p.tp_cval + r, cv);
                mirror_store(p.mir, p.tp_cidx + r, ch ? ci : 0x7fffffff);
                mirror_store(p.mir, p.tp_cnan + r, (r == 0 && v0nan) ? 1 : 0);
                const unsigned e = *(volatile const unsigned*)p.tp_seq + 1u;
                if (!tp_flag_exchange(p.tp_aflag, r, p.tp_size, p.mir, e)) set_err(p.err, B2_DEV_ERR_TIMEOUT);
                ch = false;
                for (int q = 0; q < p.tp_size; ++q) {
                    const int ii = *(volatile int*)(p.tp_cidx + q);
                    const float vv = *(volatile float*)(p.tp_cval + q);
                    if (ii != 0x7fffffff && (!ch || amax_better(vv, ii, cv, ci))) { cv = vv; ci = ii; ch = true; }
                }
                tok = ch ? ci : 0;
                v0nan = *(volatile int*)(p.tp_cnan) != 0;
            }
            if (v0nan) tok = 0;                                    // sequential scan keeps index 0
            if (p.out_tok) *p.out_tok = tok;
            if (p.st && !p.defer_tok) {
                StepState* st = p.st;
                st->next_tok = tok;
                if (pos >= st->prompt_len - 1) {
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

// ============================================================================
// Per-launch GEMV kernel (one kernel per projection; kernel-level C ABI and the
// per-layer decode path).
// ============================================================================
template <typename WT, int KMAX, int RS, bool PAIRED>
__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_kernel(const __grid_constant__ GemvParams p) {
    constexpr int ESZ = (int)sizeof(WT);
    constexpr int NM = PAIRED ? 2 : 1;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxStages;
    float* red = reinterpret_cast<float*>(empty + kGemvMaxStages);      // 8 floats
    float* part = reinterpret_cast<float*>(smem + 1024);                 // [rows_cta][NM][8] (f32) / [4] (int8)
    unsigned* amx = reinterpret_cast<unsigned*>(red + 8);                // int8: largest |x| bits
    const uint32_t row_bytes = (uint32_t)p.ld * ESZ;
    const uint32_t stage_bytes = (uint32_t)RS * row_bytes * NM;
    unsigned char* ring = smem + p.ring_offset;
    const int NS = p.nstages;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    int r0, r1;
    cta_rows(total_rows(p), p.rope ? 2 : 1, blockIdx.x, gridDim.x, r0, r1);

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
        *amx = 0u;
    }
    if constexpr (ESZ == 1)                                              // plane sums start at 0
        for (int i = tid; i < (r1 - r0) * NM * 4; i += kGemvThreads) reinterpret_cast<int*>(part)[i] = 0;
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemvConsumerWarps) {
        // producer: its copies start before griddepcontrol.wait (weights do not
        // depend on the previous kernel)
        if (lane == 0) {
            int j = 0;
            if (!gemv_produce<NM>(p, r0, r1, RS, row_bytes, ring, stage_bytes, NS, full, empty, j))
                set_err(p.err, B2_DEV_ERR_TIMEOUT);
            // drain: no copy may still be in flight when the CTA exits
            for (int i = max(0, j - NS); i < j; ++i)
                if (!mbar_wait_bounded(&full[i % NS], (uint32_t)((i / NS) & 1))) {
                    set_err(p.err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }

    const int group = warp / kGemvGroupWarps;
    const int gwarp = warp % kGemvGroupWarps;
    pdl_wait();
    const bool active = p.st ? (*(volatile int*)&p.st->active != 0) : true;
    const int pos = p.st ? *(volatile int*)&p.st->pos : p.pos_fixed;

    float2 xr[KMAX][GemvElems<WT>::EPB / 2];
    gemv_load_x<WT, KMAX>(p, xr, red, tid);
    int j = 0;
    int S = 0;
    bool ok;
    if constexpr (ESZ == 1) {
        uint32_t am = 0u;                       // the 256 slices cover x (threads s and s + 256 share one)
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
#pragma unroll
            for (int t = 0; t < 8; ++t) am = max(am, max(abs_bits(xr[k][t].x), abs_bits(xr[k][t].y)));
        S = xfix_shift_cta(am, amx);
        uint32_t xp[KMAX][16];
        xfix_from_slice<KMAX>(xr, S, xp);
        ok = gemv_consume_i8<KMAX, RS, NM>(p, r0, r1, ring, stage_bytes, NS, full, empty, j, group, lane, tid % 256,
                                           xp, reinterpret_cast<int*>(part), active);
    } else {
        ok = gemv_consume<WT, KMAX, RS, PAIRED>(p, r0, r1, ring, stage_bytes, NS, full, empty, j, group, gwarp, lane,
                                                tid % 256, xr, part, active);
    }
    if (!ok) set_err(p.err, B2_DEV_ERR_TIMEOUT);
    consumer_bar();
    if (!active) return;
    gemv_epilogue<ESZ, PAIRED>(p, r0, r1, part, pos, tid, blockIdx.x, gridDim.x, nullptr, S);
}

// ============================================================================
// int4 rows (the reference's --int4-linear / --int4-embedding format: two codes a
// byte, the even column in the low nibble; arr_i4_matvec_f32_perrow unpacks them
// to int8 and runs the int8 dot, aricode_pack.py:168-181). The same exact
// fixed-point dot as the int8 rows over the unpacked codes, so the results are
// the int8 kernel's for those codes; the stages stream the packed rows (half the
// bytes). Thread s owns the 16-byte packed blocks s, s + 256, ... = 32 codes
// each, against the planes of 32 elements of x.
// ============================================================================
struct I4Tag { unsigned char b; };
template <> struct GemvElems<I4Tag> { static constexpr int EPB = 32; };

// 8 codes (one 32-bit packed word) -> two int8x4 words, elements 0-3 and 4-7
__device__ __forceinline__ void i4_unpack8(uint32_t w, uint32_t& a, uint32_t& b) {
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    a = __vsub4(__byte_perm(lo, hi, 0x5140u) ^ 0x08080808u, 0x08080808u);   // sign-extended nibbles
    b = __vsub4(__byte_perm(lo, hi, 0x7362u) ^ 0x08080808u, 0x08080808u);
}

template <int KB, int RS>
__device__ __forceinline__ void gemv_stage_i4(const unsigned char* stage, uint32_t row_bytes, int nblk, int slotid,
                                              int lane, const uint32_t (&xp)[KB][32], int* part, int rl0, int nr) {
    constexpr int NH = RS < 8 ? RS : 8;
    constexpr int NV = NH * 4;
    constexpr int LG = Log2<NV>::v;
#pragma unroll
    for (int h0 = 0; h0 < RS; h0 += NH) {
        int acc[NH][4];
#pragma unroll
        for (int r = 0; r < NH; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[r][q] = 0;
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int b = slotid + 256 * k;
            if (b < nblk) {
#pragma unroll
                for (int r = 0; r < NH; ++r) {
                    // rows past nr read stale (in-bounds) stage bytes; never stored
                    const uint4 w = lds128(stage + (size_t)(h0 + r) * row_bytes + 16 * b);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t c0, c1;                     // elements 8q .. 8q + 3, 8q + 4 .. 8q + 7
                        i4_unpack8(ww[q], c0, c1);
                        const int g0 = 2 * q, g1 = 2 * q + 1;
                        acc[r][0] = dp4a_su(c0, xp[k][0 * 8 + g0], acc[r][0]);
                        acc[r][1] = dp4a_su(c0, xp[k][1 * 8 + g0], acc[r][1]);
                        acc[r][2] = dp4a_su(c0, xp[k][2 * 8 + g0], acc[r][2]);
                        acc[r][3] = dp4a_ss(c0, xp[k][3 * 8 + g0], acc[r][3]);
                        acc[r][0] = dp4a_su(c1, xp[k][0 * 8 + g1], acc[r][0]);
                        acc[r][1] = dp4a_su(c1, xp[k][1 * 8 + g1], acc[r][1]);
                        acc[r][2] = dp4a_su(c1, xp[k][2 * 8 + g1], acc[r][2]);
                        acc[r][3] = dp4a_ss(c1, xp[k][3 * 8 + g1], acc[r][3]);
                    }
                }
            }
        }
        int v[NV];
#pragma unroll
        for (int r = 0; r < NH; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) v[r * 4 + q] = acc[r][q];
        exchange_butterfly_i<NV>(v, lane);
        if ((lane & ((32 >> LG) - 1)) == 0) {
            const int vi = lane >> (5 - LG);
            const int r = h0 + vi / 4, pl = vi % 4;
            if (r < nr) atomicAdd(part + (rl0 + r) * 4 + pl, v[0]);
        }
    }
}

// One launch per int4 projection (per-layer path and the kernel-level C ABI): the
// int8 kernel's producer, prologue (norm, fixed point) and epilogues, the int4
// stage. p.ld = packed row bytes (16-byte multiple), p.n = codes per row.
template <int KMAX, int RS>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_i4_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxStages;
    float* red = reinterpret_cast<float*>(empty + kGemvMaxStages);
    float* part = reinterpret_cast<float*>(smem + 1024);
    unsigned* amx = reinterpret_cast<unsigned*>(red + 8);
    const uint32_t row_bytes = (uint32_t)p.ld;
    const uint32_t stage_bytes = (uint32_t)RS * row_bytes;
    unsigned char* ring = smem + p.ring_offset;
    const int NS = p.nstages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int r0, r1;
    cta_rows(total_rows(p), 1, blockIdx.x, gridDim.x, r0, r1);
    if (NS < 2 * kGemvGroups || NS > kGemvMaxStages || NS % kGemvGroups || p.stage_rows != RS || p.paired || p.rope) {
        if (tid == 0) set_err(p.err, B2_DEV_ERR_TIMEOUT);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGemvGroupWarps);
        }
        fence_mbar_init();
        *amx = 0u;
    }
    for (int i = tid; i < (r1 - r0) * 4; i += kGemvThreads) reinterpret_cast<int*>(part)[i] = 0;
    __syncthreads();
    pdl_launch_dependents();
    if (warp == kGemvConsumerWarps) {
        if (lane == 0) {
            int j = 0;
            if (!gemv_produce<1>(p, r0, r1, RS, row_bytes, ring, stage_bytes, NS, full, empty, j))
                set_err(p.err, B2_DEV_ERR_TIMEOUT);
            for (int i = max(0, j - NS); i < j; ++i)
                if (!mbar_wait_bounded(&full[i % NS], (uint32_t)((i / NS) & 1))) {
                    set_err(p.err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }
    const int group = warp / kGemvGroupWarps;
    pdl_wait();
    const bool active = p.st ? (*(volatile int*)&p.st->active != 0) : true;
    const int pos = p.st ? *(volatile int*)&p.st->pos : p.pos_fixed;
    float2 xr[KMAX][16];
    gemv_load_x<I4Tag, KMAX>(p, xr, red, tid);
    uint32_t am = 0u;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
#pragma unroll
        for (int t = 0; t < 16; ++t) am = max(am, max(abs_bits(xr[k][t].x), abs_bits(xr[k][t].y)));
    const int S = xfix_shift_cta(am, amx);
    uint32_t xp[KMAX][32];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
            float t16[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) { t16[2 * i] = xr[k][8 * hlf + i].x; t16[2 * i + 1] = xr[k][8 * hlf + i].y; }
            uint32_t w16[16];
            xfix_block(t16, S, w16);
#pragma unroll
            for (int pl = 0; pl < 4; ++pl)
#pragma unroll
                for (int g = 0; g < 4; ++g) xp[k][pl * 8 + 4 * hlf + g] = w16[pl * 4 + g];
        }
    }
    const int nblk = (int)(row_bytes >> 4);
    int j = 0;
    bool ok = true;
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, RS);
        const int slot = j % NS;
        if ((slot & 1) == group) {
            if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / NS) & 1))) { ok = false; break; }
            if (active)
                gemv_stage_i4<KMAX, RS>(ring + (size_t)slot * stage_bytes, row_bytes, nblk, tid % 256, lane, xp,
                                        reinterpret_cast<int*>(part), cur - r0, sr.nr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        ++j;
        cur += sr.nr;
    }
    if (!ok) set_err(p.err, B2_DEV_ERR_TIMEOUT);
    consumer_bar();
    if (!active) return;
    gemv_epilogue<1, false>(p, r0, r1, part, pos, tid, blockIdx.x, gridDim.x, nullptr, S);
}

}  // namespace b2
