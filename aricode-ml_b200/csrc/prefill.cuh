// prefill.cuh — batched prompt processing (many tokens per launch) on the 5th
// generation tensor cores, bit-identical to feeding the tokens one at a time.
//
// Replaces the reference's token-at-a-time prompt loop (aricode_pack.py:2203-2216),
// which runs the whole per-token forward once per prompt token. Here every
// projection of a layer is one GEMM over all prompt tokens:
//
//   planes  (prefill_planes_kernel): per token, the same RMSNorm as the decode
//           GEMV prologue (256 partials in the same order), then the exact
//           fixed-point copy X = trunc(x 2^S) of the normalised vector split into
//           byte planes P0..P3 (P0..P2 unsigned, P3 signed): [4][tokens][K] bytes.
//   GEMM    (prefill_gemm_kernel): D_p[m, t] = sum_k W[m, k] P_p[t, k] with
//           tcgen05.mma kind::i8 (int8 x uint8/int8 -> int32 in TMEM), one
//           accumulator per plane; operands staged by TMA (cp.async.bulk.tensor,
//           128-byte swizzle) into a shared-memory ring; one thread issues the
//           MMAs, one the copies, four warps run the epilogue. The int32 sums are
//           exact in any order, so D = P0 + 2^8 P1 + 2^16 P2 + 2^24 P3 is the same
//           integer the decode GEMV forms with dp4a, and the epilogue rounds it the
//           same way (f32(D 2^-S)), then applies the same per-row operations:
//           scale, bias, RoPE + 1/sqrt(dh) + KV append, residual add, SiLU * up.
//   attention (prefill_attn_kernel): for every token t the split-KV decode
//           attention over keys 0..pos(t), with the decode kernel's arithmetic
//           order (64-key chunks, lane-strided dots, the -60 tail), several tokens
//           per CTA sharing each K/V chunk.
//
// Tile: 128 weight rows (TMEM lanes) x N tokens (TMEM columns), K in 128-byte
// blocks; one accumulator per plane and matrix: one matrix N = 128 (4 x 128 TMEM
// columns), gate + up paired N = 64 (8 x 64).
#pragma once
#include <cuda.h>

#include "kernels.cuh"

namespace b2 {

constexpr int kPfRows = 128;           // weight rows per tile (MMA M)
constexpr int kPfSplitTiles = 80;      // split-K totals: the accumulator holds kPfSplitTiles x
constexpr int kPfSplitCols = 256;      // kPfSplitCols columns of 128 rows (NM * N a tile, int64 each)
constexpr int kPfSplitCounters = 512;  // tiles of a split launch (arrival counters)
constexpr int kPfKBlock = 128;         // bytes of K per stage (one 128-byte swizzle row)
constexpr int kPfEpiWarps = 8;         // epilogue warps: TMEM lane quarter w % 4, column half w / 4
constexpr int kPfThreads = (kPfEpiWarps + 3) * 32;   // + weight copies, MMAs, plane copies

enum PfEpi : int { PF_Q = 0, PF_K = 1, PF_V = 2, PF_RESID = 3, PF_SWIGLU = 4, PF_STORE = 5 };

struct PfGemmParams {
    int M;                   // weight rows
    int K;                   // row length in bytes (the matrices' ld)
    int T;                   // tokens
    int Tpad;                // plane rows per plane (tokens rounded up to the tile)
    int epi;
    const int* S;            // [T] fixed-point shift of each token's input
    const float* scale[2];   // per-row scales of the (one or two) matrices
    const float* bias;       // optional
    float* out;              // [T][ldo] (Q / residual stream / SwiGLU output / store)
    int ldo;
    // Q / K / V: RoPE at positions pos0 + t, Q scaled, K/V into the cache
    int rope;
    const float* rope_tab;
    int dh;
    float qscale;
    float* cache;            // [kv_heads][max_seq][dh]
    int max_seq;
    int pos0;
    // batched decode: token t is the next token of sequence t, at position
    // tok_pos[t], its cache rows at cache + t * cache_seq (nullptr / 0: one
    // sequence, token t at position pos0 + t)
    const int* tok_pos;
    long long cache_seq;
    int* err;
    // split K (grid z > 1): CTA z takes K blocks [z KB / Z, (z + 1) KB / Z); each adds
    // its exact dot D = P0 + 2^8 P1 + 2^16 P2 + 2^24 P3 of every (row, token) into acc
    // (64-bit integer adds: exact in any order) and the last of a tile's Z CTAs
    // (counter cnt[tile]) runs the epilogue from the totals, then clears both for the
    // next launch. acc: per tile [NM * N columns][128 rows] int64.
    unsigned long long* acc;
    unsigned* cnt;
    // tensor parallelism: out rows also written into every peer's copy of out
    Mirror mir;
    // optional timeline (B2_PF_TRACE): per CTA 8 global-timer values: start, MMA
    // thread's waits on weight / plane tiles (total ns), MMA loop end, weight and
    // plane copy threads' waits for free slots (total ns), epilogue start and end
    unsigned long long* trace;
};

struct PfAttnParams {
    const float* q;          // [T][H * dh], rotated and pre-scaled
    const float* K;          // [KVH][max_seq][dh]
    const float* V;
    float* out;              // [T][H * dh]
    float* part;             // [T][H][nsplit_max][dh + 2]
    int H, KVH, dh, max_seq, nsplit_max;
    int T, pos0;
    int* err;
    const int* n_of;         // combine only: token t sees n_of[t] + 1 keys (nullptr: pos0 + t + 1)
    int ldo;                 // out row stride (0: H * dh); tensor parallelism: this rank's heads
                             // at their columns of the whole attention output
    Mirror mir;              // and written into every peer's copy of it
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile, rows of 128 bytes in 8-row (1024-byte) swizzle atoms
// (the TMA 128-byte swizzle): start address, leading offset 16 B (unused for
// swizzled K-major), stride 1024 B between 8-row groups, descriptor version 1,
// layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::i8 instruction descriptor: D s32, A signed int8, B unsigned (planes 0-2)
// or signed (plane 3), both K-major, M = 128, N tokens
__host__ __device__ constexpr uint32_t umma_idesc_i8(int n, bool b_signed) {
    return (2u << 4) | (1u << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kPfRows >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}

// arrive on `bar` once every tcgen05 operation this thread issued has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ planes
// One CTA of 256 threads per token: x (f32 [n], row t of `x` with stride ldx) ->
// optional RMSNorm (gain g) -> S -> planes [4][Tpad][ldp] bytes (zeros past n up
// to kp), S[t]. Same operations and order as the decode GEMV prologue
// (gemv_norm_smem + xfix_shift + xfix_smem), so the planes are bit-identical.
struct PfPlanesParams {
    const float* x;
    int ldx, n;
    int norm;                // NORM_NONE / NORM_RMS
    const float* g;
    float eps;
    unsigned char* planes;   // [4][Tpad][ldp]
    int ldp, kp, Tpad;
    int* S;
};

static __global__ void __launch_bounds__(256) prefill_planes_kernel(const __grid_constant__ PfPlanesParams p) {
    extern __shared__ __align__(16) float pxs[];               // [n]
    __shared__ float red[8];
    __shared__ unsigned amx;
    const int t = blockIdx.x, tid = threadIdx.x, n = p.n;
    const float* x = p.x + (size_t)t * p.ldx;
    if (tid == 0) amx = 0u;
    for (int i = tid; i < n; i += 256) pxs[i] = x[i];
    __syncthreads();
    uint32_t am = 0u;
    if (p.norm == NORM_RMS) {
        float a = 0.0f;
        for (int i = tid; i < n; i += 256) { const float v = pxs[i]; a = ffma(v, v, a); }
        const float tot = block_reduce256(a, red);
        const float scale_a = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(tot, (float)n), p.eps)));
        for (int i = tid; i < n; i += 256) {
            const float v = fmul(fmul(pxs[i], scale_a), p.g[i]);
            pxs[i] = v;
            am = max(am, abs_bits(v));
        }
    } else {
        for (int i = tid; i < n; i += 256) am = max(am, abs_bits(pxs[i]));
    }
    am = __reduce_max_sync(0xffffffffu, am);
    if ((tid & 31) == 0) atomicMax(&amx, am);
    __syncthreads();
    const int S = xfix_shift(amx);
    if (tid == 0) p.S[t] = S;
    const float p2 = (S != kXfixBad && S <= 127) ? __uint_as_float((uint32_t)(S + 127) << 23) : 0.0f;
    // four consecutive elements per thread and pass: one 32-bit word per plane
    for (int q = tid; q * 4 < p.kp; q += 256) {
        uint32_t X[4] = {0u, 0u, 0u, 0u};
        if (S != kXfixBad) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * q + e;
                if (i < n) {
                    const float v = pxs[i];
                    X[e] = S <= 127 ? (uint32_t)__float2int_rz(__fmul_rn(v, p2)) : xfix_elem(v, S);
                }
            }
        }
        uint32_t pl[4];
        xfix_planes4(X[0], X[1], X[2], X[3], pl);
#pragma unroll
        for (int pp = 0; pp < 4; ++pp)
            *reinterpret_cast<uint32_t*>(p.planes + ((size_t)pp * p.Tpad + t) * p.ldp + 4 * q) = pl[pp];
    }
}

// ------------------------------------------------------------------ GEMM
// One CTA per (128 weight rows, N tokens) tile; NM = 2 takes the gate and up
// rows side by side (SwiGLU). Two rings in shared
// memory: weight tiles (NM x [128][128 B] per K block, streamed from HBM, deeper)
// and plane tiles (4 x [N][128 B] per K block, L2-resident), each with its own
// copy warp, so the weight stream runs ahead of the plane stream; all tiles are
// 1024-byte aligned (swizzle atoms).
// (measured on B200: the single-matrix GEMM is fastest with 128 tokens a tile --
// each MMA then reads 4 KB of weights and 4 KB of planes from shared memory for
// 128 x 128 x 32 products; 64 tokens a tile with deeper rings ran 1.4x slower)
template <int NM>
struct PfShape {
    static constexpr int N = 128 / NM;
    static constexpr int ABytes = kPfRows * kPfKBlock;            // 16 KB
    static constexpr int BBytes = N * kPfKBlock;                  // one plane tile
    static constexpr int AStage = NM * ABytes;
    static constexpr int BStage = 4 * BBytes;
    static constexpr int NSA = NM == 1 ? 4 : 3;
    static constexpr int NSB = NM == 1 ? 2 : 3;
    static constexpr int SmemBytes = 1024 + NSA * AStage + NSB * BStage + 2048;
    static constexpr int TmemCols = 512;
};

template <int NM>
__global__ void __launch_bounds__(kPfThreads, 1)
prefill_gemm_kernel(const __grid_constant__ CUtensorMap mapA0, const __grid_constant__ CUtensorMap mapA1,
                    const __grid_constant__ CUtensorMap mapB, const __grid_constant__ PfGemmParams p) {
    using Sh = PfShape<NM>;
    constexpr int N = Sh::N, NSA = Sh::NSA, NSB = Sh::NSB;
    extern __shared__ unsigned char pf_smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* ringA = sm;
    unsigned char* ringB = sm + NSA * Sh::AStage;
    uint64_t* fullA = reinterpret_cast<uint64_t*>(ringB + NSB * Sh::BStage);
    uint64_t* emptyA = fullA + NSA;
    uint64_t* fullB = emptyA + NSA;
    uint64_t* emptyB = fullB + NSB;
    uint64_t* done = emptyB + NSB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* fail = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kPfRows, n0 = blockIdx.y * N;
    const int KBall = (p.K + kPfKBlock - 1) / kPfKBlock;
    const int kb0 = (int)(blockIdx.z * (unsigned)KBall / gridDim.z);
    const int KB = (int)((blockIdx.z + 1) * (unsigned)KBall / gridDim.z) - kb0;   // this CTA's K blocks
    const bool split = gridDim.z > 1;

    if (tid == 0) {
        for (int s = 0; s < NSA; ++s) { mbar_init(&fullA[s], 1); mbar_init(&emptyA[s], 1); }
        for (int s = 0; s < NSB; ++s) { mbar_init(&fullB[s], 1); mbar_init(&emptyB[s], 1); }
        mbar_init(done, 1);
        fence_mbar_init();
        *fail = 0;
    }
    if (warp == 0) {                                          // TMEM (one CTA per SM: shared memory)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)Sh::TmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    unsigned long long* tr =
        p.trace ? p.trace + (((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer_ns();

    if (warp == kPfEpiWarps) {
        // ---- weight copies: NM tiles of K block kb
        if (lane == 0) {
            unsigned long long waited = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % NSA, r = kb / NSA;
                const unsigned long long tw = tr ? globaltimer_ns() : 0ull;
                if (r > 0 && !mbar_wait_bounded(&emptyA[s], (uint32_t)((r - 1) & 1))) { *fail = 1; break; }
                if (tr) waited += globaltimer_ns() - tw;
                unsigned char* st = ringA + (size_t)s * Sh::AStage;
                mbar_arrive_expect_tx(&fullA[s], (uint32_t)Sh::AStage);
                tma_load_2d(st, &mapA0, (kb0 + kb) * kPfKBlock, m0, &fullA[s]);
                if constexpr (NM == 2) tma_load_2d(st + Sh::ABytes, &mapA1, (kb0 + kb) * kPfKBlock, m0, &fullA[s]);
            }
            if (tr) tr[4] = waited;
        }
    } else if (warp == kPfEpiWarps + 2) {
        // ---- plane copies: the 4 plane tiles of K block kb
        if (lane == 0) {
            unsigned long long waited = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % NSB, r = kb / NSB;
                const unsigned long long tw = tr ? globaltimer_ns() : 0ull;
                if (r > 0 && !mbar_wait_bounded(&emptyB[s], (uint32_t)((r - 1) & 1))) { *fail = 1; break; }
                if (tr) waited += globaltimer_ns() - tw;
                unsigned char* st = ringB + (size_t)s * Sh::BStage;
                mbar_arrive_expect_tx(&fullB[s], (uint32_t)Sh::BStage);
#pragma unroll
                for (int pl = 0; pl < 4; ++pl)
                    tma_load_2d(st + pl * Sh::BBytes, &mapB, (kb0 + kb) * kPfKBlock, pl * p.Tpad + n0, &fullB[s]);
            }
            if (tr) tr[5] = waited;
        }
    } else if (warp == kPfEpiWarps + 1) {
        // ---- MMAs: per K block 4 steps of 32 bytes x NM matrices x 4 planes
        if (lane == 0) {
            const uint32_t id_u = umma_idesc_i8(N, false), id_s = umma_idesc_i8(N, true);
            unsigned long long wa = 0, wb = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int sa = kb % NSA, sb = kb % NSB;
                const unsigned long long t0 = tr ? globaltimer_ns() : 0ull;
                if (!mbar_wait_bounded(&fullA[sa], (uint32_t)((kb / NSA) & 1))) { *fail = 1; break; }
                const unsigned long long t1 = tr ? globaltimer_ns() : 0ull;
                if (!mbar_wait_bounded(&fullB[sb], (uint32_t)((kb / NSB) & 1))) { *fail = 1; break; }
                if (tr) { wa += t1 - t0; wb += globaltimer_ns() - t1; }
                tc_fence_after();
                const uint32_t sta = smem_u32(ringA + (size_t)sa * Sh::AStage);
                const uint32_t stb = smem_u32(ringB + (size_t)sb * Sh::BStage);
#pragma unroll
                for (int kk = 0; kk < kPfKBlock / 32; ++kk) {
#pragma unroll
                    for (int mt = 0; mt < NM; ++mt) {
                        const uint64_t ad = umma_desc_sw128(sta + mt * Sh::ABytes + 32 * kk);
#pragma unroll
                        for (int pl = 0; pl < 4; ++pl) {
                            const uint64_t bd = umma_desc_sw128(stb + pl * Sh::BBytes + 32 * kk);
                            umma_i8(tmem + (uint32_t)((mt * 4 + pl) * N), ad, bd, pl == 3 ? id_s : id_u,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                umma_commit(&emptyA[sa]);                      // both stages are free once these MMAs are done
                umma_commit(&emptyB[sb]);
            }
            umma_commit(done);
            if (tr) { tr[1] = wa; tr[2] = wb; tr[3] = globaltimer_ns(); }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = weight rows
        // m0 + 32 (w % 4) + lane, the 16-token chunks w / 4, w / 4 + 2, ... that hold
        // tokens (interleaved, so that a short tile keeps both halves busy). Per chunk
        // every global input (the residual, the RoPE rows) is requested before the
        // TMEM reads, so their latencies overlap; the tokens' shifts were staged in
        // shared memory while the MMAs ran.
        int* sS = reinterpret_cast<int*>(const_cast<int*>(fail) + 1);        // [N]
        int* sP = sS + N;                                                     // [N] positions
        for (int i = tid; i < N; i += kPfEpiWarps * 32) {
            sS[i] = n0 + i < p.T ? p.S[n0 + i] : 0;
            sP[i] = n0 + i < p.T ? (p.tok_pos ? p.tok_pos[n0 + i] : p.pos0 + n0 + i) : 0;
        }
        const int quarter = warp & 3, half = warp >> 2;
        const int m = m0 + 32 * quarter + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * quarter) << 16);
        float sc[2] = {0.0f, 0.0f}, bi = 0.0f;
        if (m < p.M) {
            sc[0] = p.scale[0][m];
            if (NM == 2) sc[1] = p.scale[1][m];
            if (p.bias) bi = p.bias[m];
        }
        const bool rope = (p.epi == PF_Q || p.epi == PF_K) && p.rope;
        const int hd = rope ? (m & ~1) % p.dh : 0;
        asm volatile("bar.sync 2, %0;" ::"n"(kPfEpiWarps * 32) : "memory");   // sS complete
        bool ok = mbar_wait_bounded(done, 0);
        tc_fence_after();
        if (tr && tid == 0) tr[6] = globaltimer_ns();
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        unsigned long long* acc = split ? p.acc + (size_t)tile * (NM * N) * kPfRows + 32 * quarter + lane : nullptr;
        bool last = true;
        if (split) {
            // this CTA's plane sums into the tile's totals (exact integer adds)
            for (int c0 = 16 * half; c0 < N && n0 + c0 < p.T; c0 += 32) {
#pragma unroll
                for (int mt = 0; mt < NM; ++mt) {
                    uint32_t r[4][16];
#pragma unroll
                    for (int pl = 0; pl < 4; ++pl) tmem_ld16(trow + (uint32_t)((mt * 4 + pl) * N + c0), r[pl]);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (ok && n0 + c0 + j < p.T && m < p.M)
                            atomicAdd(acc + (size_t)(mt * N + c0 + j) * kPfRows,
                                      (unsigned long long)xfix_dot((int)r[0][j], (int)r[1][j], (int)r[2][j], (int)r[3][j]));
                }
            }
            __threadfence();
            volatile int* lastf = const_cast<int*>(fail) + 1 + 2 * N;
            asm volatile("bar.sync 2, %0;" ::"n"(kPfEpiWarps * 32) : "memory");
            if (tid == 0) {
                const unsigned t = atomicAdd(p.cnt + tile, 1u);
                *lastf = t == gridDim.z - 1;
                if (t == gridDim.z - 1) p.cnt[tile] = 0u;      // for the next launch
            }
            asm volatile("bar.sync 2, %0;" ::"n"(kPfEpiWarps * 32) : "memory");
            last = *lastf != 0;
            if (last) __threadfence();
        }
        for (int c0 = 16 * half; last && c0 < N && n0 + c0 < p.T; c0 += 32) {
            float in0[16], in1[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;
                in0[j] = 0.0f; in1[j] = 0.0f;
                if (t < p.T && m < p.M) {
                    if (p.epi == PF_RESID) {
                        in0[j] = p.out[(size_t)t * p.ldo + m];
                    } else if (rope) {
                        const float* tr = p.rope_tab + (size_t)sP[c0 + j] * p.dh + hd;
                        in0[j] = tr[0];
                        in1[j] = tr[1];
                    }
                }
            }
            float v[NM][16];
#pragma unroll
            for (int mt = 0; mt < NM; ++mt) {
                if (split) {
                    // the totals of every split, then zeros for the next launch
                    long long D[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        unsigned long long* a = acc + (size_t)(mt * N + c0 + j) * kPfRows;
                        D[j] = (n0 + c0 + j < p.T && m < p.M) ? (long long)__ldcg(a) : 0ll;
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (n0 + c0 + j < p.T && m < p.M) acc[(size_t)(mt * N + c0 + j) * kPfRows] = 0ull;
                        v[mt][j] = xfix_value(D[j], sS[c0 + j]);
                    }
                } else {
                    uint32_t r[4][16];
#pragma unroll
                    for (int pl = 0; pl < 4; ++pl) tmem_ld16(trow + (uint32_t)((mt * 4 + pl) * N + c0), r[pl]);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int pls[4] = {(int)r[0][j], (int)r[1][j], (int)r[2][j], (int)r[3][j]};
                        v[mt][j] = xfix_row(pls, sS[c0 + j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;
                float y = fmul(v[0][j], sc[0]);
                if (p.epi == PF_SWIGLU) {
                    const float u = fmul(v[NM - 1][j], sc[NM - 1]);
                    if (ok && t < p.T && m < p.M) mirror_store(p.mir, p.out + (size_t)t * p.ldo + m, fmul(silu_f(y), u));
                    continue;
                }
                if (p.bias) y = fadd(y, bi);
                if (p.epi == PF_Q || p.epi == PF_K) {
                    // interleaved RoPE pair (2i, 2i + 1) = lanes (2i, 2i + 1) of this warp
                    const float other = __shfl_xor_sync(0xffffffffu, y, 1);
                    if (rope) {
                        const float c = in0[j], sn = in1[j];
                        y = (m & 1) ? fadd(fmul(other, sn), fmul(y, c)) : fsub(fmul(y, c), fmul(other, sn));
                    }
                }
                if (!ok || t >= p.T || m >= p.M) continue;
                if (p.epi == PF_Q) {
                    p.out[(size_t)t * p.ldo + m] = fmul(y, p.qscale);
                } else if (p.epi == PF_K || p.epi == PF_V) {
                    const int pos = sP[c0 + j];
                    const int kvh = m / p.dh, hdv = m % p.dh;
                    if (pos < p.max_seq)
                        p.cache[t * p.cache_seq + ((size_t)kvh * p.max_seq + pos) * p.dh + hdv] = y;
                    else set_err(p.err, B2_DEV_ERR_KV_OVERFLOW);
                } else if (p.epi == PF_RESID) {
                    mirror_store(p.mir, p.out + (size_t)t * p.ldo + m, fadd(y, in0[j]));
                } else {
                    mirror_store(p.mir, p.out + (size_t)t * p.ldo + m, y);
                }
            }
        }
        if (!ok) *fail = 1;
        if (tr && tid == 0) tr[7] = globaltimer_ns();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"((uint32_t)Sh::TmemCols) : "memory");
    }
    if (tid == 0 && *fail) set_err(p.err, B2_DEV_ERR_TIMEOUT);
}

// ------------------------------------------------------------------ attention
// Two launches, with the decode attention's arithmetic in the same order:
//  part:    CTA (kv head, 64-key chunk s, group of 64 tokens) copies K and V of keys
//           [64s, 64s + 64) into shared memory once; its 8 warps take the group's
//           tokens that see the chunk (token t sees keys 0 .. pos0 + t), and for
//           each of them and each query head of the kv head compute the chunk's
//           (o_s, m_s, l_s): scores as lane partials over d = lane, lane + 32, ...
//           reduced by butterflies, chunk max / exp / sum with lane L on keys L and
//           L + 32, o[d] a sequential FMA chain over the keys;
//  combine: one warp per (token, query head) merges its splits in split order
//           with the -60 tail, exactly as the decode combine does.
constexpr int kPfAttnGroup = 64;        // tokens per attention CTA
constexpr int kPfAttnWarps = 8;

inline size_t prefill_attn_smem(int G, int dh) {
    (void)G;
    return 64 + 2 * (size_t)kAttnChunk * dh * 4 + (size_t)kPfAttnWarps * kAttnChunk * 4 + 64;
}

// KD: head dimensions a lane owns (d = lane, lane + 32, ...; dh <= 32 KD, exact
// when dh == 32 KD, guarded otherwise)
template <int KD>
__global__ void __launch_bounds__(kPfAttnWarps * 32) prefill_attn_part_kernel(const __grid_constant__ PfAttnParams p) {
    extern __shared__ __align__(128) unsigned char asm_raw[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(asm_raw);
    const int G = p.H / p.KVH, dh = p.dh;
    float* Ks = reinterpret_cast<float*>(asm_raw + 64);        // [64][dh]
    float* Vs = Ks + kAttnChunk * dh;                           // [64][dh]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.x, s = blockIdx.y, g0 = blockIdx.z * kPfAttnGroup;
    float* e = Vs + kAttnChunk * dh + warp * kAttnChunk;        // [64] this warp's exponentials
    const int j0 = s * kAttnChunk;
    const int tlast = min(g0 + kPfAttnGroup, p.T) - 1;
    const int n_max = p.pos0 + tlast + 1;
    if (j0 >= n_max) return;                                    // no token of the group reaches the chunk
    const int clen = min(kAttnChunk, n_max - j0);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        const uint32_t bytes = (uint32_t)clen * dh * 4;
        mbar_arrive_expect_tx(bar, 2 * bytes);
        bulk_g2s(Ks, p.K + ((size_t)kvh * p.max_seq + j0) * dh, bytes, bar);
        bulk_g2s(Vs, p.V + ((size_t)kvh * p.max_seq + j0) * dh, bytes, bar);
    }
    __syncthreads();
    if (!mbar_wait_bounded(bar, 0)) {
        set_err(p.err, B2_DEV_ERR_TIMEOUT);
        return;
    }
    const int h0 = kvh * G;
    const int stride = dh + 2;
    // first token of the group that sees the chunk: pos0 + t + 1 > j0
    const int tfirst = max(g0, j0 - p.pos0);
    for (int t = tfirst + warp; t <= tlast; t += kPfAttnWarps) {
        const int n = p.pos0 + t + 1;
        const int len = min(kAttnChunk, n - j0);
        for (int g = 0; g < G; ++g) {
            const float* qt = p.q + (size_t)t * p.H * dh + (size_t)(h0 + g) * dh;
            const bool full = dh == 32 * KD;
            float qv[KD];
#pragma unroll
            for (int i = 0; i < KD; ++i) {
                const int d = lane + 32 * i;
                qv[i] = (full || d < dh) ? __ldg(qt + d) : 0.0f;
            }
            // scores, eight keys at a time: lane partials, then the exchange butterfly
            // (each key's total bit-identical to its own butterfly); key jj0 + lane / 4
            // ends in lanes 4k .. 4k + 3, parked in e[]
            for (int jj0 = 0; jj0 < len; jj0 += 8) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    float a = 0.0f;
                    if (jj0 + u < len) {
                        const float* kr = Ks + (jj0 + u) * dh;
#pragma unroll
                        for (int i = 0; i < KD; ++i) {
                            const int d = lane + 32 * i;
                            if (full || d < dh) a = ffma(qv[i], kr[d], a);
                        }
                    }
                    v[u] = a;
                }
                exchange_butterfly<8>(v, lane);
                if ((lane & 3) == 0 && jj0 + (lane >> 2) < len) e[jj0 + (lane >> 2)] = v[0];
            }
            __syncwarp();
            const float sc0 = lane < len ? e[lane] : 0.0f;
            const float sc1 = lane + 32 < len ? e[lane + 32] : 0.0f;
            __syncwarp();
            // chunk max (the decode order: lane-strided, then the xor tree), exp, sum
            float mx = -__int_as_float(0x7f800000);
            bool any = false;
            if (lane < len) { mx = sc0; any = true; }
            if (lane + 32 < len) { mx = any ? fmaxf(mx, sc1) : sc1; any = true; }
            for (int o = 16; o >= 1; o >>= 1) {
                const float om = __shfl_xor_sync(0xffffffffu, mx, o);
                const int oa = __shfl_xor_sync(0xffffffffu, (int)any, o);
                if (oa) { mx = any ? fmaxf(mx, om) : om; any = true; }
            }
            float a = 0.0f;
            if (lane < len) { const float v = exp_f(fsub(sc0, mx)); e[lane] = v; a = fadd(a, v); }
            if (lane + 32 < len) { const float v = exp_f(fsub(sc1, mx)); e[lane + 32] = v; a = fadd(a, v); }
            a = butterfly32(a);
            __syncwarp();
            float* pp = p.part + (((size_t)t * p.H + h0 + g) * p.nsplit_max + s) * stride;
            float o[KD];
#pragma unroll
            for (int i = 0; i < KD; ++i) o[i] = 0.0f;
            for (int jj = 0; jj < len; ++jj) {
                const float ej = e[jj];
                const float* vr = Vs + jj * dh;
#pragma unroll
                for (int i = 0; i < KD; ++i) {
                    const int d = lane + 32 * i;
                    if (full || d < dh) o[i] = ffma(ej, vr[d], o[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < KD; ++i) {
                const int d = lane + 32 * i;
                if (full || d < dh) pp[d] = o[i];
            }
            if (lane == 0) { pp[dh] = mx; pp[dh + 1] = a; }
            __syncwarp();                                       // e[] reused by the next head / token
        }
    }
}

static __global__ void __launch_bounds__(256) prefill_attn_combine_kernel(const __grid_constant__ PfAttnParams p) {
    const int lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);   // (token, query head)
    if (item >= (long long)p.T * p.H) return;
    const int t = (int)(item / p.H), h = (int)(item % p.H), dh = p.dh;
    const int n = p.n_of ? p.n_of[t] + 1 : p.pos0 + t + 1;
    const int nsplit = (n + kAttnChunk - 1) / kAttnChunk;
    const int stride = dh + 2;
    const float* base = p.part + ((size_t)t * p.H + h) * p.nsplit_max * stride;
    float M = __ldg(base + dh);
    for (int s = 1; s < nsplit; ++s) M = fmaxf(M, __ldg(base + (size_t)s * stride + dh));
    if (n < p.max_seq) M = fmaxf(M, -60.0f);
    float l = 0.0f;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
        const float* ps = base + (size_t)s * stride;
        float ov[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int d = lane + 32 * i;
            ov[i] = d < dh ? __ldg(ps + d) : 0.0f;
        }
        const float w = exp_f(fsub(__ldg(ps + dh), M));
        l = ffma(__ldg(ps + dh + 1), w, l);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = ffma(ov[i], w, o[i]);
    }
    if (n < p.max_seq) l = ffma((float)(p.max_seq - n), exp_f(fsub(-60.0f, M)), l);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < dh) mirror_store(p.mir, p.out + (size_t)t * (p.ldo ? p.ldo : p.H * dh) + (size_t)h * dh + d, fdiv(o[i], l));
    }
}

// ------------------------------------------------------------------ embedding
// x[t] = f32(q[tok_t]) * scale[tok_t] for the prompt ids at positions pos0 + t
// (the decode step's embedding, one CTA per token)
static __global__ void __launch_bounds__(256) prefill_embed_kernel(const int8_t* emb, const float* emb_s, long long ld,
                                                                  const int* ids, int pos0, int vocab, int d,
                                                                  float* x, int* err) {
    const int t = blockIdx.x;
    const int tok = ids[pos0 + t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) set_err(err, B2_DEV_ERR_BAD_TOKEN);
        return;
    }
    const float s = emb_s[tok];
    for (int i = threadIdx.x; i < d; i += 256) x[(size_t)t * d + i] = fmul((float)emb[(size_t)tok * ld + i], s);
}

// ------------------------------------------------------------------ batched decode attention
// One warp per (sequence z, kv head, 64-key chunk s): it reads the chunk's K and V
// rows straight from the cache (each lane the elements d = lane, lane + 32, ...;
// kBtKeys keys' loads in flight at a time) and computes the chunk's (o_s, m_s, l_s)
// for the kv head's query heads with the decode arithmetic: scores as lane partials
// reduced by butterflies (kBtKeys keys through one exchange butterfly, each total
// bit-identical to its own), chunk max / exp / sum with lane L on keys L and
// L + 32, o[d] a sequential FMA chain over the keys. No shared-memory staging and
// no block barriers: many warps per SM keep the cache reads in flight.
// prefill_attn_combine_kernel then merges each (sequence, head) in split order.
constexpr int kBtWarps = 8;
constexpr int kBtKeys = 4;             // keys whose loads are in flight together

template <int KD>
__global__ void __launch_bounds__(kBtWarps * 32, 3) attn_batch_part_kernel(const __grid_constant__ AttnParams p) {
    __shared__ float es[kBtWarps][kAttnChunk];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int z = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z * kBtWarps + warp;
    const int G = p.H / p.KVH, dh = p.dh;
    const int n = p.n_of[z] + 1;
    const int nsplit = (n + kAttnChunk - 1) / kAttnChunk;
    if (s >= nsplit) return;
    const bool full = dh == 32 * KD;
    const int j0 = s * kAttnChunk, len = min(kAttnChunk, n - j0);
    const float* Kc = p.K + z * p.skv + ((size_t)kvh * p.max_seq + j0) * dh;
    const float* Vc = p.V + z * p.skv + ((size_t)kvh * p.max_seq + j0) * dh;
    float* e = es[warp];
    const int stride = dh + 2;
#pragma unroll 1
    for (int g = 0; g < G; ++g) {
        const int h = kvh * G + g;
        const float* qt = p.q + z * p.sq + (size_t)h * dh;
        float qv[KD];
#pragma unroll
        for (int i = 0; i < KD; ++i) {
            const int d = lane + 32 * i;
            qv[i] = (full || d < dh) ? __ldg(qt + d) : 0.0f;
        }
#pragma unroll 1
        for (int jj0 = 0; jj0 < len; jj0 += kBtKeys) {
            float kk[kBtKeys][KD];
#pragma unroll
            for (int u = 0; u < kBtKeys; ++u)
#pragma unroll
                for (int i = 0; i < KD; ++i) {
                    const int d = lane + 32 * i;
                    kk[u][i] = (jj0 + u < len && (full || d < dh)) ? __ldcg(Kc + (size_t)(jj0 + u) * dh + d) : 0.0f;
                }
            float v[kBtKeys];
#pragma unroll
            for (int u = 0; u < kBtKeys; ++u) {
                float a = 0.0f;
#pragma unroll
                for (int i = 0; i < KD; ++i)
                    if (full || lane + 32 * i < dh) a = ffma(qv[i], kk[u][i], a);
                v[u] = a;
            }
            exchange_butterfly<kBtKeys>(v, lane);
            constexpr int LG = Log2<kBtKeys>::v;                // key jj0 + (lane >> (5 - LG))
            const int kr = lane >> (5 - LG);
            if ((lane & ((32 >> LG) - 1)) == 0 && jj0 + kr < len) e[jj0 + kr] = v[0];
        }
        __syncwarp();
        const float sc0 = lane < len ? e[lane] : 0.0f;
        const float sc1 = lane + 32 < len ? e[lane + 32] : 0.0f;
        // chunk max (lane-strided, then the xor tree), exp, sum: the decode order
        float mx = -__int_as_float(0x7f800000);
        bool any = false;
        if (lane < len) { mx = sc0; any = true; }
        if (lane + 32 < len) { mx = any ? fmaxf(mx, sc1) : sc1; any = true; }
        for (int o = 16; o >= 1; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, mx, o);
            const int oa = __shfl_xor_sync(0xffffffffu, (int)any, o);
            if (oa) { mx = any ? fmaxf(mx, om) : om; any = true; }
        }
        float a = 0.0f;
        float e0 = 0.0f, e1 = 0.0f;
        if (lane < len) { e0 = exp_f(fsub(sc0, mx)); a = fadd(a, e0); }
        if (lane + 32 < len) { e1 = exp_f(fsub(sc1, mx)); a = fadd(a, e1); }
        a = butterfly32(a);
        float o[KD];
#pragma unroll
        for (int i = 0; i < KD; ++i) o[i] = 0.0f;
#pragma unroll 1
        for (int jj0 = 0; jj0 < len; jj0 += kBtKeys) {
            float vv[kBtKeys][KD];
#pragma unroll
            for (int u = 0; u < kBtKeys; ++u)
#pragma unroll
                for (int i = 0; i < KD; ++i) {
                    const int d = lane + 32 * i;
                    vv[u][i] = (jj0 + u < len && (full || d < dh)) ? __ldcg(Vc + (size_t)(jj0 + u) * dh + d) : 0.0f;
                }
#pragma unroll
            for (int u = 0; u < kBtKeys; ++u) {
                const int jj = jj0 + u;
                const float ej = __shfl_sync(0xffffffffu, jj < 32 ? e0 : e1, jj & 31);
                if (jj < len) {
#pragma unroll
                    for (int i = 0; i < KD; ++i) o[i] = ffma(ej, vv[u][i], o[i]);
                }
            }
        }
        float* pp = p.part + z * p.spart + ((size_t)h * p.nsplit_max + s) * stride;
#pragma unroll
        for (int i = 0; i < KD; ++i) {
            const int d = lane + 32 * i;
            if (full || d < dh) pp[d] = o[i];
        }
        if (lane == 0) { pp[dh] = mx; pp[dh + 1] = a; }
        __syncwarp();                                           // e[] reused by the next head
    }
}

// ------------------------------------------------------------------ batched decode
// Greedy token of each sequence (one CTA per sequence, sample_greedy_f32 order:
// first maximum, NaN never wins, logit 0 NaN -> 0); the token is fed to the next
// step, recorded in out[step][seq], and the sequence's position advances.
struct BatchState {
    int* tok;          // [B] token each sequence feeds to the next step
    int* pos;          // [B] its position (tokens in its cache)
    int* out;          // [max_steps][B] generated ids
    int* n_steps;      // steps recorded so far (one counter)
    int max_steps;
    int max_seq;
    int* err;
};

static __global__ void __launch_bounds__(1024) batch_argmax_kernel(const float* logits, int vocab, BatchState b) {
    __shared__ float wv[32];
    __shared__ int wi[32];
    const int z = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* l = logits + (size_t)z * vocab;
    float bv = 0.0f;
    int bi = 0x7fffffff;
    for (int i = tid; i < vocab; i += 1024) {
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
    if (tid == 0) {
        float cv = 0.0f;
        int ci = 0x7fffffff;
        for (int w = 0; w < 32; ++w)
            if (wi[w] != 0x7fffffff && (ci == 0x7fffffff || amax_better(wv[w], wi[w], cv, ci))) { cv = wv[w]; ci = wi[w]; }
        const float v0 = l[0];
        const int tok = (v0 != v0 || ci == 0x7fffffff) ? 0 : ci;
        b.tok[z] = tok;
        b.pos[z] += 1;
        const int step = *b.n_steps;
        if (step < b.max_steps) b.out[(size_t)step * gridDim.x + z] = tok;
    }
}

// after the argmax of every sequence: one more recorded step
static __global__ void batch_count_kernel(BatchState b) { *b.n_steps += 1; }

// positions of a batch step: every sequence must have room for one more row
static __global__ void batch_check_kernel(BatchState b, int B) {
    const int z = blockIdx.x * blockDim.x + threadIdx.x;
    if (z < B && (b.pos[z] < 0 || b.pos[z] >= b.max_seq)) set_err(b.err, B2_DEV_ERR_KV_OVERFLOW);
}

// ------------------------------------------------------------------ host side (prefill.cu)
// Build the TMA maps and launch one GEMM: A = the weight matrix (or the gate and
// up matrices, NM = 2) int8 [M][K] with row stride K bytes; B = the planes
// [4][Tpad][ldp] bytes.
cudaError_t launch_prefill_gemm(int nm, const void* A0, const void* A1, const unsigned char* planes, int ldp,
                                const PfGemmParams& p, cudaStream_t s);
cudaError_t launch_prefill_planes(const PfPlanesParams& p, int T, cudaStream_t s);
cudaError_t launch_prefill_attn(const PfAttnParams& p, cudaStream_t s);
cudaError_t launch_batch_attn(const AttnParams& a, int nseq, int ldo, cudaStream_t s);
cudaError_t launch_batch_tail(const float* logits, int vocab, const BatchState& b, int B, cudaStream_t s);
// tensor parallelism, between two prefill launches whose outputs the ranks mirror:
// epoch e published to every rank and awaited from every rank (bounded)
cudaError_t launch_tp_sync(unsigned* flags, const Mirror& mir, int rank, int nranks, unsigned* epoch, int* err,
                           cudaStream_t s);
cudaError_t launch_batch_check(const BatchState& b, int B, cudaStream_t s);
cudaError_t launch_prefill_embed(const int8_t* emb, const float* emb_s, long long ld, const int* ids, int pos0,
                                 int vocab, int d, float* x, int T, int* err, cudaStream_t s);
// tokens per plane tile row block (the GEMM's N for one matrix)
constexpr int kPfTokenTile = 128;

}  // namespace b2
