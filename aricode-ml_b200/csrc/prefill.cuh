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
// blocks. One matrix: N = 128, 4 accumulators = 512 TMEM columns; gate + up
// paired: N = 64, 8 accumulators.
#pragma once
#include <cuda.h>

#include "kernels.cuh"

namespace b2 {

constexpr int kPfRows = 128;           // weight rows per tile (MMA M)
constexpr int kPfKBlock = 128;         // bytes of K per stage (one 128-byte swizzle row)
constexpr int kPfThreads = 192;        // warps 0-3 epilogue, warp 4 copies, warp 5 MMAs
constexpr int kPfAttnTokens = 4;       // prompt tokens per attention CTA

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
    int* err;
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
// One CTA per (128 weight rows, N tokens) tile. NM = 1: one matrix, N = 128;
// NM = 2: gate and up rows side by side (SwiGLU), N = 64. Shared memory: ring of
// NS stages, each NM A tiles [128][128 B] then 4 plane tiles [N][128 B], all
// 1024-byte aligned (swizzle atoms); then the mbarriers and the TMEM address.
template <int NM>
struct PfShape {
    static constexpr int N = 128 / NM;
    static constexpr int ABytes = kPfRows * kPfKBlock;            // 16 KB
    static constexpr int BBytes = N * kPfKBlock;                  // one plane tile
    static constexpr int StageBytes = NM * ABytes + 4 * BBytes;
    static constexpr int NS = NM == 1 ? 2 : 3;
    static constexpr int SmemBytes = 1024 + NS * StageBytes + 256;
    static constexpr int TmemCols = 512;
};

template <int NM>
__global__ void __launch_bounds__(kPfThreads, 1)
prefill_gemm_kernel(const __grid_constant__ CUtensorMap mapA0, const __grid_constant__ CUtensorMap mapA1,
                    const __grid_constant__ CUtensorMap mapB, const __grid_constant__ PfGemmParams p) {
    using Sh = PfShape<NM>;
    constexpr int N = Sh::N, NS = Sh::NS;
    extern __shared__ unsigned char pf_smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* ring = sm;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + NS * Sh::StageBytes);
    uint64_t* empty = full + NS;
    uint64_t* done = empty + NS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* fail = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kPfRows, n0 = blockIdx.y * N;
    const int KB = (p.K + kPfKBlock - 1) / kPfKBlock;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(done, 1);
        fence_mbar_init();
        *fail = 0;
    }
    if (warp == 0) {                                          // TMEM: all 512 columns (one CTA per SM)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)Sh::TmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---- copies: stage kb = NM weight tiles + the 4 plane tiles of K block kb
        if (lane == 0) {
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % NS, r = kb / NS;
                if (r > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((r - 1) & 1))) { *fail = 1; break; }
                unsigned char* st = ring + (size_t)s * Sh::StageBytes;
                mbar_arrive_expect_tx(&full[s], (uint32_t)Sh::StageBytes);
                tma_load_2d(st, &mapA0, kb * kPfKBlock, m0, &full[s]);
                if constexpr (NM == 2) tma_load_2d(st + Sh::ABytes, &mapA1, kb * kPfKBlock, m0, &full[s]);
#pragma unroll
                for (int pl = 0; pl < 4; ++pl)
                    tma_load_2d(st + NM * Sh::ABytes + pl * Sh::BBytes, &mapB, kb * kPfKBlock, pl * p.Tpad + n0,
                                &full[s]);
            }
        }
    } else if (warp == 5) {
        // ---- MMAs: per K block 4 steps of 32 bytes x NM matrices x 4 planes
        if (lane == 0) {
            const uint32_t id_u = umma_idesc_i8(N, false), id_s = umma_idesc_i8(N, true);
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % NS;
                if (!mbar_wait_bounded(&full[s], (uint32_t)((kb / NS) & 1))) { *fail = 1; break; }
                tc_fence_after();
                const uint32_t st = smem_u32(ring + (size_t)s * Sh::StageBytes);
#pragma unroll
                for (int kk = 0; kk < kPfKBlock / 32; ++kk) {
#pragma unroll
                    for (int mt = 0; mt < NM; ++mt) {
                        const uint64_t ad = umma_desc_sw128(st + mt * Sh::ABytes + 32 * kk);
#pragma unroll
                        for (int pl = 0; pl < 4; ++pl) {
                            const uint64_t bd = umma_desc_sw128(st + NM * Sh::ABytes + pl * Sh::BBytes + 32 * kk);
                            umma_i8(tmem + (uint32_t)((mt * 4 + pl) * N), ad, bd, pl == 3 ? id_s : id_u,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                umma_commit(&empty[s]);                        // the stage is free once these MMAs are done
            }
            umma_commit(done);
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32w .. 32w + 31 = weight rows m0 + 32w + lane
        const bool ok = mbar_wait_bounded(done, 0);
        tc_fence_after();
        const int m = m0 + 32 * warp + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        float sc[2] = {0.0f, 0.0f}, bi = 0.0f;
        if (m < p.M) {
            sc[0] = p.scale[0][m];
            if (NM == 2) sc[1] = p.scale[1][m];
            if (p.bias) bi = p.bias[m];
        }
        for (int c0 = 0; c0 < N; c0 += 16) {
            float v[NM][16];
#pragma unroll
            for (int mt = 0; mt < NM; ++mt) {
                uint32_t r[4][16];
#pragma unroll
                for (int pl = 0; pl < 4; ++pl) tmem_ld16(trow + (uint32_t)((mt * 4 + pl) * N + c0), r[pl]);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = n0 + c0 + j;
                    const int S = t < p.T ? p.S[t] : 0;
                    const int pls[4] = {(int)r[0][j], (int)r[1][j], (int)r[2][j], (int)r[3][j]};
                    v[mt][j] = xfix_row(pls, S);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;
                float y = fmul(v[0][j], sc[0]);
                if (p.epi == PF_SWIGLU) {
                    const float u = fmul(v[NM - 1][j], sc[NM - 1]);
                    if (ok && t < p.T && m < p.M) p.out[(size_t)t * p.ldo + m] = fmul(silu_f(y), u);
                    continue;
                }
                if (p.bias) y = fadd(y, bi);
                if (p.epi == PF_Q || p.epi == PF_K) {
                    // interleaved RoPE pair (2i, 2i + 1) = lanes (2i, 2i + 1) of this warp
                    const float other = __shfl_xor_sync(0xffffffffu, y, 1);
                    if (p.rope) {
                        const int pos = p.pos0 + (t < p.T ? t : 0);
                        const int hd = (m & ~1) % p.dh;
                        const float* tr = p.rope_tab + (size_t)pos * p.dh + hd;
                        const float c = tr[0], sn = tr[1];
                        y = (m & 1) ? fadd(fmul(other, sn), fmul(y, c)) : fsub(fmul(y, c), fmul(other, sn));
                    }
                }
                if (!ok || t >= p.T || m >= p.M) continue;
                if (p.epi == PF_Q) {
                    p.out[(size_t)t * p.ldo + m] = fmul(y, p.qscale);
                } else if (p.epi == PF_K || p.epi == PF_V) {
                    const int pos = p.pos0 + t;
                    const int kvh = m / p.dh, hd = m % p.dh;
                    if (pos < p.max_seq) p.cache[((size_t)kvh * p.max_seq + pos) * p.dh + hd] = y;
                    else set_err(p.err, B2_DEV_ERR_KV_OVERFLOW);
                } else if (p.epi == PF_RESID) {
                    float* o = p.out + (size_t)t * p.ldo + m;
                    *o = fadd(y, *o);
                } else {
                    p.out[(size_t)t * p.ldo + m] = y;
                }
            }
        }
        if (!ok) *fail = 1;
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
// CTA (kv head, group of kPfAttnTokens consecutive tokens): the K and V chunks of
// keys [64s, 64s + 64) are copied once and used by every token of the group that
// sees them; per token and query head the decode kernel's chunk arithmetic gives
// (m_s, l_s, o_s) into `part`; then the same combine with the -60 tail.
inline size_t prefill_attn_smem(int G, int dh) {
    return 64 + 2 * (size_t)kAttnChunk * dh * 4 + (size_t)kPfAttnTokens * G * dh * 4 +
           (size_t)G * kAttnChunk * 4 + 4 * (size_t)G * 4 + 64;
}

static __global__ void __launch_bounds__(kAttnThreads) prefill_attn_kernel(const __grid_constant__ PfAttnParams p) {
    extern __shared__ __align__(128) unsigned char asm_raw[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(asm_raw);
    const int G = p.H / p.KVH, dh = p.dh;
    float* Ks = reinterpret_cast<float*>(asm_raw + 64);        // [64][dh]
    float* Vs = Ks + kAttnChunk * dh;                           // [64][dh]
    float* qs = Vs + kAttnChunk * dh;                           // [tokens][G][dh]
    float* sc = qs + kPfAttnTokens * G * dh;                    // [G][64]
    float* mpart = sc + G * kAttnChunk;                         // [G]
    float* lpart = mpart + G;
    float* wtot = lpart + G;                                    // [G] combine: l
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.x, t0 = blockIdx.y * kPfAttnTokens;
    const int nt = min(kPfAttnTokens, p.T - t0);
    if (tid == 0) { mbar_init(bar, 1); fence_mbar_init(); }
    const int h0 = kvh * G;
    for (int i = tid; i < nt * G * dh; i += kAttnThreads) {
        const int tt = i / (G * dh), r = i % (G * dh);
        qs[i] = p.q[(size_t)(t0 + tt) * p.H * dh + (size_t)h0 * dh + r];
    }
    __syncthreads();
    const int n_last = p.pos0 + t0 + nt;                        // keys seen by the group's last token
    const int nsplit_all = (n_last + kAttnChunk - 1) / kAttnChunk;
    const float* Kh = p.K + (size_t)kvh * p.max_seq * dh;
    const float* Vh = p.V + (size_t)kvh * p.max_seq * dh;
    const int stride = dh + 2;
    __shared__ int s_ok;
    bool ok = true;
    for (int s = 0; s < nsplit_all; ++s) {
        const int j0 = s * kAttnChunk;
        const int clen = min(kAttnChunk, n_last - j0);
        if (tid == 0) {
            // the previous chunk's generic reads are ordered before the copy's writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint32_t bytes = (uint32_t)clen * dh * 4;
            mbar_arrive_expect_tx(bar, 2 * bytes);
            bulk_g2s(Ks, Kh + (size_t)j0 * dh, bytes, bar);
            bulk_g2s(Vs, Vh + (size_t)j0 * dh, bytes, bar);
            s_ok = mbar_wait_bounded(bar, (uint32_t)(s & 1)) ? 1 : 0;
            if (!s_ok) {
                set_err(p.err, B2_DEV_ERR_TIMEOUT);
                mbar_wait_bounded(bar, (uint32_t)(s & 1));      // last bounded wait for the copies in flight
            }
        }
        __syncthreads();
        if (!s_ok) { ok = false; break; }                        // uniform over the CTA
        mbar_wait_bounded(bar, (uint32_t)(s & 1));               // complete: each thread's own acquire
        for (int tt = 0; tt < nt; ++tt) {
            const int n = p.pos0 + t0 + tt + 1;                  // keys of this token
            if (j0 >= n) continue;                               // uniform over the CTA
            const int len = min(kAttnChunk, n - j0);
            const float* qt = qs + tt * G * dh;
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
                        if (d < dh) a = ffma(qt[g * dh + d], kv[i], a);
                    }
                    a = butterfly32(a);
                    if (lane == 0) sc[g * kAttnChunk + jj] = a;
                }
            }
            __syncthreads();
            for (int g = warp; g < G; g += kAttnThreads / 32) {
                float mx = -__int_as_float(0x7f800000);
                bool any = false;
                for (int jj = lane; jj < len; jj += 32) {
                    const float v = sc[g * kAttnChunk + jj];
                    mx = any ? fmaxf(mx, v) : v;
                    any = true;
                }
                for (int o = 16; o >= 1; o >>= 1) {
                    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
                    const int oa = __shfl_xor_sync(0xffffffffu, (int)any, o);
                    if (oa) { mx = any ? fmaxf(mx, om) : om; any = true; }
                }
                float a = 0.0f;
                for (int jj = lane; jj < len; jj += 32) {
                    const float e = exp_f(fsub(sc[g * kAttnChunk + jj], mx));
                    sc[g * kAttnChunk + jj] = e;
                    a = fadd(a, e);
                }
                a = butterfly32(a);
                if (lane == 0) { mpart[g] = mx; lpart[g] = a; }
            }
            __syncthreads();
            for (int it = tid; it < G * dh; it += kAttnThreads) {
                const int g = it / dh, d = it % dh;
                const float* e = sc + g * kAttnChunk;
                float a = 0.0f;
                for (int jj = 0; jj < len; ++jj) a = ffma(e[jj], Vs[jj * dh + d], a);
                float* pp = p.part + (((size_t)(t0 + tt) * p.H + h0 + g) * p.nsplit_max + s) * stride;
                pp[d] = a;
                if (d == 0) { pp[dh] = mpart[g]; pp[dh + 1] = lpart[g]; }
            }
            __syncthreads();                                     // sc / mpart reused by the next token
        }
    }
    if (!ok) return;
    __syncthreads();                                             // this CTA's partials are visible to it
    for (int tt = 0; tt < nt; ++tt) {
        const int n = p.pos0 + t0 + tt + 1;
        const int nsplit = (n + kAttnChunk - 1) / kAttnChunk;
        for (int g = tid; g < G; g += kAttnThreads) {
            const float* base = p.part + ((size_t)(t0 + tt) * p.H + h0 + g) * p.nsplit_max * stride;
            float M = base[dh];
            for (int s = 1; s < nsplit; ++s) M = fmaxf(M, base[(size_t)s * stride + dh]);
            if (n < p.max_seq) M = fmaxf(M, -60.0f);
            float l = 0.0f;
            for (int s = 0; s < nsplit; ++s) l = ffma(base[(size_t)s * stride + dh + 1], exp_f(fsub(base[(size_t)s * stride + dh], M)), l);
            if (n < p.max_seq) l = ffma((float)(p.max_seq - n), exp_f(fsub(-60.0f, M)), l);
            wtot[g] = l;
            mpart[g] = M;
        }
        __syncthreads();
        for (int it = tid; it < G * dh; it += kAttnThreads) {
            const int g = it / dh, d = it % dh;
            const float* base = p.part + ((size_t)(t0 + tt) * p.H + h0 + g) * p.nsplit_max * stride;
            const float M = mpart[g];
            float o = 0.0f;
            for (int s = 0; s < nsplit; ++s)
                o = ffma(base[(size_t)s * stride + d], exp_f(fsub(base[(size_t)s * stride + dh], M)), o);
            p.out[(size_t)(t0 + tt) * p.H * dh + (size_t)(h0 + g) * dh + d] = fdiv(o, wtot[g]);
        }
        __syncthreads();
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

// ------------------------------------------------------------------ host side (prefill.cu)
// Build the TMA maps and launch one GEMM: A = the weight matrix (or the gate and
// up matrices, NM = 2) int8 [M][K] with row stride K bytes; B = the planes
// [4][Tpad][ldp] bytes.
cudaError_t launch_prefill_gemm(int nm, const void* A0, const void* A1, const unsigned char* planes, int ldp,
                                const PfGemmParams& p, cudaStream_t s);
cudaError_t launch_prefill_planes(const PfPlanesParams& p, int T, cudaStream_t s);
cudaError_t launch_prefill_attn(const PfAttnParams& p, cudaStream_t s);
cudaError_t launch_prefill_embed(const int8_t* emb, const float* emb_s, long long ld, const int* ids, int pos0,
                                 int vocab, int d, float* x, int T, int* err, cudaStream_t s);
// tokens per plane tile row block (the GEMM's N for one matrix)
constexpr int kPfTokenTile = 128;

}  // namespace b2
