// token.cuh — the persistent token kernel: one launch runs a whole decode step
// (embedding, every sub-block, LM head + greedy argmax) on one CTA per SM.
//
// Why: a batch-1 step of a 7B model is 160 weight-streaming phases of 17-90 MB.
// As separate kernels each pays a few microseconds of ring fill, prologue and
// drain. Here the phases are a table walked by every CTA, and the producer warp
// streams the CTA's weight rows of phase p+1 into the shared-memory ring while
// the consumers still work on phase p or wait at the grid barrier. Weights do
// not depend on the activations, so HBM does not wait for a phase boundary.
//
// Structure of a CTA (640 threads, ~200 KB shared memory):
//   warpgroup 4    producer: one lane walks all phases, one 1-D bulk copy per
//                  stage into a ring of NS 32 KB slots (mbarrier complete_tx), at
//                  most kTkInflight copies outstanding (0: no cap beyond the
//                  ring); it also prefetches each
//                  phase's small vectors (norm gains, scales, biases) into L2;
//   warpgroups 0-3 consumers in two groups of 8 warps; stage j belongs to group
//                  j & 1 (GEMV stages, and the V chunk of an attention item);
//                  four full barriers per slot keep this exact for any slot count
//                  (tk_full);
//                  between phases, on one GPU: a consumer barrier only. Every
//                  activation a phase hands to the next (x, q, this step's K/V
//                  rows, the split partials, the attention output, the FFN
//                  hidden vector) is a (value, tag) word, tag = launch x 1024 +
//                  phase + 1, and the reader polls its words until the tags are
//                  the producing phase's (bounded to 1 s). No fence on the writer,
//                  no counter: a CTA starts a phase as soon as its inputs are
//                  there. With tensor parallelism (peer writes) and with
//                  B2_TK_TAGS=0: a grid barrier (atomic arrivals, acquire spin,
//                  bounded to 1 s) over plain floats instead.
//
// Phases (TkPhase):
//   TK_EMBED  CTA 0 writes x = embedding row (+ learned position);
//   TK_GEMV   the building blocks of gemv_kernel (gemv.cuh): prologue norm,
//             stages, epilogue (residual, RoPE + KV append, SiLU*up, GELU, argmax);
//             int8 rows as the exact fixed-point dot of gemv_stage_i8;
//   TK_ATTN   split-KV decode attention: item (query head h, 64-key split s) on
//             CTA item % grid; the V chunk arrives as a ring stage, the K chunk
//             is read straight from memory with plain loads, so that all of a
//             CTA's items are in flight at once; the
//             row of the current position comes from this step's Q/K/V phase;
//             each item writes its split's (o_s, m_s, l_s);
//   TK_ACOMB  after the grid barrier, the outputs (h, d) spread over the CTAs,
//             each merging head h's splits with the -60 tail (a separate phase:
//             no split waits for another, so no CTA's tail waits on the slowest
//             split). Arithmetic order as attn_decode_kernel (attn.cuh) and
//             oracle/refdec.c attn_head().
//
// Every value is computed by the same code and in the same order as the
// per-launch kernels, so results are bit-identical to them and to the oracle.
#pragma once
#include "kernels.cuh"

namespace b2 {

enum TkKind : int { TK_EMBED = 0, TK_GEMV = 1, TK_ATTN = 2, TK_ACOMB = 3 };
// compiled GEMV shapes: weight type, 16-byte blocks per thread per row (1, or up
// to 3: rows of at most 12 KB), rows per stage, paired (gate+up)
enum TkVariant : int {
    TV_I8_K1_R8 = 0,
    TV_I8_K1_R4_P = 1,
    TV_I8_K3_R2 = 2,
    TV_I8_K3_R1_P = 3,
    TV_F32_K1_R8 = 4,
    TV_F32_K3_R2 = 5,
};

constexpr uint32_t kTkSlotBytes = 32 * 1024;
constexpr int kTkMaxSlots = 7;                    // any count >= 3 (see tk_full)
constexpr int kTkDefaultSlots = 4;                // measured: 4 x 32 KB streams faster than 5 for Llama-2-7B
constexpr int kTkStamps = 24;                     // timeline slots per phase and CTA
constexpr int kTkInflight = 0;                    // default cap on bulk copies outstanding per CTA (0: none)
constexpr int kTkMaxSplits = 256;                 // max_seq <= 16384
constexpr int kTkGroupScratch = 64 + 4 + kTkMaxSplits;   // floats per consumer group
// shared memory: full barriers [0, 224) (4 per slot), empty barriers [224, 288),
// reduction slots [288, 320), flags [320, 352), vector-staging barrier 352
constexpr int kTkFullOffset = 0;
constexpr int kTkEmptyOffset = 224;
constexpr int kTkRedOffset = 288;
constexpr int kTkFlagOffset = 320;
constexpr int kTkVbarOffset = 352;
constexpr int kTkDbarOffset = 360;                // producer's descriptor copies
constexpr int kTkScratchOffset = 384;             // after the mbarriers and flags
constexpr int kTkDescBytes = 864;                 // one phase descriptor copy (>= sizeof(TkPhase))
constexpr int kTkDescOffset = 3072;               // >= kTkScratchOffset + 2 * kTkGroupScratch * 4
static_assert(kTkScratchOffset + 2 * kTkGroupScratch * 4 <= kTkDescOffset, "scratch layout");
static_assert(4 * kTkMaxSlots * 8 <= kTkEmptyOffset && kTkEmptyOffset + kTkMaxSlots * 8 <= kTkRedOffset, "barriers");
constexpr int kTkPartOffset = kTkDescOffset + 4 * kTkDescBytes + 32;   // 2 consumer + 2 producer copies
// 640 threads: warpgroups 0-3 consume, warpgroup 4 produces (one lane works).
// Registers are granted per warpgroup, so 5 warpgroups launch at 96 registers a
// thread (61,440 per CTA); the producer warpgroup hands registers back
// (setmaxnreg.dec) and the consumers take them (setmaxnreg.inc):
// 4 x 128 x 112 + 128 x 32 = 61,440.
constexpr int kTkThreads = kGemvConsumerThreads + 128;
constexpr int kTkProducerRegs = 32;
constexpr int kTkConsumerRegs = 112;
static_assert(4 * 128 * kTkConsumerRegs + 128 * kTkProducerRegs <= kTkThreads * 96, "register split");

struct alignas(16) TkPhase {
    int kind;
    int variant;        // TK_GEMV
    int unit;           // rows per balancing unit (2 keeps RoPE pairs in one CTA)
    int rs;             // rows per stage the variant is compiled for (paired: second matrix offset)
    int rows;           // rows per stage used (<= rs; chosen so the two groups get equal stage counts)
    int xsync;          // tensor parallelism: the barrier before this phase also waits for every rank
    int tin;            // (value, tag) inputs: the phase (of this launch) that wrote them, or -1
    int nobar;          // set on every phase of a table the tagged kernel runs: the inputs it
                        // reads from this launch are (value, tag) words, waited for word by word
    GemvParams g;
    AttnParams a;
    EmbedParams e;
};

static_assert(sizeof(TkPhase) <= kTkDescBytes && sizeof(TkPhase) % 16 == 0, "descriptor copy size");
static_assert(kTkDescOffset % 16 == 0 && kTkDescBytes % 16 == 0, "descriptor alignment");
static_assert(kTkPartOffset % 16 == 0, "part alignment");

// Copy a phase descriptor from the table (global, read-only) into shared memory,
// 16 bytes per load, across `nthreads` threads, B loads in flight per thread: its
// fields are then read at shared-memory latency instead of one dependent L2 round
// trip each.
template <int B>
__device__ __forceinline__ void tk_copy_desc(TkPhase* dst, const TkPhase* src, int t, int nthreads) {
    constexpr int NV = (int)(sizeof(TkPhase) / 16);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int w0 = t; w0 < NV; w0 += B * nthreads) {
        uint4 v[B];
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int w = w0 + u * nthreads;
            if (w < NV) v[u] = __ldg(s + w);
        }
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int w = w0 + u * nthreads;
            if (w < NV) d[w] = v[u];
        }
    }
}

struct TkParams {
    const TkPhase* phases;
    int nphases;
    int ns;             // ring slots (3 .. kTkMaxSlots)
    int ring_offset;    // bytes (128-aligned)
    unsigned* bar;      // [0] grid-barrier arrivals, [1] exits; zero between launches
    StepState* st;
    const int* prompt;
    int max_seq, max_pos, vocab;
    int inflight;       // bulk copies outstanding per CTA (1 .. ns - 1)
    int vec_offset;     // shared-memory buffer for a phase's x and norm gains (bytes, 128-aligned)
    int vec_floats;     // its capacity
    // tensor parallelism: this GPU's rank of tp_size; tp_flag[kMaxRanks] barrier
    // epochs in the exchange buffer (slot r written by rank r), mir: its peer copies
    int tp_rank, tp_size;
    unsigned* tp_flag;
    Mirror mir;
    unsigned* seq;      // launches completed on this GPU (kept apart from the step state, which
                        // the host rewrites; every rank launches in lockstep, so epochs agree)
    int final_xsync;    // the last phase's outputs went to every rank: a closing cross-rank
                        // barrier, so that no peer still writes them when the next launch starts
    // optional timeline (nullptr: off): [phase][cta][kTkStamps] global-timer stamps
    // at the phase start (after the grid barrier), when x is loaded, after the
    // prologue, after the stages and after the epilogue
    unsigned long long* trace;
};

__device__ __forceinline__ void tk_stamp(unsigned long long* tr, int k, int tid) {
    if (tr && tid == 0) tr[k] = globaltimer_ns();
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void group_bar(int group) {
    asm volatile("bar.sync %0, 256;" ::"r"(2 + group) : "memory");
}

// Ring stage j: slot j % NS, round j / NS. Its "full" barrier is one of four per
// slot (round % 4), waited with parity (round / 4) & 1. A stage belongs to one
// consumer group, j & 1 (a GEMV stage, or an attention item's V chunk),
// and for any slot count the stages j and j + 4 NS that share a barrier belong
// to the same group: each barrier's phases are waited in order by one group, so
// a parity wait never mistakes an earlier phase. The empty barrier (one per slot,
// the owner's 8 warps arrive) is waited only by the producer, in order.
__device__ __forceinline__ uint64_t* tk_full(uint64_t* full, int j, int NS) {
    return full + (j % NS) * 4 + ((j / NS) & 3);
}
__device__ __forceinline__ uint32_t tk_full_parity(int j, int NS) { return (uint32_t)((j / NS) >> 2) & 1u; }

// Producer: wait until stage j may be issued (its slot released by round - 1,
// and at most `inflight` copies outstanding); returns its full barrier or null.
__device__ __forceinline__ uint64_t* tk_issue_wait(uint64_t* full, uint64_t* empty, int NS, int j, int inflight) {
    const int slot = j % NS, round = j / NS;
    if (round > 0 && !mbar_wait_bounded(&empty[slot], (uint32_t)((round - 1) & 1))) return nullptr;
    if (inflight > 0 && j >= inflight &&
        !mbar_wait_bounded(tk_full(full, j - inflight, NS), tk_full_parity(j - inflight, NS)))
        return nullptr;
    return tk_full(full, j, NS);
}

// Grid barrier among the consumers of all CTAs: every CTA adds one arrival
// (release) and waits until `target` arrivals are visible (acquire). Bounded:
// false after ~1 s, and at once when this CTA has already failed (*abort set).
// The result is the same for every consumer thread of the CTA; `flag` alternates
// between two slots (phase parity), so one barrier publishes it.
//
// With tensor parallelism (xsync), the previous phase's outputs were also written
// into the peers' buffers: once the local barrier is complete CTA 0 publishes
// epoch `e` to every rank (tp_flag_exchange: a system-scope release, cumulative
// over the other CTAs' writes it acquired through the barrier); every CTA then
// waits for all ranks' epochs (bounded).
// xs: the cross-rank request, e.g. the next phase's xsync (read after the first
// consumer barrier, which publishes the descriptor copy other warps made).
__device__ __forceinline__ bool tk_grid_sync(unsigned* ctr, unsigned target, int tid, volatile int* flag,
                                             volatile int* abort, const int* xs = nullptr,
                                             const TkParams* P = nullptr, unsigned e = 0, int cta = 0,
                                             unsigned long long* tr = nullptr, bool entered = false) {
    if (!entered) consumer_bar();                       // entered: the caller's threads just met
    if (tid == 0) {
        const bool xsync = xs && *xs && P && P->tp_size > 1;
        bool ok = *abort == 0;
        if (ok) {
            // (with xsync no system-scope fence here: this release at gpu scope, CTA 0's
            // acquire of the count and its system-scope release of the epoch order this
            // CTA's peer copies before every rank's flag)
            if (tr) tr[8] = globaltimer_ns();
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
            const unsigned first = ld_acquire_gpu(ctr);
            if (tr) tr[9] = globaltimer_ns();
            if (first < target) {
                const uint64_t t0 = globaltimer_ns();
                for (uint32_t it = 1;; ++it) {
                    if (ld_acquire_gpu(ctr) >= target) break;
                    if ((it & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) { ok = false; break; }
                }
            }
            if (tr) tr[10] = globaltimer_ns();
            if (ok && xsync) {
                if (cta == 0) {
                    ok = tp_flag_exchange(P->tp_flag, P->tp_rank, P->tp_size, P->mir, e);
                } else {
                    const uint64_t t0 = globaltimer_ns();
                    for (uint32_t it = 1;; ++it) {
                        bool all = true;
                        for (int r = 0; r < P->tp_size; ++r) all = all && (int)(ld_acquire_sys(P->tp_flag + r) - e) >= 0;
                        if (all) break;
                        if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) { ok = false; break; }
                    }
                }
            }
        }
        *flag = ok ? 1 : 0;
    }
    consumer_bar();
    return *flag != 0;
}

// Wait for a ring stage with one decision for the whole consumer group: one thread
// waits (bounded), the group learns the outcome, then every thread takes the
// completed phase itself (returns at once) for its own acquire of the stage.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, int group, int gt, volatile int* f) {
    if (gt == 0) *f = mbar_wait_bounded(bar, parity) ? 1 : 0;
    group_bar(group);
    const bool ok = *f != 0;
    group_bar(group);
    if (ok) mbar_wait_bounded(bar, parity);
    return ok;
}

// L2 prefetch of a small read-only vector range (16-byte granules inside the
// 256-byte aligned tensors of the weight arena)
__device__ __forceinline__ void tk_prefetch(const void* ptr, size_t bytes) {
    if (!ptr || !bytes) return;
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptr) & ~(uintptr_t)15;
    const uintptr_t e = (reinterpret_cast<uintptr_t>(ptr) + bytes + 15) & ~(uintptr_t)15;
    bulk_prefetch_l2(reinterpret_cast<const void*>(a), (uint32_t)(e - a));
}

// Producer, before a GEMV phase's stages: bring the phase's small weight vectors
// (norm gains, this CTA's scales and biases, the RoPE row) into L2, so that the
// consumers' prologue and epilogue do not wait behind the weight stream in DRAM.
__device__ __forceinline__ void tk_prefetch_vectors(const GemvParams& p, int r0, int r1, int pos, bool i8) {
    if (r0 >= r1) return;
    if (p.norm != NORM_NONE) tk_prefetch(p.ng, (size_t)p.n * 4);
    if (p.norm == NORM_LN) tk_prefetch(p.nb, (size_t)p.n * 4);
    if (p.paired) {
        tk_prefetch(p.S[0] + r0, (size_t)(r1 - r0) * 4);
        tk_prefetch(p.S[1] + r0, (size_t)(r1 - r0) * 4);
        return;
    }
    int base = 0;
    for (int sg = 0; sg < p.nseg; ++sg) {
        const int lo = max(r0, base), hi = min(r1, base + p.rows[sg]);
        if (lo < hi) {
            if (i8) tk_prefetch(p.S[sg] + (lo - base), (size_t)(hi - lo) * 4);
            if (p.bias[sg]) tk_prefetch(p.bias[sg] + (lo - base), (size_t)(hi - lo) * 4);
        }
        base += p.rows[sg];
    }
    if (p.epi == EPI_QKV && p.rope) tk_prefetch(p.rope_tab + (size_t)pos * p.dh, (size_t)p.dh * 4);
}

// --------------------------------------------------------------------- attention
__device__ __forceinline__ int tk_attn_items(const AttnParams& a, int n, int& nsplit) {
    nsplit = (n + kAttnChunk - 1) / kAttnChunk;
    return a.H * nsplit;
}

// producer side: one ring stage per item carries its V chunk, so that every
// item's V is in flight at once (the consumers read the K chunks with plain
// loads; requesting them into L2 first measured no faster)
__device__ __forceinline__ bool tk_attn_produce(const AttnParams& a, int n, int cta, int ncta,
                                                unsigned char* ring, int NS, uint64_t* full, uint64_t* empty,
                                                int& j, int inflight) {
    int nsplit;
    const int items = tk_attn_items(a, n, nsplit);
    const int G = a.H / a.KVH, dh = a.dh;
    for (int it = cta; it < items; it += ncta) {
        const int h = it / nsplit, s = it % nsplit, kvh = h / G;
        const int j0 = s * kAttnChunk, len = min(kAttnChunk, n - j0);
        const uint32_t bytes = (uint32_t)len * dh * 4;
        uint64_t* bar = tk_issue_wait(full, empty, NS, j, inflight);
        if (!bar) return false;
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(ring + (size_t)(j % NS) * kTkSlotBytes, a.V + ((size_t)kvh * a.max_seq + j0) * dh, bytes, bar);
        ++j;
    }
    return true;
}

// consumer side: the owning group of each item computes it; all walk j. Every
// wait is decided once per group (group_wait), so a timeout ends the phase for
// the whole group together.
template <bool TAGS>
__device__ __forceinline__ bool tk_attn_consume(const AttnParams& a, int pos, int cta, int ncta,
                                                const unsigned char* ring, int NS, uint64_t* full,
                                                uint64_t* empty, int& j, int group, int gwarp, int lane,
                                                float* scr, volatile int* gflag,
                                                unsigned long long* tr, unsigned itag, unsigned otag) {
    // timeline (thread 0 of each group): [5] group 0's, [7] group 1's total ns
    // waiting for ring stages
    const bool stamp = tr && gwarp == 0 && lane == 0;
    unsigned long long wstage = 0;
    const int n = pos + 1;
    int nsplit;
    const int items = tk_attn_items(a, n, nsplit);
    const int G = a.H / a.KVH, dh = a.dh;
    const int gt = gwarp * 32 + lane;                   // thread index within the group
    float* sc = scr;                  // [64] scores, then exp
    float* ml = scr + 64;             // m, l
    bool tagbad = false;
    // item k of this CTA: its V chunk is ring stage j, taken by group j & 1 (as in
    // the GEMV phases); its K chunk is read from global memory
    for (int it = cta; it < items; it += ncta, ++j) {
        const int slotv = j % NS;
        if ((j & 1) != group) continue;
        const int h = it / nsplit, s = it % nsplit, kvh = h / G;
        const int j0 = s * kAttnChunk, len = min(kAttnChunk, n - j0);
        const int jnew = pos - j0;                      // this step's row, if in the chunk
        const float* knew = a.K + ((size_t)kvh * a.max_seq + pos) * dh;
        const float* vnew = a.V + ((size_t)kvh * a.max_seq + pos) * dh;
        // the chunk's earlier rows, written by earlier steps, straight from memory,
        // issued first: their latency overlaps the wait for this step's words below.
        // Scores: warp gwarp takes keys gwarp + 8 i; lane L sums d = L, L + 32, ...
        // (this step's row from the Q/K/V phase's words)
        const float* Kg = a.K + ((size_t)kvh * a.max_seq + j0) * dh;
        float kk[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int jj = gwarp + 8 * i;
#pragma unroll
            for (int ii = 0; ii < 4; ++ii) {
                const int d = lane + 32 * ii;
                kk[i][ii] = (jj < len && jj != jnew && d < dh) ? __ldcg(Kg + (size_t)jj * dh + d) : 0.0f;
            }
        }
        // loads that do not need the ring: q, and this step's K/V row when it falls
        // in the chunk (issued before the waits, so their latency overlaps them)
        const bool has_new = jnew >= 0 && jnew < len;
        float qv[4], kn[4], vn = 0.0f;
        if constexpr (TAGS) {
            // (value, tag) words written by this step's Q/K/V phase
            const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
            unsigned long long wq[4], wk[4], wv = 0ull;
            const unsigned long long* tkn = a.tkn + (size_t)kvh * dh;
            const unsigned long long* tvn = a.tvn + (size_t)kvh * dh;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                wq[i] = d < dh ? ld_tag(a.tq + (size_t)h * dh + d) : 0ull;
                wk[i] = (has_new && d < dh) ? ld_tag(tkn + d) : 0ull;
            }
            if (has_new && gt < dh) wv = ld_tag(tvn + gt);
            // the late words, all loaded again together until every tag is the phase's
            unsigned late = 0;                          // bits 0-3 q, 4-7 K row, 8 V row
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                if (d < dh && !tag_ok(wq[i], itag)) late |= 1u << i;
                if (has_new && d < dh && !tag_ok(wk[i], itag)) late |= 16u << i;
            }
            if (has_new && gt < dh && !tag_ok(wv, itag)) late |= 256u;
            while (late) {
                if (globaltimer_ns() > deadline) { tagbad = true; break; }   // values unusable; the CTA aborts after the phase
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int d = lane + 32 * i;
                    if (late & (1u << i)) wq[i] = ld_tag(a.tq + (size_t)h * dh + d);
                    if (late & (16u << i)) wk[i] = ld_tag(tkn + d);
                }
                if (late & 256u) wv = ld_tag(tvn + gt);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if ((late & (1u << i)) && tag_ok(wq[i], itag)) late &= ~(1u << i);
                    if ((late & (16u << i)) && tag_ok(wk[i], itag)) late &= ~(16u << i);
                }
                if ((late & 256u) && tag_ok(wv, itag)) late &= ~256u;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                qv[i] = d < dh ? tag_val(wq[i]) : 0.0f;
                kn[i] = (has_new && d < dh) ? tag_val(wk[i]) : 0.0f;
            }
            if (has_new && gt < dh) vn = tag_val(wv);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                qv[i] = d < dh ? __ldcg(a.q + (size_t)h * dh + d) : 0.0f;
                kn[i] = (has_new && d < dh) ? __ldcg(knew + d) : 0.0f;
            }
            vn = (has_new && gt < dh) ? __ldcg(vnew + gt) : 0.0f;
        }
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int jj = gwarp + 8 * i;
            float acc = 0.0f;
            if (jj < len) {
                const bool fresh = jj == jnew;
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    const int d = lane + 32 * ii;
                    if (d < dh) acc = ffma(qv[ii], fresh ? kn[ii] : kk[i][ii], acc);
                }
            }
            v[i] = acc;
        }
        exchange_butterfly<8>(v, lane);
        if ((lane & 3) == 0) {
            const int jj = gwarp + 8 * (lane >> 2);
            if (jj < len) sc[jj] = v[0];
        }
        group_bar(group);
        if (gwarp == 0) {                               // chunk max, exp, chunk sum
            float m = -__int_as_float(0x7f800000);
            bool any = false;
            for (int jj = lane; jj < len; jj += 32) {
                const float x = sc[jj];
                m = any ? fmaxf(m, x) : x;
                any = true;
            }
            for (int o = 16; o >= 1; o >>= 1) {
                const float om = __shfl_xor_sync(0xffffffffu, m, o);
                const int oa = __shfl_xor_sync(0xffffffffu, (int)any, o);
                if (oa) { m = any ? fmaxf(m, om) : om; any = true; }
            }
            float acc = 0.0f;
            for (int jj = lane; jj < len; jj += 32) {
                const float e = exp_f(fsub(sc[jj], m));
                sc[jj] = e;
                acc = fadd(acc, e);
            }
            acc = butterfly32(acc);
            if (lane == 0) { ml[0] = m; ml[1] = acc; }
        }
        group_bar(group);
        // o_s[d] = sum_j e_j V[j][d], j ascending (one thread per d)
        const unsigned long long tw = stamp ? globaltimer_ns() : 0ull;
        if (!group_wait(tk_full(full, j, NS), tk_full_parity(j, NS), group, gt, gflag)) return false;
        if (stamp) wstage += globaltimer_ns() - tw;
        const float* Vs = reinterpret_cast<const float*>(ring + (size_t)slotv * kTkSlotBytes);
        const int stride = dh + 2;
        // the split's (o_s, m_s, l_s), merged by the combine phase: plain stores after
        // which a grid barrier follows, or (value, tag) words
        const size_t pbase = ((size_t)h * a.nsplit_max + s) * stride;
        if (gt < dh) {
            float acc = 0.0f;
            for (int jj = 0; jj < len; ++jj)
                acc = ffma(sc[jj], jj == jnew ? vn : Vs[jj * dh + gt], acc);
            if constexpr (TAGS) {
                st_tag(a.tpart + pbase + gt, acc, otag);
                if (gt == 0) { st_tag(a.tpart + pbase + dh, ml[0], otag); st_tag(a.tpart + pbase + dh + 1, ml[1], otag); }
            } else {
                float* pp = a.part + pbase;
                pp[gt] = acc;
                if (gt == 0) { pp[dh] = ml[0]; pp[dh + 1] = ml[1]; }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slotv]);
        group_bar(group);                               // scratch reused by the next item
    }
    if (stamp) tr[group == 0 ? 5 : 7] = wstage;
    return !tagbad;
}

// Combine phase (after the attention phase's grid barrier): the H * dh outputs
// are spread over the CTAs; output (h, d) merges head h's splits in split order
// with the -60 tail, as the decode combine does (attn_decode_kernel,
// oracle/refdec.c attn_head): M = max of the m_s (and -60 when n < max_seq),
// w_s = exp(m_s - M), l = sum l_s w_s, o = sum o_s[d] w_s, out = o / l.
template <bool TAGS>
__device__ __forceinline__ bool tk_attn_combine(const AttnParams& a, int pos, int cta, int ncta, int tid,
                                                unsigned itag, unsigned otag) {
    const int n = pos + 1, dh = a.dh;
    const int nsplit = (n + kAttnChunk - 1) / kAttnChunk;
    const int stride = dh + 2;
    int r0, r1;
    cta_rows(a.H * dh, 1, cta, ncta, r0, r1);
    bool ok = true;
    for (int idx = r0 + tid; idx < r1; idx += kGemvConsumerThreads) {
        const int h = idx / dh, d = idx % dh;
        const float* base = a.part + (size_t)h * a.nsplit_max * stride;
        float M, l = 0.0f, o = 0.0f;
        if constexpr (TAGS) {
            // (value, tag) partials of the attention phase, split by split in rounds of 8
            const unsigned long long* tb = a.tpart + (size_t)h * a.nsplit_max * stride;
            const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
            M = 0.0f;
            for (int t0 = 0; t0 < nsplit; t0 += 8) {
                unsigned long long wm[8];
                unsigned late = 0;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    wm[u] = t0 + u < nsplit ? ld_tag(tb + (size_t)(t0 + u) * stride + dh) : 0ull;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (t0 + u < nsplit && !tag_ok(wm[u], itag)) late |= 1u << u;
                while (late) {                          // late words loaded again together
                    if (globaltimer_ns() > deadline) { ok = false; break; }
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (late & (1u << u)) wm[u] = ld_tag(tb + (size_t)(t0 + u) * stride + dh);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if ((late & (1u << u)) && tag_ok(wm[u], itag)) late &= ~(1u << u);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (t0 + u < nsplit) M = (t0 + u == 0) ? tag_val(wm[u]) : fmaxf(M, tag_val(wm[u]));
            }
            if (n < a.max_seq) M = fmaxf(M, -60.0f);
            for (int t0 = 0; t0 < nsplit; t0 += 8) {
                unsigned long long wm[8], wl[8], wo[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const bool in = t0 + u < nsplit;
                    const unsigned long long* pt = tb + (size_t)(t0 + u) * stride;
                    wm[u] = in ? ld_tag(pt + dh) : 0ull;
                    wl[u] = in ? ld_tag(pt + dh + 1) : 0ull;
                    wo[u] = in ? ld_tag(pt + d) : 0ull;
                }
                unsigned late = 0;                      // (normally none: m was complete above)
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (t0 + u < nsplit && !(tag_ok(wm[u], itag) && tag_ok(wl[u], itag) && tag_ok(wo[u], itag)))
                        late |= 1u << u;
                while (late) {
                    if (globaltimer_ns() > deadline) { ok = false; break; }
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        if (late & (1u << u)) {
                            const unsigned long long* pt = tb + (size_t)(t0 + u) * stride;
                            wm[u] = ld_tag(pt + dh);
                            wl[u] = ld_tag(pt + dh + 1);
                            wo[u] = ld_tag(pt + d);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if ((late & (1u << u)) && tag_ok(wm[u], itag) && tag_ok(wl[u], itag) && tag_ok(wo[u], itag))
                            late &= ~(1u << u);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (t0 + u < nsplit) {
                        const float w = exp_f(fsub(tag_val(wm[u]), M));
                        l = ffma(tag_val(wl[u]), w, l);
                        o = ffma(tag_val(wo[u]), w, o);
                    }
                }
            }
        } else if (nsplit <= 16) {
            // every split's (m, l, o[d]) in one round of loads
            float ms[16], ls[16], os[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const bool in = u < nsplit;
                const float* pt = base + (size_t)u * stride;
                ms[u] = in ? __ldcg(pt + dh) : 0.0f;
                ls[u] = in ? __ldcg(pt + dh + 1) : 0.0f;
                os[u] = in ? __ldcg(pt + d) : 0.0f;
            }
            M = ms[0];
#pragma unroll
            for (int u = 1; u < 16; ++u)
                if (u < nsplit) M = fmaxf(M, ms[u]);
            if (n < a.max_seq) M = fmaxf(M, -60.0f);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                if (u < nsplit) {
                    const float w = exp_f(fsub(ms[u], M));
                    l = ffma(ls[u], w, l);
                    o = ffma(os[u], w, o);
                }
            }
        } else {
            M = __ldcg(base + dh);
            for (int t0 = 1; t0 < nsplit; t0 += 16) {
                float ms[16];
#pragma unroll
                for (int u = 0; u < 16; ++u)
                    ms[u] = t0 + u < nsplit ? __ldcg(base + (size_t)(t0 + u) * stride + dh) : 0.0f;
#pragma unroll
                for (int u = 0; u < 16; ++u)
                    if (t0 + u < nsplit) M = fmaxf(M, ms[u]);
            }
            if (n < a.max_seq) M = fmaxf(M, -60.0f);
            for (int t0 = 0; t0 < nsplit; t0 += 16) {
                float ms[16], ls[16], os[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const bool in = t0 + u < nsplit;
                    const float* pt = base + (size_t)(t0 + u) * stride;
                    ms[u] = in ? __ldcg(pt + dh) : 0.0f;
                    ls[u] = in ? __ldcg(pt + dh + 1) : 0.0f;
                    os[u] = in ? __ldcg(pt + d) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    if (t0 + u < nsplit) {
                        const float w = exp_f(fsub(ms[u], M));
                        l = ffma(ls[u], w, l);
                        o = ffma(os[u], w, o);
                    }
                }
            }
        }
        if (n < a.max_seq) l = ffma((float)(a.max_seq - n), exp_f(fsub(-60.0f, M)), l);
        if constexpr (TAGS) mirror_st_tag(a.mir, a.tout + idx, fdiv(o, l), otag);
        else mirror_store(a.mir, a.out + idx, fdiv(o, l));
    }
    return ok;
}

// GEMV producer over the token ring: one bulk copy per matrix per stage (the
// second matrix of a paired stage starts RS rows in).
template <int NM>
__device__ __forceinline__ bool tk_gemv_produce(const GemvParams& p, int r0, int r1, int RS, int rows,
                                                uint32_t row_bytes, unsigned char* ring, int NS, uint64_t* full,
                                                uint64_t* empty, int& j, int inflight) {
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, rows);
        uint64_t* bar = tk_issue_wait(full, empty, NS, j, inflight);
        if (!bar) return false;
        const uint32_t bytes = (uint32_t)sr.nr * row_bytes;
        unsigned char* dst = ring + (size_t)(j % NS) * kTkSlotBytes;
        mbar_arrive_expect_tx(bar, bytes * NM);
        bulk_g2s(dst, reinterpret_cast<const unsigned char*>(p.W[sr.seg]) + (size_t)sr.local * row_bytes, bytes, bar);
        if constexpr (NM == 2)
            bulk_g2s(dst + (size_t)RS * row_bytes,
                     reinterpret_cast<const unsigned char*>(p.W[1]) + (size_t)sr.local * row_bytes, bytes, bar);
        ++j;
        cur += sr.nr;
    }
    return true;
}

// f32 GEMV consumers over the token ring: group j & 1 takes stage j. XREG: x slice
// in registers (long rows, gemv_consume_stage); otherwise x from shared memory
// (gemv_consume_stage_xt).
template <typename WT, int RS, int NM, int KB, bool XREG>
__device__ __forceinline__ bool tk_gemv_consume(const GemvParams& p, int r0, int r1, int rows,
                                                const unsigned char* ring, int NS, uint64_t* full, uint64_t* empty,
                                                int& j, int group, int gwarp, int lane, int slotid, const float* xs,
                                                float* part) {
    constexpr int EPB = GemvElems<WT>::EPB;
    const uint32_t row_bytes = (uint32_t)p.ld * (uint32_t)sizeof(WT);
    const int nblk = (int)(row_bytes >> 4);
    float2 xr[XREG ? 3 : 1][EPB / 2];
    if constexpr (XREG) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int b = slotid + 256 * k;
#pragma unroll
            for (int q = 0; q < EPB / 4; ++q) {
                float4 x4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (b < nblk) x4 = lds128f(xs + b * EPB + 4 * q);
                xr[k][2 * q] = make_float2(x4.x, x4.y);
                xr[k][2 * q + 1] = make_float2(x4.z, x4.w);
            }
        }
    }
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, rows);
        if ((j & 1) == group) {
            if (!mbar_wait_bounded(tk_full(full, j, NS), tk_full_parity(j, NS))) return false;
            const unsigned char* st = ring + (size_t)(j % NS) * kTkSlotBytes;
            if constexpr (XREG)
                gemv_consume_stage<WT, 3, RS, NM == 2>(st, row_bytes, nblk, slotid, lane, gwarp, xr, part,
                                                       cur - r0, sr.nr);
            else
                gemv_consume_stage_xt<WT, RS, NM, KB>(st, row_bytes, nblk, slotid, lane, gwarp, xs, part,
                                                      cur - r0, sr.nr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[j % NS]);
        }
        ++j;
        cur += sr.nr;
    }
    return true;
}

// int8 GEMV consumers over the token ring: the thread's plane words (blocks
// slotid, slotid + 256, ... of KB; xs holds the planes, xfix_smem) in registers,
// then the stages (group j & 1 takes stage j), plane sums into part[] (int32).
template <int KB, int RS, int NM>
__device__ __forceinline__ bool tk_gemv_consume_i8(const GemvParams& p, int r0, int r1, int rows,
                                                   const unsigned char* ring, int NS, uint64_t* full, uint64_t* empty,
                                                   int& j, int group, int lane, int slotid, const float* xs, int S,
                                                   int* part, unsigned long long* tr) {
    const uint32_t row_bytes = (uint32_t)p.ld;
    const int nblk = (int)(row_bytes >> 4);
    uint32_t xp[KB][16];
#pragma unroll
    for (int k = 0; k < KB; ++k) {
        const int b = slotid + 256 * k;
        const int f = xfix_swz(b);
#pragma unroll
        for (int q = 0; q < 4; ++q) {                   // plane q (chunk q ^ f)
            uint4 w = make_uint4(0u, 0u, 0u, 0u);
            if (b < nblk) w = lds128(xs + b * 16 + 4 * (q ^ f));
            xp[k][4 * q] = w.x; xp[k][4 * q + 1] = w.y; xp[k][4 * q + 2] = w.z; xp[k][4 * q + 3] = w.w;
        }
    }
    // timeline (thread 0 only): [5] before the first stage wait, [7] after it, [6] total
    // time waiting for stages
    const bool stamp = tr && threadIdx.x == 0;
    unsigned long long waited = 0;
    bool first = true;
    int cur = r0;
    while (cur < r1) {
        const StageRows sr = next_stage(p, cur, r1, rows);
        if ((j & 1) == group) {
            const unsigned long long tw = stamp ? globaltimer_ns() : 0ull;
            if (!mbar_wait_bounded(tk_full(full, j, NS), tk_full_parity(j, NS))) return false;
            if (stamp) {
                const unsigned long long t = globaltimer_ns();
                waited += t - tw;
                if (first) { tr[5] = tw; tr[7] = t; }
                first = false;
            }
            gemv_stage_i8<KB, RS, NM>(ring + (size_t)(j % NS) * kTkSlotBytes, row_bytes, nblk, slotid, lane, xp, part,
                                      cur - r0, sr.nr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[j % NS]);
        }
        ++j;
        cur += sr.nr;
    }
    if (stamp) tr[6] = waited;
    return true;
}

// --------------------------------------------------------------------- GEMV phase
// One compiled copy per weight type: any row length (blocks per thread at run
// time), rows per stage and pairing at run time. x and its norm gains are staged
// in shared memory (vec: x at [0, L), gains at [L, 2L), LN bias at [2L, 3L) with
// L = n rounded up to 16, zeros in [n, L)), normalised in place, and read by the
// stages from there.
// x as (value, tag) words -> vec[0, n), every word waited for (bounded). Thread t
// owns the word pairs t, t + 512, ..., taken U pairs at a time: their loads are in
// flight together, and while some are not yet the phase's, all of those are
// loaded again together (one round trip per round, not one per late word).
__device__ __forceinline__ bool tk_load_tagged(const unsigned long long* tx, int n, unsigned tag, float* vec, int tid) {
    constexpr int U = 4;                                // word pairs per thread per round
    const int npair = n >> 1;                           // n is a multiple of 4
    bool ok = true;
    uint64_t deadline = 0;
    for (int q0 = tid; q0 < npair; q0 += U * kGemvConsumerThreads) {
        unsigned long long a[U], b[U];
        unsigned late = 0;                              // bit u: pair u is not complete yet
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int q = q0 + u * kGemvConsumerThreads;
            if (q < npair) ld_tag2(tx + 2 * q, a[u], b[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (q0 + u * kGemvConsumerThreads < npair && !(tag_ok(a[u], tag) && tag_ok(b[u], tag))) late |= 1u << u;
        while (late) {
            if (deadline == 0) deadline = globaltimer_ns() + kWaitLimitNs;
            else if (globaltimer_ns() > deadline) { ok = false; break; }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (late & (1u << u)) ld_tag2(tx + 2 * (q0 + u * kGemvConsumerThreads), a[u], b[u]);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if ((late & (1u << u)) && tag_ok(a[u], tag) && tag_ok(b[u], tag)) late &= ~(1u << u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int q = q0 + u * kGemvConsumerThreads;
            if (q < npair) *reinterpret_cast<float2*>(vec + 2 * q) = make_float2(tag_val(a[u]), tag_val(b[u]));
        }
    }
    return ok;
}

template <typename WT, bool TAGS>
__device__ __forceinline__ bool tk_gemv(const GemvParams& p, int unit, int rs, int rows, int pos,
                                        const unsigned char* ring,
                                        int NS, uint64_t* full, uint64_t* empty, int& j, int group, int gwarp,
                                        int lane, int tid, float* red, float* part, int cta, int ncta,
                                        unsigned long long* tr, float* vec, uint64_t* vbar, uint32_t& vphase,
                                        unsigned* amx, unsigned itag, unsigned otag) {
    constexpr int ESZ = (int)sizeof(WT);
    int r0, r1;
    cta_rows(total_rows(p), unit, cta, ncta, r0, r1);
    const bool paired = p.paired != 0;
    const int n = p.n, L = (n + 15) & ~15;
    constexpr bool tagged = TAGS;
    const bool bulk = !tagged || p.norm != NORM_NONE;   // anything staged by bulk copy
    if (tid == 0 && bulk) {
        // generic-proxy writes (x by other CTAs; vec by this CTA's last phase) are
        // ordered before the bulk copies that read / overwrite them
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t nb = (uint32_t)n * 4 * ((tagged ? 0 : 1) + (p.norm != NORM_NONE) + (p.norm == NORM_LN));
        mbar_arrive_expect_tx(vbar, nb);
        if (!tagged) bulk_g2s(vec, p.x, (uint32_t)n * 4, vbar);
        if (p.norm != NORM_NONE) bulk_g2s(vec + L, p.ng, (uint32_t)n * 4, vbar);
        if (p.norm == NORM_LN) bulk_g2s(vec + 2 * L, p.nb, (uint32_t)n * 4, vbar);
    }
    for (int i = n + tid; i < L; i += kGemvConsumerThreads) vec[i] = 0.0f;     // row padding
    // part[]: [rows][NM][8] f32 warp sums (int8: [rows][NM][4] int32 plane sums),
    // then epi[]: [rows][4] epilogue inputs
    const int nm = paired ? 2 : 1;
    float* epi = part + (size_t)(r1 - r0) * nm * 8;
    if constexpr (ESZ == 1)
        for (int i = tid; i < (r1 - r0) * nm * 4; i += kGemvConsumerThreads) reinterpret_cast<int*>(part)[i] = 0;
    bool ok = true;
    if constexpr (tagged) {
        // the epilogue inputs and x word by word, their loads in flight together
        const EpiRow er = paired ? gemv_epi_load<ESZ, true>(p, r0, r1, pos, tid)
                                 : gemv_epi_load<ESZ, false>(p, r0, r1, pos, tid);
        ok = tk_load_tagged(p.tx, n, itag, vec, tid);
        gemv_epi_store(er, r1 - r0, tid, epi);
        consumer_bar();                                 // vec[0, n) and epi[] complete
        tk_stamp(tr, 8, tid);                           // timeline: every input word present
        if (bulk) {
            ok = mbar_wait_bounded(vbar, vphase & 1) && ok;
            ++vphase;
        }
    } else {
        const EpiRow er = paired ? gemv_epi_load<ESZ, true>(p, r0, r1, pos, tid)
                                 : gemv_epi_load<ESZ, false>(p, r0, r1, pos, tid);
        ok = mbar_wait_bounded(vbar, vphase & 1);
        ++vphase;
        gemv_epi_store(er, r1 - r0, tid, epi);
    }
    const uint32_t am = gemv_norm_smem(p, vec, vec + L, vec + 2 * L, red, tid);
    tk_stamp(tr, 1, tid);
    const int slotid = tid % 256;
    bool okc;
    int S = 0;
    if constexpr (ESZ == 1) {
        S = xfix_shift_cta(am, amx);                    // also publishes x, epi[] and the zeroed part[]
        xfix_smem(vec, L, S, tid);
        tk_stamp(tr, 2, tid);
        int* parti = reinterpret_cast<int*>(part);
        if (paired)
            okc = rs == 4 ? tk_gemv_consume_i8<1, 4, 2>(p, r0, r1, rows, ring, NS, full, empty, j, group, lane, slotid,
                                                        vec, S, parti, tr)
                          : tk_gemv_consume_i8<3, 1, 2>(p, r0, r1, rows, ring, NS, full, empty, j, group, lane, slotid,
                                                        vec, S, parti, tr);
        else
            okc = rs == 8 ? tk_gemv_consume_i8<1, 8, 1>(p, r0, r1, rows, ring, NS, full, empty, j, group, lane, slotid,
                                                        vec, S, parti, tr)
                          : tk_gemv_consume_i8<3, 2, 1>(p, r0, r1, rows, ring, NS, full, empty, j, group, lane, slotid,
                                                        vec, S, parti, tr);
        ok = okc && ok;
        consumer_bar();
        if (tid == 0) *amx = 0u;                        // every thread read it before its stages
        tk_stamp(tr, 3, tid);
        if (paired) gemv_epilogue<ESZ, true>(p, r0, r1, part, pos, tid, cta, ncta, epi, S, otag);
        else gemv_epilogue<ESZ, false>(p, r0, r1, part, pos, tid, cta, ncta, epi, S, otag);
        return ok;
    } else {
        consumer_bar();                                     // normalised x and epi[] visible
        tk_stamp(tr, 2, tid);
        // the stage shapes the host chose (rows per stage x matrices), compiled
        if (paired) {
            okc = rs == 4 ? tk_gemv_consume<WT, 4, 2, 1, false>(p, r0, r1, rows, ring, NS, full, empty, j, group, gwarp,
                                                                lane, slotid, vec, part)
                          : tk_gemv_consume<WT, 1, 2, 3, true>(p, r0, r1, rows, ring, NS, full, empty, j, group, gwarp,
                                                               lane, slotid, vec, part);
        } else {
            okc = rs == 8 ? tk_gemv_consume<WT, 8, 1, 1, false>(p, r0, r1, rows, ring, NS, full, empty, j, group, gwarp,
                                                                lane, slotid, vec, part)
                          : tk_gemv_consume<WT, 2, 1, 3, true>(p, r0, r1, rows, ring, NS, full, empty, j, group, gwarp,
                                                               lane, slotid, vec, part);
        }
        ok = okc && ok;
        consumer_bar();
        tk_stamp(tr, 3, tid);
        if (paired) gemv_epilogue<ESZ, true>(p, r0, r1, part, pos, tid, cta, ncta, epi, 0, otag);
        else gemv_epilogue<ESZ, false>(p, r0, r1, part, pos, tid, cta, ncta, epi, 0, otag);
        return ok;
    }
}

// VS 0: int8 weights only; VS 1: int8 and f32.
template <int VS, bool TAGS>
__device__ __forceinline__ bool tk_gemv_dispatch(const TkPhase& T, int pos, const unsigned char* ring, int NS,
                                                 uint64_t* full, uint64_t* empty, int& j, int group, int gwarp,
                                                 int lane, int tid, float* red, float* part, int cta, int ncta,
                                                 unsigned long long* tr, float* vec, uint64_t* vbar,
                                                 uint32_t& vphase, unsigned* amx, unsigned itag, unsigned otag) {
    if (VS == 1 && T.variant >= TV_F32_K1_R8)
        return tk_gemv<float, TAGS>(T.g, T.unit, T.rs, T.rows, pos, ring, NS, full, empty, j, group, gwarp, lane, tid, red, part,
                              cta, ncta, tr, vec, vbar, vphase, amx, itag, otag);
    return tk_gemv<int8_t, TAGS>(T.g, T.unit, T.rs, T.rows, pos, ring, NS, full, empty, j, group, gwarp, lane, tid, red, part, cta,
                           ncta, tr, vec, vbar, vphase, amx, itag, otag);
}

// --------------------------------------------------------------------- the kernel
// VS: weight types compiled in (0 int8, 1 int8 and f32). TAGS: the phases meet
// through (value, tag) words (one GPU; every TkPhase::nobar set by the host), or
// at grid barriers over plain floats.
template <int VS, bool TAGS>
__global__ void __launch_bounds__(kTkThreads, 1) token_kernel(const __grid_constant__ TkParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTkFullOffset);   // [4 * NS]
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kTkEmptyOffset); // [NS]
    float* red = reinterpret_cast<float*>(smem + kTkRedOffset);           // 8 floats
    volatile int* flag = reinterpret_cast<volatile int*>(smem + kTkFlagOffset);   // [0], [4] grid sync, [2..3] groups
    volatile int* abort = flag + 6;
    unsigned* amx = reinterpret_cast<unsigned*>(smem + kTkFlagOffset + 28);   // int8 GEMV: largest |x| bits
    uint64_t* vbar = reinterpret_cast<uint64_t*>(smem + kTkVbarOffset);  // vector staging
    float* vec = reinterpret_cast<float*>(smem + P.vec_offset);
    float* scratch = reinterpret_cast<float*>(smem + kTkScratchOffset);
    float* part = reinterpret_cast<float*>(smem + kTkPartOffset);
    unsigned char* ring = smem + P.ring_offset;
    const int NS = P.ns;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, ncta = gridDim.x;
    StepState* st = P.st;
    int* err = &st->err;

    // The step's inputs, read by every CTA before its first grid barrier; this
    // launch writes the step state only after its last one.
    const int active = *(volatile int*)&st->active;
    if (!active) return;
    const int pos = *(volatile int*)&st->step;
    const unsigned seq = *(volatile unsigned*)P.seq;
    int bad = 0, tok = 0;
    if (pos >= P.max_seq || (P.max_pos > 0 && pos >= P.max_pos)) {
        bad = B2_DEV_ERR_KV_OVERFLOW;
    } else {
        const int plen = *(volatile int*)&st->prompt_len;
        tok = pos < plen ? P.prompt[pos] : *(volatile int*)&st->next_tok;
        if (tok < 0 || tok >= P.vocab) bad = B2_DEV_ERR_BAD_TOKEN;
    }
    if (bad) {
        if (cta == 0 && tid == 0) { atomicCAS(err, 0, bad); st->active = 0; }
        return;
    }
    if (NS < 3 || NS > kTkMaxSlots || P.inflight < 0 || P.inflight >= NS) {
        if (cta == 0 && tid == 0) set_err(err, B2_DEV_ERR_TIMEOUT);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            for (int q = 0; q < 4; ++q) mbar_init(&full[4 * s + q], 1);
            mbar_init(&empty[s], kGemvGroupWarps);
        }
        mbar_init(vbar, 1);
        mbar_init(reinterpret_cast<uint64_t*>(smem + kTkDbarOffset), 1);
        fence_mbar_init();
        *abort = 0;
        *amx = 0u;
    }
    __syncthreads();

    if (warp >= kGemvConsumerWarps) {
        // ---------------- producer: every phase's stages, in order, never waiting
        // for a grid barrier
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTkProducerRegs));
        if (warp == kGemvConsumerWarps && lane == 0) {
            int j = 0;
            bool ok = true;
            // descriptors by bulk copy, one phase ahead ([2]: phase ph in ph & 1), so
            // that the issue of a phase's first stages never waits for its descriptor
            TkPhase* pdesc = reinterpret_cast<TkPhase*>(smem + kTkDescOffset + 2 * kTkDescBytes);
            uint64_t* dbar = reinterpret_cast<uint64_t*>(smem + kTkDbarOffset);
            mbar_arrive_expect_tx(dbar, (uint32_t)sizeof(TkPhase));
            bulk_g2s(pdesc, P.phases, (uint32_t)sizeof(TkPhase), dbar);
            int dnext = 0;                                  // phase whose descriptor copy is in flight
            for (int ph = 0; ph < P.nphases && ok; ++ph) {
                // timeline: [11] descriptor wait started, [12] done, [13] last stage issued
                unsigned long long* ptr = P.trace ? P.trace + ((size_t)ph * ncta + cta) * kTkStamps : nullptr;
                if (ptr) ptr[11] = globaltimer_ns();
                if (!mbar_wait_bounded(dbar, (uint32_t)ph & 1u)) { ok = false; break; }
                dnext = -1;
                if (ph + 1 < P.nphases) {                   // its buffer held phase ph - 1's
                    mbar_arrive_expect_tx(dbar, (uint32_t)sizeof(TkPhase));
                    bulk_g2s(pdesc + ((ph + 1) & 1), P.phases + ph + 1, (uint32_t)sizeof(TkPhase), dbar);
                    dnext = ph + 1;
                }
                if (ptr) ptr[12] = globaltimer_ns();
                const TkPhase& T = pdesc[ph & 1];
                if (T.kind == TK_GEMV) {
                    const GemvParams& p = T.g;
                    int r0, r1;
                    cta_rows(total_rows(p), T.unit, cta, ncta, r0, r1);
                    const bool i8 = T.variant < TV_F32_K1_R8;
                    const uint32_t row_bytes = (uint32_t)p.ld * (i8 ? 1u : 4u);
                    tk_prefetch_vectors(p, r0, r1, pos, i8);
                    ok = p.paired ? tk_gemv_produce<2>(p, r0, r1, T.rs, T.rows, row_bytes, ring, NS, full, empty, j,
                                                       P.inflight)
                                  : tk_gemv_produce<1>(p, r0, r1, T.rs, T.rows, row_bytes, ring, NS, full, empty, j,
                                                       P.inflight);
                } else if (T.kind == TK_ATTN) {
                    ok = tk_attn_produce(T.a, pos + 1, cta, ncta, ring, NS, full, empty, j, P.inflight);
                }
                if (ptr) ptr[13] = globaltimer_ns();
            }
            if (!ok) set_err(err, B2_DEV_ERR_TIMEOUT);
            if (dnext >= 0 && !mbar_wait_bounded(dbar, (uint32_t)dnext & 1u)) set_err(err, B2_DEV_ERR_TIMEOUT);
            for (int i = max(0, j - NS); i < j; ++i)        // no copy in flight at exit
                if (!mbar_wait_bounded(tk_full(full, i, NS), tk_full_parity(i, NS))) {
                    set_err(err, B2_DEV_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }

    // ---------------- consumers: every thread goes through the same barriers;
    // a failure anywhere in the CTA sets *abort and ends the walk for all of them
    // at the next phase boundary
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTkConsumerRegs));
    const int group = warp / kGemvGroupWarps;
    const int gwarp = warp % kGemvGroupWarps;
    float* gscr = scratch + group * kTkGroupScratch;
    volatile int* gflag = flag + 2 + group;
    int j = 0;
    unsigned arrivals = 0;
    uint32_t vphase = 0;                                // phases of vbar used so far
    TkPhase* cdesc = reinterpret_cast<TkPhase*>(smem + kTkDescOffset);      // [2]: phase ph in ph & 1
    tk_copy_desc<1>(cdesc, P.phases, tid, kGemvConsumerThreads);
    consumer_bar();
    const unsigned tbase = seq * 1024u + 1u;            // tag of phase ph: tbase + ph
    for (int ph = 0; ph < P.nphases; ++ph) {
        const TkPhase& T = cdesc[ph & 1];
        if (ph > 0) {
            // every consumer thread meets here first: the descriptor of phase ph (copied
            // by other threads during phase ph - 1) is complete only after this barrier,
            // so T is read after it and every thread takes the same path below
            consumer_bar();
            if constexpr (TAGS) {
                // the inputs are (value, tag) words: no grid barrier
                if (*abort) break;
            } else {
                arrivals += (unsigned)ncta;
                unsigned long long* trb = P.trace ? P.trace + ((size_t)ph * ncta + cta) * kTkStamps : nullptr;
                if (!tk_grid_sync(P.bar, arrivals, tid, flag + 4 * (ph & 1), abort, &T.xsync, &P,
                                  seq * 1024u + (unsigned)ph, cta, trb, true)) {
                    if (tid == 0) *abort = 1;
                    break;
                }
            }
        }
        const unsigned otag = tbase + (unsigned)ph;
        const unsigned itag = tbase + (unsigned)T.tin;
        unsigned long long* tr = P.trace ? P.trace + ((size_t)ph * ncta + cta) * kTkStamps : nullptr;
        tk_stamp(tr, 0, tid);
        // the next phase's descriptor, by the last consumer warps (in place after the
        // next grid barrier; the buffer it overwrites was last read in phase ph - 1)
        if (ph + 1 < P.nphases && tid >= kGemvConsumerThreads - 64)
            tk_copy_desc<1>(cdesc + ((ph + 1) & 1), P.phases + ph + 1, tid - (kGemvConsumerThreads - 64), 64);
        bool ok = true;
        if (T.kind == TK_EMBED) {
            if (cta == 0) {
                const EmbedParams& e = T.e;
                for (int i = tid; i < e.d; i += kGemvConsumerThreads) {
                    float v;
                    if (e.emb_i8 == 2) {
                        const int b = reinterpret_cast<const unsigned char*>(e.emb)[(size_t)tok * e.ld + (i >> 1)];
                        v = fmul((float)((((b >> ((i & 1) * 4)) & 15) ^ 8) - 8), e.emb_s[tok]);
                    } else if (e.emb_i8) {
                        const int8_t q = reinterpret_cast<const int8_t*>(e.emb)[(size_t)tok * e.ld + i];
                        v = fmul((float)q, e.emb_s[tok]);
                    } else {
                        v = reinterpret_cast<const float*>(e.emb)[(size_t)tok * e.ld + i];
                    }
                    if (e.pos_tab) v = fadd(v, e.pos_tab[(size_t)pos * e.d + i]);
                    if constexpr (TAGS) st_tag(e.tx + i, v, otag);
                    else e.x[i] = v;
                }
            }
        } else if (T.kind == TK_GEMV) {
            ok = tk_gemv_dispatch<VS, TAGS>(T, pos, ring, NS, full, empty, j, group, gwarp, lane, tid, red, part, cta,
                                      ncta, tr, vec, vbar, vphase, amx, itag, otag);
            // this phase's generic writes of vec before the next phase's bulk copies into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        } else if (T.kind == TK_ACOMB) {
            ok = tk_attn_combine<TAGS>(T.a, pos, cta, ncta, tid, itag, otag);
        } else {
            tk_stamp(tr, 1, tid);
            tk_stamp(tr, 2, tid);
            ok = tk_attn_consume<TAGS>(T.a, pos, cta, ncta, ring, NS, full, empty, j, group, gwarp, lane, gscr, gflag, tr,
                                 itag, otag);
            if (tr) {
                consumer_bar();
                tk_stamp(tr, 3, tid);
            }
        }
        if (tr) {
            consumer_bar();
            tk_stamp(tr, 4, tid);
        }
        if (!ok) *abort = 1;
    }
    if (P.final_xsync && P.tp_size > 1) {
        consumer_bar();
        if (!*abort) {
            arrivals += (unsigned)ncta;
            const int one = 1;
            if (!tk_grid_sync(P.bar, arrivals, tid, flag + 4 * (P.nphases & 1), abort, &one, &P,
                              seq * 1024u + (unsigned)P.nphases, cta) && tid == 0)
                *abort = 1;
        }
    }
    consumer_bar();
    if (tid == 0) {
        if (*abort) set_err(err, B2_DEV_ERR_TIMEOUT);
        __threadfence();
        const unsigned t = atomicAdd(P.bar + 1, 1u);
        if (t == (unsigned)ncta - 1) {                  // every CTA is past its last barrier
            if (!*abort) {
                st->pos = pos;
                st->step = pos + 1;
            }
            *P.seq = seq + 1u;
            P.bar[0] = 0u;
            P.bar[1] = 0u;
            __threadfence();
        }
    }
}

// Host side (token.cu, where the kernel is instantiated): set the dynamic shared
// memory of variant (vs, tags) and report how many CTAs fit an SM; launch one step.
cudaError_t tk_prepare(int vs, bool tags, size_t smem, int* per_sm);
cudaError_t tk_launch(int vs, bool tags, const cudaLaunchConfig_t& cfg, const TkParams& P);

}  // namespace b2
