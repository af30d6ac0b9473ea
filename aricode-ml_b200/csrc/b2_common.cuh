// b2_common.cuh — device helpers shared by the decode kernels (sm_100a).
//
// * explicit-rounding arithmetic (no implicit FMA contraction), so every kernel
//   performs exactly the operation sequence written in oracle/refdec.c;
// * own exp in f32/f64 (Cody & Waite reduction + Taylor series), bit-identical to
//   the oracle's b2o_exp_f / b2o_exp_d;
// * PTX wrappers: mbarrier, 1-D bulk async copy (TMA engine), programmatic
//   dependent launch, global timer;
// * bounded waits: every spin carries a ~1 s limit and reports B2_DEV_ERR_TIMEOUT.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace b2 {

// device error codes written to the step state's err word
enum : int {
    B2_DEV_OK = 0,
    B2_DEV_ERR_TIMEOUT = 1,
    B2_DEV_ERR_KV_OVERFLOW = 2,
    B2_DEV_ERR_BAD_TOKEN = 3,
};

constexpr uint64_t kWaitLimitNs = 1000000000ull;   // 1 s per wait

// ------------------------------------------------------------------ arithmetic
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double ddiv(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ double dfma(double a, double b, double c) { return __fma_rn(a, b, c); }

__device__ __forceinline__ float pow2f_bits(int e) { return __int_as_float((e + 127) << 23); }
__device__ __forceinline__ double pow2d_bits(int e) {
    return __longlong_as_double((long long)(e + 1023) << 52);
}

// f32 exp: same steps and constants as b2o_exp_f (oracle/refdec.c)
__device__ __forceinline__ float exp_f(float x) {
    if (x != x) return x;
    if (x > 0x1.62e42ep+6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p+6f) return 0.0f;
    const float kf = rintf(fmul(x, 0x1.715476p+0f));
    float r = ffma(-kf, 0x1.63p-1f, x);
    r = ffma(-kf, -0x1.bd0106p-13f, r);
    float p = 0x1.a01a02p-13f;
    p = ffma(p, r, 0x1.6c16c2p-10f);
    p = ffma(p, r, 0x1.111112p-7f);
    p = ffma(p, r, 0x1.555556p-5f);
    p = ffma(p, r, 0x1.555556p-3f);
    p = ffma(p, r, 0x1.0p-1f);
    p = ffma(p, r, 1.0f);
    p = ffma(p, r, 1.0f);
    const int k = (int)kf;
    if (k > 127) return fmul(fmul(p, pow2f_bits(127)), pow2f_bits(k - 127));
    if (k < -126) return fmul(fmul(p, pow2f_bits(k + 64)), pow2f_bits(-64));
    return fmul(p, pow2f_bits(k));
}

// f64 exp: same steps and constants as b2o_exp_d (clamped to [-700, 700])
__device__ __forceinline__ double exp_d(double x) {
    if (x != x) return x;
    if (x > 700.0) x = 700.0;
    if (x < -700.0) x = -700.0;
    const double kd = rint(dmul(x, 0x1.71547652b82fep+0));
    double r = dfma(-kd, 0x1.62e42p-1, x);
    r = dfma(-kd, 0x1.fdf473de6af28p-22, r);
    double p = 0x1.6124613a86d09p-33;
    p = dfma(p, r, 0x1.1eed8eff8d898p-29);
    p = dfma(p, r, 0x1.ae64567f544e4p-26);
    p = dfma(p, r, 0x1.27e4fb7789f5cp-22);
    p = dfma(p, r, 0x1.71de3a556c734p-19);
    p = dfma(p, r, 0x1.a01a01a01a01ap-16);
    p = dfma(p, r, 0x1.a01a01a01a01ap-13);
    p = dfma(p, r, 0x1.6c16c16c16c17p-10);
    p = dfma(p, r, 0x1.1111111111111p-7);
    p = dfma(p, r, 0x1.5555555555555p-5);
    p = dfma(p, r, 0x1.5555555555555p-3);
    p = dfma(p, r, 0x1.0p-1);
    p = dfma(p, r, 1.0);
    p = dfma(p, r, 1.0);
    return dmul(p, pow2d_bits((int)kd));
}

// silu(g) = g / (1 + exp(-g)) in f64, narrowed to f32 (b2o_silu)
__device__ __forceinline__ float silu_f(float g) {
    const double x = (double)g;
    return (float)ddiv(x, dadd(1.0, exp_d(-x)));
}

// tanh-GELU in f64 with the |2z| > 20 clamp (b2o_gelu / gelu_f32 in the reference)
__device__ __forceinline__ float gelu_f(float xf) {
    const double x = (double)xf;
    const double c = 0.7978845608028654;
    const double inner = dmul(c, dadd(x, dmul(dmul(dmul(0.044715, x), x), x)));
    const double two_inner = dmul(2.0, inner);
    double t;
    if (two_inner > 20.0) t = 1.0;
    else if (two_inner < -20.0) t = -1.0;
    else t = __dsub_rn(1.0, ddiv(2.0, dadd(exp_d(two_inner), 1.0)));
    return (float)dmul(dmul(0.5, x), dadd(1.0, t));
}

// int8 x4 (one 32-bit word) -> exact f32 values via the 2^23 magic number:
// (b ^ 0x80) in the low byte of 0x4B000000 is 2^23 + b + 128; subtracting
// 2^23 + 128 is exact.
__device__ __forceinline__ float i8_to_f(uint32_t u_xored, int i) {
    const uint32_t bits = __byte_perm(u_xored, 0x4B000000u, 0x7440u + (uint32_t)i);
    return fsub(__uint_as_float(bits), 8388736.0f);
}

// 32-lane XOR butterfly (strides 16, 8, 4, 2, 1): v <- v + v[lane ^ s]
__device__ __forceinline__ float butterfly32(float v) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) v = fadd(v, __shfl_xor_sync(0xffffffffu, v, s));
    return v;
}

// ------------------------------------------------------------------ time / errors
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------ PDL
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ------------------------------------------------------------------ mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or ~2 us pass, instead of spinning through issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(2000u) : "memory");
    return ok != 0;
}

// bounded wait on an mbarrier phase; false after ~1 s (caller reports the timeout)
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if ((it & 7u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// (value, tag) words: one aligned 8-byte access carries an f32 and the tag of the
// phase that wrote it, so a reader that sees the tag has the value with it (no
// fence on either side; the tag changes every phase and launch, so an old word
// never passes for a new one)
__device__ __forceinline__ void st_tag(unsigned long long* p, float v, unsigned tag) {
    const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// system scope: the words may come from a peer GPU's stores (tensor parallelism)
__device__ __forceinline__ unsigned long long ld_tag(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ void ld_tag2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool tag_ok(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float tag_val(unsigned long long w) { return __uint_as_float((unsigned)w); }
// the value of a word whose tag must be `tag`: polls (bounded by the deadline;
// false after it, with the last value)
__device__ __forceinline__ bool tag_wait(const unsigned long long* p, unsigned tag, unsigned long long& w,
                                         uint64_t deadline) {
    for (uint32_t it = 0; !tag_ok(w, tag); ++it) {
        if ((it & 15u) == 15u && globaltimer_ns() > deadline) return false;
        w = ld_tag(p);
    }
    return true;
}

// 1-D bulk copy global -> shared (TMA engine), completion signalled on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// L2 prefetch of a global range through the bulk engine (no smem involved)
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ float4 lds128f(const void* p) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(smem_u32(p)));
    return v;
}

// ------------------------------------------------------------------ step state
// Device-resident decode state: the host never writes it between steps, so
// a whole generation replays captured graphs with no host round trips.
struct StepState {
    int step;          // steps executed so far (= position of the next token)
    int pos;           // position of the token being processed by this step
    int prompt_len;    // tokens in the prompt
    int max_new;       // tokens to generate
    int next_tok;      // argmax of the last LM-head step
    int n_out;         // generated ids written to out_ids
    int active;        // 0 once the generation finished (EOS / limit) or failed
    int eos;           // -1: none
    int err;           // B2_DEV_ERR_*
    unsigned rng;      // sampling: LCG state before this step's advance
    int pad[6];
};

// ------------------------------------------------------------------ tensor parallelism
// Up to kMaxRanks GPUs split each matrix by output rows (attention by heads). A
// phase whose output every rank needs writes each value into its own buffer and,
// through NVLink peer mappings, into the same offset of every peer's buffer:
// Mirror holds the byte distance from the local buffer to each peer's copy.
constexpr int kMaxRanks = 8;
struct Mirror {
    long long delta[kMaxRanks - 1];
    int n;                 // peers (0: single GPU)
};

template <typename T>
__device__ __forceinline__ void mirror_store(const Mirror& m, T* p, T v) {
    *p = v;
    for (int i = 0; i < m.n; ++i) *reinterpret_cast<T*>(reinterpret_cast<char*>(p) + m.delta[i]) = v;
}

// a (value, tag) word here and in every peer's copy of the buffer (system scope:
// the peers read them)
__device__ __forceinline__ void mirror_st_tag(const Mirror& m, unsigned long long* p, float v, unsigned tag) {
    const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
    if (m.n == 0) {
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
        return;
    }
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
    for (int i = 0; i < m.n; ++i)
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(reinterpret_cast<char*>(p) + m.delta[i]), "l"(w)
                     : "memory");
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Publish epoch e in slot `rank` of the flag array f on every rank, then wait
// until every rank's slot has reached e (wrap-safe). One system-scope fence
// before the relaxed flag stores makes them a release: every write this thread
// has observed (the other CTAs' outputs and peer copies, acquired through the
// local grid barrier) is visible on every rank before its flag. Bounded: false
// after ~1 s.
__device__ __forceinline__ bool tp_flag_exchange(unsigned* f, int rank, int nranks, const Mirror& m, unsigned e) {
    __threadfence_system();
    st_relaxed_sys(f + rank, e);
    for (int i = 0; i < m.n; ++i)
        st_relaxed_sys(reinterpret_cast<unsigned*>(reinterpret_cast<char*>(f + rank) + m.delta[i]), e);
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        bool all = true;
        for (int r = 0; r < nranks; ++r) all = all && (int)(ld_acquire_sys(f + r) - e) >= 0;
        if (all) return true;
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

}  // namespace b2
