/*
 * refdec.c — CPU oracle for the int8 decoder decode path (see refdec.h).
 *
 * TEST INFRASTRUCTURE: loaded only by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py. Never part of the product path.
 *
 * Build: gcc -O2 -march=x86-64-v3 -ffp-contract=off -pthread -fPIC -shared (Makefile)
 * (-ffp-contract=off keeps every a*b+c as two roundings unless written fmaf();
 * the CUDA kernels use __fmul_rn/__fadd_rn/__fmaf_rn for the same reason).
 */
#include "refdec.h"

#include <math.h>
#include <pthread.h>
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#endif
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------
 * Tiny persistent thread pool: parallel_for(n, fn, ctx) splits [0,n) into
 * g_threads contiguous ranges. Every row / head is computed by exactly one
 * thread in the same order, so results do not depend on the thread count.
 * ------------------------------------------------------------------------ */
typedef void (*range_fn)(void* ctx, int64_t i0, int64_t i1);

static int g_threads = 1;
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t g_cv_job = PTHREAD_COND_INITIALIZER;
static pthread_cond_t g_cv_done = PTHREAD_COND_INITIALIZER;
static int g_pool_size = 0;              /* worker threads alive (excl. caller) */
static uint64_t g_job_gen = 0;
static int g_job_pending = 0;
static range_fn g_job_fn;
static void* g_job_ctx;
static int64_t g_job_n;
static int g_job_parts;

static void run_part(int part) {
    const int64_t per = (g_job_n + g_job_parts - 1) / g_job_parts;
    const int64_t i0 = (int64_t)part * per;
    int64_t i1 = i0 + per;
    if (i1 > g_job_n) i1 = g_job_n;
    if (i0 < i1) g_job_fn(g_job_ctx, i0, i1);
}

static void* worker_main(void* arg) {
    const int part = (int)(intptr_t)arg;        /* 1..pool_size */
    uint64_t seen = 0;
    pthread_mutex_lock(&g_mu);
    for (;;) {
        while (g_job_gen == seen) pthread_cond_wait(&g_cv_job, &g_mu);
        seen = g_job_gen;
        const int active = part < g_job_parts;
        pthread_mutex_unlock(&g_mu);
        if (active) run_part(part);
        pthread_mutex_lock(&g_mu);
        if (active && --g_job_pending == 0) pthread_cond_signal(&g_cv_done);
    }
    return NULL;
}

static void parallel_for(int64_t n, range_fn fn, void* ctx) {
    const int parts = g_threads;
    if (parts <= 1 || n < 2) { fn(ctx, 0, n); return; }
    pthread_mutex_lock(&g_mu);
    while (g_pool_size < parts - 1) {
        pthread_t th;
        if (pthread_create(&th, NULL, worker_main, (void*)(intptr_t)(g_pool_size + 1)) != 0) break;
        pthread_detach(th);
        g_pool_size++;
    }
    const int use = g_pool_size + 1 < parts ? g_pool_size + 1 : parts;
    g_job_fn = fn; g_job_ctx = ctx; g_job_n = n; g_job_parts = use;
    g_job_pending = use - 1;
    g_job_gen++;
    pthread_cond_broadcast(&g_cv_job);
    pthread_mutex_unlock(&g_mu);
    run_part(0);
    pthread_mutex_lock(&g_mu);
    while (g_job_pending > 0) pthread_cond_wait(&g_cv_done, &g_mu);
    pthread_mutex_unlock(&g_mu);
}

void b2o_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int  b2o_get_threads(void) { return g_threads; }

/* ------------------------------------------------------------------------
 * exp, own implementation (no libm exp on the compared path).
 * Method: Cody & Waite argument reduction x = k*ln2 + r with a two-piece ln2
 * (hi piece short enough that k*hi is exact), exp(r) by its Taylor series in
 * Horner form with fused multiply-adds, then an exact scale by 2^k built from
 * exponent bits. Coefficients are 1/i! rounded to the working precision.
 * Identical operation sequence in aricode-ml_b200/csrc/b2_math.cuh.
 * ------------------------------------------------------------------------ */
static inline float pow2f_bits(int e) { /* 2^e for -126 <= e <= 127 */
    union { uint32_t u; float f; } v; v.u = (uint32_t)(e + 127) << 23; return v.f;
}
static inline double pow2d_bits(int e) { /* 2^e for -1022 <= e <= 1023 */
    union { uint64_t u; double f; } v; v.u = (uint64_t)(e + 1023) << 52; return v.f;
}

float b2o_exp_f(float x) {
    if (x != x) return x;
    if (x > 0x1.62e42ep+6f) return INFINITY;          /* > ln(FLT_MAX) */
    if (x < -0x1.9fe368p+6f) return 0.0f;             /* < ln(2^-150) */
    const float kf = rintf(x * 0x1.715476p+0f);       /* round(x*log2 e) */
    float r = fmaf(-kf, 0x1.63p-1f, x);               /* ln2 hi = 0.693359375 */
    r = fmaf(-kf, -0x1.bd0106p-13f, r);               /* ln2 lo */
    float p = 0x1.a01a02p-13f;                        /* 1/7! */
    p = fmaf(p, r, 0x1.6c16c2p-10f);                  /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f);                   /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f);                   /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f);                   /* 1/3! */
    p = fmaf(p, r, 0x1.0p-1f);                        /* 1/2! */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = (int)kf;
    if (k > 127) return (p * pow2f_bits(127)) * pow2f_bits(k - 127);
    if (k < -126) return (p * pow2f_bits(k + 64)) * pow2f_bits(-64);
    return p * pow2f_bits(k);
}

double b2o_exp_d(double x) {
    if (x != x) return x;
    if (x > 700.0) x = 700.0;                         /* reference math_exp clamp */
    if (x < -700.0) x = -700.0;
    const double kd = rint(x * 0x1.71547652b82fep+0);
    double r = fma(-kd, 0x1.62e42p-1, x);             /* ln2 hi (k*hi exact) */
    r = fma(-kd, 0x1.fdf473de6af28p-22, r);           /* ln2 lo */
    double p = 0x1.6124613a86d09p-33;                 /* 1/13! */
    p = fma(p, r, 0x1.1eed8eff8d898p-29);             /* 1/12! */
    p = fma(p, r, 0x1.ae64567f544e4p-26);             /* 1/11! */
    p = fma(p, r, 0x1.27e4fb7789f5cp-22);             /* 1/10! */
    p = fma(p, r, 0x1.71de3a556c734p-19);             /* 1/9!  */
    p = fma(p, r, 0x1.a01a01a01a01ap-16);             /* 1/8!  */
    p = fma(p, r, 0x1.a01a01a01a01ap-13);             /* 1/7!  */
    p = fma(p, r, 0x1.6c16c16c16c17p-10);             /* 1/6!  */
    p = fma(p, r, 0x1.1111111111111p-7);              /* 1/5!  */
    p = fma(p, r, 0x1.5555555555555p-5);              /* 1/4!  */
    p = fma(p, r, 0x1.5555555555555p-3);              /* 1/3!  */
    p = fma(p, r, 0x1.0p-1);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    return p * pow2d_bits((int)kd);
}

/* silu via f64 promote-then-narrow (reference: arr_f32_silu, aricode_pack.py:614-625) */
float b2o_silu(float g) {
    const double x = (double)g;
    return (float)(x / (1.0 + b2o_exp_d(-x)));
}

/* tanh-GELU exactly as gelu_f32 (aricode_pack.py:539-572), f64 scalar code */
float b2o_gelu(float xf) {
    const double x = (double)xf;
    const double c = 0.7978845608028654;
    const double inner = c * (x + 0.044715 * x * x * x);
    const double two_inner = 2.0 * inner;
    double t;
    if (two_inner > 20.0) t = 1.0;
    else if (two_inner < -20.0) t = -1.0;
    else t = 1.0 - 2.0 / (b2o_exp_d(two_inner) + 1.0);
    return (float)(0.5 * x * (1.0 + t));
}

/* ------------------------------------------------------------------------
 * Quantiser — tools/aricode_pack.py:3356-3379 with numpy float32 semantics:
 *   scale = max|row| / 127 (f32), safe = scale>0 ? scale : 1,
 *   q = clip(round_half_even(row / safe), -128, 127); stored scale keeps 0.
 * ------------------------------------------------------------------------ */
void b2o_quantize_rows(const float* W, int64_t m, int64_t n,
                       int8_t* q, int64_t ldq, float* scale) {
    for (int64_t r = 0; r < m; ++r) {
        const float* row = W + r * n;
        float mx = 0.0f;
        for (int64_t c = 0; c < n; ++c) { float a = fabsf(row[c]); if (a > mx) mx = a; }
        const float s = mx / 127.0f;
        const float safe = s > 0.0f ? s : 1.0f;
        int8_t* qr = q + r * ldq;
        for (int64_t c = 0; c < n; ++c) {
            float v = rintf(row[c] / safe);
            if (v < -128.0f) v = -128.0f;
            if (v > 127.0f) v = 127.0f;
            qr[c] = (int8_t)v;
        }
        for (int64_t c = n; c < ldq; ++c) qr[c] = 0;
        scale[r] = s;
    }
}

/* ------------------------------------------------------------------------
 * 256-partial reduction (norms and dot products): partial j sits in warp j/32,
 * lane j%32; each warp butterflies (XOR strides 16, 8, 4, 2, 1:
 * p[L] <- p[L] + p[L^s]); warps combine as ((W0+W1)+(W2+W3)) + ((W4+W5)+(W6+W7)).
 * ------------------------------------------------------------------------ */
static float butterfly32(float* p) {
    float t[32];
    for (int s = 16; s >= 1; s >>= 1) {
        for (int L = 0; L < 32; ++L) t[L] = p[L] + p[L ^ s];
        memcpy(p, t, sizeof(t));
    }
    return p[0];
}

static float reduce256(float* s) {
    float W[8];
    for (int w = 0; w < 8; ++w) W[w] = butterfly32(s + 32 * w);
    return ((W[0] + W[1]) + (W[2] + W[3])) + ((W[4] + W[5]) + (W[6] + W[7]));
}

/* ------------------------------------------------------------------------
 * int8 rows (arr_i8_matvec_f32_perrow; call sites tools/aricode_pack.py:183,
 * :1789-1808, attention_gqa_kv_i8.ari:149-151): the dot product is computed
 * exactly on a fixed-point copy of x and rounded once, so it has no association
 * order (integer sums are exact in any order) and any thread layout on the GPU
 * gives these bits:
 *   max|x| < 2^E (frexp exponent), S = 31 - E, X_i = trunc(x_i * 2^S), |X_i| < 2^31;
 *   D = sum_i w_i * X_i (exact in int64), dot = f32((double)D * 2^-S), one rounding;
 *   y = dot * scale (f32).
 * Truncating x to 31 bits below its largest element errs by at most 2^-31 max|x|
 * per element, far below the rounding of an f32 accumulation. A NaN or an
 * infinity in x makes every row NaN.
 * ------------------------------------------------------------------------ */
int b2o_xfix(const float* x, int64_t n, int32_t* X) {
    uint32_t amax = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        u &= 0x7fffffffu;                       /* non-negative floats order as their bits */
        if (u > amax) amax = u;
    }
    if (amax >= 0x7f800000u) return B2O_XFIX_BAD;
    if (amax == 0) {
        memset(X, 0, (size_t)n * sizeof(int32_t));
        return 0;
    }
    float am;
    memcpy(&am, &amax, 4);
    int E;
    frexp((double)am, &E);
    const int S = 31 - E;
    const double p = ldexp(1.0, S);
    for (int64_t i = 0; i < n; ++i) X[i] = (int32_t)((double)x[i] * p);   /* exact product, truncation */
    return S;
}

float b2o_dot_i8x(const int8_t* w, const int32_t* X, int64_t n, int S) {
    if (S == B2O_XFIX_BAD) return NAN;
    int64_t D = 0;
    for (int64_t i = 0; i < n; ++i) D += (int64_t)w[i] * (int64_t)X[i];
    return (float)((double)D * ldexp(1.0, -S));
}

/* ------------------------------------------------------------------------
 * f32 rows, shared order (the CUDA GEMV uses the same):
 *  - the row is viewed as 16-byte blocks (4 f32); elements past n are 0 and so
 *    is x there;
 *  - slot s in 0..255 owns blocks s, s+256, s+512, ... in ascending order and
 *    keeps four accumulators a[t] over element t of each block (fused
 *    multiply-add); slot partial = (a0 + a1) + (a2 + a3);
 *  - the 256 slot partials go through reduce256().
 * ------------------------------------------------------------------------ */
float b2o_dot_f32(const float* w, const float* x, int64_t n) {
    const int64_t nblk = (n + 3) / 4;
    float part[256];
    for (int sl = 0; sl < 256; ++sl) {
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t b = sl; b < nblk; b += 256) {
            for (int t = 0; t < 4; ++t) {
                const int64_t k = 4 * b + t;
                const float wv = k < n ? w[k] : 0.0f;
                const float xv = k < n ? x[k] : 0.0f;
                a[t] = fmaf(wv, xv, a[t]);
            }
        }
        part[sl] = (a[0] + a[1]) + (a[2] + a[3]);
    }
    return reduce256(part);
}

/* ------------------------------------------------------------------------
 * Two more restatements of the int8 matvec, used to measure how far the exact
 * fixed-point dot above (the one the GPU reproduces bit for bit) sits from the
 * reference's own arithmetic and from a high-precision truth:
 *
 *  - f32 accumulation as README.md:128-131 describes the builtin
 *    arr_i8_matvec_f32(_perrow): 8 codes sign-extended (vpmovsxbd), converted to
 *    f32 (vcvtdq2ps), one vfmadd231ps per 8 lanes into one accumulator vector,
 *    lane l holding the elements 8b + l. The builtin's source (codegen_builtins.c
 *    of the aric compiler) is not in the reference tree, so its horizontal sum
 *    and tail handling are restated in the usual AVX2 form: fold the upper 128
 *    bits onto the lower (l, l+4), then the upper 64 (l, l+2), then the odd lane,
 *    i.e. ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)); the n % 8 tail elements follow
 *    one by one with fmaf. Then y = dot * scale.
 *  - f64 accumulation: every product and sum in double, rounded to f32 once
 *    after the scale (truth model for the matvec; everything else in the model
 *    keeps the reference's f32 arithmetic).
 *
 * b2o_set_matvec_mode selects which one b2o_gemv_i8 and the whole-model step
 * use: 0 the fixed-point dot (default), 1 f32 accumulation, 2 f64. Mode 2 also
 * takes the f32-weight projections in f64.
 * ------------------------------------------------------------------------ */
static int g_matvec_mode = 0;
void b2o_set_matvec_mode(int mode) { g_matvec_mode = (mode >= 0 && mode <= 2) ? mode : 0; }
int  b2o_get_matvec_mode(void) { return g_matvec_mode; }

float b2o_dot_i8_f32acc(const int8_t* w, const float* x, int64_t n) {
    float a[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const int64_t n8 = n / 8 * 8;
#if defined(__AVX2__) && defined(__FMA__)
    /* the described instruction sequence itself: vpmovsxbd, vcvtdq2ps, vfmadd231ps */
    __m256 acc = _mm256_setzero_ps();
    for (int64_t b = 0; b < n8; b += 8) {
        const __m256i wi = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + b)));
        acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(wi), _mm256_loadu_ps(x + b), acc);
    }
    _mm256_storeu_ps(a, acc);
#else
    for (int64_t b = 0; b < n8; b += 8)
        for (int l = 0; l < 8; ++l) a[l] = fmaf((float)w[b + l], x[b + l], a[l]);
#endif
    float t = ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
    for (int64_t i = n8; i < n; ++i) t = fmaf((float)w[i], x[i], t);
    return t;
}

double b2o_dot_i8_f64(const int8_t* w, const float* x, int64_t n) {
    double t = 0.0;
    for (int64_t i = 0; i < n; ++i) t += (double)w[i] * (double)x[i];
    return t;
}

static double dot_f32_f64(const float* w, const float* x, int64_t n) {
    double t = 0.0;
    for (int64_t i = 0; i < n; ++i) t += (double)w[i] * (double)x[i];
    return t;
}

typedef struct {
    const void* W; int64_t ld; const float* scale; const float* x; int64_t n; float* y;
    const int32_t* X; int S; int mode;
} gemv_ctx;

static void gemv_i8_range(void* c, int64_t r0, int64_t r1) {
    const gemv_ctx* g = (const gemv_ctx*)c;
    const int8_t* W = (const int8_t*)g->W;
    if (g->mode == 1)
        for (int64_t r = r0; r < r1; ++r) g->y[r] = b2o_dot_i8_f32acc(W + r * g->ld, g->x, g->n) * g->scale[r];
    else if (g->mode == 2)
        for (int64_t r = r0; r < r1; ++r)
            g->y[r] = (float)(b2o_dot_i8_f64(W + r * g->ld, g->x, g->n) * (double)g->scale[r]);
    else
        for (int64_t r = r0; r < r1; ++r) g->y[r] = b2o_dot_i8x(W + r * g->ld, g->X, g->n, g->S) * g->scale[r];
}
static void gemv_f32_range(void* c, int64_t r0, int64_t r1) {
    const gemv_ctx* g = (const gemv_ctx*)c;
    const float* W = (const float*)g->W;
    if (g->mode == 2)
        for (int64_t r = r0; r < r1; ++r) g->y[r] = (float)dot_f32_f64(W + r * g->ld, g->x, g->n);
    else
        for (int64_t r = r0; r < r1; ++r) g->y[r] = b2o_dot_f32(W + r * g->ld, g->x, g->n);
}

void b2o_gemv_i8(const int8_t* W, int64_t ld, const float* scale, const float* x,
                 int64_t m, int64_t n, float* y) {
    int32_t* X = NULL;
    int S = 0;
    if (g_matvec_mode == 0) {
        X = (int32_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
        if (!X) abort();
        S = b2o_xfix(x, n, X);
    }
    gemv_ctx g = {W, ld, scale, x, n, y, X, S, g_matvec_mode};
    parallel_for(m, gemv_i8_range, &g);
    free(X);
}

void b2o_gemv_f32(const float* W, int64_t ld, const float* x,
                  int64_t m, int64_t n, float* y) {
    gemv_ctx g = {W, ld, NULL, x, n, y, NULL, 0, g_matvec_mode};
    parallel_for(m, gemv_f32_range, &g);
}

/* int4 rows: the reference's builtin unpacks each row's nibbles into int8 (low
 * nibble = even column, sign-extended) and runs its int8 dot on them
 * (aricode_pack.py:168-181); here the unpacked row goes through the selected int8
 * matvec mode. */
void b2o_unpack_i4(const uint8_t* packed, int64_t n, int8_t* codes) {
    for (int64_t i = 0; i < n; ++i) {
        const int v = (packed[i >> 1] >> ((i & 1) * 4)) & 15;
        codes[i] = (int8_t)((v ^ 8) - 8);
    }
}

typedef struct { const uint8_t* W; int64_t ld; const float* scale; const float* x; int64_t n; float* y;
                 const int32_t* X; int S; int mode; } gemv4_ctx;

static void gemv_i4_range(void* c, int64_t r0, int64_t r1) {
    const gemv4_ctx* g = (const gemv4_ctx*)c;
    int8_t* row = (int8_t*)malloc((size_t)(g->n > 0 ? g->n : 1));
    if (!row) abort();
    for (int64_t r = r0; r < r1; ++r) {
        b2o_unpack_i4(g->W + r * g->ld, g->n, row);
        if (g->mode == 1) g->y[r] = b2o_dot_i8_f32acc(row, g->x, g->n) * g->scale[r];
        else if (g->mode == 2) g->y[r] = (float)(b2o_dot_i8_f64(row, g->x, g->n) * (double)g->scale[r]);
        else g->y[r] = b2o_dot_i8x(row, g->X, g->n, g->S) * g->scale[r];
    }
    free(row);
}

void b2o_gemv_i4(const uint8_t* W, int64_t ld, const float* scale, const float* x,
                 int64_t m, int64_t n, float* y) {
    int32_t* X = NULL;
    int S = 0;
    if (g_matvec_mode == 0) {
        X = (int32_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
        if (!X) abort();
        S = b2o_xfix(x, n, X);
    }
    gemv4_ctx g = {W, ld, scale, x, n, y, X, S, g_matvec_mode};
    parallel_for(m, gemv_i4_range, &g);
    free(X);
}

/* rmsnorm_affine_f32 (aricode_pack.py:585-607): x * (1/sqrt(mean(x^2)+eps)), then * g */
void b2o_rmsnorm(const float* x, const float* g, int d, float eps, float* y) {
    float s[256];
    for (int j = 0; j < 256; ++j) {
        float a = 0.0f;
        for (int i = j; i < d; i += 256) a = fmaf(x[i], x[i], a);
        s[j] = a;
    }
    const float ms = reduce256(s) / (float)d;
    const float inv = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < d; ++i) y[i] = (x[i] * inv) * g[i];
}

/* layernorm_affine_f32 (aricode_pack.py:503-521): two-pass stats, affine in f64 */
void b2o_layernorm(const float* x, const float* g, const float* b, int d, float eps, float* y) {
    float s[256];
    for (int j = 0; j < 256; ++j) {
        float a = 0.0f;
        for (int i = j; i < d; i += 256) a = a + x[i];
        s[j] = a;
    }
    const float mean = reduce256(s) / (float)d;
    for (int j = 0; j < 256; ++j) {
        float a = 0.0f;
        for (int i = j; i < d; i += 256) { const float dx = x[i] - mean; a = fmaf(dx, dx, a); }
        s[j] = a;
    }
    const float var = reduce256(s) / (float)d;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < d; ++i) {
        const float t = (x[i] - mean) * inv;
        y[i] = (float)((double)t * (double)g[i] + (double)b[i]);
    }
}

/* ------------------------------------------------------------------------
 * RoPE — rope_f32.ari:34-55 (table in f64, stored f32) and :69-72 (interleaved pairs)
 * ------------------------------------------------------------------------ */
void b2o_rope_table(int max_seq, int d_head, double theta, float* table) {
    const double log_theta = log(theta);
    const int half = d_head / 2;
    for (int pos = 0; pos < max_seq; ++pos) {
        for (int i = 0; i < half; ++i) {
            const double exponent = 0.0 - 2.0 * (double)i / (double)d_head;
            const double freq = exp(exponent * log_theta);
            const double angle = (double)pos * freq;
            table[pos * d_head + 2 * i] = (float)cos(angle);
            table[pos * d_head + 2 * i + 1] = (float)sin(angle);
        }
    }
}

void b2o_rope_apply(float* v, const float* table, int pos, int d_head) {
    const float* row = table + (int64_t)pos * d_head;
    for (int i = 0; i < d_head / 2; ++i) {
        const float x0 = v[2 * i], x1 = v[2 * i + 1];
        const float c = row[2 * i], s = row[2 * i + 1];
        v[2 * i] = x0 * c - x1 * s;
        v[2 * i + 1] = x0 * s + x1 * c;
    }
}

/* ------------------------------------------------------------------------
 * Decode attention for one step — restates _gqa_score_head_i8
 * (attention_gqa_kv_i8.ari:97-117): scores = Kc[0..n]·q, the max_seq-n inactive
 * tail entries are -60, softmax over all max_seq, out = Vc[0..n]^T p.
 * Split order shared with the CUDA kernel (chunks of B2O_ATT_CHUNK keys):
 *   score_j   : 32-lane dot, lane L sums d = L, L+32, ... by fmaf, butterfly;
 *   m_s       : max of the chunk's scores;
 *   e_j       : exp_f(score_j - m_s);
 *   l_s       : lane L adds e_{j0+L}, e_{j0+L+32}, ... ; butterfly;
 *   o_s[d]    : fmaf over j ascending;
 *   combine   : M = max_s m_s (and -60 when n < max_seq); w_s = exp_f(m_s - M);
 *               l = fmaf(l_s, w_s, l), o = fmaf(o_s, w_s, o) over s ascending;
 *               tail: l = fmaf(max_seq - n, exp_f(-60 - M), l); out = o / l.
 * ------------------------------------------------------------------------ */
static void attn_head(const float* q, const float* K, const float* V, int dh, int n,
                      int max_seq, float* out) {
    const int nsplit = n < 1 ? 1 : (n + B2O_ATT_CHUNK - 1) / B2O_ATT_CHUNK;
    float* ms = (float*)malloc(sizeof(float) * (size_t)nsplit);
    float* ls = (float*)malloc(sizeof(float) * (size_t)nsplit);
    float* os = (float*)malloc(sizeof(float) * (size_t)nsplit * (size_t)dh);
    float sc[B2O_ATT_CHUNK], e[B2O_ATT_CHUNK];
    for (int s = 0; s < nsplit; ++s) {
        const int j0 = s * B2O_ATT_CHUNK;
        const int len = (n - j0) < B2O_ATT_CHUNK ? (n - j0) : B2O_ATT_CHUNK;
        for (int jj = 0; jj < len; ++jj) {
            const float* kr = K + (int64_t)(j0 + jj) * dh;
            float p[32];
            for (int L = 0; L < 32; ++L) {
                float a = 0.0f;
                for (int d = L; d < dh; d += 32) a = fmaf(q[d], kr[d], a);
                p[L] = a;
            }
            sc[jj] = butterfly32(p);
        }
        float m = sc[0];
        for (int jj = 1; jj < len; ++jj) m = fmaxf(m, sc[jj]);
        for (int jj = 0; jj < len; ++jj) e[jj] = b2o_exp_f(sc[jj] - m);
        float p[32];
        for (int L = 0; L < 32; ++L) {
            float a = 0.0f;
            for (int jj = L; jj < len; jj += 32) a = a + e[jj];
            p[L] = a;
        }
        ms[s] = m;
        ls[s] = butterfly32(p);
        for (int d = 0; d < dh; ++d) {
            float a = 0.0f;
            for (int jj = 0; jj < len; ++jj) a = fmaf(e[jj], V[(int64_t)(j0 + jj) * dh + d], a);
            os[(int64_t)s * dh + d] = a;
        }
    }
    float M = ms[0];
    for (int s = 1; s < nsplit; ++s) M = fmaxf(M, ms[s]);
    if (n < max_seq) M = fmaxf(M, -60.0f);
    float l = 0.0f;
    for (int d = 0; d < dh; ++d) out[d] = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
        const float w = b2o_exp_f(ms[s] - M);
        l = fmaf(ls[s], w, l);
        for (int d = 0; d < dh; ++d) out[d] = fmaf(os[(int64_t)s * dh + d], w, out[d]);
    }
    if (n < max_seq) l = fmaf((float)(max_seq - n), b2o_exp_f(-60.0f - M), l);
    for (int d = 0; d < dh; ++d) out[d] = out[d] / l;
    free(ms); free(ls); free(os);
}

typedef struct { const float *q, *Kc, *Vc; int group, d_head, n, max_seq; float* out; } attn_ctx;

static void attn_range(void* c, int64_t h0, int64_t h1) {
    const attn_ctx* a = (const attn_ctx*)c;
    for (int64_t h = h0; h < h1; ++h) {
        const int64_t off = (h / a->group) * (int64_t)a->max_seq * a->d_head;
        attn_head(a->q + h * a->d_head, a->Kc + off, a->Vc + off, a->d_head, a->n, a->max_seq,
                  a->out + h * a->d_head);
    }
}

void b2o_attn_decode(const float* q, const float* Kc, const float* Vc,
                     int n_heads, int n_kv_heads, int d_head, int n, int max_seq,
                     float* out) {
    attn_ctx a = {q, Kc, Vc, n_heads / n_kv_heads, d_head, n, max_seq, out};
    parallel_for(n_heads, attn_range, &a);
}

/* sample_greedy_f32 (sampling_f32.ari:10-24): strict '>' -> first max wins, NaN never wins */
int32_t b2o_argmax(const float* v, int64_t n) {
    float best = v[0];
    int32_t bi = 0;
    for (int64_t i = 1; i < n; ++i)
        if (v[i] > best) { best = v[i]; bi = (int32_t)i; }
    return bi;
}

/* ------------------------------------------------------------------------
 * Sampling beyond greedy (sampling_f32.ari:31-153, driven by the decoder loop at
 * aricode_pack.py:2186-2306):
 *   rng_state = rng_state * 1103515245 + 12345  (32-bit wrap-around), then
 *   unit = (rng_state & 65535) / 65536.0, advanced once per loop step (prompt
 *   steps included: the loop evaluates the head and samples on every step);
 *   topk:K:T first keeps the K largest distinct values (K passes of "largest
 *   value below the previous one", values below the K-th become -1e6; K <= 0
 *   keeps only the first maximum, K >= n changes nothing);
 *   temperature T <= 0 returns the greedy id; otherwise l = f32(l * (1/T)),
 *   e = exp(l - max) in f64 stored as f32 while the f64 e's are summed in index
 *   order, p = f32(p * (1/sum)), and the id is the first whose running f64 sum of
 *   p exceeds unit (n - 1 if none does). The f64 exp is b2o_exp_d (the aric
 *   compiler's math_exp is not in the reference tree).
 * ------------------------------------------------------------------------ */
uint32_t b2o_lcg_next(uint32_t state) { return state * 1103515245u + 12345u; }

void b2o_topk_filter(float* l, int64_t n, int k) {
    if (k >= n) return;
    if (k <= 0) {
        const int32_t best = b2o_argmax(l, n);
        for (int64_t j = 0; j < n; ++j)
            if (j != best) l[j] = -1.0e6f;
        return;
    }
    double prev = 1.0e30, kth = (double)l[0];
    for (int pass = 0; pass < k; ++pass) {
        double cur = -1.0e30;
        for (int64_t i = 0; i < n; ++i) {
            const double v = (double)l[i];
            if (v < prev && v > cur) cur = v;
        }
        kth = cur;
        prev = cur;
    }
    for (int64_t j = 0; j < n; ++j)
        if ((double)l[j] < kth) l[j] = -1.0e6f;
}

int32_t b2o_sample_temperature(float* l, int64_t n, double temperature, double unit) {
    if (temperature <= 0.0) return b2o_argmax(l, n);
    const double inv_t = 1.0 / temperature;
    for (int64_t i = 0; i < n; ++i) l[i] = (float)((double)l[i] * inv_t);
    double mx = (double)l[0];
    for (int64_t i = 1; i < n; ++i)
        if ((double)l[i] > mx) mx = (double)l[i];
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double e = b2o_exp_d((double)l[i] - mx);
        l[i] = (float)e;
        sum = sum + e;
    }
    const double inv_sum = 1.0 / sum;
    for (int64_t i = 0; i < n; ++i) l[i] = (float)((double)l[i] * inv_sum);
    double cum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        cum = cum + (double)l[i];
        if (cum > unit) return (int32_t)i;
    }
    return (int32_t)(n - 1);
}

int32_t b2o_sample(float* l, int64_t n, int mode, int top_k, double temperature, uint32_t* rng) {
    if (mode == B2O_SAMPLE_GREEDY) return b2o_argmax(l, n);
    if (mode == B2O_SAMPLE_TOPK) b2o_topk_filter(l, n, top_k);
    *rng = b2o_lcg_next(*rng);
    const double unit = (double)(int32_t)(*rng & 65535u) / 65536.0;
    return b2o_sample_temperature(l, n, temperature, unit);
}

/* ------------------------------------------------------------------------
 * Synthetic weights: splitmix64 of a (seed, tensor, index) key; four 16-bit
 * uniforms summed (Irwin-Hall(4), centred) and scaled to the requested std.
 * Integer maths + one f32 multiply, so the GPU generator is bit-identical.
 * ------------------------------------------------------------------------ */
static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float b2o_synth_value(uint64_t seed, uint64_t tensor_id, uint64_t index, float stdv) {
    const uint64_t key = seed * 0xD1B54A32D192ED03ull + tensor_id * 0xA0761D6478BD642Full + index;
    const uint64_t z = splitmix64(key);
    const int32_t s = (int32_t)(z & 0xFFFF) + (int32_t)((z >> 16) & 0xFFFF) +
                      (int32_t)((z >> 32) & 0xFFFF) + (int32_t)(z >> 48) - 131070;
    const float c = stdv * 0x1.bb67aep-16f;           /* 1/std of the centred sum */
    return (float)s * c;
}

typedef struct { uint64_t seed, tid; int64_t n; float stdv; int64_t r0, c0, c1, ldq; int8_t* q; float* scale; float* out; } synth_ctx;

static void synth_fill_range(void* c, int64_t r0, int64_t r1) {
    const synth_ctx* s = (const synth_ctx*)c;
    for (int64_t r = r0; r < r1; ++r)
        for (int64_t k = 0; k < s->n; ++k)
            s->out[r * s->n + k] = b2o_synth_value(s->seed, s->tid, (uint64_t)(r * s->n + k), s->stdv);
}

void b2o_synth_fill_f32(uint64_t seed, uint64_t tensor_id, int64_t m, int64_t n,
                        float stdv, float* out) {
    synth_ctx s = {seed, tensor_id, n, stdv, 0, 0, 0, 0, NULL, NULL, out};
    parallel_for(m, synth_fill_range, &s);
}

static void synth_quant_range(void* c, int64_t i0, int64_t i1);

void b2o_synth_quant_rows(uint64_t seed, uint64_t tensor_id, int64_t n, float stdv,
                          int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                          int8_t* q, int64_t ldq, float* scale) {
    synth_ctx s = {seed, tensor_id, n, stdv, r0, c0, c1, ldq, q, scale, NULL};
    parallel_for(r1 - r0, synth_quant_range, &s);
}

static void synth_quant_range(void* cv, int64_t i0, int64_t i1) {
    const synth_ctx* S = (const synth_ctx*)cv;
    const uint64_t seed = S->seed, tensor_id = S->tid;
    const int64_t n = S->n, r0 = S->r0, c0 = S->c0, c1 = S->c1, ldq = S->ldq;
    const float stdv = S->stdv;
    int8_t* q = S->q; float* scale = S->scale;
    for (int64_t r = r0 + i0; r < r0 + i1; ++r) {
        float mx = 0.0f;
        for (int64_t c = 0; c < n; ++c) {
            const float a = fabsf(b2o_synth_value(seed, tensor_id, (uint64_t)(r * n + c), stdv));
            if (a > mx) mx = a;
        }
        const float s = mx / 127.0f;
        const float safe = s > 0.0f ? s : 1.0f;
        int8_t* qr = q + (r - r0) * ldq;
        for (int64_t c = c0; c < c1; ++c) {
            float v = rintf(b2o_synth_value(seed, tensor_id, (uint64_t)(r * n + c), stdv) / safe);
            if (v < -128.0f) v = -128.0f;
            if (v > 127.0f) v = 127.0f;
            qr[c - c0] = (int8_t)v;
        }
        for (int64_t c = c1 - c0; c < ldq; ++c) qr[c] = 0;
        scale[r - r0] = s;
    }
}

/* ------------------------------------------------------------------------
 * Whole decoder — gen_decoder_main (aricode_pack.py:2068-2344) with the
 * per-token forward of gen_forward (aricode_pack.py:1629-2032).
 * ------------------------------------------------------------------------ */
int b2o_state_init(const b2o_model* m, b2o_state* s) {
    memset(s, 0, sizeof(*s));
    s->n_slots = m->n_kv_slots;
    s->K = (float**)calloc((size_t)m->n_kv_slots, sizeof(float*));
    s->V = (float**)calloc((size_t)m->n_kv_slots, sizeof(float*));
    s->kv_elems = (size_t*)calloc((size_t)m->n_kv_slots, sizeof(size_t));
    if (!s->K || !s->V || !s->kv_elems) return -1;
    for (int b = 0; b < m->n_blocks; ++b) {
        const b2o_block* B = &m->blocks[b];
        if (B->type != B2O_SB_ATTN) continue;
        const size_t e = (size_t)B->n_kv_heads * m->max_seq * B->d_head;
        s->kv_elems[B->kv_slot] = e;
        s->K[B->kv_slot] = (float*)calloc(e, sizeof(float));
        s->V[B->kv_slot] = (float*)calloc(e, sizeof(float));
        if (!s->K[B->kv_slot] || !s->V[B->kv_slot]) return -1;
    }
    s->x = (float*)calloc((size_t)m->d, sizeof(float));
    s->h = (float*)calloc((size_t)m->d, sizeof(float));
    s->q = (float*)calloc((size_t)m->max_heads, sizeof(float));
    s->k = (float*)calloc((size_t)m->max_kv_dim, sizeof(float));
    s->v = (float*)calloc((size_t)m->max_kv_dim, sizeof(float));
    s->att = (float*)calloc((size_t)m->max_heads, sizeof(float));
    s->f1 = (float*)calloc((size_t)m->max_ffn + 1, sizeof(float));
    s->f3 = (float*)calloc((size_t)m->max_ffn + 1, sizeof(float));
    s->logits = (float*)calloc((size_t)m->vocab, sizeof(float));
    s->count = 0;
    return (s->x && s->h && s->q && s->k && s->v && s->att && s->f1 && s->f3 && s->logits)
               ? 0 : -1;
}

void b2o_state_free(b2o_state* s) {
    for (int i = 0; i < s->n_slots; ++i) { free(s->K[i]); free(s->V[i]); }
    free(s->K); free(s->V); free(s->kv_elems);
    free(s->x); free(s->h); free(s->q); free(s->k); free(s->v);
    free(s->att); free(s->f1); free(s->f3); free(s->logits);
    memset(s, 0, sizeof(*s));
}

void b2o_state_reset(const b2o_model* m, b2o_state* s) {
    (void)m;
    for (int i = 0; i < s->n_slots; ++i) {
        if (s->K[i]) memset(s->K[i], 0, s->kv_elems[i] * sizeof(float));
        if (s->V[i]) memset(s->V[i], 0, s->kv_elems[i] * sizeof(float));
    }
    s->count = 0;
}

void b2o_state_fill_kv(const b2o_model* m, b2o_state* s, int count, uint64_t seed) {
    if (count > m->max_seq) count = m->max_seq;
    for (int b = 0; b < m->n_blocks; ++b) {
        const b2o_block* B = &m->blocks[b];
        if (B->type != B2O_SB_ATTN) continue;
        for (int kh = 0; kh < B->n_kv_heads; ++kh)
            for (int pos = 0; pos < count; ++pos)
                for (int i = 0; i < B->d_head; ++i) {
                    const int64_t at = ((int64_t)kh * m->max_seq + pos) * B->d_head + i;
                    s->K[B->kv_slot][at] = b2o_synth_value(seed, 0xC0DE0000ull + 2 * b, (uint64_t)at, 1.0f);
                    s->V[B->kv_slot][at] = b2o_synth_value(seed, 0xC0DE0001ull + 2 * b, (uint64_t)at, 1.0f);
                }
    }
    s->count = count;
}

/* projection with the reference's bias rule: int8 weights add a bias only when
 * the op has one (emit_linear, aricode_pack.py:182-185); f32 weights always add
 * one (arr_f32_matvec takes W,x,b and the ops without a bias pass a zero-filled
 * buffer, e.g. attention_gqa_kv_f32.ari:226-270). */
static void proj(const b2o_mat* M, const float* b, const float* x, int64_t m, int64_t n,
                 float* y) {
    if (M->is_i8) {
        if (M->is_i8 == 2) b2o_gemv_i4((const uint8_t*)M->w, M->ld, M->s, x, m, n, y);
        else b2o_gemv_i8((const int8_t*)M->w, M->ld, M->s, x, m, n, y);
        if (b) for (int64_t i = 0; i < m; ++i) y[i] = y[i] + b[i];
    } else {
        b2o_gemv_f32((const float*)M->w, M->ld, x, m, n, y);
        for (int64_t i = 0; i < m; ++i) y[i] = y[i] + (b ? b[i] : 0.0f);
    }
}

static void norm(int kind, const float* x, const float* g, const float* b, int d, float eps,
                 float* y) {
    if (kind == B2O_NORM_RMS) b2o_rmsnorm(x, g, d, eps, y);
    else b2o_layernorm(x, g, b, d, eps, y);
}

int32_t b2o_step(const b2o_model* m, b2o_state* s, int32_t tok, float* logits, int want_logits) {
    const int d = m->d, pos = s->count;
    if (pos >= m->max_seq) return -1;
    if (tok < 0 || tok >= m->vocab) return -2;

    /* embedding: f32(q) * scale — the reference's f64 product rounded to f32 is the
     * same value (aricode_pack.py:2254-2265); positional add in f32 (:2275-2284) */
    if (m->emb.is_i8 == 2) {          /* int4 rows: nibble, sign-extended (aricode_pack.py:2226-2249) */
        const uint8_t* row = (const uint8_t*)m->emb.w + (int64_t)tok * m->emb.ld;
        for (int i = 0; i < d; ++i) {
            const int v = (row[i >> 1] >> ((i & 1) * 4)) & 15;
            s->x[i] = (float)((v ^ 8) - 8) * m->emb.s[tok];
        }
    } else if (m->emb.is_i8) {
        const int8_t* row = (const int8_t*)m->emb.w + (int64_t)tok * m->emb.ld;
        for (int i = 0; i < d; ++i) s->x[i] = (float)row[i] * m->emb.s[tok];
    } else {
        memcpy(s->x, (const float*)m->emb.w + (int64_t)tok * m->emb.ld, sizeof(float) * d);
    }
    if (m->pos)
        for (int i = 0; i < d; ++i) s->x[i] = s->x[i] + m->pos[(int64_t)pos * d + i];

    for (int bi = 0; bi < m->n_blocks; ++bi) {
        const b2o_block* B = &m->blocks[bi];
        norm(B->norm, s->x, B->ng, B->nb, d, m->eps, s->h);      /* save_residual keeps x */
        if (B->type == B2O_SB_ATTN) {
            const int H = B->n_heads, KVH = B->n_kv_heads, dh = B->d_head;
            const int qd = H * dh, kd = KVH * dh;
            const float qscale = (float)(1.0 / sqrt((double)dh));
            float* Kl = s->K[B->kv_slot];
            float* Vl = s->V[B->kv_slot];
            proj(&B->k, B->bk, s->h, kd, d, s->k);
            proj(&B->v, B->bv, s->h, kd, d, s->v);
            proj(&B->q, B->bq, s->h, qd, d, s->q);
            for (int kh = 0; kh < KVH; ++kh) {
                float* kr = s->k + kh * dh;
                if (B->rope) b2o_rope_apply(kr, m->rope, pos, dh);
                memcpy(Kl + ((int64_t)kh * m->max_seq + pos) * dh, kr, sizeof(float) * dh);
                memcpy(Vl + ((int64_t)kh * m->max_seq + pos) * dh, s->v + kh * dh,
                       sizeof(float) * dh);
            }
            for (int h = 0; h < H; ++h) {
                float* qr = s->q + h * dh;
                if (B->rope) b2o_rope_apply(qr, m->rope, pos, dh);
                for (int i = 0; i < dh; ++i) qr[i] = qr[i] * qscale;
            }
            b2o_attn_decode(s->q, Kl, Vl, H, KVH, dh, pos + 1, m->max_seq, s->att);
            proj(&B->o, B->bo, s->att, d, qd, s->h);
        } else if (B->ffn_kind == B2O_FFN_SWIGLU) {
            proj(&B->w1, NULL, s->h, B->d_ffn, d, s->f1);
            proj(&B->w3, NULL, s->h, B->d_ffn, d, s->f3);
            for (int i = 0; i < B->d_ffn; ++i) s->f3[i] = b2o_silu(s->f1[i]) * s->f3[i];
            proj(&B->w2, NULL, s->f3, d, B->d_ffn, s->h);
        } else {
            proj(&B->w1, B->b1, s->h, B->d_ffn, d, s->f1);
            for (int i = 0; i < B->d_ffn; ++i) s->f1[i] = b2o_gelu(s->f1[i]);
            proj(&B->w2, B->b2, s->f1, d, B->d_ffn, s->h);
        }
        for (int i = 0; i < d; ++i) s->x[i] = s->h[i] + s->x[i];   /* add_residual */
    }
    s->count = pos + 1;
    if (!want_logits) return 0;
    norm(m->fn_kind, s->x, m->fn_g, m->fn_b, d, m->eps, s->h);
    proj(&m->lm, m->lm_b, s->h, m->vocab, d, s->logits);
    if (logits) memcpy(logits, s->logits, sizeof(float) * (size_t)m->vocab);
    return b2o_argmax(s->logits, m->vocab);
}

int b2o_generate_ex(const b2o_model* m, b2o_state* s, const int32_t* prompt, int n_prompt,
                    int max_new, int32_t eos, int mode, int top_k, double temperature, uint32_t seed,
                    int32_t* out_ids) {
    if (n_prompt <= 0) return 0;
    const int total = n_prompt + max_new - 1;
    uint32_t rng = seed;
    int32_t cur = 0;
    int n_out = 0;
    for (int t = 0; t < total; ++t) {
        if (t < n_prompt) cur = prompt[t];
        const int32_t r = b2o_step(m, s, cur, NULL, 1);
        if (r < 0) return r == -1 ? -1 : -2;
        const int32_t nxt = b2o_sample(s->logits, m->vocab, mode, top_k, temperature, &rng);
        if (t >= n_prompt - 1) {
            if (eos >= 0 && nxt == eos) break;
            out_ids[n_out++] = nxt;
        }
        cur = nxt;
    }
    return n_out;
}

int b2o_generate(const b2o_model* m, b2o_state* s, const int32_t* prompt, int n_prompt,
                 int max_new, int32_t* out_ids) {
    if (n_prompt <= 0) return 0;
    const int total = n_prompt + max_new - 1;
    int32_t cur = 0;
    int n_out = 0;
    for (int t = 0; t < total; ++t) {
        if (t < n_prompt) cur = prompt[t];
        const int need = t >= n_prompt - 1;    /* the LM head only where it is printed */
        const int32_t nxt = b2o_step(m, s, cur, NULL, need);
        if (nxt < 0) return nxt == -1 ? -1 : -2;
        if (need) { out_ids[n_out++] = nxt; cur = nxt; }
    }
    return n_out;
}
