/*
 * refdec.h — CPU oracle for the int8 decoder decode path.
 *
 * TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load this library, and only as the
 * checker or the timed CPU baseline. The product path (the CUDA library under
 * aricode-ml_b200/) never calls it.
 *
 * What it restates (reference = AriCodeLabs/aricode-ml):
 *   - per-row int8 quantiser            tools/aricode_pack.py:3356-3379
 *   - arr_i8_matvec_f32_perrow          call sites tools/aricode_pack.py:183, :1789-1808,
 *                                       attention_gqa_kv_i8.ari:149-151, :191
 *   - arr_f32_matvec (f32 projections)  attention_kv_f32.ari:122-140, attention_gqa_kv_f32.ari:226-270
 *   - rmsnorm_affine_f32                tools/aricode_pack.py:585-607
 *   - layernorm_affine_f32              tools/aricode_pack.py:503-521
 *   - silu_mul_f32 / arr_f32_silu       tools/aricode_pack.py:614-632
 *   - gelu_f32                          tools/aricode_pack.py:539-572
 *   - rope_alloc_f32 / rope_apply_f32   rope_f32.ari:34-55, :69-72
 *   - _gqa_score_head_i8 (+ -60 tail)   attention_gqa_kv_i8.ari:97-117, attention_kv_f32.ari:134-162
 *   - attn_gqa_kv_step_i8/_f32          attention_gqa_kv_i8.ari:119-195, attention_gqa_kv_f32.ari:170-274
 *   - attn_mh_kv_step_f32               attention_mh_kv_f32.ari:101-152
 *   - sample_greedy_f32                 sampling_f32.ari:10-24
 *   - decoder main loop                 tools/aricode_pack.py:2068-2344
 *
 * The reference's arithmetic lives in builtins of the external `aric` compiler
 * (codegen_builtins.c), which is not in the reference tree; its AVX2 lane/tree
 * order is unrecoverable. This oracle therefore fixes ONE association order per
 * reduction (documented at each function) and the CUDA kernels use exactly the
 * same order, so GPU results are bit-identical to this oracle. The oracle is
 * pinned against the reference's own fixtures: packer bytes (codes/scales),
 * the RoPE golden vector, the KV-attention invariants and the tiny decoder
 * examples' PyTorch greedy tokens (tests/golden/).
 */
#ifndef B2_REFDEC_H
#define B2_REFDEC_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar maths shared bit-for-bit with the CUDA kernels ---- */
float  b2o_exp_f(float x);      /* own f32 exp: Cody-Waite reduction + degree-7 Taylor */
double b2o_exp_d(double x);     /* own f64 exp: clamp [-700,700], Cody-Waite + degree-13 Taylor */
float  b2o_silu(float g);       /* (float)(g / (1 + exp(-g))) in f64 */
float  b2o_gelu(float x);       /* tanh-GELU in f64, clamp |2z|>20 */

/* ---- per-row int8 quantiser (numpy float32 semantics) ---- */
void b2o_quantize_rows(const float* W, int64_t m, int64_t n,
                       int8_t* q, int64_t ldq, float* scale);

/* ---- matvecs: y[j] = scale[j] * dot(W[j,:], x)  /  y[j] = dot(W[j,:], x) ---- */
void b2o_gemv_i8(const int8_t* W, int64_t ld, const float* scale, const float* x,
                 int64_t m, int64_t n, float* y);
void b2o_gemv_f32(const float* W, int64_t ld, const float* x,
                  int64_t m, int64_t n, float* y);
/* int4 rows (arr_i4_matvec_f32_perrow, aricode_pack.py:168-181: the nibbles of a
 * row unpacked to int8 codes, then the int8 matvec): packed [m][ld bytes] */
void b2o_unpack_i4(const uint8_t* packed, int64_t n, int8_t* codes);
void b2o_gemv_i4(const uint8_t* W, int64_t ld, const float* scale, const float* x,
                 int64_t m, int64_t n, float* y);
/* int8 rows: x as 32-bit block fixed point X = trunc(x * 2^S); returns S, or
 * B2O_XFIX_BAD when x holds a NaN or an infinity (every row is then NaN) */
#define B2O_XFIX_BAD (-100000)
int b2o_xfix(const float* x, int64_t n, int32_t* X);
/* one row: f32(sum w*X exactly, times 2^-S) */
float b2o_dot_i8x(const int8_t* w, const int32_t* X, int64_t n, int S);
/* f32 rows: dot product in the shared order, exposed for tests */
float b2o_dot_f32(const float* w, const float* x, int64_t n);
/* int8 rows, for measuring tolerances: f32 8-lane FMA accumulation as the
 * reference's builtin is described (README.md:128-131), and f64 accumulation */
float  b2o_dot_i8_f32acc(const int8_t* w, const float* x, int64_t n);
double b2o_dot_i8_f64(const int8_t* w, const float* x, int64_t n);
/* which matvec b2o_gemv_i8 / b2o_step use: 0 fixed-point (the GPU's bits, default),
 * 1 f32 accumulation, 2 f64 accumulation (f32-weight matvecs too) */
void b2o_set_matvec_mode(int mode);
int  b2o_get_matvec_mode(void);

/* ---- norms ---- */
void b2o_rmsnorm(const float* x, const float* g, int d, float eps, float* y);
void b2o_layernorm(const float* x, const float* g, const float* b, int d, float eps, float* y);

/* ---- RoPE ---- */
void b2o_rope_table(int max_seq, int d_head, double theta, float* table);
void b2o_rope_apply(float* v, const float* table, int pos, int d_head);

/* ---- attention over a KV cache (one decode step, split-KV order) ----
 * q:  [n_heads * d_head] (already rotated and scaled)
 * Kc, Vc: [n_kv_heads][max_seq][d_head]
 * out: [n_heads * d_head]; n = number of valid keys (count+1). */
#define B2O_ATT_CHUNK 64
void b2o_attn_decode(const float* q, const float* Kc, const float* Vc,
                     int n_heads, int n_kv_heads, int d_head, int n, int max_seq,
                     float* out);

/* ---- sampling ---- */
int32_t b2o_argmax(const float* v, int64_t n);
enum { B2O_SAMPLE_GREEDY = 0, B2O_SAMPLE_TEMPERATURE = 1, B2O_SAMPLE_TOPK = 2 };
uint32_t b2o_lcg_next(uint32_t state);
/* sample_topk_filter_f32 / sample_temperature_f32 (in place, like the reference) */
void    b2o_topk_filter(float* logits, int64_t n, int k);
int32_t b2o_sample_temperature(float* logits, int64_t n, double temperature, double unit);
/* one loop step's choice: greedy, or advance *rng and sample (logits overwritten) */
int32_t b2o_sample(float* logits, int64_t n, int mode, int top_k, double temperature, uint32_t* rng);

/* ---- synthetic weights (counter-based, identical on the GPU) ---- */
float b2o_synth_value(uint64_t seed, uint64_t tensor_id, uint64_t index, float stdv);
void  b2o_synth_fill_f32(uint64_t seed, uint64_t tensor_id, int64_t m, int64_t n,
                         float stdv, float* out);
/* generate rows [r0,r1) x cols [c0,c1) of an m x n tensor and quantise each row over
 * its FULL width (scales are per global row); q has row stride ldq. */
void  b2o_synth_quant_rows(uint64_t seed, uint64_t tensor_id, int64_t n, float stdv,
                           int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                           int8_t* q, int64_t ldq, float* scale);

/* ---- whole decoder ----
 * The model is the embedding, a list of pre-norm residual sub-blocks
 * (save_residual, norm, op, add_residual) and a final norm + LM head, as the
 * reference's decoder mode packs it (aricode_pack.py:2068-2344). */
enum { B2O_SB_ATTN = 0, B2O_SB_FFN = 1 };
enum { B2O_NORM_RMS = 0, B2O_NORM_LN = 1 };
enum { B2O_FFN_SWIGLU = 0, B2O_FFN_GELU = 1 };

/* a matrix: is_i8 1 = int8 codes + per-row scales, 2 = int4 codes packed two per
 * byte (even column in the low nibble; ld in bytes) + per-row scales, 0 = f32;
 * rows padded to ld elements */
typedef struct { int is_i8; const void* w; const float* s; int64_t ld; } b2o_mat;

typedef struct {
    int type;                 /* B2O_SB_ATTN / B2O_SB_FFN */
    int norm;                 /* B2O_NORM_RMS / B2O_NORM_LN */
    const float* ng; const float* nb;
    /* attention: multi_head_attention_gqa_kv (rope=1) or multi_head_attention_kv */
    int rope, n_heads, n_kv_heads, d_head, kv_slot;
    b2o_mat q, k, v, o;
    const float *bq, *bk, *bv, *bo;     /* NULL: none (f32 weights then add +0) */
    /* feed-forward: swiglu (w1=gate, w3=up, w2=down) or linear-gelu-linear (w1, w2) */
    int ffn_kind, d_ffn;
    b2o_mat w1, w3, w2;
    const float *b1, *b2;
} b2o_block;

typedef struct {
    int vocab, d, max_seq, n_blocks, n_kv_slots;
    float eps;
    b2o_mat emb;                          /* [vocab, d] */
    const float* pos; int max_pos;        /* learned positions or NULL */
    const b2o_block* blocks;
    int fn_kind; const float* fn_g; const float* fn_b;
    b2o_mat lm; const float* lm_b;        /* [vocab, d] + bias */
    const float* rope;                    /* [max_seq, d_head] (RoPE sub-blocks) */
    int max_heads, max_kv_dim, max_ffn;   /* scratch sizing */
} b2o_model;

typedef struct {
    float** K;           /* per kv slot: [n_kv_heads][max_seq][d_head] */
    float** V;
    size_t* kv_elems;
    int n_slots;
    int count;
    float *x, *h, *q, *k, *v, *att, *f1, *f3, *logits;
} b2o_state;

int  b2o_state_init(const b2o_model* m, b2o_state* s);
void b2o_state_free(b2o_state* s);
void b2o_state_reset(const b2o_model* m, b2o_state* s);
/* Benchmark helper: fill KV rows [0, count) of every attention sub-block with
 * synthetic values (unit std) and set the position to count, so a decode sample
 * can start mid-sequence without a CPU prefill. */
void b2o_state_fill_kv(const b2o_model* m, b2o_state* s, int count, uint64_t seed);
/* One token through the whole model: returns argmax id (want_logits=1) or 0,
 * -1 on KV overflow (nothing written), -2 on a bad token id. */
int32_t b2o_step(const b2o_model* m, b2o_state* s, int32_t tok, float* logits, int want_logits);
/* Greedy generation with the reference loop structure (total = P + N - 1 steps,
 * emit argmax for t >= P-1). Returns number of ids written, or -1 on overflow. */
int b2o_generate(const b2o_model* m, b2o_state* s, const int32_t* prompt, int n_prompt,
                 int max_new, int32_t* out_ids);

/* The reference loop with a sampler (the head runs and the rng advances on every
 * step, prompt steps included) and an EOS id (eos < 0: none; generation stops
 * before emitting it). Returns ids written, -1 on overflow, -2 on a bad id. */
int b2o_generate_ex(const b2o_model* m, b2o_state* s, const int32_t* prompt, int n_prompt,
                    int max_new, int32_t eos, int mode, int top_k, double temperature, uint32_t seed,
                    int32_t* out_ids);

/* worker threads for matvecs/attention (pthreads); 1 = single-threaded like the reference */
void b2o_set_threads(int n);
int  b2o_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
