/*
 * b2dec.h — C ABI of the B200 decode library (libb2dec.so).
 *
 * Plain pointers and sizes only. Every function returns an int status (B2_OK or a
 * negative B2_E_* code) and never aborts the process. The library is built for
 * sm_100a; device pointers below are CUDA global-memory addresses on the device
 * the call runs on, `stream` is a cudaStream_t (NULL = the legacy default stream).
 *
 * Reference = AriCodeLabs/aricode-ml. The reference has no native library of its
 * own: its packer (tools/aricode_pack.py) emits `.ari` source whose decode loop
 * calls builtins of the external `aric` compiler. The model-level calls below
 * replace the packed binary's main() (gen_decoder_main, aricode_pack.py:2068-2344,
 * driven by tools/run_decoder.py); the kernel-level calls replace the builtins and
 * .ari step functions listed beside them.
 */
#ifndef B2DEC_H
#define B2DEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    B2_OK = 0,
    B2_E_INVALID = -1,      /* bad argument / shape */
    B2_E_IO = -2,           /* blob file unreadable */
    B2_E_FORMAT = -3,       /* blob or plan malformed, checksum mismatch */
    B2_E_CUDA = -4,         /* CUDA runtime error (see b2_last_error) */
    B2_E_OOM = -5,          /* device allocation failed */
    B2_E_KV_OVERFLOW = -6,  /* position >= max_seq (reference: step returns -1) */
    B2_E_UNSUPPORTED = -7,
    B2_E_DEVICE = -8,       /* device-side error word set (timeout, bad token id) */
    B2_E_COMM = -9          /* tensor-parallel exchange failed */
};

typedef struct b2_ctx b2_ctx;

/* ---------------------------------------------------------------- model level */

/* Load a packed model (<out>.b2blob from `python -m aricode-ml_b200.pack
 * --target b200`) onto `device`: weights, KV cache and workspaces are allocated
 * once; the per-token step is captured into CUDA graphs. plan_json NULL uses the
 * plan embedded in the blob.
 * Replaces: the packed binary's start-up — weight load gen_load
 * (aricode_pack.py:1476-1611) and state allocation gen_scratch (:1222-1466). */
int b2_create(const char* blob_path, const char* plan_json, int device, b2_ctx** out);

/* Same, with weights synthesised on the device from (seed, std): int8 weights are
 * drawn per tensor from a counter-based generator and quantised per row exactly
 * like the packer; norm gains 1, norm/linear biases 0. No reference counterpart
 * (the reference always packs a checkpoint); used for models too large to stage
 * through a host checkpoint. */
int b2_create_synthetic(const char* plan_json, uint64_t seed, float stdv, int device,
                        b2_ctx** out);

/* Tensor parallelism over tp_size GPUs, one process (and context) per GPU: rank
 * tp_rank holds its share of every matrix (Q/K/V by heads, O, gate, up, down and
 * the LM head by output rows) and computes exactly those rows of the one-GPU
 * step, so tokens and logits are bit-identical to one GPU. The step runs as one
 * token-kernel launch per rank; outputs every rank needs are written into the
 * peers' buffers over NVLink and the phase barriers span the ranks.
 * Set-up: b2_create_synthetic_tp on every rank, b2_tp_handle (64 bytes per rank),
 * exchange the handles between the processes, b2_tp_connect with all of them in
 * rank order. Every rank must then make the same calls in the same order (steps,
 * prefill, generate, decode). A rank that stops makes the others' waits time out
 * (B2_E_DEVICE after about 1 s); the contexts must then be recreated. Logits
 * returned by b2_step hold only this rank's vocabulary rows.
 * Replaces: the plan's b2_create(blob, plan, device, tp_rank, tp_size, nccl_id);
 * the reference itself runs on one CPU thread and has no counterpart. */
int b2_create_synthetic_tp(const char* plan_json, uint64_t seed, float stdv, int device, int tp_rank,
                           int tp_size, b2_ctx** out);
/* The same from a packed blob: each rank reads the blob once (checksummed) and
 * keeps its rows of every row-split tensor and the whole of every replicated one;
 * then b2_tp_handle / b2_tp_connect as above. The packer's --tp only records the
 * degree; any blob whose head counts, d_model, d_ffn and vocab divide by tp_size
 * loads. Same limits as the synthetic form (int8 attention weights, no attention
 * biases, SwiGLU feed-forward blocks).
 * Replaces: b2_create(blob, plan, device, tp_rank, tp_size, ...) of the plan. */
int b2_create_tp(const char* blob_path, const char* plan_json, int device, int tp_rank, int tp_size,
                 b2_ctx** out);
int b2_tp_handle(b2_ctx* ctx, void* handle, int len);
int b2_tp_connect(b2_ctx* ctx, const void* handles, int len);

int b2_destroy(b2_ctx* ctx);

/* Forget the sequence: position 0, no generated ids (KV contents need no zeroing:
 * positions >= count are never read).
 * Replaces: attn_gqa_kv_reset_i8 (attention_gqa_kv_i8.ari:82-92),
 * attn_mh_kv_reset_f32 (attention_mh_kv_f32.ari:78-87). */
int b2_reset(b2_ctx* ctx);

/* One token through the model: next_tok = greedy argmax of the logits; logits
 * (vocab floats, host) optional. n_seq > 1: one token for each sequence of the
 * batched state (b2_batch_init with that many sequences), as b2_batch_step. Returns B2_E_KV_OVERFLOW, writing
 * nothing, when the position has reached max_seq.
 * Replaces: one iteration of the decoder loop (aricode_pack.py:2203-2324). */
int b2_step(b2_ctx* ctx, const int32_t* tok, int n_seq, int32_t* next_tok, float* logits);

/* Feed n tokens without evaluating the LM head (results-equivalent to n steps;
 * the reference evaluates and discards the head on every prompt token). */
int b2_prefill(b2_ctx* ctx, const int32_t* toks, int n);

/* Whole greedy generation from host buffers: total = n_prompt + max_new - 1 steps,
 * ids emitted for t >= n_prompt - 1, stop before emitting `eos` (eos < 0: none).
 * out_ids holds max_new entries. Returns B2_E_KV_OVERFLOW (with *n_out ids) when
 * the steps would pass max_seq.
 * Replaces: gen_decoder_main (aricode_pack.py:2068-2344) + run_decoder.py:62-151. */
int b2_generate(b2_ctx* ctx, const int32_t* prompt, int n_prompt, int max_new, int32_t eos,
                int32_t* out_ids, int* n_out);

/* Device-resident decode loop pieces (no host round trips; for benchmarks and
 * streaming hosts): rewind the position (KV rows < pos are kept; next_tok is the
 * token fed at pos), then enqueue n decode steps whose argmax feeds the next
 * step. Both only enqueue work on the context's stream. */
int b2_set_position(b2_ctx* ctx, int pos, int32_t next_tok);

/* Batched decode: n_seq independent sequences, each with its own KV
 * cache (n_seq x max_seq positions), advanced one token each per step. Every
 * projection of a step is one tensor-core GEMM over the n_seq tokens (tcgen05
 * kind::i8 over the byte planes of each token's fixed-point activations), whose
 * rows equal the one-sequence GEMV bit for bit; attention runs per sequence over
 * its own cache; the LM head covers every sequence and the greedy token of each
 * is fed to its next step. So every sequence's ids and logits are those it would
 * get decoded alone. Needs a plan the batched prefill covers (Llama family) and
 * n_seq <= 512. With tensor parallelism (b2_create_tp / b2_create_synthetic_tp)
 * every rank makes the same calls with the same arguments: each runs its rows of
 * every GEMM, its heads and its vocabulary rows, writes them into every rank's
 * copy and waits (bounded) for the others after each exchange, so ids and logits
 * are the one-GPU ones on every rank. A rank more than about 1 s behind the
 * others at an exchange makes their waits time out (B2_E_DEVICE): synchronise the
 * ranks on the host after b2_batch_init.
 *   b2_batch_init       allocate the caches and an output record of max_steps steps
 *   b2_batch_reset      every sequence back to position 0, record emptied
 *   b2_batch_prefill    prompt tokens of one sequence (no LM head), batched
 *   b2_batch_step       one token per sequence (n_seq ids in, n_seq greedy ids out,
 *                       optional logits [n_seq][vocab]); b2_step with n_seq equal
 *                       to the batch does the same
 *   b2_batch_decode_async  n steps on the device, each feeding its greedy ids on
 *   b2_batch_read_output   the recorded ids [steps][n_seq]
 *   b2_batch_generate   prompts [n_seq][n_prompt] -> out [n_seq][max_new]: prefill
 *                       of every prompt, then max_new batched steps
 * The reference decodes one sequence at a time; this replaces running its decoder
 * loop (aricode_pack.py:2068-2344) once per sequence. */
int b2_batch_init(b2_ctx* ctx, int n_seq, int max_steps);
int b2_batch_reset(b2_ctx* ctx);
int b2_batch_prefill(b2_ctx* ctx, int seq, const int32_t* toks, int n);
int b2_batch_step(b2_ctx* ctx, const int32_t* toks, int32_t* next, float* logits);
int b2_batch_decode_async(b2_ctx* ctx, int n_steps);
int b2_batch_read_output(b2_ctx* ctx, int32_t* ids, int max_steps, int* n_steps);
int b2_batch_generate(b2_ctx* ctx, const int32_t* prompts, int n_prompt, int max_new, int32_t* out_ids);

/* Token choice after the LM head: mode 0 greedy (the default), 1 temperature
 * softmax, 2 top-k then temperature, with the reference's 32-bit LCG
 * (state = state * 1103515245 + 12345, draw = (state & 65535) / 65536) seeded
 * with `seed` at every new sequence (b2_reset, b2_generate) and advanced on every
 * step, prompt steps included, as the reference loop does. A plan packed with
 * --sample / --rng-seed starts with those settings. Not with tensor parallelism
 * (B2_E_UNSUPPORTED). Returns the settings to the sequence start at the current
 * position.
 * Replaces: sample_temperature_f32 / sample_topk_filter_f32 (sampling_f32.ari:31-153)
 * and the sampling branch of the decoder loop (aricode_pack.py:2186-2306). */
enum { B2_SAMPLE_GREEDY = 0, B2_SAMPLE_TEMPERATURE = 1, B2_SAMPLE_TOPK = 2 };
int b2_set_sampling(b2_ctx* ctx, int mode, int top_k, double temperature, uint32_t seed);

/* Fill KV rows [0, count) of every attention sub-block with synthetic values and
 * set the position to count: value of element ((kv_head * max_seq + pos) * d_head
 * + i) of sub-block b (index in the plan's block list) is the synthetic generator's
 * value for (seed, tensor 0xC0DE0000 + 2b for K / + 2b + 1 for V, that index,
 * std 1). Lets a test or benchmark start decoding mid-sequence with the same
 * cache as the oracle's b2o_state_fill_kv, without a prefill. No reference
 * counterpart. */
int b2_fill_kv_synthetic(b2_ctx* ctx, int count, uint64_t seed);
int b2_decode_async(b2_ctx* ctx, int n_steps);
int b2_sync(b2_ctx* ctx);
int b2_read_output(b2_ctx* ctx, int32_t* ids, int max_ids, int* n_ids);

/* Launch the model's graphs and copies on `stream` (cudaStream_t, NULL = legacy
 * default stream) instead of the context's private stream, e.g. to time them
 * with the caller's events. The context does not take ownership. */
int b2_set_stream(b2_ctx* ctx, void* stream);

/* Numeric properties: "weight_bytes", "kv_bytes_per_pos", "kernels_per_step",
 * "max_seq", "vocab", "position", "n_out", "device_err", "sm_count",
 * "token_kernel" (1: one persistent launch per step), "token_tags" (1: its phases
 * meet through tagged words instead of grid barriers), "prefill_batched". */
int b2_query(b2_ctx* ctx, const char* key, double* value);

/* Last error message of ctx (or of the last failed create when ctx is NULL). */
int b2_last_error(b2_ctx* ctx, char* buf, int len);

/* ---------------------------------------------------------------- kernel level
 * Device pointers in and out; nothing is allocated and nothing synchronises. */

/* y[j] = scale[j] * sum_k W[j,k] x[k] (+ bias[j]), W int8 row-major with row
 * stride ld (ld % 16 == 0, zero padding past n), f32 accumulation.
 * Replaces: arr_i8_matvec_f32_perrow + arr_f32_add_scaled
 * (aricode_pack.py:183-184; attention_gqa_kv_i8.ari:149-151, :191). */
int b2_gemv_i8_rowscale(const int8_t* W, int64_t ld, const float* scale, const float* x,
                        const float* bias, float* y, int m, int n, void* stream);

/* The same for int4 rows in the reference's --int4-linear format (two codes a
 * byte, even column in the low nibble, ld = packed bytes per row, ld % 16 == 0,
 * n even): the exact int8 dot over the unpacked codes, streaming the packed rows.
 * Replaces: arr_i4_matvec_f32_perrow + bias add (aricode_pack.py:168-181). */
int b2_gemv_i4_rowscale(const uint8_t* W, int64_t ld, const float* scale, const float* x, const float* bias,
                        float* y, int m, int n, void* stream);

/* The same for T input vectors at once, on the tensor cores (tcgen05 kind::i8
 * over the byte planes of each vector's fixed-point copy): Y[t][j] = scale[j] *
 * dot(W[j,:], X[t,:]) (+ bias[j]), bit-identical to T calls of
 * b2_gemv_i8_rowscale. X [T][ldx] f32, Y [T][ldy] f32; rows (tokens) padded
 * planes need b2_gemm_i8_rowscale_workspace(T, ld) bytes of workspace (16-byte
 * aligned, no initialisation).
 * Replaces: the batched linear loop the packer emits for seq > 1
 * (aricode_pack.py:186-210: one arr_i8_matvec_f32_perrow per row of the input). */
size_t b2_gemm_i8_rowscale_workspace(int T, int64_t ld);
int b2_gemm_i8_rowscale(const int8_t* W, int64_t ld, const float* scale, const float* X, int64_t ldx,
                        const float* bias, float* Y, int64_t ldy, int m, int n, int T, void* workspace,
                        size_t workspace_bytes, void* stream);

/* y = W x + bias (bias NULL adds 0), W f32 with row stride ld (ld % 4 == 0).
 * Replaces: arr_f32_matvec (attention_kv_f32.ari:122-140, attention_mh_kv_f32.ari:150). */
int b2_gemv_f32(const float* W, int64_t ld, const float* x, const float* bias, float* y,
                int m, int n, void* stream);

/* Replaces: rmsnorm_affine_f32 (aricode_pack.py:585-607). */
int b2_rmsnorm(const float* x, const float* g, float* y, int d, float eps, void* stream);

/* Replaces: layernorm_affine_f32 (aricode_pack.py:503-521). */
int b2_layernorm(const float* x, const float* g, const float* b, float* y, int d, float eps,
                 void* stream);

/* Rotate n_vec consecutive d_head-wide vectors in place with table row pos.
 * Replaces: rope_apply_f32 / arr_f32_rope_apply_pairs (rope_f32.ari:69-72). */
int b2_rope_apply(float* v, const float* table, int pos, int d_head, int n_vec, void* stream);

/* Decode attention for one step: q [n_heads*d_head] (rotated, pre-scaled),
 * K/V caches [n_kv_heads][max_seq][d_head] (16-byte aligned, d_head % 4 == 0,
 * d_head <= 256), n valid keys, inactive tail = -60.
 * workspace: b2_attn_decode_workspace() bytes of device memory, zero-filled
 * before the first call (the kernel leaves it zero again).
 * Replaces: _gqa_score_head_i8 (attention_gqa_kv_i8.ari:97-117) /
 * the scoring half of attn_kv_step_f32 (attention_kv_f32.ari:134-162). */
size_t b2_attn_decode_workspace(int n_heads, int n_kv_heads, int d_head, int max_seq);
int b2_attn_decode(const float* q, const float* K, const float* V, float* out, int n_heads,
                   int n_kv_heads, int d_head, int n, int max_seq, void* workspace,
                   size_t workspace_bytes, void* stream);

/* b2_attn_decode without a workspace argument, for callers that cannot allocate
 * device memory (a host framework that owns the device's memory and forbids
 * library cudaMalloc calls, or an FFI binding with no device allocator). No
 * counterpart in the reference. Its scratch is a fixed device array of
 * B2_ATTN_STATIC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit; problems needing more scratch than that (n_heads * ceil(max_seq/64) *
 * (d_head+2) * 4 + n_kv_heads * 4 bytes) return B2_E_INVALID, with the reason in
 * b2_last_error(NULL, ...). The first call on a device looks the array up on that
 * device, so make it before any stream capture; the address found there is kept
 * for the life of the process, so a host that resets the device (cudaDeviceReset)
 * must not call this entry point on that device afterwards. All calls share the
 * array: calls that overlap on the GPU race. Allocates nothing. */
#define B2_ATTN_STATIC_SCRATCH_BYTES (4u << 20)
int b2_attn_decode_static(const float* q, const float* K, const float* V, float* out,
                          int n_heads, int n_kv_heads, int d_head, int n, int max_seq,
                          void* stream);

/* out[0] = first index of the maximum (NaN never wins; logits[0] NaN -> 0).
 * Replaces: sample_greedy_f32 (sampling_f32.ari:10-24). */
int b2_argmax(const float* v, int64_t n, int32_t* out, void* stream);

/* h[i] = silu(g[i]) * u[i] (silu in f64, narrowed). Replaces: silu_mul_f32
 * (aricode_pack.py:626-632). */
int b2_silu_mul(const float* g, const float* u, float* h, int n, void* stream);

/* y[i] = tanh-GELU(x[i]) in f64. Replaces: gelu_f32 (aricode_pack.py:539-572). */
int b2_gelu(const float* x, float* y, int n, void* stream);

/* Per-row symmetric int8: scale = max|row|/127, q = clip(rint(row/scale)).
 * Replaces: the packer's per-row quantiser (aricode_pack.py:3356-3379). */
int b2_quantize_rows(const float* W, int64_t m, int64_t n, int8_t* q, int64_t ldq,
                     float* scale, void* stream);

/* Synthetic weights: rows [r0,r1) x cols [c0,c1) of an m x n tensor quantised per
 * FULL row. No reference counterpart (synthetic-checkpoint generator). */
int b2_synth_quant_rows(uint64_t seed, uint64_t tensor_id, int64_t n, float stdv, int64_t r0,
                        int64_t r1, int64_t c0, int64_t c1, int8_t* q, int64_t ldq,
                        float* scale, void* stream);
int b2_synth_fill_f32(uint64_t seed, uint64_t tensor_id, int64_t m, int64_t n, float stdv,
                      float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
