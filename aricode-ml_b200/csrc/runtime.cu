// runtime.cu — model context, blob loader, launch plan, CUDA-graph decode loop and
// the C ABI of include/b2dec.h.
//
// One context = one model on one device. Weights live in one arena (one H2D copy
// of the blob's data region), the KV cache in another, activations and scratch in
// a third. The per-token step (embedding, every sub-block, LM head) is captured
// once into two CUDA graphs — with and without the LM head — whose kernels are
// chained by programmatic dependent launch. The decode state (position, next
// token, generated ids, EOS/limit flag, error word) lives on the device, so a
// whole generation is a sequence of graph launches with no host round trips.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/b2dec.h"
#include "json.h"
#include "prefill.cuh"
#include "token.cuh"

using namespace b2;

namespace {

thread_local std::string g_last_create_error;

struct DevMat {
    const void* w = nullptr;
    const float* s = nullptr;
    int rows = 0, cols = 0;
    int ld = 0;
    bool i8 = false;        // int8 or int4 codes with per-row scales
    bool i4 = false;        // int4: two codes a byte, ld in bytes
};

struct NormRef {
    int kind = NORM_RMS;
    const float* g = nullptr;
    const float* b = nullptr;
};

struct Block {
    bool attn = false;
    NormRef norm;
    // attention
    bool rope = false;
    int H = 0, KVH = 0, dh = 0;        // this rank's heads (all of them on one GPU)
    int head0 = 0, H_all = 0;          // first query head of this rank, heads of the model
    DevMat q, k, v, o;
    const float* bias[4] = {nullptr, nullptr, nullptr, nullptr};
    float* K = nullptr;
    float* V = nullptr;
    // feed-forward
    bool swiglu = false;
    int d_ffn = 0;                     // of the model
    int ffn_local = 0, ffn0 = 0;       // this rank's hidden rows and the first of them
    DevMat w1, w3, w2;
    const float* b1 = nullptr;
    const float* b2 = nullptr;
};

struct TensorInfo {
    int dtype = 0;          // 1 int8, 2 f32
    long long rows = 0, cols = 0, ld = 0;
    size_t off = 0, nbytes = 0;
    bool two_d = false;
};

uint64_t fnv1a64(const std::string& s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (unsigned char c : s) { h ^= c; h *= 0x100000001b3ull; }
    return h;
}

// blob checksum (same as blob.checksum in Python)
uint64_t checksum_words(const unsigned char* p, size_t n, uint64_t first_word) {
    uint64_t tot = 0;
    const size_t nw = n / 8;
    for (size_t i = 0; i < nw; ++i) {
        uint64_t w;
        std::memcpy(&w, p + 8 * i, 8);
        tot += (w ^ ((first_word + i) * 0x9E3779B97F4A7C15ull)) * 0xBF58476D1CE4E5B9ull;
    }
    if (n % 8) {
        uint64_t w = 0;
        std::memcpy(&w, p + 8 * nw, n % 8);
        tot += (w ^ ((first_word + nw) * 0x9E3779B97F4A7C15ull)) * 0xBF58476D1CE4E5B9ull;
    }
    return tot;
}

struct Err : std::runtime_error {
    int code;
    Err(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(expr)                                                                              \
    do {                                                                                      \
        cudaError_t _e = (expr);                                                              \
        if (_e != cudaSuccess)                                                                \
            throw Err(B2_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e));         \
    } while (0)

}  // namespace

struct b2_ctx {
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;       // launches and copies
    cudaStream_t cap_stream = nullptr;   // private stream the graphs are captured on
    bool own_stream = false;
    std::string err;

    int vocab = 0, d = 0, max_seq = 0, max_pos = 0, token_bytes = 4;
    float eps = 1e-5f;
    DevMat emb;
    const float* pos_tab = nullptr;
    NormRef fnorm;
    DevMat lm;
    const float* lm_b = nullptr;
    std::vector<Block> blocks;
    int rope_dh = 0;
    double rope_theta = 0.0;

    void* d_weights = nullptr;
    size_t weight_bytes = 0;
    std::map<std::string, TensorInfo> tensors;
    void* d_kv = nullptr;
    size_t kv_bytes = 0, kv_bytes_per_pos = 0;
    void* d_work = nullptr;
    size_t work_bytes = 0;

    float* rope_tab = nullptr;
    float* x = nullptr;
    float* q = nullptr;
    float* att = nullptr;
    float* f = nullptr;
    float* logits = nullptr;
    float* attn_part = nullptr;
    // token kernel: the activations as (value, tag) words (x, q, attention output,
    // FFN hidden vector, this step's K / V rows); the split partials reuse attn_part
    unsigned long long *tx = nullptr, *tq = nullptr, *tatt = nullptr, *tf = nullptr, *tkn = nullptr, *tvn = nullptr;
    bool tk_tags = false;   // the token kernel's phases meet through tagged words, not grid barriers
    unsigned* attn_cnt = nullptr;
    int attn_nsplit_max = 1;
    float* amax_val = nullptr;
    int* amax_idx = nullptr;
    int* amax_v0nan = nullptr;
    unsigned* amax_cnt = nullptr;
    StepState* st = nullptr;
    int* prompt = nullptr;
    int* out_ids = nullptr;
    StepState* h_st = nullptr;     // pinned mirror

    cudaGraphExec_t g_prefill = nullptr, g_decode = nullptr;
    int kernels_prefill = 0, kernels_decode = 0;
    bool pdl = true;               // programmatic dependent launch between kernels
    // persistent token kernel (token.cuh): one launch per step
    bool token = false;
    int token_vs = 0;              // compiled variant set (0 int8 only, 1 int8 + f32)
    TkPhase* d_phases = nullptr;   // [prefill phases][decode phases]
    int nph_prefill = 0, nph_decode = 0;
    unsigned* tk_bar = nullptr;    // grid-barrier counters, zero between launches
    int n_attn_cnt = 0;
    int tk_ns = 0, tk_ring_offset = 0, tk_inflight = kTkInflight, tk_vec_offset = 0, tk_vec_floats = 0;
    size_t tk_smem = 0;
    std::string token_why;         // why the per-layer kernels are used instead
    unsigned long long* d_trace = nullptr;   // token-kernel timeline (B2_TK_TRACE)
    std::string trace_path;
    std::vector<int> trace_kinds;  // per phase of both tables: kind, or 10 + GEMV variant
    int host_step = 0;
    unsigned* tk_seq = nullptr;    // token-kernel launches completed (cross-rank epochs)
    int tk_final_xsync[2] = {0, 0};  // per table (prefill, decode): last phase mirrored
    // tensor parallelism: rank tp_rank of tp_size GPUs (one process each). The
    // exchange buffer holds what every rank reads whole (x, attention output,
    // FFN hidden vector) and the cross-rank flags; peers write into it through
    // CUDA IPC mappings.
    int tp_rank = 0, tp_size = 1;
    bool tp_connected = false;
    void* d_xch = nullptr;
    size_t xch_bytes = 0;
    void* peer_base[kMaxRanks] = {};
    Mirror mir{};
    unsigned* tp_flag = nullptr;   // [kMaxRanks] barrier epochs
    unsigned* tp_aflag = nullptr;  // [kMaxRanks] argmax epochs
    float* tp_cval = nullptr;      // [kMaxRanks] each rank's best logit
    int* tp_cidx = nullptr;
    int* tp_cnan = nullptr;
    // sampling beyond greedy (b2_set_sampling): a sampler kernel follows the LM head
    int samp_mode = 0, samp_k = 0;
    double samp_t = 0.0;
    unsigned seed = 0, rng = 0;    // rng: LCG state before the next step's advance
    double* samp_e = nullptr;
    // batched prefill (prefill.cuh): whether the plan is covered, and its workspace
    bool pf_ok = false;
    std::string pf_why;
    void* pf_base = nullptr;
    int pf_tmax = 0, pf_ldp = 0;
    unsigned char* pf_planes = nullptr;
    int* pf_S = nullptr;
    float *pf_x = nullptr, *pf_q = nullptr, *pf_att = nullptr, *pf_f = nullptr, *pf_part = nullptr;
    // tensor parallelism: the prefill's x, attention output and FFN hidden rows of every
    // rank, in the exchange buffer (the peers write their rows), and the flags and
    // epoch of the barriers between its launches
    float *pfx_x = nullptr, *pfx_att = nullptr, *pfx_f = nullptr;
    unsigned* tp_pflag = nullptr;
    unsigned* tp_pepoch = nullptr;     // this rank's count of those barriers (device)
    float* pfx_logits = nullptr;       // batched decode's logits [pf_tmax][vocab]
    int pfx_tmax = 0;
    unsigned long long* pf_acc = nullptr;   // split-K dot totals of the tensor-core GEMM (zero between launches)
    unsigned* pf_cnt = nullptr;     // its per-tile arrival counters
    // batched decode (b2_batch_init): bt_n sequences, each with its own KV cache
    int bt_n = 0, bt_max_steps = 0;
    void* bt_base = nullptr;
    std::vector<float*> bt_K, bt_V;          // per block: [bt_n][KVH][max_seq][dh] (attention blocks)
    long long bt_seq_stride = 0;             // floats between two sequences' caches of one block
    int *bt_tok = nullptr, *bt_pos = nullptr, *bt_out = nullptr, *bt_nsteps = nullptr, *bt_ids = nullptr;
    float *bt_logits = nullptr, *bt_part = nullptr;
    unsigned* bt_cnt = nullptr;
    std::vector<int> bt_pos_host;
    int bt_steps_host = 0;
    cudaGraphExec_t g_batch = nullptr;

    ~b2_ctx() {
        if (device >= 0) cudaSetDevice(device);
        if (g_prefill) cudaGraphExecDestroy(g_prefill);
        if (g_decode) cudaGraphExecDestroy(g_decode);
        if (d_weights) cudaFree(d_weights);
        if (d_kv) cudaFree(d_kv);
        if (d_work) cudaFree(d_work);
        if (d_phases) cudaFree(d_phases);
        if (d_trace) cudaFree(d_trace);
        if (pf_base) cudaFree(pf_base);
        if (g_batch) cudaGraphExecDestroy(g_batch);
        if (bt_base) cudaFree(bt_base);
        for (int r = 0; r < kMaxRanks; ++r)
            if (peer_base[r]) cudaIpcCloseMemHandle(peer_base[r]);
        if (d_xch) cudaFree(d_xch);
        if (h_st) cudaFreeHost(h_st);
        if (own_stream && stream) cudaStreamDestroy(stream);
        if (cap_stream) cudaStreamDestroy(cap_stream);
    }

    // ------------------------------------------------------------ tensors
    const TensorInfo& tinfo(const std::string& name) const {
        auto it = tensors.find(name);
        if (it == tensors.end()) throw Err(B2_E_FORMAT, "blob has no tensor '" + name + "'");
        return it->second;
    }
    const float* vec(const b2json::Value& v, long long expect) const {
        if (v.is_null()) return nullptr;
        const TensorInfo& t = tinfo(v.as_str());
        if (t.dtype != 2 || t.two_d || t.cols != expect)
            throw Err(B2_E_FORMAT, "tensor '" + v.str + "' must be f32 [" + std::to_string(expect) + "]");
        return reinterpret_cast<const float*>(static_cast<char*>(d_weights) + t.off);
    }
    DevMat mat(const std::string& name, long long rows, long long cols) const {
        const TensorInfo& t = tinfo(name);
        if (!t.two_d || t.rows != rows || t.cols != cols)
            throw Err(B2_E_FORMAT, "tensor '" + name + "' must be [" + std::to_string(rows) + ", " +
                                       std::to_string(cols) + "]");
        DevMat m;
        m.w = static_cast<char*>(d_weights) + t.off;
        m.rows = (int)rows;
        m.cols = (int)cols;
        m.ld = (int)t.ld;
        m.i8 = t.dtype == 1 || t.dtype == 3;
        m.i4 = t.dtype == 3;
        if (m.i4 && (cols % 2 || t.ld * 2 < cols))
            throw Err(B2_E_FORMAT, "int4 tensor '" + name + "' must have an even row length");
        if (m.i8) {
            if (t.ld % 16) throw Err(B2_E_FORMAT, "int8 tensor '" + name + "' row stride not 16-aligned");
            if (cols > kXfixMaxN)
                throw Err(B2_E_UNSUPPORTED, "int8 tensor '" + name + "' has rows longer than " +
                                                std::to_string(kXfixMaxN) + " codes (the exact dot's int32 sums)");
            b2json::Value sname;
            sname.kind = b2json::Value::String;
            sname.str = name + "_scales";
            m.s = vec(sname, rows);
        } else if (t.ld % 4) {
            throw Err(B2_E_FORMAT, "f32 tensor '" + name + "' row stride not 4-aligned");
        }
        if ((reinterpret_cast<uintptr_t>(m.w) & 15) != 0)
            throw Err(B2_E_FORMAT, "tensor '" + name + "' not 16-byte aligned");
        return m;
    }
    NormRef norm_of(const b2json::Value& n) const {
        NormRef r;
        const std::string& kind = n["kind"].as_str("norm.kind");
        if (kind == "rms") r.kind = NORM_RMS;
        else if (kind == "ln") r.kind = NORM_LN;
        else throw Err(B2_E_FORMAT, "unknown norm kind " + kind);
        r.g = vec(n["g"], d);
        if (r.kind == NORM_LN) r.b = vec(n["b"], d);
        return r;
    }
};

namespace {

// ------------------------------------------------------------------ plan -> tensor shapes
struct Need {
    std::string name;
    int dtype;            // 1 int8 (+ _scales), 2 f32
    long long rows, cols; // cols = 0: 1-D of length rows
    int init;             // synthetic: 0 random, 1 ones, 2 zeros
    long long row0 = 0;   // tensor parallelism: first row of this rank's share
};

// Tensor shapes of a plan; with tp > 1 the row-split tensors (Q/K/V by heads,
// O, gate, up, down and the LM head by output rows) are this rank's share.
std::vector<Need> plan_needs(const b2json::Value& plan, int tp = 1, int rank = 0) {
    std::vector<Need> out;
    const long long d = plan["d_model"].as_int("d_model"), vocab = plan["vocab"].as_int("vocab");
    auto split = [&](Need n) {
        if (tp > 1) {
            if (n.rows % tp) throw Err(B2_E_UNSUPPORTED, "tensor '" + n.name + "' rows do not split over the ranks");
            n.rows /= tp;
            n.row0 = n.rows * rank;
        }
        out.push_back(n);
    };
    auto no_tp = [&](const char* what) {
        if (tp > 1) throw Err(B2_E_UNSUPPORTED, std::string("tensor parallelism does not cover ") + what);
    };
    auto norm = [&](const b2json::Value& n) {
        out.push_back({n["g"].as_str(), 2, d, 0, 1});
        if (n["kind"].as_str() == "ln") out.push_back({n["b"].as_str(), 2, d, 0, 2});
    };
    out.push_back({plan["embedding"].as_str(), 1, vocab, d, 0});
    if (plan.has("pos_embedding"))
        out.push_back({plan["pos_embedding"].as_str(), 2, plan["max_pos"].as_int(), d, 0});
    const b2json::Value& blocks = plan["blocks"];
    for (size_t i = 0; i < blocks.size(); ++i) {
        const b2json::Value& b = blocks[i];
        norm(b["norm"]);
        if (b["type"].as_str() == "attn") {
            const long long H = b["n_heads"].as_int(), KVH = b["n_kv_heads"].as_int(),
                            dh = b["d_head"].as_int();
            const int dt = b["dtype"].as_str() == "i8" ? 1 : 2;
            if (tp > 1 && (H % tp || KVH % tp)) throw Err(B2_E_UNSUPPORTED, "heads do not split over the ranks");
            if (dt != 1) no_tp("f32 attention weights");
            split({b["q"].as_str(), dt, H * dh, d, 0});
            split({b["k"].as_str(), dt, KVH * dh, d, 0});
            split({b["v"].as_str(), dt, KVH * dh, d, 0});
            split({b["o"].as_str(), dt, d, H * dh, 0});
            if (b.has("bias")) {
                no_tp("attention biases");
                const b2json::Value& bs = b["bias"];
                const char* proj[4] = {"q", "k", "v", "o"};
                const long long len[4] = {H * dh, KVH * dh, KVH * dh, d};
                for (int k = 0; k < 4; ++k)              // a missing projection bias adds 0
                    if (bs.has(proj[k])) out.push_back({bs[proj[k]].as_str(), 2, len[k], 0, 0});
            }
        } else if (b["kind"].as_str() == "swiglu") {
            const long long ffn = b["d_ffn"].as_int();
            split({b["gate"].as_str(), 1, ffn, d, 0});
            split({b["up"].as_str(), 1, ffn, d, 0});
            split({b["down"].as_str(), 1, d, ffn, 0});
        } else {
            no_tp("GELU feed-forward blocks");
            const long long ffn = b["d_ffn"].as_int();
            out.push_back({b["fc1"].as_str(), 1, ffn, d, 0});
            out.push_back({b["fc1_b"].as_str(), 2, ffn, 0, 0});
            out.push_back({b["fc2"].as_str(), 1, d, ffn, 0});
            out.push_back({b["fc2_b"].as_str(), 2, d, 0, 0});
        }
    }
    norm(plan["final_norm"]);
    split({plan["lm_head"]["W"].as_str(), 1, vocab, d, 0});
    split({plan["lm_head"]["b"].as_str(), 2, vocab, 0, 2});
    return out;
}

long long pad_ld(long long cols, int dtype) { return dtype == 1 ? (cols + 15) / 16 * 16 : (cols + 3) / 4 * 4; }

// ------------------------------------------------------------------ model assembly
void setup_device(b2_ctx* c, int device) {
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) throw Err(B2_E_INVALID, "device index out of range");
    c->device = device;
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) throw Err(B2_E_UNSUPPORTED, "this library is built for sm_100a (B200)");
    c->sm_count = prop.multiProcessorCount;
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking));
    c->own_stream = true;
}

void assemble(b2_ctx* c, const b2json::Value& plan) {
    if (plan["format"].is_null() || plan["format"].as_str() != "b200-decode-plan")
        throw Err(B2_E_FORMAT, "not a b200 decode plan");
    c->vocab = (int)plan["vocab"].as_int();
    c->d = (int)plan["d_model"].as_int();
    c->max_seq = (int)plan["max_seq"].as_int();
    c->token_bytes = plan.has("token_bytes") ? (int)plan["token_bytes"].as_int() : 4;
    c->eps = plan.has("eps") ? (float)plan["eps"].as_num() : 1e-5f;
    c->max_pos = plan.has("max_pos") ? (int)plan["max_pos"].as_int() : 0;
    if (c->d <= 0 || c->vocab <= 0 || c->max_seq <= 0) throw Err(B2_E_FORMAT, "bad plan dimensions");
    c->emb = c->mat(plan["embedding"].as_str(), c->vocab, c->d);
    if (plan.has("pos_embedding")) {
        c->pos_tab = static_cast<const float*>(c->mat(plan["pos_embedding"].as_str(), c->max_pos, c->d).w);
        if (c->mat(plan["pos_embedding"].as_str(), c->max_pos, c->d).ld != c->d)
            throw Err(B2_E_FORMAT, "positional embedding rows must be unpadded");
    }
    const b2json::Value& blocks = plan["blocks"];
    size_t kv_total = 0;
    for (size_t i = 0; i < blocks.size(); ++i) {
        const b2json::Value& b = blocks[i];
        Block B;
        B.norm = c->norm_of(b["norm"]);
        if (b["type"].as_str() == "attn") {
            B.attn = true;
            B.rope = b["rope"].as_bool();
            B.H = (int)b["n_heads"].as_int();
            B.KVH = (int)b["n_kv_heads"].as_int();
            B.dh = (int)b["d_head"].as_int();
            if (B.H <= 0 || B.KVH <= 0 || B.H % B.KVH || B.dh <= 0 || B.dh > 256 || B.dh % 4)
                throw Err(B2_E_UNSUPPORTED, "attention needs n_heads % n_kv_heads == 0 and head_dim "
                                            "a multiple of 4 up to 256");
            if (B.rope && (B.dh % 2)) throw Err(B2_E_FORMAT, "RoPE needs an even head_dim");
            B.H_all = B.H;
            if (B.H % c->tp_size || B.KVH % c->tp_size || c->d % c->tp_size)
                throw Err(B2_E_UNSUPPORTED, "heads or d_model do not split over the ranks");
            B.H /= c->tp_size;                      // this rank's query and KV heads
            B.KVH /= c->tp_size;
            B.head0 = c->tp_rank * B.H;
            const int qd = B.H * B.dh, kd = B.KVH * B.dh;
            B.q = c->mat(b["q"].as_str(), qd, c->d);
            B.k = c->mat(b["k"].as_str(), kd, c->d);
            B.v = c->mat(b["v"].as_str(), kd, c->d);
            B.o = c->mat(b["o"].as_str(), c->d / c->tp_size, B.H_all * B.dh);
            if (B.q.i8 != B.k.i8 || B.q.i8 != B.v.i8 || B.q.i8 != B.o.i8)
                throw Err(B2_E_FORMAT, "attention projections must share one dtype");
            if (b.has("bias")) {
                const b2json::Value& bs = b["bias"];
                B.bias[0] = c->vec(bs["q"], qd);
                B.bias[1] = c->vec(bs["k"], kd);
                B.bias[2] = c->vec(bs["v"], kd);
                B.bias[3] = c->vec(bs["o"], c->d / c->tp_size);
            }
            if (B.rope) {
                const double th = b["theta"].as_num("theta");
                if (c->rope_dh && (c->rope_dh != B.dh || c->rope_theta != th))
                    throw Err(B2_E_UNSUPPORTED, "RoPE sub-blocks must share head_dim and theta");
                c->rope_dh = B.dh;
                c->rope_theta = th;
            }
            kv_total += 2ull * B.KVH * c->max_seq * B.dh;
        } else {
            B.d_ffn = (int)b["d_ffn"].as_int();
            if (B.d_ffn % c->tp_size) throw Err(B2_E_UNSUPPORTED, "d_ffn does not split over the ranks");
            B.ffn_local = B.d_ffn / c->tp_size;
            B.ffn0 = c->tp_rank * B.ffn_local;
            if (b["kind"].as_str() == "swiglu") {
                B.swiglu = true;
                B.w1 = c->mat(b["gate"].as_str(), B.ffn_local, c->d);
                B.w3 = c->mat(b["up"].as_str(), B.ffn_local, c->d);
                B.w2 = c->mat(b["down"].as_str(), c->d / c->tp_size, B.d_ffn);
                if (!B.w1.i8 || !B.w3.i8 || !B.w2.i8)
                    throw Err(B2_E_UNSUPPORTED, "swiglu_ffn weights must be int8 (--quantize int8)");
            } else {
                B.w1 = c->mat(b["fc1"].as_str(), B.d_ffn, c->d);
                B.w2 = c->mat(b["fc2"].as_str(), c->d, B.d_ffn);
                B.b1 = c->vec(b["fc1_b"], B.d_ffn);
                B.b2 = c->vec(b["fc2_b"], c->d);
                if (!B.w1.i8 || !B.w2.i8)
                    throw Err(B2_E_UNSUPPORTED, "linear weights must be int8 (--quantize int8)");
            }
        }
        c->blocks.push_back(B);
    }
    if (plan.has("generation")) {                 // --sample / --rng-seed of the packer
        const b2json::Value& g = plan["generation"];
        if (g.has("sample_mode")) c->samp_mode = (int)g["sample_mode"].as_int();
        if (g.has("top_k")) c->samp_k = (int)g["top_k"].as_int();
        if (g.has("temperature")) c->samp_t = g["temperature"].as_num();
        if (g.has("rng_seed") && !g["rng_seed"].is_null()) c->seed = (unsigned)(long long)g["rng_seed"].as_num();
        c->rng = c->seed;
        if (c->samp_mode < 0 || c->samp_mode > 2) throw Err(B2_E_FORMAT, "unknown sample mode in the plan");
        if (c->samp_mode && c->tp_size > 1) throw Err(B2_E_UNSUPPORTED, "sampling needs every logit on one GPU");
    }
    c->fnorm = c->norm_of(plan["final_norm"]);
    if (c->vocab % c->tp_size) throw Err(B2_E_UNSUPPORTED, "vocab does not split over the ranks");
    c->lm = c->mat(plan["lm_head"]["W"].as_str(), c->vocab / c->tp_size, c->d);
    c->lm_b = c->vec(plan["lm_head"]["b"], c->vocab / c->tp_size);
    if (!c->lm.i8 || !c->emb.i8) throw Err(B2_E_UNSUPPORTED, "embedding and LM head must be int8");

    // ---- KV cache arena
    c->kv_bytes = kv_total * sizeof(float);
    c->kv_bytes_per_pos = c->kv_bytes / (size_t)c->max_seq;
    if (c->kv_bytes) {
        if (cudaMalloc(&c->d_kv, c->kv_bytes) != cudaSuccess) throw Err(B2_E_OOM, "KV cache allocation failed");
        CK(cudaMemsetAsync(c->d_kv, 0, c->kv_bytes, c->stream));
    }
    float* kvp = static_cast<float*>(c->d_kv);
    for (Block& B : c->blocks) {
        if (!B.attn) continue;
        const size_t e = (size_t)B.KVH * c->max_seq * B.dh;
        B.K = kvp; kvp += e;
        B.V = kvp; kvp += e;
    }

    // ---- activations + scratch arena
    int max_q = 1, max_q_all = 1, max_ffn = 1, max_H = 1, max_KVH = 1, max_dh = 1;
    for (const Block& B : c->blocks) {
        if (B.attn) {
            max_q = std::max(max_q, B.H * B.dh);
            max_q_all = std::max(max_q_all, B.H_all * B.dh);
            max_H = std::max(max_H, B.H);
            max_KVH = std::max(max_KVH, B.KVH);
            max_dh = std::max(max_dh, B.dh);
        } else {
            max_ffn = std::max(max_ffn, B.d_ffn);
        }
    }
    c->attn_nsplit_max = (c->max_seq + kAttnChunk - 1) / kAttnChunk;
    std::vector<std::pair<void**, size_t>> plan_mem;
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    size_t off = 0;
    std::vector<size_t> offs;
    auto add = [&](size_t bytes) { offs.push_back(off); off += al(bytes); return offs.size() - 1; };
    const size_t i_rope = add(c->rope_dh ? (size_t)c->max_seq * c->rope_dh * 4 : 16);
    const size_t i_q = add((size_t)max_q * 4);
    const size_t i_seq = add(4);
    const size_t i_logits = add((size_t)c->vocab * 4);
    const size_t i_part = add((size_t)max_H * c->attn_nsplit_max * (max_dh + 2) * 8);   // token kernel: (value, tag) pairs
    const size_t i_acnt = add((size_t)std::max(max_H, max_KVH) * 4);   // per query head (token kernel)
    const size_t i_aval = add((size_t)c->sm_count * 4);
    const size_t i_aidx = add((size_t)c->sm_count * 4);
    const size_t i_anan = add(4);
    const size_t i_amcnt = add(4);
    const size_t i_tkbar = add(8);
    const size_t i_st = add(sizeof(StepState));
    const size_t i_prompt = add((size_t)c->max_seq * 4);
    const size_t i_out = add((size_t)c->max_seq * 4);
    const size_t i_samp = add((size_t)c->vocab * 8);
    const size_t i_tq = add((size_t)max_q * 8);
    const size_t i_tkn = add((size_t)max_KVH * max_dh * 8);
    const size_t i_tvn = add((size_t)max_KVH * max_dh * 8);
    c->work_bytes = off;
    if (cudaMalloc(&c->d_work, c->work_bytes) != cudaSuccess) throw Err(B2_E_OOM, "workspace allocation failed");
    CK(cudaMemsetAsync(c->d_work, 0, c->work_bytes, c->stream));
    char* w = static_cast<char*>(c->d_work);
    c->rope_tab = reinterpret_cast<float*>(w + offs[i_rope]);
    c->q = reinterpret_cast<float*>(w + offs[i_q]);
    c->tk_seq = reinterpret_cast<unsigned*>(w + offs[i_seq]);
    // exchange buffer: x, attention output, FFN hidden vector (whole, on every
    // rank), then the cross-rank flags and argmax candidates
    {
        size_t xo = 0;
        auto xadd = [&](size_t bytes) { const size_t o = xo; xo += al(bytes); return o; };
        const size_t o_x = xadd((size_t)c->d * 4), o_att = xadd((size_t)max_q_all * 4),
                     o_f = xadd((size_t)max_ffn * 4), o_fl = xadd(kMaxRanks * 4), o_afl = xadd(kMaxRanks * 4),
                     o_cv = xadd(kMaxRanks * 4), o_ci = xadd(kMaxRanks * 4), o_cn = xadd(kMaxRanks * 4),
                     o_tx = xadd((size_t)c->d * 8), o_tatt = xadd((size_t)max_q_all * 8),
                     o_tf = xadd((size_t)max_ffn * 8);
        // tensor parallelism: the batched prefill's exchanged activations
        const size_t pfT = c->tp_size > 1
                               ? (size_t)std::min(512, (c->max_seq + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile)
                               : 0;
        const size_t o_pfx = xadd(pfT * c->d * 4), o_pfa = xadd(pfT * max_q_all * 4), o_pff = xadd(pfT * max_ffn * 4),
                     o_pfl = xadd(kMaxRanks * 4), o_pep = xadd(4), o_plg = xadd(pfT * c->vocab * 4);
        c->xch_bytes = xo;
        if (cudaMalloc(&c->d_xch, c->xch_bytes) != cudaSuccess) throw Err(B2_E_OOM, "exchange buffer allocation failed");
        CK(cudaMemsetAsync(c->d_xch, 0, c->xch_bytes, c->stream));
        char* xb = static_cast<char*>(c->d_xch);
        c->x = reinterpret_cast<float*>(xb + o_x);
        c->att = reinterpret_cast<float*>(xb + o_att);
        c->f = reinterpret_cast<float*>(xb + o_f);
        c->tp_flag = reinterpret_cast<unsigned*>(xb + o_fl);
        c->tp_aflag = reinterpret_cast<unsigned*>(xb + o_afl);
        c->tp_cval = reinterpret_cast<float*>(xb + o_cv);
        c->tp_cidx = reinterpret_cast<int*>(xb + o_ci);
        c->tp_cnan = reinterpret_cast<int*>(xb + o_cn);
        // the token kernel's tagged x, attention output and FFN hidden vector: with
        // tensor parallelism the peers write their rows here
        c->tx = reinterpret_cast<unsigned long long*>(xb + o_tx);
        c->tatt = reinterpret_cast<unsigned long long*>(xb + o_tatt);
        c->tf = reinterpret_cast<unsigned long long*>(xb + o_tf);
        if (pfT) {
            c->pfx_tmax = (int)pfT;
            c->pfx_x = reinterpret_cast<float*>(xb + o_pfx);
            c->pfx_att = reinterpret_cast<float*>(xb + o_pfa);
            c->pfx_f = reinterpret_cast<float*>(xb + o_pff);
            c->tp_pflag = reinterpret_cast<unsigned*>(xb + o_pfl);
            c->tp_pepoch = reinterpret_cast<unsigned*>(xb + o_pep);
            c->pfx_logits = reinterpret_cast<float*>(xb + o_plg);
        }
    }
    c->logits = reinterpret_cast<float*>(w + offs[i_logits]);
    c->attn_part = reinterpret_cast<float*>(w + offs[i_part]);
    c->attn_cnt = reinterpret_cast<unsigned*>(w + offs[i_acnt]);
    c->amax_val = reinterpret_cast<float*>(w + offs[i_aval]);
    c->amax_idx = reinterpret_cast<int*>(w + offs[i_aidx]);
    c->amax_v0nan = reinterpret_cast<int*>(w + offs[i_anan]);
    c->amax_cnt = reinterpret_cast<unsigned*>(w + offs[i_amcnt]);
    c->tk_bar = reinterpret_cast<unsigned*>(w + offs[i_tkbar]);
    c->n_attn_cnt = std::max(max_H, max_KVH);
    c->st = reinterpret_cast<StepState*>(w + offs[i_st]);
    c->prompt = reinterpret_cast<int*>(w + offs[i_prompt]);
    c->out_ids = reinterpret_cast<int*>(w + offs[i_out]);
    c->samp_e = reinterpret_cast<double*>(w + offs[i_samp]);
    c->tq = reinterpret_cast<unsigned long long*>(w + offs[i_tq]);
    c->tkn = reinterpret_cast<unsigned long long*>(w + offs[i_tkn]);
    c->tvn = reinterpret_cast<unsigned long long*>(w + offs[i_tvn]);

    // RoPE table in f64 via libm, stored f32 (rope_alloc_f32, rope_f32.ari:34-55)
    if (c->rope_dh) {
        std::vector<float> tab((size_t)c->max_seq * c->rope_dh);
        const double log_theta = std::log(c->rope_theta);
        const int half = c->rope_dh / 2;
        for (int pos = 0; pos < c->max_seq; ++pos)
            for (int i = 0; i < half; ++i) {
                const double exponent = 0.0 - 2.0 * (double)i / (double)c->rope_dh;
                const double freq = std::exp(exponent * log_theta);
                const double angle = (double)pos * freq;
                tab[(size_t)pos * c->rope_dh + 2 * i] = (float)std::cos(angle);
                tab[(size_t)pos * c->rope_dh + 2 * i + 1] = (float)std::sin(angle);
            }
        CK(cudaMemcpyAsync(c->rope_tab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaStreamSynchronize(c->stream));
    }
    CK(cudaMallocHost(&c->h_st, sizeof(StepState)));
    std::memset(c->h_st, 0, sizeof(StepState));

    // batched prefill covers one-GPU Llama-family plans: RMSNorm, int8 RoPE attention,
    // int8 SwiGLU, no learned positions
    c->pf_ok = false;
    const char* pe = std::getenv("B2_PREFILL_BATCHED");
    if (pe && pe[0] == '0') c->pf_why = "batched prefill disabled (B2_PREFILL_BATCHED=0)";
    else if (c->pos_tab) c->pf_why = "learned positional embedding";
    else if (c->emb.i4 || c->lm.i4) c->pf_why = "int4 weights";
    else {
        c->pf_ok = true;
        for (const Block& B : c->blocks) {
            if (B.norm.kind != NORM_RMS) { c->pf_ok = false; c->pf_why = "LayerNorm"; }
            else if (B.attn && (!B.q.i8 || !B.rope)) { c->pf_ok = false; c->pf_why = "f32 or RoPE-less attention"; }
            else if (B.attn && (B.dh > 256 || B.dh % 4)) { c->pf_ok = false; c->pf_why = "head_dim"; }
            else if (!B.attn && !B.swiglu) { c->pf_ok = false; c->pf_why = "GELU feed-forward"; }
        }
    }
}

// ------------------------------------------------------------------ one step's launches
// One operation of a step: what the per-layer path launches as one kernel and
// the token kernel runs as one phase.
struct Op {
    int kind = TK_GEMV;
    bool i8 = true;
    bool mirror = false;      // its output is written to every rank (tensor parallelism)
    GemvParams g{};
    AttnParams a{};
    EmbedParams e{};
};

std::vector<Op> build_ops(b2_ctx* c, bool with_head) {
    std::vector<Op> ops;
    const bool tp = c->tp_size > 1;
    auto gemv = [&](const GemvParams& g, bool i8, bool mirror = false) {
        Op o; o.kind = TK_GEMV; o.g = g; o.i8 = i8; o.mirror = tp && mirror;
        if (o.mirror) o.g.mir = c->mir;
        ops.push_back(o);
    };
    const int d_local = c->d / c->tp_size, d0 = c->tp_rank * d_local;   // this rank's rows of x
    EmbedParams ep{};
    ep.emb = c->emb.w; ep.emb_i8 = c->emb.i4 ? 2 : (c->emb.i8 ? 1 : 0); ep.emb_s = c->emb.s; ep.ld = c->emb.ld;
    ep.pos_tab = c->pos_tab; ep.max_pos = c->max_pos;
    ep.d = c->d; ep.vocab = c->vocab; ep.max_seq = c->max_seq;
    ep.prompt = c->prompt; ep.st = c->st; ep.x = c->x;
    { Op o; o.kind = TK_EMBED; o.e = ep; ops.push_back(o); }

    for (const Block& B : c->blocks) {
        GemvParams p{};
        p.st = c->st;
        p.err = &c->st->err;
        p.eps = c->eps;
        p.norm = B.norm.kind;
        p.ng = B.norm.g;
        p.nb = B.norm.b;
        p.x = c->x;
        p.n = c->d;
        if (B.attn) {
            // Q/K/V projections + RoPE + scale + KV append
            p.W[0] = B.q.w; p.W[1] = B.k.w; p.W[2] = B.v.w;
            p.S[0] = B.q.s; p.S[1] = B.k.s; p.S[2] = B.v.s;
            p.bias[0] = B.bias[0]; p.bias[1] = B.bias[1]; p.bias[2] = B.bias[2];
            p.rows[0] = B.q.rows; p.rows[1] = B.k.rows; p.rows[2] = B.v.rows;
            p.nseg = 3; p.ld = B.q.ld;
            p.epi = EPI_QKV;
            p.rope = B.rope;
            p.rope_tab = c->rope_tab;
            p.dh = B.dh;
            p.qscale = (float)(1.0 / std::sqrt((double)B.dh));
            p.qout = c->q;
            p.kcache = B.K; p.vcache = B.V;
            p.max_seq = c->max_seq;
            gemv(p, B.q.i8);

            AttnParams a{};
            a.q = c->q; a.K = B.K; a.V = B.V; a.out = c->att + (size_t)B.head0 * B.dh;
            a.part = c->attn_part; a.counters = c->attn_cnt;
            a.H = B.H; a.KVH = B.KVH; a.dh = B.dh; a.max_seq = c->max_seq;
            a.nsplit_max = c->attn_nsplit_max;
            a.st = c->st; a.err = &c->st->err;
            if (tp) a.mir = c->mir;
            { Op op; op.kind = TK_ATTN; op.a = a; ops.push_back(op); }
            // token kernel: the splits are merged in a phase of their own (the
            // per-layer attention kernel merges them itself)
            { Op op; op.kind = TK_ACOMB; op.a = a; op.mirror = tp; ops.push_back(op); }

            GemvParams o{};
            o.st = c->st; o.err = &c->st->err;
            o.W[0] = B.o.w; o.S[0] = B.o.s; o.bias[0] = B.bias[3];
            o.rows[0] = B.o.rows; o.nseg = 1; o.ld = B.o.ld;
            o.x = c->att; o.n = B.o.cols; o.norm = NORM_NONE;
            o.epi = EPI_RESID; o.y = c->x + d0; o.resid = c->x + d0;
            gemv(o, B.o.i8, true);
        } else if (B.swiglu) {
            p.W[0] = B.w1.w; p.W[1] = B.w3.w;
            p.S[0] = B.w1.s; p.S[1] = B.w3.s;
            p.rows[0] = B.ffn_local; p.rows[1] = B.ffn_local;
            p.nseg = 2; p.paired = 1; p.ld = B.w1.ld;
            p.epi = EPI_SWIGLU; p.y = c->f + B.ffn0;
            gemv(p, true, true);

            GemvParams dn{};
            dn.st = c->st; dn.err = &c->st->err;
            dn.W[0] = B.w2.w; dn.S[0] = B.w2.s;
            dn.rows[0] = d_local; dn.nseg = 1; dn.ld = B.w2.ld;
            dn.x = c->f; dn.n = B.d_ffn; dn.norm = NORM_NONE;
            dn.epi = EPI_RESID; dn.y = c->x + d0; dn.resid = c->x + d0;
            gemv(dn, true, true);
        } else {
            p.W[0] = B.w1.w; p.S[0] = B.w1.s; p.bias[0] = B.b1;
            p.rows[0] = B.d_ffn; p.nseg = 1; p.ld = B.w1.ld; p.i4 = B.w1.i4;
            p.epi = EPI_GELU; p.y = c->f;
            gemv(p, true);

            GemvParams f2{};
            f2.st = c->st; f2.err = &c->st->err;
            f2.W[0] = B.w2.w; f2.S[0] = B.w2.s; f2.bias[0] = B.b2;
            f2.rows[0] = c->d; f2.nseg = 1; f2.ld = B.w2.ld; f2.i4 = B.w2.i4;
            f2.x = c->f; f2.n = B.d_ffn; f2.norm = NORM_NONE;
            f2.epi = EPI_RESID; f2.y = c->x; f2.resid = c->x;
            gemv(f2, true);
        }
    }
    if (with_head) {
        GemvParams h{};
        h.st = c->st; h.err = &c->st->err;
        h.W[0] = c->lm.w; h.S[0] = c->lm.s; h.bias[0] = c->lm_b;
        h.rows[0] = c->lm.rows; h.nseg = 1; h.ld = c->lm.ld; h.i4 = c->lm.i4;
        h.x = c->x; h.n = c->d;
        h.norm = c->fnorm.kind; h.ng = c->fnorm.g; h.nb = c->fnorm.b; h.eps = c->eps;
        h.row_base = c->tp_rank * c->lm.rows;
        h.epi = EPI_ARGMAX; h.y = c->logits + h.row_base;
        if (tp) {
            h.mir = c->mir;
            h.tp_rank = c->tp_rank; h.tp_size = c->tp_size; h.tp_seq = c->tk_seq;
            h.tp_cval = c->tp_cval; h.tp_cidx = c->tp_cidx; h.tp_cnan = c->tp_cnan; h.tp_aflag = c->tp_aflag;
        }
        h.amax_val = c->amax_val; h.amax_idx = c->amax_idx; h.amax_v0nan = c->amax_v0nan;
        h.amax_count = c->amax_cnt; h.out_ids = c->out_ids;
        h.defer_tok = c->samp_mode != 0;
        gemv(h, true);
    }
    return ops;
}

// per-layer path: one kernel per operation, chained by programmatic dependent launch
int enqueue_step(b2_ctx* c, bool with_head, cudaStream_t s) {
    const std::vector<Op> ops = build_ops(c, with_head);
    int n = 0;
    for (const Op& o : ops) {
        if (o.kind == TK_ACOMB) continue;
        if (o.kind == TK_EMBED) CK(launch_embed(o.e, s, c->pdl));
        else if (o.kind == TK_ATTN) CK(launch_attn(o.a, s, c->pdl));
        else if (o.g.i4) CK(launch_gemv_i4(o.g, s, c->pdl, c->sm_count));
        else CK(launch_gemv(o.g, o.i8, s, c->pdl, c->sm_count));
        ++n;
    }
    return n;
}

// the sampler after the LM head (sampling modes only); returns kernels launched
int enqueue_sampler(b2_ctx* c, cudaStream_t s) {
    if (!c->samp_mode) return 0;
    SampleParams sp{};
    sp.logits = c->logits; sp.e = c->samp_e; sp.vocab = c->vocab;
    sp.mode = c->samp_mode; sp.top_k = c->samp_k; sp.temperature = c->samp_t;
    sp.st = c->st; sp.out_ids = c->out_ids;
    sample_kernel<<<1, kSampleThreads, 0, s>>>(sp);
    CK(cudaGetLastError());
    return 1;
}


// ------------------------------------------------------------------ token kernel
// The phase of one operation; false (with the reason) when its shape is outside
// what the token kernel is compiled for.
bool tk_phase_of(const b2_ctx* c, const Op& o, TkPhase& T, size_t& part_bytes, size_t& vec_floats,
                 std::string& why) {
    T = TkPhase{};
    T.kind = o.kind;
    if (o.kind == TK_EMBED) {
        T.e = o.e;
        return true;
    }
    if (o.kind == TK_ACOMB) {
        T.a = o.a;
        return true;
    }
    if (o.kind == TK_ATTN) {
        T.a = o.a;
        if (o.a.dh > 128 || o.a.dh % 4) { why = "head_dim above 128"; return false; }
        if (c->attn_nsplit_max > kTkMaxSplits) { why = "max_seq above 16384"; return false; }
        return true;
    }
    T.g = o.g;
    const GemvParams& g = o.g;
    if (g.i4) { why = "int4 weights (per-layer int4 kernel)"; return false; }
    const size_t row_bytes = (size_t)g.ld * (o.i8 ? 1 : 4);
    const int K = (int)((row_bytes / 16 + 255) / 256);
    if (K < 1 || K > 3) { why = "weight rows longer than 12 KB"; return false; }
    const bool paired = g.paired != 0;
    if (o.i8) {
        if (K == 1) { T.variant = paired ? TV_I8_K1_R4_P : TV_I8_K1_R8; T.rs = paired ? 4 : 8; }
        else { T.variant = paired ? TV_I8_K3_R1_P : TV_I8_K3_R2; T.rs = paired ? 1 : 2; }
    } else {
        if (paired) { why = "paired f32 weights"; return false; }
        if (K == 1) { T.variant = TV_F32_K1_R8; T.rs = 8; }
        else { T.variant = TV_F32_K3_R2; T.rs = 2; }
    }
    if ((size_t)T.rs * row_bytes * (paired ? 2 : 1) > kTkSlotBytes) { why = "stage above 32 KB"; return false; }
    T.unit = g.rope ? 2 : 1;
    long long total = paired ? g.rows[0] : 0;
    if (!paired)
        for (int k = 0; k < g.nseg; ++k) total += g.rows[k];
    const long long units = (total + T.unit - 1) / T.unit;
    const long long rows_cta = (units + c->sm_count - 1) / c->sm_count * T.unit;
    part_bytes = std::max(part_bytes, (size_t)rows_cta * ((paired ? 2 : 1) * 8 + 4) * sizeof(float));
    T.rows = T.rs;                      // rows per stage (the compiled capacity: all of it is computed)
    // x and its norm gains staged in shared memory: n % 4 (16-byte bulk copies),
    // 16-aligned pointers, L = n rounded up to 16 covering the padded rows
    const size_t L = ((size_t)g.n + 15) & ~(size_t)15;
    const size_t nv = L * (1 + (g.norm != NORM_NONE) + (g.norm == NORM_LN));
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (g.n % 4 || !al16(g.x) || (g.norm != NORM_NONE && !al16(g.ng)) || (g.norm == NORM_LN && !al16(g.nb)) ||
        (size_t)g.ld * (o.i8 ? 1 : 4) > L * (o.i8 ? 1 : 4)) {
        why = "input vector not stageable";
        return false;
    }
    vec_floats = std::max(vec_floats, nv);
    return true;
}

// Let the phases of a table meet through (value, tag) words instead of grid
// barriers. Every activation a phase reads from this launch gets its tagged
// twin and the index of the phase that wrote it; false (table unchanged in its
// meaning) when some input has no twin.
bool tk_tag_table(b2_ctx* c, std::vector<TkPhase>& ph, size_t first, size_t count) {
    int wx = -1, wq = -1, wpart = -1, watt = -1, wf = -1;
    std::vector<TkPhase> out(ph.begin() + first, ph.begin() + first + count);
    for (size_t i = 0; i < out.size(); ++i) {
        TkPhase& T = out[i];
        const int idx = (int)i;
        if (T.kind == TK_EMBED) {
            T.e.tx = c->tx;
            wx = idx;
            continue;
        }
        T.nobar = 1;
        if (T.kind == TK_ATTN) {
            if (wq < 0) return false;
            T.a.tq = c->tq; T.a.tkn = c->tkn; T.a.tvn = c->tvn;
            T.a.tpart = reinterpret_cast<unsigned long long*>(c->attn_part);
            T.tin = wq;
            wpart = idx;
            continue;
        }
        if (T.kind == TK_ACOMB) {
            if (wpart < 0 || T.a.out < c->att) return false;
            T.a.tpart = reinterpret_cast<unsigned long long*>(c->attn_part);
            T.a.tout = c->tatt + (T.a.out - c->att);
            T.tin = wpart;
            watt = idx;
            continue;
        }
        GemvParams& g = T.g;
        if (g.x == c->x) { g.tx = c->tx; T.tin = wx; }
        else if (g.x == c->att) { g.tx = c->tatt; T.tin = watt; }
        else if (g.x == c->f) { g.tx = c->tf; T.tin = wf; }
        else return false;
        if (T.tin < 0) return false;
        if (g.epi == EPI_QKV) {
            g.ty = c->tq; g.tkn = c->tkn; g.tvn = c->tvn;
            wq = idx;
        } else if (g.epi == EPI_RESID) {
            if (g.y < c->x || g.y >= c->x + c->d || g.resid != g.y) return false;
            g.ty = c->tx + (g.y - c->x);
            g.tresid = c->tx + (g.resid - c->x);
            wx = idx;
        } else if (g.epi == EPI_SWIGLU || g.epi == EPI_GELU) {
            if (g.y < c->f) return false;
            g.ty = c->tf + (g.y - c->f);
            wf = idx;
        } else if (g.epi != EPI_ARGMAX) {
            return false;
        }
    }
    std::copy(out.begin(), out.end(), ph.begin() + first);
    return true;
}

bool tk_prepare_kernel(b2_ctx* c, int vs) {
    int per_sm = 0;
    CK(tk_prepare(vs, c->tk_tags, c->tk_smem, &per_sm));
    return per_sm >= 1;
}

// Build both phase tables (prefill: no LM head; decode: with it) and size the
// kernel's shared memory; leaves c->token false with c->token_why otherwise.
void setup_token(b2_ctx* c) {
    c->token = false;
    const char* env = std::getenv("B2_TOKEN_KERNEL");
    if (env && env[0] == '0') { c->token_why = "per-layer kernels requested (B2_TOKEN_KERNEL=0)"; return; }
    int coop = 0;
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device));
    if (!coop) { c->token_why = "no cooperative launch"; return; }
    std::vector<TkPhase> ph;
    size_t part = 0, vec_floats = 0;
    std::string why;
    bool f32 = false;
    for (int head = 0; head < 2; ++head) {
        bool prev_mirror = false;
        for (const Op& o : build_ops(c, head == 1)) {
            TkPhase T;
            if (!tk_phase_of(c, o, T, part, vec_floats, why)) { c->token_why = why; return; }
            if (T.kind == TK_GEMV && T.variant >= TV_F32_K1_R8) f32 = true;
            T.xsync = prev_mirror ? 1 : 0;              // the outputs it reads came from every rank
            prev_mirror = o.mirror;
            ph.push_back(T);
        }
        c->tk_final_xsync[head] = prev_mirror ? 1 : 0;
        if (head == 0) c->nph_prefill = (int)ph.size();
        else c->nph_decode = (int)ph.size() - c->nph_prefill;
    }
    // phase tags and cross-rank epochs are launch count x 1024 + phase: a table of
    // 1024 or more phases would give phase 1024 + k of one launch the tag of phase k
    // of the next one
    if (std::max(c->nph_prefill, c->nph_decode) >= 1024) {
        c->token_why = "more than 1023 phases (phase tags)";
        return;
    }
    // tagged words between phases instead of grid barriers (with tensor
    // parallelism the peers' rows arrive as tagged words too, no cross-rank barrier)
    c->tk_tags = false;
    const char* tg = std::getenv("B2_TK_TAGS");
    if (!(tg && tg[0] == '0')) {
        std::vector<TkPhase> tagged = ph;
        if (tk_tag_table(c, tagged, 0, (size_t)c->nph_prefill) &&
            tk_tag_table(c, tagged, (size_t)c->nph_prefill, (size_t)c->nph_decode)) {
            ph.swap(tagged);
            c->tk_tags = true;
        }
    }
    const size_t vec_off = (kTkPartOffset + part + 127) & ~(size_t)127;
    const size_t ring_off = (vec_off + vec_floats * 4 + 127) & ~(size_t)127;
    c->tk_vec_offset = (int)vec_off;
    c->tk_vec_floats = (int)vec_floats;
    const size_t smem_max = 226 * 1024;             // dynamic; the static argmax slots need the rest
    if (ring_off + 3 * (size_t)kTkSlotBytes > smem_max) { c->token_why = "too many rows per CTA"; return; }
    const int ns_fit = std::min((int)((smem_max - ring_off) / kTkSlotBytes), kTkMaxSlots);
    int ns = std::min(ns_fit, kTkDefaultSlots);
    if (const char* sl = std::getenv("B2_TK_SLOTS"))             // tuning: 3 .. what fits
        ns = std::max(3, std::min(ns_fit, std::atoi(sl)));
    c->tk_ns = ns;
    c->tk_ring_offset = (int)ring_off;
    c->tk_smem = ring_off + (size_t)ns * kTkSlotBytes;
    const char* inf = std::getenv("B2_TK_INFLIGHT");          // tuning: 0 = no cap
    c->tk_inflight = inf ? std::max(0, std::min(ns - 1, std::atoi(inf))) : std::min(kTkInflight, ns - 1);
    c->token_vs = f32 ? 1 : 0;
    if (!tk_prepare_kernel(c, f32 ? 1 : 0)) {
        c->token_why = "token kernel does not fit an SM";
        return;
    }
    if (c->d_phases) { cudaFree(c->d_phases); c->d_phases = nullptr; }
    if (cudaMalloc(&c->d_phases, ph.size() * sizeof(TkPhase)) != cudaSuccess)
        throw Err(B2_E_OOM, "phase table allocation failed");
    CK(cudaMemcpy(c->d_phases, ph.data(), ph.size() * sizeof(TkPhase), cudaMemcpyHostToDevice));
    c->token = true;
    c->token_why.clear();
    const char* tr = std::getenv("B2_TK_TRACE");
    if (tr && tr[0] && !c->d_trace) {
        const size_t n = (size_t)std::max(c->nph_prefill, c->nph_decode) * c->sm_count * kTkStamps;
        if (cudaMalloc(&c->d_trace, n * sizeof(unsigned long long)) != cudaSuccess)
            throw Err(B2_E_OOM, "trace allocation failed");
        CK(cudaMemset(c->d_trace, 0, n * sizeof(unsigned long long)));
        c->trace_path = tr;
        c->trace_kinds.clear();
        for (const TkPhase& T : ph) c->trace_kinds.push_back(T.kind == TK_GEMV ? 10 + T.variant : T.kind);
    }
}

// one step as one cooperative launch (all CTAs resident: the grid barriers need it)
void launch_token(b2_ctx* c, bool with_head, cudaStream_t s) {
    TkParams P{};
    P.phases = c->d_phases + (with_head ? c->nph_prefill : 0);
    P.nphases = with_head ? c->nph_decode : c->nph_prefill;
    P.ns = c->tk_ns;
    P.ring_offset = c->tk_ring_offset;
    P.bar = c->tk_bar;
    P.st = c->st;
    P.prompt = c->prompt;
    P.max_seq = c->max_seq;
    P.max_pos = c->pos_tab ? c->max_pos : 0;
    P.vocab = c->vocab;
    P.trace = c->d_trace;
    P.inflight = c->tk_inflight;
    P.vec_offset = c->tk_vec_offset;
    P.vec_floats = c->tk_vec_floats;
    P.seq = c->tk_seq;
    P.tp_rank = c->tp_rank;
    P.tp_size = c->tp_size;
    P.tp_flag = c->tp_flag;
    P.mir = c->mir;
    P.final_xsync = with_head ? c->tk_final_xsync[1] : c->tk_final_xsync[0];
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)c->sm_count);
    cfg.blockDim = dim3(kTkThreads);
    cfg.dynamicSmemBytes = c->tk_smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    CK(tk_launch(c->token_vs, c->tk_tags, cfg, P));
}

// ------------------------------------------------------------------ batched prefill
void prefill_workspace(b2_ctx* c) {
    if (c->pf_base) return;
    int ld_max = 16, qd = 1, ffn = 1, H = 1, dh = 1;
    for (const Block& B : c->blocks) {
        if (B.attn) {
            ld_max = std::max({ld_max, B.q.ld, B.o.ld});
            qd = std::max(qd, B.H_all * B.dh);
            H = std::max(H, B.H);
            dh = std::max(dh, B.dh);
        } else {
            ld_max = std::max({ld_max, B.w1.ld, B.w2.ld});
            ffn = std::max(ffn, B.d_ffn);
        }
    }
    c->pf_ldp = (ld_max + 127) / 128 * 128;
    c->pf_tmax = std::min(512, (c->max_seq + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile);
    const size_t T = (size_t)c->pf_tmax;
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    const size_t b_planes = al(4 * T * c->pf_ldp), b_S = al(T * 4), b_x = al(T * c->d * 4),
                 b_q = al(T * qd * 4), b_f = al(T * ffn * 4),
                 b_part = al(T * H * (size_t)c->attn_nsplit_max * (dh + 2) * 4);
    const size_t b_acc = al((size_t)kPfSplitTiles * kPfSplitCols * kPfRows * 8), b_cnt = al(kPfSplitCounters * 4);
    const size_t total = b_planes + b_S + b_x + 2 * b_q + b_f + b_part + b_acc + b_cnt;
    if (cudaMalloc(&c->pf_base, total) != cudaSuccess) throw Err(B2_E_OOM, "prefill workspace allocation failed");
    char* w = static_cast<char*>(c->pf_base);
    c->pf_planes = reinterpret_cast<unsigned char*>(w); w += b_planes;
    c->pf_S = reinterpret_cast<int*>(w); w += b_S;
    c->pf_x = reinterpret_cast<float*>(w); w += b_x;
    c->pf_q = reinterpret_cast<float*>(w); w += b_q;
    c->pf_att = reinterpret_cast<float*>(w); w += b_q;
    c->pf_f = reinterpret_cast<float*>(w); w += b_f;
    if (c->tp_size > 1) {                       // the exchanged ones: in the exchange buffer
        if (c->pfx_tmax < c->pf_tmax) throw Err(B2_E_INVALID, "prefill exchange region too small");
        c->pf_x = c->pfx_x; c->pf_att = c->pfx_att; c->pf_f = c->pfx_f;
    }
    c->pf_part = reinterpret_cast<float*>(w); w += b_part;
    c->pf_acc = reinterpret_cast<unsigned long long*>(w); w += b_acc;
    c->pf_cnt = reinterpret_cast<unsigned*>(w);
    // plane rows past the chunk's tokens must read as zeros; the split-K totals and
    // counters start (and are left by every launch) at zero
    CK(cudaMemsetAsync(c->pf_planes, 0, b_planes, c->stream));
    CK(cudaMemsetAsync(c->pf_acc, 0, b_acc + b_cnt, c->stream));
}

// Tokens [p0, p0 + T) of the device id buffer `ids` through every sub-block, no LM
// head: the KV cache ends as n decode steps would leave it, bit for bit. seq >= 0:
// sequence seq of the batched state (its own cache).
void enqueue_prefill_chunk(b2_ctx* c, int p0, int T, cudaStream_t s, const int* ids = nullptr, int seq = -1) {
    if (!ids) ids = c->prompt;
    int* err = &c->st->err;
    const int Tpad = (T + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile;
    auto planes = [&](const float* x, int ldx, int n, const NormRef* nr) {
        PfPlanesParams pp{};
        pp.x = x; pp.ldx = ldx; pp.n = n;
        pp.norm = nr ? nr->kind : NORM_NONE; pp.g = nr ? nr->g : nullptr; pp.eps = c->eps;
        pp.planes = c->pf_planes; pp.ldp = c->pf_ldp; pp.kp = c->pf_ldp; pp.Tpad = Tpad; pp.S = c->pf_S;
        CK(launch_prefill_planes(pp, T, s));
    };
    // tensor parallelism: a rank's rows of x, its heads of the attention output and its
    // columns of the FFN hidden go to every rank's copy (mirrored stores), and a flag
    // barrier follows each such launch before any rank reads the whole row
    const bool tp = c->tp_size > 1;
    const Mirror nomir{};
    const Mirror& mir = tp ? c->mir : nomir;
    const int d0 = c->tp_rank * (c->d / c->tp_size);
    auto sync = [&]() {
        if (tp) CK(launch_tp_sync(c->tp_pflag, c->mir, c->tp_rank, c->tp_size, c->tp_pepoch, err, s));
    };
    auto gemm = [&](int nm, const DevMat& A, const DevMat* A1, int epi, float* out, int ldo, const float* bias,
                    const Block* B, float* cache) {
        PfGemmParams g{};
        g.mir = (epi == PF_RESID || epi == PF_SWIGLU || epi == PF_STORE) ? mir : nomir;
        g.M = A.rows; g.K = A.ld; g.T = T; g.Tpad = Tpad; g.epi = epi; g.S = c->pf_S;
        g.scale[0] = A.s; g.scale[1] = A1 ? A1->s : A.s; g.bias = bias;
        g.out = out; g.ldo = ldo; g.err = err; g.pos0 = p0; g.max_seq = c->max_seq;
        if (B) { g.rope = B->rope; g.rope_tab = c->rope_tab; g.dh = B->dh; g.qscale = (float)(1.0 / std::sqrt((double)B->dh)); }
        g.cache = cache;
        g.acc = c->pf_acc; g.cnt = c->pf_cnt;
        CK(launch_prefill_gemm(nm, A.w, A1 ? A1->w : nullptr, c->pf_planes, c->pf_ldp, g, s));
    };
    CK(launch_prefill_embed(static_cast<const int8_t*>(c->emb.w), c->emb.s, c->emb.ld, ids, p0, c->vocab,
                            c->d, c->pf_x, T, err, s));
    for (size_t bi = 0; bi < c->blocks.size(); ++bi) {
        const Block& B = c->blocks[bi];
        planes(c->pf_x, c->d, c->d, &B.norm);
        if (B.attn) {
            const int qd = B.H * B.dh;
            float* Kc = seq < 0 ? B.K : c->bt_K[bi] + (size_t)seq * c->bt_seq_stride;
            float* Vc = seq < 0 ? B.V : c->bt_V[bi] + (size_t)seq * c->bt_seq_stride;
            gemm(1, B.q, nullptr, PF_Q, c->pf_q, qd, B.bias[0], &B, nullptr);
            gemm(1, B.k, nullptr, PF_K, nullptr, 0, B.bias[1], &B, Kc);
            gemm(1, B.v, nullptr, PF_V, nullptr, 0, B.bias[2], &B, Vc);
            PfAttnParams a{};
            const int qall = B.H_all * B.dh;
            a.q = c->pf_q; a.K = Kc; a.V = Vc; a.out = c->pf_att + (size_t)B.head0 * B.dh; a.ldo = qall;
            a.mir = mir; a.part = c->pf_part;
            a.H = B.H; a.KVH = B.KVH; a.dh = B.dh; a.max_seq = c->max_seq; a.nsplit_max = c->attn_nsplit_max;
            a.T = T; a.pos0 = p0; a.err = err;
            CK(launch_prefill_attn(a, s));
            sync();
            planes(c->pf_att, qall, qall, nullptr);
            gemm(1, B.o, nullptr, PF_RESID, c->pf_x + d0, c->d, B.bias[3], nullptr, nullptr);
            sync();
        } else {
            gemm(2, B.w1, &B.w3, PF_SWIGLU, c->pf_f + B.ffn0, B.d_ffn, nullptr, nullptr, nullptr);
            sync();
            planes(c->pf_f, B.d_ffn, B.d_ffn, nullptr);
            gemm(1, B.w2, nullptr, PF_RESID, c->pf_x + d0, c->d, nullptr, nullptr, nullptr);
            sync();
        }
    }
}

void enqueue_prefill(b2_ctx* c, int p0, int n, cudaStream_t s, const int* ids = nullptr, int seq = -1) {
    prefill_workspace(c);
    for (int done = 0; done < n; done += c->pf_tmax)
        enqueue_prefill_chunk(c, p0 + done, std::min(c->pf_tmax, n - done), s, ids, seq);
}

// ------------------------------------------------------------------ batched decode
BatchState batch_state(b2_ctx* c) {
    BatchState b{};
    b.tok = c->bt_tok; b.pos = c->bt_pos; b.out = c->bt_out; b.n_steps = c->bt_nsteps;
    b.max_steps = c->bt_max_steps; b.max_seq = c->max_seq; b.err = &c->st->err;
    return b;
}

// One step of every sequence: the token each feeds (bt_tok) at its position
// (bt_pos) through the model on the tensor cores (one GEMM over the bt_n tokens
// per projection, each row the exact dot of the one-sequence path), decode
// attention per sequence over its own cache, the LM head for every sequence, the
// greedy token fed back and recorded.
void enqueue_batch_step(b2_ctx* c, cudaStream_t s) {
    const int Bn = c->bt_n;
    int* err = &c->st->err;
    const BatchState bs = batch_state(c);
    CK(launch_batch_check(bs, Bn, s));
    const int Tpad = (Bn + kPfTokenTile - 1) / kPfTokenTile * kPfTokenTile;
    auto planes = [&](const float* x, int ldx, int n, const NormRef* nr) {
        PfPlanesParams pp{};
        pp.x = x; pp.ldx = ldx; pp.n = n;
        pp.norm = nr ? nr->kind : NORM_NONE; pp.g = nr ? nr->g : nullptr; pp.eps = c->eps;
        pp.planes = c->pf_planes; pp.ldp = c->pf_ldp; pp.kp = c->pf_ldp; pp.Tpad = Tpad; pp.S = c->pf_S;
        CK(launch_prefill_planes(pp, Bn, s));
    };
    // tensor parallelism: a rank's rows of x, its heads of the attention output and its
    // columns of the FFN hidden go to every rank's copy (mirrored stores), and a flag
    // barrier follows each such launch before any rank reads the whole row
    const bool tp = c->tp_size > 1;
    const Mirror nomir{};
    const Mirror& mir = tp ? c->mir : nomir;
    const int d0 = c->tp_rank * (c->d / c->tp_size);
    auto sync = [&]() {
        if (tp) CK(launch_tp_sync(c->tp_pflag, c->mir, c->tp_rank, c->tp_size, c->tp_pepoch, err, s));
    };
    auto gemm = [&](int nm, const DevMat& A, const DevMat* A1, int epi, float* out, int ldo, const float* bias,
                    const Block* B, float* cache) {
        PfGemmParams g{};
        g.mir = (epi == PF_RESID || epi == PF_SWIGLU || epi == PF_STORE) ? mir : nomir;
        g.M = A.rows; g.K = A.ld; g.T = Bn; g.Tpad = Tpad; g.epi = epi; g.S = c->pf_S;
        g.scale[0] = A.s; g.scale[1] = A1 ? A1->s : A.s; g.bias = bias;
        g.out = out; g.ldo = ldo; g.err = err; g.pos0 = 0; g.max_seq = c->max_seq;
        g.tok_pos = c->bt_pos; g.cache_seq = c->bt_seq_stride;
        if (B) { g.rope = B->rope; g.rope_tab = c->rope_tab; g.dh = B->dh; g.qscale = (float)(1.0 / std::sqrt((double)B->dh)); }
        g.cache = cache;
        g.acc = c->pf_acc; g.cnt = c->pf_cnt;
        CK(launch_prefill_gemm(nm, A.w, A1 ? A1->w : nullptr, c->pf_planes, c->pf_ldp, g, s));
    };
    CK(launch_prefill_embed(static_cast<const int8_t*>(c->emb.w), c->emb.s, c->emb.ld, c->bt_tok, 0, c->vocab, c->d,
                            c->pf_x, Bn, err, s));
    for (size_t bi = 0; bi < c->blocks.size(); ++bi) {
        const Block& B = c->blocks[bi];
        planes(c->pf_x, c->d, c->d, &B.norm);
        if (B.attn) {
            const int qd = B.H * B.dh;
            gemm(1, B.q, nullptr, PF_Q, c->pf_q, qd, B.bias[0], &B, nullptr);
            gemm(1, B.k, nullptr, PF_K, nullptr, 0, B.bias[1], &B, c->bt_K[bi]);
            gemm(1, B.v, nullptr, PF_V, nullptr, 0, B.bias[2], &B, c->bt_V[bi]);
            const int qall = B.H_all * B.dh;
            AttnParams a{};
            a.q = c->pf_q; a.K = c->bt_K[bi]; a.V = c->bt_V[bi]; a.out = c->pf_att + (size_t)B.head0 * B.dh;
            a.mir = mir; a.part = c->bt_part; a.counters = c->bt_cnt;
            a.H = B.H; a.KVH = B.KVH; a.dh = B.dh; a.max_seq = c->max_seq; a.nsplit_max = c->attn_nsplit_max;
            a.st = nullptr; a.err = err; a.n_of = c->bt_pos;
            a.sq = qd; a.skv = c->bt_seq_stride; a.spart = (long long)B.H * c->attn_nsplit_max * (B.dh + 2);
            CK(launch_batch_attn(a, Bn, qall, s));
            sync();
            planes(c->pf_att, qall, qall, nullptr);
            gemm(1, B.o, nullptr, PF_RESID, c->pf_x + d0, c->d, B.bias[3], nullptr, nullptr);
            sync();
        } else {
            gemm(2, B.w1, &B.w3, PF_SWIGLU, c->pf_f + B.ffn0, B.d_ffn, nullptr, nullptr, nullptr);
            sync();
            planes(c->pf_f, B.d_ffn, B.d_ffn, nullptr);
            gemm(1, B.w2, nullptr, PF_RESID, c->pf_x + d0, c->d, nullptr, nullptr, nullptr);
            sync();
        }
    }
    // the LM head: each rank its vocabulary rows, into every rank's logits; every
    // rank then takes the same greedy ids from the whole rows
    planes(c->pf_x, c->d, c->d, &c->fnorm);
    gemm(1, c->lm, nullptr, PF_STORE, c->bt_logits + (size_t)c->tp_rank * c->lm.rows, c->vocab, c->lm_b, nullptr,
         nullptr);
    sync();
    CK(launch_batch_tail(c->bt_logits, c->vocab, bs, Bn, s));
}

void batch_init(b2_ctx* c, int n, int max_steps) {
    if (!c->pf_ok) throw Err(B2_E_UNSUPPORTED, "batched decode needs a plan the tensor-core path covers: " + c->pf_why);
    if (n < 1 || n > 512 || max_steps < 1) throw Err(B2_E_INVALID, "batch size 1..512 and max_steps >= 1");
    if (c->bt_base) throw Err(B2_E_INVALID, "batched state already initialised");
    prefill_workspace(c);
    if (n > c->pf_tmax) throw Err(B2_E_UNSUPPORTED, "batch larger than the prefill tile capacity");
    size_t kv = 0;
    int H = 1, dh = 1;
    for (const Block& B : c->blocks)
        if (B.attn) {
            kv += 2ull * n * B.KVH * c->max_seq * B.dh;
            H = std::max(H, B.H);
            dh = std::max(dh, B.dh);
        }
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t b_kv = al(kv * 4), b_i = al((size_t)n * 4), b_out = al((size_t)max_steps * n * 4),
                 b_ids = al((size_t)c->max_seq * 4), b_log = c->tp_size > 1 ? 0 : al((size_t)n * c->vocab * 4),
                 b_part = al((size_t)n * H * c->attn_nsplit_max * (dh + 2) * 4), b_cnt = al((size_t)n * H * 4);
    const size_t total = b_kv + 2 * b_i + b_out + 256 + b_ids + b_log + b_part + b_cnt;
    if (cudaMalloc(&c->bt_base, total) != cudaSuccess) throw Err(B2_E_OOM, "batched state allocation failed");
    char* w = static_cast<char*>(c->bt_base);
    float* kvp = reinterpret_cast<float*>(w); w += b_kv;
    c->bt_tok = reinterpret_cast<int*>(w); w += b_i;
    c->bt_pos = reinterpret_cast<int*>(w); w += b_i;
    c->bt_out = reinterpret_cast<int*>(w); w += b_out;
    c->bt_nsteps = reinterpret_cast<int*>(w); w += 256;
    c->bt_ids = reinterpret_cast<int*>(w); w += b_ids;
    c->bt_logits = reinterpret_cast<float*>(w); w += b_log;
    if (c->tp_size > 1) c->bt_logits = c->pfx_logits;   // every rank writes its rows into every copy
    c->bt_part = reinterpret_cast<float*>(w); w += b_part;
    c->bt_cnt = reinterpret_cast<unsigned*>(w);
    c->bt_K.assign(c->blocks.size(), nullptr);
    c->bt_V.assign(c->blocks.size(), nullptr);
    for (size_t bi = 0; bi < c->blocks.size(); ++bi) {
        const Block& B = c->blocks[bi];
        if (!B.attn) continue;
        const size_t per = (size_t)n * B.KVH * c->max_seq * B.dh;
        c->bt_K[bi] = kvp; kvp += per;
        c->bt_V[bi] = kvp; kvp += per;
        c->bt_seq_stride = (long long)B.KVH * c->max_seq * B.dh;
    }
    c->bt_n = n;
    c->bt_max_steps = max_steps;
    CK(cudaMemsetAsync(c->bt_tok, 0, 2 * b_i + b_out + 256, c->stream));
    CK(cudaMemsetAsync(c->bt_cnt, 0, b_cnt, c->stream));
    c->bt_pos_host.assign(n, 0);
    c->bt_steps_host = 0;
    // one step as a graph (fixed pointers; positions and tokens live on the device)
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
    try {
        enqueue_batch_step(c, c->cap_stream);
    } catch (...) {
        cudaStreamEndCapture(c->cap_stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    CK(cudaStreamEndCapture(c->cap_stream, &g));
    const cudaError_t e = cudaGraphInstantiate(&c->g_batch, g, 0);
    cudaGraphDestroy(g);
    CK(e);
    CK(cudaStreamSynchronize(c->stream));
}

// the batched path reports device errors through the step state's error word
void batch_begin(b2_ctx* c) {
    if (!c->bt_base) throw Err(B2_E_INVALID, "batched decode not initialised (b2_batch_init)");
    CK(cudaMemsetAsync(&c->st->err, 0, sizeof(int), c->stream));
}

void capture_graphs_once(b2_ctx* c);

void capture_graphs(b2_ctx* c) {
    const char* env = std::getenv("B2_NO_PDL");
    c->pdl = !(env && env[0] == '1');
    setup_token(c);
    if (c->tp_size > 1 && !c->token)
        throw Err(B2_E_UNSUPPORTED, "tensor parallelism needs the token kernel: " + c->token_why);
    if (c->token) {
        try {
            capture_graphs_once(c);
            return;
        } catch (const Err& e) {
            if (c->tp_size > 1) throw;
            cudaGetLastError();
            c->token = false;
            c->token_why = std::string("graph capture failed: ") + e.what();
        }
    }
    try {
        capture_graphs_once(c);
    } catch (const Err&) {
        if (!c->pdl) throw;
        cudaGetLastError();            // clear, then capture without PDL edges
        c->pdl = false;
        capture_graphs_once(c);
    }
}

void capture_graphs_once(b2_ctx* c) {
    if (c->g_prefill) { cudaGraphExecDestroy(c->g_prefill); c->g_prefill = nullptr; }
    if (c->g_decode) { cudaGraphExecDestroy(c->g_decode); c->g_decode = nullptr; }
    for (int head = 0; head < 2; ++head) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
        int n = 0;
        try {
            if (c->token) {
                launch_token(c, head == 1, c->cap_stream);
                n = 1;
            } else {
                n = enqueue_step(c, head == 1, c->cap_stream);
            }
            if (head == 1) n += enqueue_sampler(c, c->cap_stream);
        } catch (...) {
            cudaStreamEndCapture(c->cap_stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        CK(cudaStreamEndCapture(c->cap_stream, &g));
        cudaGraphExec_t ex = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        CK(e);
        if (head) { c->g_decode = ex; c->kernels_decode = n; }
        else { c->g_prefill = ex; c->kernels_prefill = n; }
    }
}

// grid-barrier and last-CTA counters back to zero (they are zero after every
// completed step; a step that timed out may leave them set)
void clear_tickets(b2_ctx* c, cudaStream_t s) {
    CK(cudaMemsetAsync(c->tk_bar, 0, 2 * sizeof(unsigned), s));
    CK(cudaMemsetAsync(c->amax_cnt, 0, sizeof(unsigned), s));
    CK(cudaMemsetAsync(c->attn_cnt, 0, (size_t)c->n_attn_cnt * sizeof(unsigned), s));
}

void upload_state(b2_ctx* c, int step, int prompt_len, int max_new, int next_tok, int eos) {
    StepState& h = *c->h_st;
    std::memset(&h, 0, sizeof(h));
    h.step = step;
    h.pos = step;
    h.prompt_len = prompt_len;
    h.max_new = max_new;
    h.next_tok = next_tok;
    h.n_out = 0;
    h.active = 1;
    h.eos = eos;
    h.err = 0;
    h.rng = c->rng;
    CK(cudaMemcpyAsync(c->st, c->h_st, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    clear_tickets(c, c->stream);
}

int fetch_state(b2_ctx* c) {
    CK(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    c->host_step = c->h_st->step;
    c->rng = c->h_st->rng;
    if (c->h_st->err == B2_DEV_ERR_KV_OVERFLOW) throw Err(B2_E_KV_OVERFLOW, "KV cache overflow on the device");
    if (c->h_st->err == B2_DEV_ERR_BAD_TOKEN) throw Err(B2_E_INVALID, "token id outside the vocabulary");
    if (c->h_st->err) throw Err(B2_E_DEVICE, "device wait timed out (error word " +
                                                 std::to_string(c->h_st->err) + ")");
    return B2_OK;
}

// The blob's header and tensor table (file offsets relative to its data region)
struct BlobIndex {
    std::map<std::string, TensorInfo> tensors;
    uint64_t data_off = 0, data_bytes = 0, csum = 0;
};

BlobIndex read_blob_index(FILE* f, std::string* embedded_plan) {
    BlobIndex ix;
    unsigned char hdr[64];
    if (std::fread(hdr, 1, 64, f) != 64 || std::memcmp(hdr, "B2DBLOB1", 8) != 0)
        throw Err(B2_E_FORMAT, "not a b200 decode blob");
    uint32_t ver, ntens, plan_len;
    uint64_t table_off, plan_off;
    std::memcpy(&ver, hdr + 8, 4);
    std::memcpy(&ntens, hdr + 12, 4);
    std::memcpy(&table_off, hdr + 16, 8);
    std::memcpy(&ix.data_off, hdr + 24, 8);
    std::memcpy(&ix.data_bytes, hdr + 32, 8);
    std::memcpy(&ix.csum, hdr + 40, 8);
    std::memcpy(&plan_len, hdr + 48, 4);
    std::memcpy(&plan_off, hdr + 56, 8);
    if (ver != 1) throw Err(B2_E_FORMAT, "unsupported blob version");
    std::vector<unsigned char> table((size_t)ntens * 128);
    if (std::fseek(f, (long)table_off, SEEK_SET) || std::fread(table.data(), 1, table.size(), f) != table.size())
        throw Err(B2_E_FORMAT, "truncated tensor table");
    embedded_plan->resize(plan_len);
    if (std::fseek(f, (long)plan_off, SEEK_SET) ||
        std::fread(&(*embedded_plan)[0], 1, plan_len, f) != plan_len)
        throw Err(B2_E_FORMAT, "truncated plan");
    for (uint32_t i = 0; i < ntens; ++i) {
        const unsigned char* e = table.data() + 128 * (size_t)i;
        char name[65] = {0};
        std::memcpy(name, e, 64);
        TensorInfo t;
        uint32_t dtype, ndim;
        uint64_t s0, s1, ld, off, nb;
        std::memcpy(&dtype, e + 64, 4);
        std::memcpy(&ndim, e + 68, 4);
        std::memcpy(&s0, e + 72, 8);
        std::memcpy(&s1, e + 80, 8);
        std::memcpy(&ld, e + 88, 8);
        std::memcpy(&off, e + 96, 8);
        std::memcpy(&nb, e + 104, 8);
        t.dtype = (int)dtype;
        t.two_d = ndim == 2;
        t.rows = (long long)(t.two_d ? s0 : 1);
        t.cols = (long long)(t.two_d ? s1 : s0);
        t.ld = (long long)ld;
        t.off = (size_t)off;
        t.nbytes = (size_t)nb;
        if ((dtype < 1 || dtype > 3) || off + nb > ix.data_bytes)
            throw Err(B2_E_FORMAT, std::string("bad table entry for ") + name);
        ix.tensors[name] = t;
    }
    return ix;
}

// One byte range of the blob's data region and where it goes in the weight arena.
struct CopyRange { uint64_t src, bytes; size_t dst; };

// Stream the blob's whole data region through two pinned buffers, checksumming it
// on the host as it passes and copying the parts in `ranges` (sorted by src, not
// overlapping) to the weight arena.
void stream_blob(b2_ctx* c, FILE* f, const BlobIndex& ix, const std::vector<CopyRange>& ranges) {
    const size_t chunk = 64ull << 20;
    unsigned char* pin[2] = {nullptr, nullptr};
    CK(cudaMallocHost(&pin[0], chunk));
    CK(cudaMallocHost(&pin[1], chunk));
    struct PinFree { unsigned char** p; ~PinFree() { cudaFreeHost(p[0]); cudaFreeHost(p[1]); } } pf{pin};
    cudaEvent_t ev[2];
    CK(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
    struct EvFree { cudaEvent_t* e; ~EvFree() { cudaEventDestroy(e[0]); cudaEventDestroy(e[1]); } } ef{ev};
    if (std::fseek(f, (long)ix.data_off, SEEK_SET)) throw Err(B2_E_FORMAT, "truncated data region");
    uint64_t sum = 0;
    size_t done = 0, ri = 0;
    int k = 0;
    bool used[2] = {false, false};
    while (done < ix.data_bytes) {
        const size_t n = std::min(chunk, (size_t)ix.data_bytes - done);
        if (used[k]) CK(cudaEventSynchronize(ev[k]));
        if (std::fread(pin[k], 1, n, f) != n) throw Err(B2_E_FORMAT, "truncated data region");
        sum += checksum_words(pin[k], n, done / 8);
        while (ri < ranges.size() && ranges[ri].src + ranges[ri].bytes <= done) ++ri;
        for (size_t r = ri; r < ranges.size() && ranges[r].src < done + n; ++r) {
            const uint64_t lo = std::max<uint64_t>(ranges[r].src, done);
            const uint64_t hi = std::min<uint64_t>(ranges[r].src + ranges[r].bytes, done + n);
            if (lo < hi)
                CK(cudaMemcpyAsync(static_cast<char*>(c->d_weights) + ranges[r].dst + (lo - ranges[r].src),
                                   pin[k] + (lo - done), hi - lo, cudaMemcpyHostToDevice, c->stream));
        }
        CK(cudaEventRecord(ev[k], c->stream));
        used[k] = true;
        done += n;
        k ^= 1;
    }
    CK(cudaStreamSynchronize(c->stream));
    if (sum != ix.csum) throw Err(B2_E_FORMAT, "blob checksum mismatch");
}

void load_blob(b2_ctx* c, const char* path, std::string* embedded_plan) {
    FILE* f = std::fopen(path, "rb");
    if (!f) throw Err(B2_E_IO, std::string("cannot open blob ") + path);
    struct Closer { FILE* f; ~Closer() { std::fclose(f); } } closer{f};
    BlobIndex ix = read_blob_index(f, embedded_plan);
    c->tensors = ix.tensors;
    if (cudaMalloc(&c->d_weights, ix.data_bytes) != cudaSuccess) throw Err(B2_E_OOM, "weight allocation failed");
    c->weight_bytes = ix.data_bytes;
    stream_blob(c, f, ix, {CopyRange{0, ix.data_bytes, 0}});
}

// Tensor parallelism from a packed blob: this rank's rows of every row-split
// tensor (plan_needs) and the whole of every replicated one, laid out in a new
// arena with the blob's row strides; the whole data region is still read once
// for the checksum.
void load_blob_rank(b2_ctx* c, const char* path, const char* plan_json) {
    FILE* f = std::fopen(path, "rb");
    if (!f) throw Err(B2_E_IO, std::string("cannot open blob ") + path);
    struct Closer { FILE* f; ~Closer() { std::fclose(f); } } closer{f};
    std::string embedded;
    BlobIndex ix = read_blob_index(f, &embedded);
    const b2json::Value plan = b2json::parse(plan_json ? std::string(plan_json) : embedded);
    std::vector<Need> needs = plan_needs(plan, c->tp_size, c->tp_rank);
    std::vector<CopyRange> ranges;
    size_t off = 0;
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    auto take = [&](const std::string& name, long long row0, long long rows) {
        auto it = ix.tensors.find(name);
        if (it == ix.tensors.end()) throw Err(B2_E_FORMAT, "blob has no tensor '" + name + "'");
        const TensorInfo& t = it->second;
        const size_t esz = t.dtype == 1 ? 1 : 4;
        TensorInfo loc = t;
        const size_t row_bytes = t.two_d ? (size_t)t.ld * esz : esz;       // 1-D: one element a row
        const long long full = t.two_d ? t.rows : t.cols;
        if (row0 + rows > full) throw Err(B2_E_FORMAT, "tensor '" + name + "' is smaller than the plan says");
        if (t.two_d) loc.rows = rows; else loc.cols = rows;
        loc.nbytes = (size_t)rows * row_bytes;
        loc.off = off;
        ranges.push_back({t.off + (uint64_t)row0 * row_bytes, loc.nbytes, off});
        off = al(off + loc.nbytes);
        c->tensors[name] = loc;
    };
    for (const Need& nd : needs) {
        if (c->tensors.count(nd.name)) continue;
        take(nd.name, nd.row0, nd.rows);
        if (nd.dtype == 1) take(nd.name + "_scales", nd.row0, nd.rows);
    }
    std::sort(ranges.begin(), ranges.end(), [](const CopyRange& a, const CopyRange& b) { return a.src < b.src; });
    if (cudaMalloc(&c->d_weights, off) != cudaSuccess) throw Err(B2_E_OOM, "weight allocation failed");
    c->weight_bytes = off;
    stream_blob(c, f, ix, ranges);
    assemble(c, plan);
}

void synth_weights(b2_ctx* c, const b2json::Value& plan, uint64_t seed, float stdv) {
    std::vector<Need> needs = plan_needs(plan, c->tp_size, c->tp_rank);
    size_t off = 0;
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    for (const Need& nd : needs) {
        if (c->tensors.count(nd.name)) continue;
        TensorInfo t;
        t.dtype = nd.dtype;
        t.two_d = nd.cols > 0;
        t.rows = t.two_d ? nd.rows : 1;
        t.cols = t.two_d ? nd.cols : nd.rows;
        t.ld = t.two_d ? pad_ld(nd.cols, nd.dtype) : t.cols;
        t.nbytes = (size_t)t.rows * t.ld * (nd.dtype == 1 ? 1 : 4);
        t.off = off;
        off = al(off + t.nbytes);
        c->tensors[nd.name] = t;
        if (nd.dtype == 1) {
            TensorInfo s;
            s.dtype = 2; s.two_d = false; s.rows = 1; s.cols = nd.rows; s.ld = nd.rows;
            s.nbytes = (size_t)nd.rows * 4;
            s.off = off;
            off = al(off + s.nbytes);
            c->tensors[nd.name + "_scales"] = s;
        }
    }
    if (cudaMalloc(&c->d_weights, off) != cudaSuccess) throw Err(B2_E_OOM, "weight allocation failed");
    c->weight_bytes = off;
    char* base = static_cast<char*>(c->d_weights);
    for (const Need& nd : needs) {
        const TensorInfo& t = c->tensors[nd.name];
        const uint64_t tid = fnv1a64(nd.name);
        if (nd.dtype == 1) {
            const TensorInfo& s = c->tensors[nd.name + "_scales"];
            const long long rows = t.rows;
            synth_quant_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, c->stream>>>(
                seed, tid, t.cols, stdv, nd.row0, nd.row0 + rows, 0, t.cols, reinterpret_cast<int8_t*>(base + t.off),
                t.ld, reinterpret_cast<float*>(base + s.off));
        } else if (nd.init == 0) {
            if (nd.row0) throw Err(B2_E_UNSUPPORTED, "random f32 tensors are not split");
            const long long tot = t.rows * t.ld;
            synth_fill_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, c->stream>>>(
                seed, tid, t.rows, t.cols, t.ld, stdv, reinterpret_cast<float*>(base + t.off));
        } else {
            const long long tot = t.rows * t.ld;
            fill_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, c->stream>>>(
                reinterpret_cast<float*>(base + t.off), tot, nd.init == 1 ? 1.0f : 0.0f);
        }
        CK(cudaGetLastError());
    }
    CK(cudaStreamSynchronize(c->stream));
}

int fail(b2_ctx* c, const Err& e) {
    if (c) c->err = e.what();
    else g_last_create_error = e.what();
    return e.code;
}

template <typename F>
int guarded(b2_ctx* c, F&& f) {
    if (!c) return B2_E_INVALID;
    try {
        cudaSetDevice(c->device);
        return f();
    } catch (const Err& e) {
        return fail(c, e);
    } catch (const std::exception& e) {
        c->err = e.what();
        return B2_E_FORMAT;
    }
}

int create_common(b2_ctx** out, int device, const std::function<void(b2_ctx*)>& body, int tp_rank = 0,
                  int tp_size = 1) {
    if (!out) return B2_E_INVALID;
    *out = nullptr;
    if (tp_size < 1 || tp_size > kMaxRanks || tp_rank < 0 || tp_rank >= tp_size) return B2_E_INVALID;
    auto c = std::make_unique<b2_ctx>();
    c->device = -1;
    c->tp_rank = tp_rank;
    c->tp_size = tp_size;
    try {
        setup_device(c.get(), device);
        body(c.get());
        if (tp_size == 1) {                             // with ranks: after b2_tp_connect
            capture_graphs(c.get());
            upload_state(c.get(), 0, 0, 0, 0, -1);
        }
        CK(cudaStreamSynchronize(c->stream));
    } catch (const Err& e) {
        g_last_create_error = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_last_create_error = e.what();
        return B2_E_FORMAT;
    }
    *out = c.release();
    return B2_OK;
}

}  // namespace

// Timeline of the last token-kernel step (B2_TK_TRACE=<file>): "B2TRACE1", then
// int32 nphases, ncta, stamps per phase, the phase kinds of the decode table (0
// embed, 2 attention, 10 + GEMV variant), then u64 [nphases][ncta][stamps]
// global-timer stamps (see TkParams::trace).
void dump_trace(b2_ctx* c) {
    const int nph = c->nph_decode, ncta = c->sm_count;
    std::vector<unsigned long long> t((size_t)nph * ncta * kTkStamps);
    if (cudaMemcpy(t.data(), c->d_trace, t.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return;
    FILE* f = std::fopen(c->trace_path.c_str(), "wb");
    if (!f) return;
    std::fwrite("B2TRACE1", 1, 8, f);
    std::fwrite(&nph, 4, 1, f);
    std::fwrite(&ncta, 4, 1, f);
    const int ns = kTkStamps;
    std::fwrite(&ns, 4, 1, f);
    std::fwrite(c->trace_kinds.data() + c->nph_prefill, 4, (size_t)nph, f);
    std::fwrite(t.data(), 8, t.size(), f);
    std::fclose(f);
}

// message for b2_last_error(NULL, ...) from the context-free entry points
void b2_internal_set_error(const std::string& msg) { g_last_create_error = msg; }

// ===================================================================== C ABI
extern "C" {

int b2_create(const char* blob_path, const char* plan_json, int device, b2_ctx** out) {
    if (!blob_path) return B2_E_INVALID;
    return create_common(out, device, [&](b2_ctx* c) {
        std::string embedded;
        load_blob(c, blob_path, &embedded);
        const b2json::Value plan = b2json::parse(plan_json ? std::string(plan_json) : embedded);
        assemble(c, plan);
    });
}

int b2_create_synthetic(const char* plan_json, uint64_t seed, float stdv, int device, b2_ctx** out) {
    if (!plan_json) return B2_E_INVALID;
    return create_common(out, device, [&](b2_ctx* c) {
        const b2json::Value plan = b2json::parse(plan_json);
        synth_weights(c, plan, seed, stdv);
        assemble(c, plan);
    });
}

int b2_create_tp(const char* blob_path, const char* plan_json, int device, int tp_rank, int tp_size,
                 b2_ctx** out) {
    if (!blob_path) return B2_E_INVALID;
    return create_common(out, device, [&](b2_ctx* c) { load_blob_rank(c, blob_path, plan_json); }, tp_rank,
                         tp_size);
}

int b2_create_synthetic_tp(const char* plan_json, uint64_t seed, float stdv, int device, int tp_rank,
                           int tp_size, b2_ctx** out) {
    if (!plan_json) return B2_E_INVALID;
    return create_common(out, device, [&](b2_ctx* c) {
        const b2json::Value plan = b2json::parse(plan_json);
        synth_weights(c, plan, seed, stdv);
        assemble(c, plan);
    }, tp_rank, tp_size);
}

int b2_tp_handle(b2_ctx* ctx, void* handle, int len) {
    return guarded(ctx, [&] {
        if (!handle || len < (int)sizeof(cudaIpcMemHandle_t)) return B2_E_INVALID;
        cudaIpcMemHandle_t h;
        CK(cudaIpcGetMemHandle(&h, ctx->d_xch));
        std::memcpy(handle, &h, sizeof(h));
        return B2_OK;
    });
}

int b2_tp_connect(b2_ctx* ctx, const void* handles, int len) {
    return guarded(ctx, [&] {
        const int N = ctx->tp_size;
        if (N < 2 || ctx->tp_connected || !handles || len != N * (int)sizeof(cudaIpcMemHandle_t))
            return B2_E_INVALID;
        const char* hp = static_cast<const char*>(handles);
        Mirror m{};
        for (int r = 0; r < N; ++r) {
            if (r == ctx->tp_rank) continue;
            cudaIpcMemHandle_t h;
            std::memcpy(&h, hp + (size_t)r * sizeof(h), sizeof(h));
            CK(cudaIpcOpenMemHandle(&ctx->peer_base[r], h, cudaIpcMemLazyEnablePeerAccess));
            m.delta[m.n++] = static_cast<char*>(ctx->peer_base[r]) - static_cast<char*>(ctx->d_xch);
        }
        ctx->mir = m;
        capture_graphs(ctx);
        upload_state(ctx, 0, 0, 0, 0, -1);
        CK(cudaStreamSynchronize(ctx->stream));
        ctx->tp_connected = true;
        return B2_OK;
    });
}

int b2_destroy(b2_ctx* ctx) {
    if (!ctx) return B2_E_INVALID;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->d_trace) dump_trace(ctx);
    delete ctx;
    return B2_OK;
}

unsigned lcg_advance(unsigned s, long long n) {
    for (long long i = 0; i < n; ++i) s = s * 1103515245u + 12345u;
    return s;
}

int b2_reset(b2_ctx* ctx) {
    return guarded(ctx, [&] {
        ctx->rng = ctx->seed;
        upload_state(ctx, 0, 0, 0, 0, -1);
        CK(cudaStreamSynchronize(ctx->stream));
        ctx->host_step = 0;
        return B2_OK;
    });
}

int b2_step(b2_ctx* ctx, const int32_t* tok, int n_seq, int32_t* next_tok, float* logits) {
    return guarded(ctx, [&]() -> int {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (n_seq > 1) {
            if (n_seq != ctx->bt_n) throw Err(B2_E_UNSUPPORTED, "n_seq must equal the b2_batch_init batch");
            return b2_batch_step(ctx, tok, next_tok, logits);
        }
        if (!tok || n_seq != 1) return B2_E_INVALID;
        if (ctx->host_step >= ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "position reached max_seq");
        if (tok[0] < 0 || tok[0] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
        const int t = ctx->host_step;
        CK(cudaMemcpyAsync(ctx->prompt + t, tok, 4, cudaMemcpyHostToDevice, ctx->stream));
        upload_state(ctx, t, t + 1, 1 << 30, 0, -1);
        CK(cudaGraphLaunch(ctx->g_decode, ctx->stream));
        if (logits)
            CK(cudaMemcpyAsync(logits, ctx->logits, (size_t)ctx->vocab * 4, cudaMemcpyDeviceToHost, ctx->stream));
        fetch_state(ctx);
        if (next_tok) next_tok[0] = ctx->h_st->next_tok;
        return B2_OK;
    });
}

int b2_prefill(b2_ctx* ctx, const int32_t* toks, int n) {
    return guarded(ctx, [&] {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (n < 0 || (n > 0 && !toks)) return B2_E_INVALID;
        if (ctx->host_step + n > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "prefill passes max_seq");
        for (int i = 0; i < n; ++i)
            if (toks[i] < 0 || toks[i] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
        const int t = ctx->host_step;
        if (n) CK(cudaMemcpyAsync(ctx->prompt + t, toks, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
        // the reference samples (and advances its generator) on prompt steps too
        if (ctx->samp_mode) ctx->rng = lcg_advance(ctx->rng, n);
        if (ctx->pf_ok && n >= 2) {
            upload_state(ctx, t + n, t + n, 1 << 30, 0, -1);
            enqueue_prefill(ctx, t, n, ctx->stream);
            fetch_state(ctx);
            return B2_OK;
        }
        upload_state(ctx, t, t + n, 1 << 30, 0, -1);
        for (int i = 0; i < n; ++i) CK(cudaGraphLaunch(ctx->g_prefill, ctx->stream));
        fetch_state(ctx);
        return B2_OK;
    });
}

int b2_generate(b2_ctx* ctx, const int32_t* prompt, int n_prompt, int max_new, int32_t eos,
                int32_t* out_ids, int* n_out) {
    return guarded(ctx, [&] {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (n_out) *n_out = 0;
        if (!prompt || n_prompt <= 0 || max_new < 0 || (max_new > 0 && !out_ids)) return B2_E_INVALID;
        if (max_new == 0) return B2_OK;
        for (int i = 0; i < n_prompt; ++i)
            if (prompt[i] < 0 || prompt[i] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
        const int np = std::min(n_prompt, ctx->max_seq);
        CK(cudaMemcpyAsync(ctx->prompt, prompt, (size_t)np * 4, cudaMemcpyHostToDevice, ctx->stream));
        // a new sequence: the generator restarts at the seed and advances once per
        // prompt step before the first emitted token (the prefill graph runs no head)
        ctx->rng = ctx->samp_mode ? lcg_advance(ctx->seed, (long long)std::min(n_prompt, ctx->max_seq + 1) - 1)
                                  : ctx->seed;
        const long long total = (long long)n_prompt + max_new - 1;
        const int steps = (int)std::min<long long>(total, ctx->max_seq);
        // prompt steps before the last one: one batched prefill when the plan is covered
        const int pre = ctx->pf_ok ? std::min(n_prompt - 1, steps) : 0;
        upload_state(ctx, pre, n_prompt, max_new, 0, eos);
        if (pre >= 1) enqueue_prefill(ctx, 0, pre, ctx->stream);
        for (int t = pre; t < steps; ++t)
            CK(cudaGraphLaunch(t < n_prompt - 1 ? ctx->g_prefill : ctx->g_decode, ctx->stream));
        CK(cudaMemcpyAsync(out_ids, ctx->out_ids, (size_t)max_new * 4, cudaMemcpyDeviceToHost, ctx->stream));
        fetch_state(ctx);
        if (n_out) *n_out = ctx->h_st->n_out;
        if (total > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "generation passes max_seq");
        return B2_OK;
    });
}

int b2_set_position(b2_ctx* ctx, int pos, int32_t next_tok) {
    return guarded(ctx, [&] {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (pos < 0 || pos > ctx->max_seq || next_tok < 0 || next_tok >= ctx->vocab) return B2_E_INVALID;
        // enqueued on the stream (no host synchronisation): one tiny kernel
        clear_tickets(ctx, ctx->stream);
        set_state_kernel<<<1, 1, 0, ctx->stream>>>(ctx->st, pos, pos, 1 << 30, next_tok, -1);
        CK(cudaGetLastError());
        ctx->host_step = pos;
        return B2_OK;
    });
}

int b2_batch_init(b2_ctx* ctx, int n_seq, int max_steps) {
    return guarded(ctx, [&] {
        batch_init(ctx, n_seq, max_steps);
        return B2_OK;
    });
}

int b2_batch_reset(b2_ctx* ctx) {
    return guarded(ctx, [&] {
        batch_begin(ctx);
        CK(cudaMemsetAsync(ctx->bt_pos, 0, (size_t)ctx->bt_n * 4, ctx->stream));
        CK(cudaMemsetAsync(ctx->bt_nsteps, 0, sizeof(int), ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
        ctx->bt_pos_host.assign(ctx->bt_n, 0);
        ctx->bt_steps_host = 0;
        return B2_OK;
    });
}

int b2_batch_prefill(b2_ctx* ctx, int seq, const int32_t* toks, int n) {
    return guarded(ctx, [&] {
        batch_begin(ctx);
        if (seq < 0 || seq >= ctx->bt_n || n < 0 || (n > 0 && !toks)) return B2_E_INVALID;
        const int p0 = ctx->bt_pos_host[seq];
        if (p0 + n > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "prefill passes max_seq");
        for (int i = 0; i < n; ++i)
            if (toks[i] < 0 || toks[i] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
        if (n == 0) return B2_OK;
        CK(cudaMemcpyAsync(ctx->bt_ids + p0, toks, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
        enqueue_prefill(ctx, p0, n, ctx->stream, ctx->bt_ids, seq);
        const int np = p0 + n;
        CK(cudaMemcpyAsync(ctx->bt_pos + seq, &np, 4, cudaMemcpyHostToDevice, ctx->stream));
        fetch_state(ctx);
        ctx->bt_pos_host[seq] = np;
        return B2_OK;
    });
}

int b2_batch_step(b2_ctx* ctx, const int32_t* toks, int32_t* next, float* logits) {
    return guarded(ctx, [&] {
        batch_begin(ctx);
        if (!toks) return B2_E_INVALID;
        for (int z = 0; z < ctx->bt_n; ++z) {
            if (toks[z] < 0 || toks[z] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
            if (ctx->bt_pos_host[z] >= ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "a sequence reached max_seq");
        }
        if (ctx->bt_steps_host >= ctx->bt_max_steps) throw Err(B2_E_INVALID, "output record full (max_steps)");
        CK(cudaMemcpyAsync(ctx->bt_tok, toks, (size_t)ctx->bt_n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaGraphLaunch(ctx->g_batch, ctx->stream));
        if (next) CK(cudaMemcpyAsync(next, ctx->bt_tok, (size_t)ctx->bt_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        if (logits)
            CK(cudaMemcpyAsync(logits, ctx->bt_logits, (size_t)ctx->bt_n * ctx->vocab * 4, cudaMemcpyDeviceToHost,
                               ctx->stream));
        fetch_state(ctx);
        for (int& p : ctx->bt_pos_host) ++p;
        ++ctx->bt_steps_host;
        return B2_OK;
    });
}

int b2_batch_decode_async(b2_ctx* ctx, int n_steps) {
    return guarded(ctx, [&] {
        if (!ctx->bt_base) throw Err(B2_E_INVALID, "batched decode not initialised (b2_batch_init)");
        if (n_steps < 0) return B2_E_INVALID;
        for (int p : ctx->bt_pos_host)
            if (p + n_steps > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "decode passes max_seq");
        if (ctx->bt_steps_host + n_steps > ctx->bt_max_steps) throw Err(B2_E_INVALID, "output record full (max_steps)");
        for (int i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(ctx->g_batch, ctx->stream));
        for (int& p : ctx->bt_pos_host) p += n_steps;
        ctx->bt_steps_host += n_steps;
        return B2_OK;
    });
}

int b2_batch_read_output(b2_ctx* ctx, int32_t* ids, int max_steps, int* n_steps) {
    return guarded(ctx, [&] {
        if (!ctx->bt_base || !ids) return B2_E_INVALID;
        fetch_state(ctx);
        const int n = std::min(max_steps, ctx->bt_steps_host);
        if (n > 0) {
            CK(cudaMemcpyAsync(ids, ctx->bt_out, (size_t)n * ctx->bt_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
            CK(cudaStreamSynchronize(ctx->stream));
        }
        if (n_steps) *n_steps = n;
        return B2_OK;
    });
}

int b2_batch_generate(b2_ctx* ctx, const int32_t* prompts, int n_prompt, int max_new, int32_t* out_ids) {
    return guarded(ctx, [&] {
        if (!ctx->bt_base) throw Err(B2_E_INVALID, "batched decode not initialised (b2_batch_init)");
        if (!prompts || n_prompt <= 0 || max_new <= 0 || !out_ids) return B2_E_INVALID;
        if (n_prompt + max_new - 1 > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "generation passes max_seq");
        if (max_new > ctx->bt_max_steps) throw Err(B2_E_INVALID, "max_new above the output record (max_steps)");
        const int Bn = ctx->bt_n;
        for (long long i = 0; i < (long long)Bn * n_prompt; ++i)
            if (prompts[i] < 0 || prompts[i] >= ctx->vocab) throw Err(B2_E_INVALID, "token id outside the vocabulary");
        batch_begin(ctx);
        CK(cudaMemsetAsync(ctx->bt_nsteps, 0, sizeof(int), ctx->stream));
        // every prompt but its last token through the batched prefill, sequence by sequence
        std::vector<int32_t> last(Bn), pos(Bn, n_prompt - 1);
        for (int z = 0; z < Bn; ++z) {
            const int32_t* pz = prompts + (size_t)z * n_prompt;
            if (n_prompt > 1) {
                CK(cudaMemcpyAsync(ctx->bt_ids, pz, (size_t)(n_prompt - 1) * 4, cudaMemcpyHostToDevice, ctx->stream));
                enqueue_prefill(ctx, 0, n_prompt - 1, ctx->stream, ctx->bt_ids, z);
                CK(cudaStreamSynchronize(ctx->stream));            // bt_ids is reused by the next sequence
            }
            last[z] = pz[n_prompt - 1];
        }
        CK(cudaMemcpyAsync(ctx->bt_pos, pos.data(), (size_t)Bn * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaMemcpyAsync(ctx->bt_tok, last.data(), (size_t)Bn * 4, cudaMemcpyHostToDevice, ctx->stream));
        for (int i = 0; i < max_new; ++i) CK(cudaGraphLaunch(ctx->g_batch, ctx->stream));
        std::vector<int32_t> rec((size_t)max_new * Bn);
        CK(cudaMemcpyAsync(rec.data(), ctx->bt_out, rec.size() * 4, cudaMemcpyDeviceToHost, ctx->stream));
        fetch_state(ctx);
        for (int z = 0; z < Bn; ++z)
            for (int i = 0; i < max_new; ++i) out_ids[(size_t)z * max_new + i] = rec[(size_t)i * Bn + z];
        ctx->bt_pos_host.assign(Bn, n_prompt - 1 + max_new);
        ctx->bt_steps_host = max_new;
        return B2_OK;
    });
}

int b2_set_sampling(b2_ctx* ctx, int mode, int top_k, double temperature, uint32_t seed) {
    return guarded(ctx, [&] {
        if (mode < 0 || mode > 2) return B2_E_INVALID;
        if (mode && ctx->tp_size > 1) throw Err(B2_E_UNSUPPORTED, "sampling needs every logit on one GPU");
        const bool recapture = mode != ctx->samp_mode || (mode && (top_k != ctx->samp_k || temperature != ctx->samp_t));
        ctx->samp_mode = mode;
        ctx->samp_k = top_k;
        ctx->samp_t = temperature;
        ctx->seed = seed;
        ctx->rng = seed;
        if (recapture) capture_graphs(ctx);
        upload_state(ctx, ctx->host_step, ctx->host_step, 1 << 30, 0, -1);
        CK(cudaStreamSynchronize(ctx->stream));
        return B2_OK;
    });
}

int b2_fill_kv_synthetic(b2_ctx* ctx, int count, uint64_t seed) {
    return guarded(ctx, [&] {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (count < 0 || count > ctx->max_seq) return B2_E_INVALID;
        for (size_t b = 0; b < ctx->blocks.size(); ++b) {
            const Block& B = ctx->blocks[b];
            if (!B.attn || count == 0) continue;
            const long long n = (long long)B.KVH * count * B.dh;
            const unsigned grid = (unsigned)((n + 255) / 256);
            const int kv0 = ctx->tp_rank * B.KVH;
            synth_kv_kernel<<<grid, 256, 0, ctx->stream>>>(seed, 0xC0DE0000ull + 2 * b, B.K, B.KVH, kv0,
                                                           ctx->max_seq, B.dh, count);
            synth_kv_kernel<<<grid, 256, 0, ctx->stream>>>(seed, 0xC0DE0001ull + 2 * b, B.V, B.KVH, kv0,
                                                           ctx->max_seq, B.dh, count);
            CK(cudaGetLastError());
        }
        upload_state(ctx, count, count, 1 << 30, 0, -1);
        CK(cudaStreamSynchronize(ctx->stream));
        ctx->host_step = count;
        return B2_OK;
    });
}

int b2_decode_async(b2_ctx* ctx, int n_steps) {
    return guarded(ctx, [&] {
        if (!ctx->g_decode) throw Err(B2_E_INVALID, "ranks not connected (b2_tp_connect)");
        if (n_steps < 0) return B2_E_INVALID;
        if (ctx->host_step + n_steps > ctx->max_seq) throw Err(B2_E_KV_OVERFLOW, "decode passes max_seq");
        for (int i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(ctx->g_decode, ctx->stream));
        ctx->host_step += n_steps;
        return B2_OK;
    });
}

int b2_sync(b2_ctx* ctx) {
    return guarded(ctx, [&] { return fetch_state(ctx); });
}

int b2_read_output(b2_ctx* ctx, int32_t* ids, int max_ids, int* n_ids) {
    return guarded(ctx, [&] {
        fetch_state(ctx);
        const int n = std::min(max_ids, ctx->h_st->n_out);
        if (n > 0) {
            CK(cudaMemcpyAsync(ids, ctx->out_ids, (size_t)n * 4, cudaMemcpyDeviceToHost, ctx->stream));
            CK(cudaStreamSynchronize(ctx->stream));
        }
        if (n_ids) *n_ids = n;
        return B2_OK;
    });
}

int b2_set_stream(b2_ctx* ctx, void* stream) {
    return guarded(ctx, [&] {
        // graphs were captured on the private capture stream and launch on any stream
        CK(cudaStreamSynchronize(ctx->stream));
        if (ctx->own_stream) CK(cudaStreamDestroy(ctx->stream));
        ctx->stream = static_cast<cudaStream_t>(stream);
        ctx->own_stream = false;
        return B2_OK;
    });
}

int b2_query(b2_ctx* ctx, const char* key, double* value) {
    if (!ctx || !key || !value) return B2_E_INVALID;
    const std::string k(key);
    if (k == "weight_bytes") *value = (double)ctx->weight_bytes;
    else if (k == "kv_bytes_per_pos") *value = (double)ctx->kv_bytes_per_pos;
    else if (k == "kernels_per_step") *value = ctx->kernels_decode;
    else if (k == "kernels_per_prefill_step") *value = ctx->kernels_prefill;
    else if (k == "max_seq") *value = ctx->max_seq;
    else if (k == "vocab") *value = ctx->vocab;
    else if (k == "position") *value = ctx->host_step;
    else if (k == "n_out") *value = ctx->h_st->n_out;
    else if (k == "device_err") *value = ctx->h_st->err;
    else if (k == "sm_count") *value = ctx->sm_count;
    else if (k == "pdl") *value = ctx->pdl ? 1 : 0;
    else if (k == "token_kernel") *value = ctx->token ? 1 : 0;
    else if (k == "token_tags") *value = ctx->token && ctx->tk_tags ? 1 : 0;
    else if (k == "prefill_batched") *value = ctx->pf_ok ? 1 : 0;
    else if (k == "batch") *value = ctx->bt_n;
    else return B2_E_INVALID;
    return B2_OK;
}

int b2_last_error(b2_ctx* ctx, char* buf, int len) {
    if (!buf || len <= 0) return B2_E_INVALID;
    const std::string& m = ctx ? ctx->err : g_last_create_error;
    std::snprintf(buf, (size_t)len, "%s", m.c_str());
    return B2_OK;
}

}  // extern "C"
