// b2run.cpp — the stdin-tokens front end: a drop-in for the packed decoder
// binary that tools/run_decoder.py drives (aricode_pack.py:2147-2173 wire
// format, :2321 output), running the model on the B200 through libb2dec.so.
//
//   <out>            a symlink to this program, written by the packer next to
//   <out>.b2blob     the blob; run with no arguments (run_decoder.py starts it as
//                    "./<name>" in the blob's directory)
//
// stdin:  [u32 LE prompt_len][u32 LE seed][prompt_len token ids, each tb bytes LE]
//         with tb = 1 (vocab <= 256), 2 (<= 65536) or 4; the seed drives the
//         sampler when the plan's --sample is not greedy (a greedy plan reads and
//         ignores it). With --input-format embedded the prompt comes from the
//         plan's prompt file instead (raw tb-byte ids) and the seed is --rng-seed.
// stdout: every generated id as a decimal line, flushed as it is produced:
//         total = prompt_len + max_new - 1 steps, the ids of steps t >= prompt_len - 1,
//         stopping before an --eos-token id.
// Exit status: 0 done, 2 bad input (wire format, token ids, prompt longer than
// --max-prompt-tokens), 3 the KV cache would overflow (max_seq), 4 library error.
// Usage: b2run [blob] ; B2_DEVICE selects the GPU (default 0).
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/b2dec.h"
#include "json.h"

namespace {

int fail(int code, const std::string& msg) {
    std::fprintf(stderr, "b2run: %s\n", msg.c_str());
    return code;
}

bool read_exact(FILE* f, void* dst, size_t n) { return std::fread(dst, 1, n, f) == n; }

int token_width(long long vocab) { return vocab <= 256 ? 1 : (vocab <= 65536 ? 2 : 4); }

uint32_t le32(const unsigned char* b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

std::vector<int32_t> decode_ids(const std::vector<unsigned char>& raw, int tb) {
    std::vector<int32_t> ids(raw.size() / tb);
    for (size_t i = 0; i < ids.size(); ++i) {
        uint32_t v = 0;
        for (int k = 0; k < tb; ++k) v |= (uint32_t)raw[i * tb + k] << (8 * k);
        ids[i] = (int32_t)v;
    }
    return ids;
}

// the plan embedded in the blob: header bytes 48..63 hold its length and offset
bool read_plan(const std::string& blob, std::string* plan) {
    FILE* f = std::fopen(blob.c_str(), "rb");
    if (!f) return false;
    unsigned char hdr[64];
    bool ok = read_exact(f, hdr, 64) && std::memcmp(hdr, "B2DBLOB1", 8) == 0;
    if (ok) {
        uint32_t len;
        uint64_t off;
        std::memcpy(&len, hdr + 48, 4);
        std::memcpy(&off, hdr + 56, 8);
        plan->resize(len);
        ok = std::fseek(f, (long)off, SEEK_SET) == 0 && read_exact(f, &(*plan)[0], len);
    }
    std::fclose(f);
    return ok;
}

std::string last_error(b2_ctx* c) {
    char buf[512];
    b2_last_error(c, buf, sizeof(buf));
    return buf;
}

}  // namespace

int main(int argc, char** argv) {
    const std::string blob = argc > 1 ? std::string(argv[1]) : std::string(argv[0]) + ".b2blob";
    std::string plan_s;
    if (!read_plan(blob, &plan_s)) return fail(2, "cannot read the plan of " + blob);
    b2json::Value plan;
    try {
        plan = b2json::parse(plan_s);
    } catch (const std::exception& e) {
        return fail(2, std::string("malformed plan: ") + e.what());
    }
    const long long vocab = plan["vocab"].as_int();
    const int tb = token_width(vocab);
    long long max_new = 16, max_prompt = 512;
    int32_t eos = -1;
    int mode = 0, top_k = 0;
    double temperature = 0.0;
    uint32_t seed = 20260502u;
    std::string input_format = "stdin-tokens", prompt_file;
    if (plan.has("generation")) {
        const b2json::Value& g = plan["generation"];
        if (g.has("max_new_tokens")) max_new = g["max_new_tokens"].as_int();
        if (g.has("max_prompt_tokens")) max_prompt = g["max_prompt_tokens"].as_int();
        if (g.has("eos_token")) eos = (int32_t)g["eos_token"].as_int();
        if (g.has("sample_mode")) mode = (int)g["sample_mode"].as_int();
        if (g.has("top_k")) top_k = (int)g["top_k"].as_int();
        if (g.has("temperature")) temperature = g["temperature"].as_num();
        if (g.has("rng_seed")) seed = (uint32_t)(long long)g["rng_seed"].as_num();
        if (g.has("input_format")) input_format = g["input_format"].as_str();
        if (g.has("prompt_file")) prompt_file = g["prompt_file"].as_str();
    }

    // ---- the prompt (and the per-call seed) before any GPU work
    std::vector<int32_t> prompt;
    if (input_format == "embedded") {
        FILE* f = std::fopen(prompt_file.c_str(), "rb");
        if (!f) return fail(2, "cannot open the embedded prompt file " + prompt_file);
        std::vector<unsigned char> raw;
        unsigned char buf[4096];
        size_t n;
        while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) raw.insert(raw.end(), buf, buf + n);
        std::fclose(f);
        if (raw.size() % tb) return fail(2, "embedded prompt file is not a whole number of token ids");
        prompt = decode_ids(raw, tb);
    } else {
        unsigned char hdr[8];
        if (!read_exact(stdin, hdr, 8)) return fail(2, "stdin ended inside the 8-byte header (length, seed)");
        const uint32_t len = le32(hdr);
        seed = le32(hdr + 4);
        if ((long long)len > max_prompt)
            return fail(2, "prompt of " + std::to_string(len) + " tokens is longer than --max-prompt-tokens " +
                               std::to_string(max_prompt));
        std::vector<unsigned char> raw((size_t)len * tb);
        if (len && !read_exact(stdin, raw.data(), raw.size()))
            return fail(2, "stdin ended inside the prompt (" + std::to_string(len) + " ids of " +
                               std::to_string(tb) + " bytes expected)");
        prompt = decode_ids(raw, tb);
    }
    for (int32_t t : prompt)
        if (t < 0 || t >= vocab) return fail(2, "token id " + std::to_string(t) + " outside the vocabulary");

    // ---- the model
    const char* dev_env = std::getenv("B2_DEVICE");
    const int device = dev_env ? std::atoi(dev_env) : 0;
    b2_ctx* ctx = nullptr;
    if (b2_create(blob.c_str(), nullptr, device, &ctx) != B2_OK) return fail(4, "b2_create: " + last_error(nullptr));
    struct Destroy { b2_ctx* c; ~Destroy() { b2_destroy(c); } } destroy{ctx};
    if (mode && b2_set_sampling(ctx, mode, top_k, temperature, seed) != B2_OK)
        return fail(4, "b2_set_sampling: " + last_error(ctx));

    // the reference loop: steps t < P - 1 only fill the cache (their head output is
    // not printed; b2_prefill advances the sampler's generator for them), then one
    // step per emitted id
    const long long P = (long long)prompt.size();
    const long long total = P + max_new - 1;
    if (P > 1) {
        const int rc = b2_prefill(ctx, prompt.data(), (int)(P - 1));
        if (rc == B2_E_KV_OVERFLOW) return fail(3, "prompt longer than the KV cache: " + last_error(ctx));
        if (rc != B2_OK) return fail(4, "b2_prefill: " + last_error(ctx));
    }
    int32_t cur = P ? prompt[P - 1] : 0;
    for (long long t = P > 1 ? P - 1 : 0; t < total; ++t) {
        if (t < P) cur = prompt[t];
        int32_t next = 0;
        const int rc = b2_step(ctx, &cur, 1, &next, nullptr);
        if (rc == B2_E_KV_OVERFLOW) return fail(3, "KV cache full at step " + std::to_string(t));
        if (rc != B2_OK) return fail(4, "b2_step: " + last_error(ctx));
        if (t >= P - 1) {
            if (eos >= 0 && next == eos) break;
            std::printf("%d\n", next);
            std::fflush(stdout);
        }
        cur = next;
    }
    return 0;
}
