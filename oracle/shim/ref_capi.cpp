// TEST INFRASTRUCTURE -- a C entry layer over the reference's own
// vortexrt::Gemma3Model (src/gemma3.cpp, compiled unmodified from the
// reference tree), so Python tests and the CPU baseline can drive the
// reference token loop.  Every call catches the reference's exceptions and
// returns -1 with the message copied into `err`.

#include "vortexrt/gemma3.hpp"

#include <cstring>
#include <exception>
#include <memory>
#include <string>

namespace {

struct RefModel {
    std::unique_ptr<vortexrt::VulkanContext> ctx;
    std::unique_ptr<vortexrt::Gemma3Model> model;
};

void put_err(char* err, std::size_t n, const char* msg) {
    if (err && n) {
        std::strncpy(err, msg, n - 1);
        err[n - 1] = 0;
    }
}

std::string lanes_path(unsigned lanes) { return "lanes=" + std::to_string(lanes); }

} // namespace

extern "C" {

void* vrt_ref_open(const char* path, unsigned subgroup, unsigned lane_override, int fusion,
                   unsigned threads, char* err, std::size_t errlen) {
    try {
        auto m = std::make_unique<RefModel>();
        m->ctx = std::make_unique<vortexrt::VulkanContext>(subgroup, threads);
        m->model = std::make_unique<vortexrt::Gemma3Model>(
            path, *m->ctx, lanes_path(64), std::string{}, "argmax", lanes_path(32), std::string{},
            "gelu_mul", lanes_path(16), std::string{}, lanes_path(8), std::string{}, lane_override);
        if (fusion == 0) m->model->set_projection_fusion_enabled(false);
        if (fusion == 1) m->model->set_projection_fusion_enabled(true);
        return m.release();
    } catch (const std::exception& e) {
        put_err(err, errlen, e.what());
        return nullptr;
    }
}

void vrt_ref_close(void* h) { delete static_cast<RefModel*>(h); }

void vrt_ref_set_threads(void* h, unsigned threads) {
    static_cast<RefModel*>(h)->ctx->set_threads(threads);
}

// u32 out[10]: context, d, L, ff, H, KV, hd, vd, vocab, window; f32 outf[3]: eps, theta_g, theta_l
int vrt_ref_config(void* h, unsigned* out, float* outf, unsigned* policy) {
    const auto& c = static_cast<RefModel*>(h)->model->config();
    const unsigned v[10] = {c.context_length, c.embedding_length, c.block_count,
                            c.feed_forward_length, c.head_count, c.head_count_kv, c.head_dim,
                            c.value_dim, c.vocab_size, c.sliding_window};
    std::memcpy(out, v, sizeof(v));
    outf[0] = c.rms_epsilon;
    outf[1] = c.global_rope_base;
    outf[2] = c.local_rope_base;
    auto& m = *static_cast<RefModel*>(h)->model;
    policy[0] = m.narrow_q8_lane_count();
    policy[1] = m.projection_fusion_enabled() ? 1u : 0u;
    policy[2] = m.fused_ffn_enabled() ? 1u : 0u;
    return 0;
}

void vrt_ref_reset(void* h) { static_cast<RefModel*>(h)->model->reset_cache(); }

// Runs Gemma3Model::decode_token (or run_single_token when single != 0).
int vrt_ref_decode(void* h, unsigned token, unsigned position, std::size_t top_k, int single,
                   float* hidden, unsigned* ids, float* logits, std::size_t* n_top, char* err,
                   std::size_t errlen) {
    try {
        auto& m = *static_cast<RefModel*>(h)->model;
        const auto r = single ? m.run_single_token(token, top_k) : m.decode_token(token, position, top_k);
        if (hidden) std::memcpy(hidden, r.hidden.data(), r.hidden.size() * sizeof(float));
        for (std::size_t i = 0; i < r.top_tokens.size(); ++i) {
            if (ids) ids[i] = r.top_tokens[i].token_id;
            if (logits) logits[i] = r.top_tokens[i].logit;
        }
        if (n_top) *n_top = r.top_tokens.size();
        return 0;
    } catch (const std::exception& e) {
        put_err(err, errlen, e.what());
        return -1;
    }
}

int vrt_ref_generate(void* h, const unsigned* prompt, std::size_t n, std::size_t max_new,
                     unsigned* out_ids, std::size_t* out_n, char* text, std::size_t text_cap,
                     char* err, std::size_t errlen) {
    try {
        auto& m = *static_cast<RefModel*>(h)->model;
        std::vector<std::uint32_t> p(prompt, prompt + n);
        const auto g = m.generate_greedy_tokens(p, max_new);
        for (std::size_t i = 0; i < g.token_ids.size(); ++i) out_ids[i] = g.token_ids[i];
        *out_n = g.token_ids.size();
        if (text && text_cap) put_err(text, text_cap, g.text.c_str());
        return 0;
    } catch (const std::exception& e) {
        put_err(err, errlen, e.what());
        return -1;
    }
}

int vrt_ref_tokenize(void* h, const char* text, int add_bos, unsigned* out, std::size_t cap,
                     std::size_t* n, char* err, std::size_t errlen) {
    try {
        const auto ids = static_cast<RefModel*>(h)->model->tokenize(text, add_bos != 0);
        *n = ids.size();
        for (std::size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
        return 0;
    } catch (const std::exception& e) {
        put_err(err, errlen, e.what());
        return -1;
    }
}

} // extern "C"
