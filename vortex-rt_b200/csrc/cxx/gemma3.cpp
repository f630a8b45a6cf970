// vortexrt::Gemma3Model and vortexrt::Gemma3Tokenizer.  The model runs every
// token step on the GPU through the C ABI (vrt_model_*); the tokenizer and
// piece decoding stay on the host, with the reference's rules.

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>

#include "vortexrt/gemma3.hpp"
#include "vortexrt_b200.h"

namespace vrt {
int fail(int code, const char* fmt, ...);  // runtime.cu: records vrt_last_error()
}

namespace vortexrt {
namespace {

const std::string kSpaceMarker = "\xE2\x96\x81";  // U+2581

int hex_digit(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
}

// "<0xHH>" -> byte value, or -1
int byte_piece(const std::string& s) {
    if (s.size() != 6 || s[0] != '<' || s[1] != '0' || s[2] != 'x' || s[5] != '>') return -1;
    const int hi = hex_digit(s[3]), lo = hex_digit(s[4]);
    return (hi < 0 || lo < 0) ? -1 : (hi << 4) | lo;
}

[[noreturn]] void raise(const char* what) { throw std::runtime_error(std::string(what) + vrt_last_error()); }

}  // namespace

// ------------------------------------------------------------- tokenizer

Gemma3Tokenizer::Gemma3Tokenizer(const GgufFile& g, std::uint32_t vocab) {
    const auto* toks = g.find_metadata("tokenizer.ggml.tokens");
    const auto* scores = g.find_metadata("tokenizer.ggml.scores");
    const auto* types = g.find_metadata("tokenizer.ggml.token_type");
    if (!toks || !scores || !types || !toks->is_array() || !scores->is_array() || !types->is_array() ||
        toks->array.size() != vocab || scores->array.size() != vocab || types->array.size() != vocab) {
        throw std::runtime_error("Gemma 3 tokenizer metadata is incomplete");
    }
    byte_ids_.fill(std::numeric_limits<std::uint32_t>::max());
    pieces_.resize(vocab);
    index_.reserve(vocab);
    for (std::uint32_t id = 0; id < vocab; ++id) {
        const auto piece = toks->array[id].as_string();
        const auto score = scores->array[id].as_f64();
        const auto type = types->array[id].as_i64();
        if (piece) pieces_[id] = *piece;
        if (!piece || !score || !type) continue;
        if (*type == 6) {
            const int b = byte_piece(*piece);
            if (b >= 0) {
                byte_ids_[static_cast<std::size_t>(b)] = id;
                continue;
            }
        }
        if (*type != 1 && *type != 4) continue;
        const float sc = static_cast<float>(*score);
        auto it = index_.find(*piece);
        if (it == index_.end() || sc > it->second.score) index_[*piece] = Entry{id, sc};
        max_piece_ = std::max(max_piece_, piece->size());
    }
    if (const auto* sp = g.find_metadata("tokenizer.ggml.add_space_prefix")) add_space_prefix_ = sp->as_bool().value_or(false);
    unk_ = static_cast<std::uint32_t>(std::min<std::uint64_t>(g.metadata_u64("tokenizer.ggml.unknown_token_id").value_or(3),
                                                              vocab - 1u));
    const auto bos = g.metadata_u64("tokenizer.ggml.bos_token_id").value_or(2);
    if (bos >= vocab) throw std::runtime_error("Gemma 3 BOS token id is out of range");
    bos_ = static_cast<std::uint32_t>(bos);
    eos_ = g.metadata_u64("tokenizer.ggml.eos_token_id").value_or(1);
}

std::vector<std::uint32_t> Gemma3Tokenizer::tokenize(const std::string& text, bool add_bos) const {
    if (index_.empty()) throw std::runtime_error("Gemma 3 tokenizer index is unavailable");
    // whitespace runs collapse to one marker
    std::string s;
    s.reserve(text.size() + 3);
    bool in_space = false;
    for (const unsigned char c : text) {
        if (c == ' ' || c == '\t' || c == '\r' || c == '\n') {
            if (!in_space) s += kSpaceMarker;
            in_space = true;
        } else {
            s.push_back(static_cast<char>(c));
            in_space = false;
        }
    }
    if (add_space_prefix_ && !s.empty() && s.compare(0, kSpaceMarker.size(), kSpaceMarker) != 0) {
        s.insert(0, kSpaceMarker);
    }
    // best-score segmentation; an unmatched byte costs 100
    const std::size_t n = s.size();
    const float ninf = -std::numeric_limits<float>::infinity();
    std::vector<float> best(n + 1, ninf);
    std::vector<std::size_t> from(n + 1, std::numeric_limits<std::size_t>::max());
    std::vector<std::uint32_t> tok(n + 1, std::numeric_limits<std::uint32_t>::max());
    best[0] = 0.0f;
    for (std::size_t i = 0; i < n; ++i) {
        if (!std::isfinite(best[i])) continue;
        bool any = false;
        const std::size_t lim = std::min(max_piece_, n - i);
        for (std::size_t len = 1; len <= lim; ++len) {
            const auto it = index_.find(s.substr(i, len));
            if (it == index_.end()) continue;
            any = true;
            const float cand = best[i] + it->second.score;
            if (cand > best[i + len]) {
                best[i + len] = cand;
                from[i + len] = i;
                tok[i + len] = it->second.id;
            }
        }
        if (!any) {
            std::uint32_t id = byte_ids_[static_cast<unsigned char>(s[i])];
            if (id == std::numeric_limits<std::uint32_t>::max()) id = unk_;
            const float cand = best[i] - 100.0f;
            if (cand > best[i + 1]) {
                best[i + 1] = cand;
                from[i + 1] = i;
                tok[i + 1] = id;
            }
        }
    }
    if (n && !std::isfinite(best[n])) throw std::runtime_error("Gemma 3 tokenizer could not segment prompt");
    std::vector<std::uint32_t> rev;
    for (std::size_t at = n; at != 0; at = from[at]) {
        if (from[at] == std::numeric_limits<std::size_t>::max() || tok[at] == std::numeric_limits<std::uint32_t>::max()) {
            throw std::runtime_error("Gemma 3 tokenizer backtracking failed");
        }
        rev.push_back(tok[at]);
    }
    std::vector<std::uint32_t> out;
    out.reserve(rev.size() + 1);
    if (add_bos) out.push_back(bos_);
    out.insert(out.end(), rev.rbegin(), rev.rend());
    return out;
}

std::string Gemma3Tokenizer::token_piece(std::uint32_t id) const {
    return id < pieces_.size() ? pieces_[id] : std::string{};
}

std::string Gemma3Tokenizer::decode_piece(std::uint32_t id) const {
    if (id <= 3) return {};
    std::string p = token_piece(id);
    const int b = byte_piece(p);
    if (b >= 0) return std::string(1, static_cast<char>(b));
    for (std::size_t at = 0; (at = p.find(kSpaceMarker, at)) != std::string::npos; ++at) p.replace(at, kSpaceMarker.size(), " ");
    return p;
}

// ------------------------------------------------------------------ model

Gemma3Model::Gemma3Model(const std::string& gguf_path, VulkanContext& context, const std::string&,
                         const std::string&, const std::string& argmax_spirv, const std::string& q8_matvec_32_spirv,
                         const std::string&, const std::string& gelu_mul_spirv, const std::string& q8_matvec_16_spirv,
                         const std::string&, const std::string& q8_matvec_8_spirv, const std::string&,
                         std::uint32_t q8_lane_override)
    : context_(context) {
    // lane policy of the reference constructor (src/gemma3.cpp:94-172): the
    // requested variant must have been named; on a GPU the auto choice
    // follows the warp width (32)
    std::uint32_t lanes = q8_lane_override ? q8_lane_override : context.capabilities().subgroup_size;
    if (lanes != 8 && lanes != 16 && lanes != 32 && lanes != 64) {
        if (q8_lane_override) throw std::runtime_error("Q8 lane override must be 0, 8, 16, 32, or 64");
        lanes = 64;
    }
    const std::string* path = lanes == 32 ? &q8_matvec_32_spirv : lanes == 16 ? &q8_matvec_16_spirv
                              : lanes == 8 ? &q8_matvec_8_spirv : nullptr;
    if (path && path->empty()) throw std::runtime_error("Requested Q8 lane variant is unavailable");
    narrow_q8_lane_count_ = lanes;
    fuse_projections_ = context.capabilities().device_type != VK_PHYSICAL_DEVICE_TYPE_CPU;
    ffn_available_ = !gelu_mul_spirv.empty();
    argmax_available_ = !argmax_spirv.empty();

    GgufFile g(gguf_path);
    if (g.metadata_string("general.architecture") != std::optional<std::string>{"gemma3"}) {
        throw std::runtime_error("Gemma3Model requires general.architecture=gemma3");
    }
    vrt_model_options opt;
    vrt_model_options_default(&opt);
    if (vrt_model_load(context.native(), gguf_path.c_str(), &opt, &model_) != VRT_OK) raise("Gemma3Model: ");
    vrt_gemma3_config c{};
    vrt_model_config(model_, &c);
    config_ = Gemma3Config{c.context_length, c.embedding_length, c.block_count, c.feed_forward_length, c.head_count,
                           c.head_count_kv, c.head_dim, c.value_dim, c.vocab_size, c.sliding_window, c.rms_epsilon,
                           c.global_rope_base, c.local_rope_base};
    tokenizer_ = std::make_unique<Gemma3Tokenizer>(g, config_.vocab_size);
}

Gemma3Model::~Gemma3Model() { vrt_model_destroy(model_); }

void Gemma3Model::reset_cache() {
    if (vrt_model_reset(model_) != VRT_OK) raise("reset_cache: ");
    next_position_ = 0;
}

Gemma3SingleTokenResult Gemma3Model::decode_token(std::uint32_t token, std::uint32_t position, std::size_t top_k) {
    if (position != next_position_) throw std::runtime_error("Gemma 3 decode positions must be contiguous");
    if (position >= config_.context_length) throw std::runtime_error("Gemma 3 context length exceeded");
    Gemma3SingleTokenResult r;
    r.hidden.resize(config_.embedding_length);
    const std::size_t k = std::min<std::size_t>(top_k, config_.vocab_size);
    std::vector<std::uint32_t> ids(std::max<std::size_t>(k, 1));
    std::vector<float> logits(ids.size());
    const int rc = vrt_decode_step(model_, token, position, static_cast<std::uint32_t>(k), r.hidden.data(), ids.data(),
                                   logits.data());
    if (rc != VRT_OK) {
        const std::string msg = vrt_last_error();
        reset_cache();
        throw std::runtime_error(msg);
    }
    for (std::size_t i = 0; i < k; ++i) r.top_tokens.push_back(Gemma3TopToken{ids[i], logits[i], token_piece(ids[i])});
    ++next_position_;
    return r;
}

Gemma3SingleTokenResult Gemma3Model::run_single_token(std::uint32_t token, std::size_t top_k) {
    reset_cache();
    auto r = decode_token(token, 0, top_k);
    reset_cache();
    return r;
}

std::vector<std::uint32_t> Gemma3Model::tokenize(const std::string& text, bool add_bos) const {
    return tokenizer_->tokenize(text, add_bos);
}

std::string Gemma3Model::token_piece(std::uint32_t id) const { return tokenizer_->token_piece(id); }
std::string Gemma3Model::decode_piece(std::uint32_t id) const { return tokenizer_->decode_piece(id); }

Gemma3GenerationResult Gemma3Model::generate_greedy_tokens(const std::vector<std::uint32_t>& prompt,
                                                           std::size_t max_new) {
    reset_cache();
    Gemma3GenerationResult out;
    if (max_new == 0) return out;
    if (prompt.empty()) throw std::runtime_error("Gemma 3 prompt produced no input tokens");
    std::vector<std::uint32_t> ids(max_new);
    std::uint32_t n = 0;
    if (vrt_generate_greedy(model_, prompt.data(), static_cast<std::uint32_t>(prompt.size()),
                            static_cast<std::uint32_t>(max_new), ids.data(), &n) != VRT_OK) {
        const std::string msg = vrt_last_error();
        reset_cache();
        throw std::runtime_error(msg);
    }
    std::uint32_t pos = 0;
    vrt_model_next_token(model_, nullptr, &pos);
    next_position_ = pos;
    for (std::uint32_t i = 0; i < n; ++i) {
        out.token_ids.push_back(ids[i]);
        if (ids[i] == tokenizer_->eos()) break;
        out.text += decode_piece(ids[i]);
    }
    return out;
}

Gemma3GenerationResult Gemma3Model::generate_greedy(const std::string& prompt, std::size_t max_new) {
    if (max_new == 0) {
        reset_cache();
        return {};
    }
    return generate_greedy_tokens(tokenize(prompt, true), max_new);
}

Gemma3GenerationResult Gemma3Model::generate_greedy_from_bos(std::size_t max_new) {
    if (max_new == 0) {
        reset_cache();
        return {};
    }
    return generate_greedy_tokens({tokenizer_->bos()}, max_new);
}

}  // namespace vortexrt

// ------------------------------------------------------ tokenizer C entry

struct vrt_tokenizer {
    std::unique_ptr<vortexrt::GgufFile> g;
    std::unique_ptr<vortexrt::Gemma3Tokenizer> t;
};

extern "C" {

VRT_API int vrt_tokenizer_open(const char* gguf_path, vrt_tokenizer** out) {
    try {
        auto tk = std::make_unique<vrt_tokenizer>();
        tk->g = std::make_unique<vortexrt::GgufFile>(gguf_path);
        const auto* emb = tk->g->find_tensor("token_embd.weight");
        if (!emb || emb->dimensions.size() != 2) throw std::runtime_error("Unsupported token_embd.weight layout");
        tk->t = std::make_unique<vortexrt::Gemma3Tokenizer>(*tk->g, static_cast<std::uint32_t>(emb->dimensions[1]));
        *out = tk.release();
        return VRT_OK;
    } catch (const std::exception& e) {
        return vrt::fail(VRT_E_IO, "%s", e.what());
    }
}

VRT_API void vrt_tokenizer_close(vrt_tokenizer* t) { delete t; }

VRT_API int vrt_tokenize(vrt_tokenizer* t, const char* text, int add_bos, uint32_t* out, size_t cap, size_t* n) {
    try {
        const auto ids = t->t->tokenize(text, add_bos != 0);
        *n = ids.size();
        for (std::size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
        return VRT_OK;
    } catch (const std::exception& e) {
        return vrt::fail(VRT_E_INVALID, "%s", e.what());
    }
}

VRT_API int vrt_token_piece(vrt_tokenizer* t, uint32_t id, int decoded, char* out, size_t cap, size_t* n) {
    const std::string s = decoded ? t->t->decode_piece(id) : t->t->token_piece(id);
    *n = s.size();
    if (cap) {
        const std::size_t m = std::min(cap - 1, s.size());
        std::memcpy(out, s.data(), m);
        out[m] = 0;
    }
    return VRT_OK;
}

}  // extern "C"
