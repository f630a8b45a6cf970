// Gemma 3 Q8_0 model with the public interface of the Vortex-RT reference's
// Gemma3Model (include/vortexrt/gemma3.hpp:19-117 of the reference), running
// the whole token step on the GPU (vrt_model_* of include/vortexrt_b200.h).
//
// Kept: constructor signature (the SPIR-V paths are accepted and ignored; a
// non-empty argmax path still selects the fused LM-head argmax for top_k 1,
// the q8 lane override is validated and reported), config(), the fusion /
// lane accessors, run_single_token, reset_cache, decode_token (positions
// must be contiguous), tokenize, generate_greedy{,_tokens,_from_bos}, the
// result structs, and std::runtime_error on failure (the KV cache is reset
// when a decode step fails, as in the reference).
// Lifted: one-KV-head and < 4 GiB limits (any head_count_kv dividing
// head_count, 64-bit offsets).
#pragma once

#include "vortexrt/gguf.hpp"
#include "vortexrt/vulkan_context.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

struct vrt_model;

namespace vortexrt {

struct Gemma3Config {
    std::uint32_t context_length = 0;
    std::uint32_t embedding_length = 0;
    std::uint32_t block_count = 0;
    std::uint32_t feed_forward_length = 0;
    std::uint32_t head_count = 0;
    std::uint32_t head_count_kv = 0;
    std::uint32_t head_dim = 0;
    std::uint32_t value_dim = 0;
    std::uint32_t vocab_size = 0;
    std::uint32_t sliding_window = 0;
    float rms_epsilon = 1.0e-6f;
    float global_rope_base = 1.0e6f;
    float local_rope_base = 1.0e4f;
};

struct Gemma3TopToken {
    std::uint32_t token_id = 0;
    float logit = 0.0f;
    std::string piece;
};

struct Gemma3SingleTokenResult {
    std::vector<float> hidden;
    std::vector<Gemma3TopToken> top_tokens;
};

struct Gemma3GenerationResult {
    std::vector<std::uint32_t> token_ids;
    std::string text;
};

class Gemma3Tokenizer;

class Gemma3Model {
public:
    Gemma3Model(const std::string& gguf_path, VulkanContext& context, const std::string& q8_matvec_spirv,
                const std::string& q8_matvec_u8_spirv = {}, const std::string& argmax_spirv = {},
                const std::string& q8_matvec_32_spirv = {}, const std::string& q8_matvec_u8_32_spirv = {},
                const std::string& gelu_mul_spirv = {}, const std::string& q8_matvec_16_spirv = {},
                const std::string& q8_matvec_u8_16_spirv = {}, const std::string& q8_matvec_8_spirv = {},
                const std::string& q8_matvec_u8_8_spirv = {}, std::uint32_t q8_lane_override = 0);
    ~Gemma3Model();
    Gemma3Model(const Gemma3Model&) = delete;
    Gemma3Model& operator=(const Gemma3Model&) = delete;

    [[nodiscard]] const Gemma3Config& config() const noexcept { return config_; }
    [[nodiscard]] bool projection_fusion_enabled() const noexcept { return fuse_projections_; }
    void set_projection_fusion_enabled(bool enabled) noexcept { fuse_projections_ = enabled; }
    [[nodiscard]] std::uint32_t narrow_q8_lane_count() const noexcept { return narrow_q8_lane_count_; }
    [[nodiscard]] bool fused_ffn_enabled() const noexcept { return fuse_projections_ && ffn_available_; }

    [[nodiscard]] Gemma3SingleTokenResult run_single_token(std::uint32_t token_id, std::size_t top_k = 8);
    void reset_cache();
    [[nodiscard]] Gemma3SingleTokenResult decode_token(std::uint32_t token_id, std::uint32_t position,
                                                       std::size_t top_k = 1);
    [[nodiscard]] std::vector<std::uint32_t> tokenize(const std::string& text, bool add_bos = true) const;
    [[nodiscard]] Gemma3GenerationResult generate_greedy(const std::string& prompt, std::size_t max_new_tokens);
    [[nodiscard]] Gemma3GenerationResult generate_greedy_tokens(const std::vector<std::uint32_t>& prompt_tokens,
                                                                std::size_t max_new_tokens);
    [[nodiscard]] Gemma3GenerationResult generate_greedy_from_bos(std::size_t max_new_tokens);

    // Extensions
    [[nodiscard]] std::string token_piece(std::uint32_t token_id) const;
    [[nodiscard]] std::string decode_piece(std::uint32_t token_id) const;
    [[nodiscard]] vrt_model* native() const noexcept { return model_; }

private:
    VulkanContext& context_;
    vrt_model* model_ = nullptr;
    std::unique_ptr<Gemma3Tokenizer> tokenizer_;
    Gemma3Config config_{};
    bool fuse_projections_ = true;
    bool ffn_available_ = false;
    bool argmax_available_ = false;
    std::uint32_t narrow_q8_lane_count_ = 32;
    std::uint32_t next_position_ = 0;
};

// Host tokenizer of the GGUF vocabulary with the reference's rules
// (src/gemma3.cpp:289-454 index, 1895-2062 tokenize, 1237-1299 pieces):
// whitespace runs -> one U+2581, optional space prefix, Viterbi over pieces
// of type 1/4 by score, byte-piece fallback (<0xHH>, type 6) at -100, else
// the unknown id; BOS prepended on request.
class Gemma3Tokenizer {
public:
    explicit Gemma3Tokenizer(const GgufFile& gguf, std::uint32_t vocab_size);
    [[nodiscard]] std::vector<std::uint32_t> tokenize(const std::string& text, bool add_bos) const;
    [[nodiscard]] std::string token_piece(std::uint32_t id) const;
    [[nodiscard]] std::string decode_piece(std::uint32_t id) const;
    [[nodiscard]] std::uint32_t bos() const noexcept { return bos_; }
    [[nodiscard]] std::uint64_t eos() const noexcept { return eos_; }

private:
    struct Entry {
        std::uint32_t id = 0;
        float score = 0.0f;
    };
    std::vector<std::string> pieces_;
    std::unordered_map<std::string, Entry> index_;
    std::array<std::uint32_t, 256> byte_ids_{};
    std::size_t max_piece_ = 0;
    std::uint32_t unk_ = 3, bos_ = 2;
    std::uint64_t eos_ = 1;
    bool add_space_prefix_ = false;
};

}  // namespace vortexrt
