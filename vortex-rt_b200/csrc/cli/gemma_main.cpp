// vortexrt-gemma: command line of the Vortex-RT reference (src/gemma_main.cpp)
// over the B200 backend.  Same flags and the same report lines that the
// reference's CI greps ("Layers:", "Prompt token ids:", "Generated token ids:",
// "TEXT_BEGIN"/"TEXT_END", "Top logits:", "Final hidden checksum:",
// "Validation: OK").  Additions: --prompt-ids a,b,c and no 128-token cap on
// --generate; --q8-lanes and --projection-fusion are accepted and reported.

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <iomanip>
#include <iostream>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "vortexrt/gemma3.hpp"
#include "vortexrt/vulkan_context.hpp"

namespace {

struct Args {
    std::string model, device, prompt, prompt_ids, fusion = "auto";
    std::uint32_t token_id = 2, lanes = 0;
    std::size_t top_k = 8, generate = 0;
};

std::uint64_t number(const std::string& s, const char* flag, std::uint64_t max) {
    std::size_t used = 0;
    unsigned long long v = 0;
    try {
        v = std::stoull(s, &used, 10);
    } catch (...) {
        used = 0;
    }
    if (used != s.size() || v > max) throw std::runtime_error(std::string(flag) + " expects an integer <= " + std::to_string(max));
    return v;
}

const char* kUsage =
    "usage: vortexrt-gemma <model.gguf> [options]\n"
    "  --token-id N          input token id (default: 2/BOS)\n"
    "  --top-k N             display top logits; 0 skips LM head\n"
    "  --prompt TEXT         tokenize/prefill a text prompt before generation\n"
    "  --prompt-ids A,B,...  prefill these token ids (no tokenizer)\n"
    "  --generate N          greedy-generate N tokens with KV cache\n"
    "  --projection-fusion auto|on|off\n"
    "  --q8-lanes auto|8|16|32|64\n"
    "  --device <index|name> CUDA device selector\n";

Args parse(int argc, char** argv) {
    if (argc < 2) throw std::runtime_error(kUsage);
    Args a;
    a.model = argv[1];
    if (a.model == "--help" || a.model == "-h") {
        std::cout << kUsage;
        std::exit(0);
    }
    for (int i = 2; i < argc; ++i) {
        const std::string f = argv[i];
        auto val = [&]() -> std::string {
            if (i + 1 >= argc) throw std::runtime_error(f + " requires a value");
            return argv[++i];
        };
        if (f == "--token-id") a.token_id = static_cast<std::uint32_t>(number(val(), "--token-id", 0xffffffffu));
        else if (f == "--top-k") a.top_k = number(val(), "--top-k", std::numeric_limits<std::uint32_t>::max());
        else if (f == "--prompt") a.prompt = val();
        else if (f == "--prompt-ids") a.prompt_ids = val();
        else if (f == "--generate") a.generate = number(val(), "--generate", 1u << 16);
        else if (f == "--projection-fusion") {
            a.fusion = val();
            if (a.fusion != "auto" && a.fusion != "on" && a.fusion != "off") {
                throw std::runtime_error("--projection-fusion must be auto, on, or off");
            }
        } else if (f == "--q8-lanes") {
            const std::string v = val();
            if (v == "auto") a.lanes = 0;
            else {
                a.lanes = static_cast<std::uint32_t>(number(v, "--q8-lanes", 64));
                if (a.lanes != 8 && a.lanes != 16 && a.lanes != 32 && a.lanes != 64) {
                    throw std::runtime_error("--q8-lanes must be auto, 8, 16, 32, or 64");
                }
            }
        } else if (f == "--device") a.device = val();
        else if (f == "--help" || f == "-h") {
            std::cout << kUsage;
            std::exit(0);
        } else throw std::runtime_error("unknown argument: " + f);
    }
    return a;
}

std::string escape(const std::string& s) {
    std::ostringstream o;
    for (const unsigned char c : s) {
        if (c == '\n') o << "\\n";
        else if (c == '\r') o << "\\r";
        else if (c == '\t') o << "\\t";
        else if (c >= 32 && c < 127) o << static_cast<char>(c);
        else o << "\\x" << std::hex << std::setw(2) << std::setfill('0') << static_cast<unsigned>(c) << std::dec
               << std::setfill(' ');
    }
    return o.str();
}

double ms_since(std::chrono::steady_clock::time_point t) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count();
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const Args a = parse(argc, argv);
        const auto t_runtime = std::chrono::steady_clock::now();
        vortexrt::VulkanContext ctx(a.device);
        const auto t_model = std::chrono::steady_clock::now();
        // SPIR-V arguments are accepted by the constructor for source compatibility
        vortexrt::Gemma3Model model(a.model, ctx, "q8_matvec", "q8_matvec_u8", "argmax", "q8_matvec_32",
                                    "q8_matvec_u8_32", "gelu_mul", "q8_matvec_16", "q8_matvec_u8_16", "q8_matvec_8",
                                    "q8_matvec_u8_8", a.lanes);
        if (a.fusion == "on") model.set_projection_fusion_enabled(true);
        if (a.fusion == "off") model.set_projection_fusion_enabled(false);
        const double load_ms = ms_since(t_model), setup_ms = ms_since(t_runtime);
        const auto& c = model.config();
        std::cout << "Vortex-RT Gemma 3 runtime (B200 backend)\n"
                  << "  GPU: " << ctx.capabilities().name << "\n"
                  << "  Layers: " << c.block_count << "\n"
                  << "  Hidden: " << c.embedding_length << "\n"
                  << "  FFN: " << c.feed_forward_length << "\n"
                  << "  Heads: " << c.head_count << " / KV " << c.head_count_kv << "\n"
                  << "  Head dim: " << c.head_dim << "\n"
                  << "  Sliding window: " << c.sliding_window << "\n"
                  << "  Vocab: " << c.vocab_size << "\n"
                  << "  Narrow Q8 kernel: " << model.narrow_q8_lane_count() << " lanes\n"
                  << "  Projection fusion: " << (model.projection_fusion_enabled() ? "enabled" : "disabled") << "\n"
                  << "  Fused FFN: " << (model.fused_ffn_enabled() ? "enabled" : "disabled") << "\n"
                  << "  Model load: " << load_ms << " ms\n"
                  << "  Runtime setup: " << setup_ms << " ms\n";
        if (a.generate) {
            std::cout << "  Greedy generation from BOS: " << a.generate << " token(s)\n";
            std::vector<std::uint32_t> prompt;
            if (!a.prompt_ids.empty()) {
                std::stringstream ss(a.prompt_ids);
                std::string item;
                while (std::getline(ss, item, ',')) prompt.push_back(static_cast<std::uint32_t>(number(item, "--prompt-ids", 0xffffffffu)));
            } else {
                prompt = model.tokenize(a.prompt, true);
            }
            std::cout << "  Prompt token ids:";
            for (auto id : prompt) std::cout << " " << id;
            std::cout << "\n";
            const auto t0 = std::chrono::steady_clock::now();
            const auto g = model.generate_greedy_tokens(prompt, a.generate);
            const double gen_ms = ms_since(t0);
            std::cout << "  Generated token ids:";
            for (auto id : g.token_ids) std::cout << " " << id;
            std::cout << "\n  Generation time: " << gen_ms << " ms\n"
                      << "  Throughput: " << (gen_ms > 0 ? g.token_ids.size() * 1000.0 / gen_ms : 0.0) << " tok/s\n"
                      << "  Generated text: \"" << escape(g.text) << "\"\n"
                      << "TEXT_BEGIN\n" << g.text << "\nTEXT_END\n"
                      << "  Validation: OK\n";
            return 0;
        }
        std::cout << "  Token: " << a.token_id << "\n";
        const auto t0 = std::chrono::steady_clock::now();
        const auto r = model.run_single_token(a.token_id, a.top_k);
        const double fwd_ms = ms_since(t0);
        double checksum = 0.0, sq = 0.0;
        float max_abs = 0.0f;
        for (std::size_t i = 0; i < r.hidden.size(); ++i) {
            const float v = r.hidden[i];
            if (!std::isfinite(v)) throw std::runtime_error("final hidden state is non-finite");
            checksum += static_cast<double>(v) * static_cast<double>(i + 1);
            sq += static_cast<double>(v) * v;
            max_abs = std::max(max_abs, std::fabs(v));
        }
        std::cout << "  Forward time: " << fwd_ms << " ms\n"
                  << "  Final hidden RMS: " << std::sqrt(sq / static_cast<double>(r.hidden.size())) << "\n"
                  << "  Final hidden max abs: " << max_abs << "\n"
                  << "  Final hidden checksum: " << std::setprecision(12) << checksum << "\n";
        if (!r.top_tokens.empty()) {
            std::cout << "  Top logits:\n";
            for (std::size_t i = 0; i < r.top_tokens.size(); ++i) {
                std::cout << "    " << i + 1 << ": id=" << r.top_tokens[i].token_id << " logit=" << r.top_tokens[i].logit
                          << " piece=\"" << escape(r.top_tokens[i].piece) << "\"\n";
            }
        }
        std::cout << "  Validation: OK\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "vortexrt-gemma: " << e.what() << "\n";
        return 1;
    }
}
