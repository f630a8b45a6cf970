// TEST INFRASTRUCTURE -- host bodies for the Vulkan-layer classes that the
// reference's unmodified src/gemma3.cpp links against (11 symbols: Buffer,
// Q8MatVecPipeline::run_staged*, ArgmaxPipeline).  Each body computes what the
// reference's shader computes, on host threads, in the shader's own order:
//
//   shaders/q8_matvec*.comp:36-69   per-lane fp32 partial sums over Q8_0
//                                   blocks strided by the lane count, then a
//                                   shared-memory tree reduction
//   shaders/gelu_mul.comp:17-31     gate = gelu_tanh(gate) * up
//   shaders/argmax.comp:30-107      argmax, ties -> lower index, NaN never wins
//
// The checks and messages follow src/q8_matvec.cpp (801-930, 933-1358,
// 1360-2004, 2007-2447, 2450-2890) and src/argmax.cpp:503-567.  Rows are split
// across threads; a row's arithmetic never depends on the thread count.
//
// Built with -ffp-contract=off so every product and sum rounds separately.

#include "vortexrt/argmax.hpp"
#include "vortexrt/buffer.hpp"
#include "vortexrt/q8_matvec.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <thread>
#include <vector>

namespace vortexrt {
namespace {

constexpr std::uint64_t kBlockElems = 32;
constexpr std::uint64_t kBlockBytes = 34;

float half_to_float(std::uint16_t h) {
    const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
    std::uint32_t exponent = (h >> 10) & 31u;
    std::uint32_t mantissa = h & 1023u;
    std::uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mantissa & 0x400u) == 0) {
                mantissa <<= 1;
                --e;
            }
            mantissa &= 0x3ffu;
            bits = sign | (static_cast<std::uint32_t>(e + 127) << 23) | (mantissa << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent - 15u + 127u) << 23) | (mantissa << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

std::uint64_t mul_checked(std::uint64_t a, std::uint64_t b, const char* what) {
    if (a != 0 && b > std::numeric_limits<std::uint64_t>::max() / a) {
        throw std::runtime_error(what);
    }
    return a * b;
}

std::uint64_t add_checked(std::uint64_t a, std::uint64_t b, const char* what) {
    if (b > std::numeric_limits<std::uint64_t>::max() - a) {
        throw std::runtime_error(what);
    }
    return a + b;
}

// One output row, exactly as one workgroup of the restated shader.
float shader_row(const unsigned char* w, std::uint64_t row_base, std::uint32_t input_dim,
                 const float* x, std::uint32_t lanes, float* partial) {
    const std::uint32_t blocks = input_dim / 32u;
    for (std::uint32_t lane = 0; lane < lanes; ++lane) {
        float sum = 0.0f;
        for (std::uint32_t b = lane; b < blocks; b += lanes) {
            const std::uint64_t base = row_base + static_cast<std::uint64_t>(b) * 34u;
            const std::uint16_t bits =
                static_cast<std::uint16_t>(w[base] | (static_cast<unsigned>(w[base + 1]) << 8));
            const float d = half_to_float(bits);
            for (std::uint32_t k = 0; k < 32u; ++k) {
                const int q = static_cast<std::int8_t>(w[base + 2 + k]);
                const float prod = d * static_cast<float>(q);
                sum = sum + prod * x[b * 32u + k];
            }
        }
        partial[lane] = sum;
    }
    for (std::uint32_t stride = lanes / 2; stride > 0; stride >>= 1) {
        for (std::uint32_t lane = 0; lane < stride; ++lane) {
            partial[lane] += partial[lane + stride];
        }
    }
    return partial[0];
}

void matvec_rows(const unsigned char* w, std::uint64_t offset, std::uint32_t input_dim,
                 std::uint32_t output_dim, const float* x, float* y, std::uint32_t lanes,
                 unsigned threads) {
    const std::uint64_t row_bytes = static_cast<std::uint64_t>(input_dim) / 32u * 34u;
    auto work = [&](std::uint32_t r0, std::uint32_t r1) {
        std::vector<float> partial(lanes);
        for (std::uint32_t r = r0; r < r1; ++r) {
            y[r] = shader_row(w, offset + r * row_bytes, input_dim, x, lanes, partial.data());
        }
    };
    threads = std::max(1u, std::min<unsigned>(threads, output_dim / 64u + 1u));
    if (threads == 1) {
        work(0, output_dim);
        return;
    }
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < threads; ++t) {
        const auto r0 = static_cast<std::uint32_t>(static_cast<std::uint64_t>(output_dim) * t / threads);
        const auto r1 = static_cast<std::uint32_t>(static_cast<std::uint64_t>(output_dim) * (t + 1) / threads);
        pool.emplace_back(work, r0, r1);
    }
    for (auto& th : pool) th.join();
}

float gelu_tanh(float x) {
    constexpr float kSqrt2OverPi = 0.7978845608028654f;
    constexpr float kCubic = 0.044715f;
    const float x3 = x * x * x;
    return 0.5f * x * (1.0f + std::tanh(kSqrt2OverPi * (x + kCubic * x3)));
}

void check_matrix(const Buffer& weights, std::uint32_t offset, std::uint32_t input_dim,
                  std::uint32_t output_dim, const char* prefix) {
    if (input_dim == 0 || output_dim == 0) {
        throw std::runtime_error(std::string(prefix) + " dimensions must be non-zero");
    }
    if ((input_dim % kBlockElems) != 0) {
        throw std::runtime_error(std::string(prefix) + " input_dim must be divisible by 32");
    }
    if ((offset & 3u) != 0u) {
        throw std::runtime_error(std::string(prefix) + " weight byte offset must be 4-byte aligned");
    }
    const std::uint64_t row_bytes = mul_checked(input_dim / kBlockElems, kBlockBytes, "row byte size overflow");
    const std::uint64_t bytes = mul_checked(output_dim, row_bytes, "matrix byte size overflow");
    if (add_checked(offset, bytes, "weight range overflow") > weights.size()) {
        throw std::runtime_error(std::string(prefix) + " weight buffer is too small");
    }
}

std::uint32_t lanes_from_path(const std::string& path) {
    // "lanes=N" selects the restated q8_matvec_N shader; anything else is the 64-lane one.
    if (path.rfind("lanes=", 0) == 0) {
        const unsigned long v = std::stoul(path.substr(6));
        if (v == 8 || v == 16 || v == 32 || v == 64) return static_cast<std::uint32_t>(v);
        throw std::runtime_error("oracle shim: unsupported lane count " + path);
    }
    if (path.empty()) throw std::runtime_error("failed to open SPIR-V: ");
    return 64;
}

} // namespace

Buffer::Buffer(VulkanContext& context, VkDeviceSize size, VkBufferUsageFlags, VkMemoryPropertyFlags)
    : context_(context), size_(size), bytes_(static_cast<std::size_t>(size), 0) {
    if (size == 0) throw std::runtime_error("Buffer size must be non-zero");
}

void Buffer::upload(const void* data, std::size_t bytes, VkDeviceSize offset) {
    if (offset > size_ || bytes > size_ - offset) throw std::runtime_error("Buffer upload out of range");
    if (bytes) std::memcpy(bytes_.data() + offset, data, bytes);
}

void Buffer::download(void* data, std::size_t bytes, VkDeviceSize offset) const {
    if (offset > size_ || bytes > size_ - offset) throw std::runtime_error("Buffer download out of range");
    if (bytes) std::memcpy(data, bytes_.data() + offset, bytes);
}

Q8MatVecPipeline::Q8MatVecPipeline(VulkanContext& context, const std::string& spirv_path,
                                   const std::string&, const std::string& gelu_mul_spirv_path)
    : context_(context), lanes_(lanes_from_path(spirv_path)),
      ffn_available_(!gelu_mul_spirv_path.empty()) {}

void Q8MatVecPipeline::run(Buffer& weights, Buffer& input, Buffer& output,
                           std::uint32_t weight_byte_offset, std::uint32_t input_dim,
                           std::uint32_t output_dim) {
    check_matrix(weights, weight_byte_offset, input_dim, output_dim, "Q8MatVecPipeline");
    if (static_cast<std::uint64_t>(input_dim) * 4u > input.size()) {
        throw std::runtime_error("Q8MatVecPipeline input buffer is too small");
    }
    if (static_cast<std::uint64_t>(output_dim) * 4u > output.size()) {
        throw std::runtime_error("Q8MatVecPipeline output buffer is too small");
    }
    matvec_rows(weights.data(), weight_byte_offset, input_dim, output_dim,
                reinterpret_cast<const float*>(input.data()), reinterpret_cast<float*>(output.data()),
                lanes_, context_.threads());
}

void Q8MatVecPipeline::run_staged(Buffer& weights, Buffer& input, Buffer& output,
                                  Buffer& staging_input, Buffer& staging_output,
                                  const void* host_input, std::size_t host_input_bytes,
                                  void* host_output, std::size_t host_output_bytes,
                                  std::uint32_t weight_byte_offset, std::uint32_t input_dim,
                                  std::uint32_t output_dim) {
    if (host_input == nullptr) {
        throw std::runtime_error("Q8MatVecPipeline::run_staged received null host input");
    }
    const bool readback = host_output != nullptr;
    check_matrix(weights, weight_byte_offset, input_dim, output_dim, "Q8MatVecPipeline");
    const std::uint64_t in_bytes = static_cast<std::uint64_t>(input_dim) * 4u;
    const std::uint64_t out_bytes = static_cast<std::uint64_t>(output_dim) * 4u;
    if (in_bytes > input.size() || out_bytes > output.size()) {
        throw std::runtime_error("Q8MatVecPipeline device buffer is too small");
    }
    if (in_bytes > staging_input.size() || (readback && out_bytes > staging_output.size())) {
        throw std::runtime_error("Q8MatVecPipeline staging buffer is too small");
    }
    if (host_input_bytes < in_bytes || (readback && host_output_bytes < out_bytes)) {
        throw std::runtime_error("Q8MatVecPipeline host buffer is too small");
    }
    input.upload(host_input, in_bytes);
    run(weights, input, output, weight_byte_offset, input_dim, output_dim);
    if (readback) output.download(host_output, out_bytes);
}

void Q8MatVecPipeline::run_staged_ffn(Buffer& weights, Buffer& input, Buffer& workspace,
                                      Buffer& staging_input, Buffer& staging_output,
                                      const void* host_input, std::size_t host_input_bytes,
                                      void* host_output, std::size_t host_output_bytes,
                                      std::uint32_t gate_off, std::uint32_t up_off,
                                      std::uint32_t down_off, std::uint32_t input_dim,
                                      std::uint32_t ffn_dim, std::uint32_t output_dim) {
    if (!ffn_available_) throw std::runtime_error("Q8MatVecPipeline fused FFN path is unavailable");
    if (host_input == nullptr || host_output == nullptr) {
        throw std::runtime_error("Q8MatVecPipeline::run_staged_ffn received null host buffer");
    }
    if (input_dim == 0 || ffn_dim == 0 || output_dim == 0 || (input_dim % 32u) != 0 ||
        (ffn_dim % 32u) != 0) {
        throw std::runtime_error("Q8 fused FFN dimensions must be non-zero and Q8 aligned");
    }
    if ((gate_off & 3u) || (up_off & 3u) || (down_off & 3u)) {
        throw std::runtime_error("Q8 fused FFN weight offsets must be 4-byte aligned");
    }
    check_matrix(weights, gate_off, input_dim, ffn_dim, "Q8 fused FFN gate");
    check_matrix(weights, up_off, input_dim, ffn_dim, "Q8 fused FFN up");
    check_matrix(weights, down_off, ffn_dim, output_dim, "Q8 fused FFN down");
    const std::uint64_t in_bytes = static_cast<std::uint64_t>(input_dim) * 4u;
    const std::uint64_t ffn_bytes = static_cast<std::uint64_t>(ffn_dim) * 4u;
    const std::uint64_t out_bytes = static_cast<std::uint64_t>(output_dim) * 4u;
    if (in_bytes > input.size() || in_bytes > staging_input.size() || host_input_bytes < in_bytes ||
        2 * ffn_bytes + out_bytes > workspace.size() || out_bytes > staging_output.size() ||
        host_output_bytes < out_bytes) {
        throw std::runtime_error("Q8 fused FFN activation/staging buffer is too small");
    }
    input.upload(host_input, in_bytes);
    const float* x = reinterpret_cast<const float*>(input.data());
    float* ws = reinterpret_cast<float*>(workspace.data());
    float* gate = ws;
    float* up = ws + ffn_dim;
    float* y = ws + 2u * static_cast<std::size_t>(ffn_dim);
    matvec_rows(weights.data(), gate_off, input_dim, ffn_dim, x, gate, lanes_, context_.threads());
    matvec_rows(weights.data(), up_off, input_dim, ffn_dim, x, up, lanes_, context_.threads());
    for (std::uint32_t i = 0; i < ffn_dim; ++i) gate[i] = gelu_tanh(gate[i]) * up[i];
    matvec_rows(weights.data(), down_off, ffn_dim, output_dim, gate, y, lanes_, context_.threads());
    std::memcpy(host_output, y, out_bytes);
}

namespace {

template <std::size_t N>
void run_packed(Q8MatVecPipeline& self, std::uint32_t lanes, unsigned threads, Buffer& weights,
                Buffer& input, Buffer& output, const void* host_input,
                std::size_t host_input_bytes, void* host_output, std::size_t host_output_bytes,
                const std::array<std::uint32_t, N>& offsets, std::uint32_t input_dim,
                const std::array<std::uint32_t, N>& dims, const char* prefix) {
    (void)self;
    if (host_input == nullptr || host_output == nullptr) {
        throw std::runtime_error(std::string(prefix) + " received null host buffer");
    }
    if (input_dim == 0 || (input_dim % 32u) != 0) {
        throw std::runtime_error(std::string(prefix) + " input_dim must be non-zero and divisible by 32");
    }
    const std::uint64_t in_bytes = static_cast<std::uint64_t>(input_dim) * 4u;
    if (in_bytes > input.size() || host_input_bytes < in_bytes) {
        throw std::runtime_error(std::string(prefix) + " input buffer is too small");
    }
    std::uint64_t total = 0;
    for (std::size_t i = 0; i < N; ++i) {
        if (dims[i] == 0) throw std::runtime_error(std::string(prefix) + " output dimensions must be non-zero");
        check_matrix(weights, offsets[i], input_dim, dims[i], prefix);
        total += static_cast<std::uint64_t>(dims[i]) * 4u;
    }
    if (total > output.size() || host_output_bytes < total) {
        throw std::runtime_error(std::string(prefix) + " output buffer is too small");
    }
    input.upload(host_input, in_bytes);
    float* out = reinterpret_cast<float*>(output.data());
    std::size_t cursor = 0;
    for (std::size_t i = 0; i < N; ++i) {
        matvec_rows(weights.data(), offsets[i], input_dim, dims[i],
                    reinterpret_cast<const float*>(input.data()), out + cursor, lanes, threads);
        cursor += dims[i];
    }
    output.download(host_output, total);
}

} // namespace

void Q8MatVecPipeline::run_staged_pair(Buffer& weights, Buffer& input, Buffer& output, Buffer&,
                                       Buffer&, const void* host_input,
                                       std::size_t host_input_bytes, void* host_output,
                                       std::size_t host_output_bytes,
                                       const std::array<std::uint32_t, 2>& offsets,
                                       std::uint32_t input_dim,
                                       const std::array<std::uint32_t, 2>& dims) {
    run_packed<2>(*this, lanes_, context_.threads(), weights, input, output, host_input,
                  host_input_bytes, host_output, host_output_bytes, offsets, input_dim, dims,
                  "Q8MatVecPipeline::run_staged_pair");
}

void Q8MatVecPipeline::run_staged_triplet(Buffer& weights, Buffer& input, Buffer& output, Buffer&,
                                          Buffer&, const void* host_input,
                                          std::size_t host_input_bytes, void* host_output,
                                          std::size_t host_output_bytes,
                                          const std::array<std::uint32_t, 3>& offsets,
                                          std::uint32_t input_dim,
                                          const std::array<std::uint32_t, 3>& dims) {
    run_packed<3>(*this, lanes_, context_.threads(), weights, input, output, host_input,
                  host_input_bytes, host_output, host_output_bytes, offsets, input_dim, dims,
                  "Q8MatVecPipeline::run_staged_triplet");
}

ArgmaxPipeline::ArgmaxPipeline(VulkanContext& context, const std::string& spirv_path)
    : context_(context) {
    if (spirv_path.empty()) throw std::runtime_error("failed to open SPIR-V: ");
}

void ArgmaxPipeline::run(Buffer& input, Buffer& output, std::uint32_t element_count) {
    if (element_count == 0) throw std::runtime_error("ArgmaxPipeline requires non-zero input");
    if (static_cast<std::uint64_t>(element_count) * 4u > input.size()) {
        throw std::runtime_error("ArgmaxPipeline input buffer is too small");
    }
    if (sizeof(ArgmaxResult) > output.size()) {
        throw std::runtime_error("ArgmaxPipeline output buffer is too small");
    }
    const float* v = reinterpret_cast<const float*>(input.data());
    float best_value = -std::numeric_limits<float>::infinity();
    std::uint32_t best_index = 0xffffffffu;
    for (std::uint32_t i = 0; i < element_count; ++i) {
        const float c = v[i];
        if (std::isnan(c)) continue;
        if (c > best_value || (c == best_value && i < best_index)) {
            best_value = c;
            best_index = i;
        }
    }
    ArgmaxResult r{best_index, best_value};
    output.upload(&r, sizeof(r));
}

} // namespace vortexrt
