// Host restatement of the reference's Q8MatVecPipeline interface
// (include/vortexrt/q8_matvec.hpp:17-100).  TEST INFRASTRUCTURE: the bodies
// (oracle/shim/shim.cpp) compute what shaders/q8_matvec*.comp and
// shaders/gelu_mul.comp compute, on host threads.
#pragma once

#include "vortexrt/buffer.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>

namespace vortexrt {

class Q8MatVecPipeline {
public:
    // `spirv_path` selects the lane count of the restated shader: the
    // reference passes the path of q8_matvec{,_32,_16,_8}.spv; the oracle
    // passes "lanes=N".
    Q8MatVecPipeline(VulkanContext& context, const std::string& spirv_path,
                     const std::string& u8_spirv_path = {},
                     const std::string& gelu_mul_spirv_path = {});
    ~Q8MatVecPipeline() = default;
    Q8MatVecPipeline(const Q8MatVecPipeline&) = delete;
    Q8MatVecPipeline& operator=(const Q8MatVecPipeline&) = delete;

    [[nodiscard]] bool using_native_u8() const noexcept { return false; }
    [[nodiscard]] bool ffn_available() const noexcept { return ffn_available_; }
    [[nodiscard]] std::uint32_t lanes() const noexcept { return lanes_; }

    void run(Buffer& weights, Buffer& input, Buffer& output, std::uint32_t weight_byte_offset,
             std::uint32_t input_dim, std::uint32_t output_dim);

    void run_staged(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                    Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                    void* host_output, std::size_t host_output_bytes,
                    std::uint32_t weight_byte_offset, std::uint32_t input_dim,
                    std::uint32_t output_dim);

    void run_staged_ffn(Buffer& weights, Buffer& input, Buffer& workspace, Buffer& staging_input,
                        Buffer& staging_output, const void* host_input,
                        std::size_t host_input_bytes, void* host_output,
                        std::size_t host_output_bytes, std::uint32_t gate_weight_byte_offset,
                        std::uint32_t up_weight_byte_offset,
                        std::uint32_t down_weight_byte_offset, std::uint32_t input_dim,
                        std::uint32_t ffn_dim, std::uint32_t output_dim);

    void run_staged_pair(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                         Buffer& staging_output, const void* host_input,
                         std::size_t host_input_bytes, void* host_output,
                         std::size_t host_output_bytes,
                         const std::array<std::uint32_t, 2>& weight_byte_offsets,
                         std::uint32_t input_dim,
                         const std::array<std::uint32_t, 2>& output_dims);

    void run_staged_triplet(Buffer& weights, Buffer& input, Buffer& output,
                            Buffer& staging_input, Buffer& staging_output,
                            const void* host_input, std::size_t host_input_bytes,
                            void* host_output, std::size_t host_output_bytes,
                            const std::array<std::uint32_t, 3>& weight_byte_offsets,
                            std::uint32_t input_dim,
                            const std::array<std::uint32_t, 3>& output_dims);

private:
    VulkanContext& context_;
    std::uint32_t lanes_ = 64;
    bool ffn_available_ = false;
};

} // namespace vortexrt
