// Q8_0 mat-vec with the interface of the reference's Q8MatVecPipeline
// (include/vortexrt/q8_matvec.hpp:17-100 of the reference).  Every run*
// call is synchronous, validates dimensions, 4-byte aligned offsets and
// buffer ranges, and throws std::runtime_error on failure, as the reference
// does.  The SPIR-V path arguments are accepted and ignored; the fused FFN
// is available when a gelu_mul path is given, as in the reference.
#pragma once

#include "vortexrt/buffer.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>

namespace vortexrt {

class Q8MatVecPipeline {
public:
    Q8MatVecPipeline(VulkanContext& context, const std::string& spirv_path,
                     const std::string& u8_spirv_path = {}, const std::string& gelu_mul_spirv_path = {});
    ~Q8MatVecPipeline() = default;
    Q8MatVecPipeline(const Q8MatVecPipeline&) = delete;
    Q8MatVecPipeline& operator=(const Q8MatVecPipeline&) = delete;

    [[nodiscard]] bool using_native_u8() const noexcept { return true; }
    [[nodiscard]] bool ffn_available() const noexcept { return ffn_available_; }

    void run(Buffer& weights, Buffer& input, Buffer& output, std::uint32_t weight_byte_offset,
             std::uint32_t input_dim, std::uint32_t output_dim);

    void run_staged(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                    Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                    void* host_output, std::size_t host_output_bytes, std::uint32_t weight_byte_offset,
                    std::uint32_t input_dim, std::uint32_t output_dim);

    void run_staged_ffn(Buffer& weights, Buffer& input, Buffer& workspace, Buffer& staging_input,
                        Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                        void* host_output, std::size_t host_output_bytes,
                        std::uint32_t gate_weight_byte_offset, std::uint32_t up_weight_byte_offset,
                        std::uint32_t down_weight_byte_offset, std::uint32_t input_dim,
                        std::uint32_t ffn_dim, std::uint32_t output_dim);

    void run_staged_pair(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                         Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                         void* host_output, std::size_t host_output_bytes,
                         const std::array<std::uint32_t, 2>& weight_byte_offsets, std::uint32_t input_dim,
                         const std::array<std::uint32_t, 2>& output_dims);

    void run_staged_triplet(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                            Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                            void* host_output, std::size_t host_output_bytes,
                            const std::array<std::uint32_t, 3>& weight_byte_offsets, std::uint32_t input_dim,
                            const std::array<std::uint32_t, 3>& output_dims);

private:
    VulkanContext& context_;
    bool ffn_available_ = false;
};

}  // namespace vortexrt
