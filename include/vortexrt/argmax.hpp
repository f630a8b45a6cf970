// Argmax with the interface of the reference's ArgmaxPipeline
// (include/vortexrt/argmax.hpp:12-32 of the reference); runs vrt_argmax.
// Rule: largest value, ties -> lower index, NaN never wins.
#pragma once

#include "vortexrt/buffer.hpp"

#include <cstdint>
#include <string>

namespace vortexrt {

struct ArgmaxResult {
    std::uint32_t index = 0;
    float value = 0.0f;
};

static_assert(sizeof(ArgmaxResult) == 8);

class ArgmaxPipeline {
public:
    // `spirv_path` is accepted for source compatibility and ignored.
    ArgmaxPipeline(VulkanContext& context, const std::string& spirv_path);
    ~ArgmaxPipeline() = default;
    ArgmaxPipeline(const ArgmaxPipeline&) = delete;
    ArgmaxPipeline& operator=(const ArgmaxPipeline&) = delete;

    // Synchronous: `output` holds an ArgmaxResult when it returns.
    void run(Buffer& input, Buffer& output, std::uint32_t element_count);

private:
    VulkanContext& context_;
};

}  // namespace vortexrt
