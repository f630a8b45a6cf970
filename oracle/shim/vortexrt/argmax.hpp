// Host restatement of the reference's ArgmaxPipeline interface
// (include/vortexrt/argmax.hpp:12-32).  TEST INFRASTRUCTURE.
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
    ArgmaxPipeline(VulkanContext& context, const std::string& spirv_path);
    ~ArgmaxPipeline() = default;
    ArgmaxPipeline(const ArgmaxPipeline&) = delete;
    ArgmaxPipeline& operator=(const ArgmaxPipeline&) = delete;

    void run(Buffer& input, Buffer& output, std::uint32_t element_count);

private:
    VulkanContext& context_;
};

} // namespace vortexrt
