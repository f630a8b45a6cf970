// Host-memory Buffer with the reference's interface (include/vortexrt/buffer.hpp:11-42).
// TEST INFRASTRUCTURE for the oracle build of the reference's src/gemma3.cpp.
#pragma once

#include "vortexrt/vulkan_context.hpp"

#include <cstddef>
#include <vector>

namespace vortexrt {

class Buffer {
public:
    Buffer(VulkanContext& context, VkDeviceSize size, VkBufferUsageFlags usage,
           VkMemoryPropertyFlags memory_properties);
    ~Buffer() = default;
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;

    [[nodiscard]] VkDeviceSize size() const noexcept { return size_; }
    [[nodiscard]] unsigned char* data() noexcept { return bytes_.data(); }
    [[nodiscard]] const unsigned char* data() const noexcept { return bytes_.data(); }
    [[nodiscard]] VulkanContext& context() const noexcept { return context_; }

    void upload(const void* data, std::size_t bytes, VkDeviceSize offset = 0);
    void download(void* data, std::size_t bytes, VkDeviceSize offset = 0) const;

private:
    VulkanContext& context_;
    VkDeviceSize size_ = 0;
    std::vector<unsigned char> bytes_;
};

} // namespace vortexrt
