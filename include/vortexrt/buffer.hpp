// Device buffer with the interface of the reference's Buffer
// (include/vortexrt/buffer.hpp:11-42 of the reference).  Memory is device
// memory of the context's GPU (vrt_alloc); upload/download are synchronous
// copies.  Usage and memory-property flags are accepted and recorded.
#pragma once

#include "vortexrt/vulkan_context.hpp"

#include <cstddef>

namespace vortexrt {

class Buffer {
public:
    Buffer(VulkanContext& context, VkDeviceSize size, VkBufferUsageFlags usage,
           VkMemoryPropertyFlags memory_properties);
    ~Buffer();
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;

    [[nodiscard]] void* handle() const noexcept { return ptr_; }      // device pointer
    [[nodiscard]] void* device_ptr() const noexcept { return ptr_; }
    [[nodiscard]] VkDeviceSize size() const noexcept { return size_; }
    [[nodiscard]] bool host_visible() const noexcept {
        return (memory_properties_ & VK_MEMORY_PROPERTY_HOST_VISIBLE_BIT) != 0;
    }
    [[nodiscard]] bool host_coherent() const noexcept {
        return (memory_properties_ & VK_MEMORY_PROPERTY_HOST_COHERENT_BIT) != 0;
    }
    [[nodiscard]] VulkanContext& context() const noexcept { return context_; }

    void upload(const void* data, std::size_t bytes, VkDeviceSize offset = 0);
    void download(void* data, std::size_t bytes, VkDeviceSize offset = 0) const;

private:
    VulkanContext& context_;
    void* ptr_ = nullptr;
    VkDeviceSize size_ = 0;
    VkMemoryPropertyFlags memory_properties_ = 0;
};

}  // namespace vortexrt
