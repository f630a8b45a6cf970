// Host-only stand-in for the reference's Vulkan context header
// (include/vortexrt/vulkan_context.hpp:13-145).  TEST INFRASTRUCTURE: it lets
// the reference's unmodified src/gemma3.cpp compile on a machine without a
// graphics stack, so the oracle is the reference's own token loop.  Only the
// names gemma3.cpp touches are provided.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

using VkDeviceSize = std::uint64_t;
using VkBufferUsageFlags = std::uint32_t;
using VkMemoryPropertyFlags = std::uint32_t;

enum VkPhysicalDeviceType {
    VK_PHYSICAL_DEVICE_TYPE_OTHER = 0,
    VK_PHYSICAL_DEVICE_TYPE_INTEGRATED_GPU = 1,
    VK_PHYSICAL_DEVICE_TYPE_DISCRETE_GPU = 2,
    VK_PHYSICAL_DEVICE_TYPE_VIRTUAL_GPU = 3,
    VK_PHYSICAL_DEVICE_TYPE_CPU = 4,
};

constexpr VkBufferUsageFlags VK_BUFFER_USAGE_TRANSFER_SRC_BIT = 0x1;
constexpr VkBufferUsageFlags VK_BUFFER_USAGE_TRANSFER_DST_BIT = 0x2;
constexpr VkBufferUsageFlags VK_BUFFER_USAGE_STORAGE_BUFFER_BIT = 0x20;
constexpr VkMemoryPropertyFlags VK_MEMORY_PROPERTY_DEVICE_LOCAL_BIT = 0x1;
constexpr VkMemoryPropertyFlags VK_MEMORY_PROPERTY_HOST_VISIBLE_BIT = 0x2;
constexpr VkMemoryPropertyFlags VK_MEMORY_PROPERTY_HOST_COHERENT_BIT = 0x4;

namespace vortexrt {

struct DeviceCapabilities {
    std::string name = "oracle-host";
    VkPhysicalDeviceType device_type = VK_PHYSICAL_DEVICE_TYPE_CPU;
    std::uint32_t subgroup_size = 8;
};

class VulkanContext {
public:
    explicit VulkanContext(std::uint32_t subgroup_size = 8, unsigned threads = 1) {
        caps_.subgroup_size = subgroup_size;
        threads_ = threads == 0 ? 1 : threads;
    }
    [[nodiscard]] const DeviceCapabilities& capabilities() const noexcept { return caps_; }
    [[nodiscard]] unsigned threads() const noexcept { return threads_; }
    void set_threads(unsigned t) noexcept { threads_ = t == 0 ? 1 : t; }

private:
    DeviceCapabilities caps_{};
    unsigned threads_ = 1;
};

} // namespace vortexrt
