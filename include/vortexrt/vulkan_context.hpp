// Device context with the interface of the Vortex-RT reference's
// VulkanContext (include/vortexrt/vulkan_context.hpp:13-145 of the reference),
// backed by a CUDA device (vrt_ctx of include/vortexrt_b200.h).  The class and
// type names are kept so code written against the reference compiles
// unchanged; no Vulkan is involved.  The Vk* names below are plain integer
// aliases that carry the same meaning in the Buffer interface.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

struct vrt_ctx;

using VkDeviceSize = std::uint64_t;
using VkBufferUsageFlags = std::uint32_t;
using VkMemoryPropertyFlags = std::uint32_t;
using VkSubgroupFeatureFlags = std::uint32_t;

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
    std::string name;
    std::uint32_t device_index = 0;
    std::uint32_t vendor_id = 0x10de;
    std::uint32_t device_id = 0;
    VkPhysicalDeviceType device_type = VK_PHYSICAL_DEVICE_TYPE_DISCRETE_GPU;
    std::uint32_t api_version = 0;
    std::uint32_t subgroup_size = 32;  // CUDA warp
    VkSubgroupFeatureFlags subgroup_ops = 0;
    bool fp16 = true;
    bool int8 = true;
    bool storage8 = true;
    bool storage16 = true;
    float timestamp_period_ns = 1.0f;
    std::uint32_t timestamp_valid_bits = 64;
    VkDeviceSize non_coherent_atom_size = 1;
    VkDeviceSize device_local_bytes = 0;
    std::uint32_t sm_count = 0;
};

class VulkanContext {
public:
    // `device_selector`: a device index, or a substring of the device name;
    // empty = VORTEXRT_DEVICE environment variable, else device 0
    // (the selection rule of the reference, src/vulkan_context.cpp:116-123).
    explicit VulkanContext(std::string device_selector = {});
    ~VulkanContext();
    VulkanContext(const VulkanContext&) = delete;
    VulkanContext& operator=(const VulkanContext&) = delete;

    [[nodiscard]] const DeviceCapabilities& capabilities() const noexcept { return caps_; }
    [[nodiscard]] vrt_ctx* native() const noexcept { return ctx_; }
    void synchronize();

private:
    vrt_ctx* ctx_ = nullptr;
    DeviceCapabilities caps_{};
};

}  // namespace vortexrt
