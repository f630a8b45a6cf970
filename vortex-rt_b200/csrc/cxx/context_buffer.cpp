// vortexrt::VulkanContext and vortexrt::Buffer over the C ABI (CUDA device
// context and device allocations).

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "vortexrt/buffer.hpp"
#include "vortexrt/vulkan_context.hpp"
#include "vortexrt_b200.h"

namespace vortexrt {
namespace {

void check(int rc, const char* what) {
    if (rc != VRT_OK) throw std::runtime_error(std::string(what) + ": " + vrt_last_error());
}

bool all_digits(const std::string& s) {
    if (s.empty()) return false;
    for (char c : s)
        if (c < '0' || c > '9') return false;
    return true;
}

}  // namespace

VulkanContext::VulkanContext(std::string selector) {
    if (selector.empty()) {
        if (const char* env = std::getenv("VORTEXRT_DEVICE")) selector = env;
    }
    int device = 0;
    if (all_digits(selector)) {
        device = std::stoi(selector);
    } else if (!selector.empty()) {
        // name substring: probe devices 0..15
        bool found = false;
        for (int d = 0; d < 16 && !found; ++d) {
            vrt_ctx* c = nullptr;
            if (vrt_ctx_create(d, &c) != VRT_OK) break;
            vrt_device_info info{};
            vrt_ctx_info(c, &info);
            vrt_ctx_destroy(c);
            if (std::string(info.name).find(selector) != std::string::npos) {
                device = d;
                found = true;
            }
        }
        if (!found) throw std::runtime_error("No CUDA device matches selector: " + selector);
    }
    check(vrt_ctx_create(device, &ctx_), "VulkanContext");
    vrt_device_info info{};
    check(vrt_ctx_info(ctx_, &info), "VulkanContext");
    caps_.name = info.name;
    caps_.device_index = static_cast<std::uint32_t>(info.device);
    caps_.subgroup_size = info.warp_size;
    caps_.device_local_bytes = info.global_mem_bytes;
    caps_.sm_count = static_cast<std::uint32_t>(info.sm_count);
    caps_.api_version = static_cast<std::uint32_t>(info.cc_major * 10 + info.cc_minor);
}

VulkanContext::~VulkanContext() { vrt_ctx_destroy(ctx_); }

void VulkanContext::synchronize() { check(vrt_ctx_synchronize(ctx_), "synchronize"); }

Buffer::Buffer(VulkanContext& context, VkDeviceSize size, VkBufferUsageFlags, VkMemoryPropertyFlags props)
    : context_(context), size_(size), memory_properties_(props) {
    if (size == 0) throw std::runtime_error("Buffer size must be non-zero");
    check(vrt_alloc(context.native(), static_cast<size_t>(size), &ptr_), "Buffer allocation");
}

Buffer::~Buffer() { vrt_free(context_.native(), ptr_); }

void Buffer::upload(const void* data, std::size_t bytes, VkDeviceSize offset) {
    if (offset > size_ || bytes > size_ - offset) throw std::runtime_error("Buffer upload out of range");
    if (!bytes) return;
    check(vrt_upload(context_.native(), static_cast<char*>(ptr_) + offset, data, bytes), "Buffer upload");
}

void Buffer::download(void* data, std::size_t bytes, VkDeviceSize offset) const {
    if (offset > size_ || bytes > size_ - offset) throw std::runtime_error("Buffer download out of range");
    if (!bytes) return;
    check(vrt_download(context_.native(), data, static_cast<const char*>(ptr_) + offset, bytes), "Buffer download");
}

}  // namespace vortexrt
