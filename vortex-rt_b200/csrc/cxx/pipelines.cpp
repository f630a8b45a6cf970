// vortexrt::Q8MatVecPipeline and vortexrt::ArgmaxPipeline over the C ABI.
// Validation order and messages follow the reference (src/q8_matvec.cpp:
// 801-930, 933-1358, 1360-2004, 2007-2890; src/argmax.cpp:503-567); every
// call is synchronous like the reference's fence-waited submits.

#include <limits>
#include <stdexcept>
#include <string>

#include "vortexrt/argmax.hpp"
#include "vortexrt/q8_matvec.hpp"
#include "vortexrt_b200.h"

namespace vortexrt {
namespace {

void check(int rc) {
    if (rc != VRT_OK) throw std::runtime_error(vrt_last_error());
}

std::uint64_t mul(std::uint64_t a, std::uint64_t b, const char* what) {
    if (a && b > std::numeric_limits<std::uint64_t>::max() / a) throw std::runtime_error(what);
    return a * b;
}

std::uint64_t matrix_bytes(std::uint32_t in, std::uint32_t out, const char* what) {
    return mul(out, mul(in / 32u, 34u, what), what);
}

void validate_single(Buffer& w, std::uint32_t off, std::uint32_t in, std::uint32_t out) {
    if (in == 0 || out == 0) throw std::runtime_error("Q8MatVecPipeline dimensions must be non-zero");
    if (in % 32u) throw std::runtime_error("Q8MatVecPipeline input_dim must be divisible by 32");
    if (off & 3u) throw std::runtime_error("Q8MatVecPipeline weight byte offset must be 4-byte aligned");
    if (static_cast<std::uint64_t>(off) + matrix_bytes(in, out, "Q8MatVecPipeline matrix byte size overflow") > w.size()) {
        throw std::runtime_error("Q8MatVecPipeline weight buffer is too small");
    }
}

}  // namespace

Q8MatVecPipeline::Q8MatVecPipeline(VulkanContext& context, const std::string&, const std::string&,
                                   const std::string& gelu_mul_spirv_path)
    : context_(context), ffn_available_(!gelu_mul_spirv_path.empty()) {}

void Q8MatVecPipeline::run(Buffer& weights, Buffer& input, Buffer& output, std::uint32_t off, std::uint32_t in,
                           std::uint32_t out) {
    validate_single(weights, off, in, out);
    if (static_cast<std::uint64_t>(in) * 4u > input.size()) throw std::runtime_error("Q8MatVecPipeline input buffer is too small");
    if (static_cast<std::uint64_t>(out) * 4u > output.size()) throw std::runtime_error("Q8MatVecPipeline output buffer is too small");
    check(vrt_q8_gemv(context_.native(), weights.device_ptr(), weights.size(), off,
                      static_cast<const float*>(input.device_ptr()), static_cast<float*>(output.device_ptr()), in, out,
                      nullptr));
    context_.synchronize();
}

void Q8MatVecPipeline::run_staged(Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
                                  Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                                  void* host_output, std::size_t host_output_bytes, std::uint32_t off,
                                  std::uint32_t in, std::uint32_t out) {
    if (!host_input) throw std::runtime_error("Q8MatVecPipeline::run_staged received null host input");
    const bool readback = host_output != nullptr;
    validate_single(weights, off, in, out);
    const std::uint64_t ib = static_cast<std::uint64_t>(in) * 4u, ob = static_cast<std::uint64_t>(out) * 4u;
    if (ib > input.size() || ob > output.size()) throw std::runtime_error("Q8MatVecPipeline device buffer is too small");
    if (ib > staging_input.size() || (readback && ob > staging_output.size())) {
        throw std::runtime_error("Q8MatVecPipeline staging buffer is too small");
    }
    if (host_input_bytes < ib || (readback && host_output_bytes < ob)) {
        throw std::runtime_error("Q8MatVecPipeline host buffer is too small");
    }
    input.upload(host_input, ib);
    check(vrt_q8_gemv(context_.native(), weights.device_ptr(), weights.size(), off,
                      static_cast<const float*>(input.device_ptr()), static_cast<float*>(output.device_ptr()), in, out,
                      nullptr));
    if (readback) output.download(host_output, ob);
    else context_.synchronize();
}

void Q8MatVecPipeline::run_staged_ffn(Buffer& weights, Buffer& input, Buffer& workspace, Buffer& staging_input,
                                      Buffer& staging_output, const void* host_input, std::size_t host_input_bytes,
                                      void* host_output, std::size_t host_output_bytes, std::uint32_t gate_off,
                                      std::uint32_t up_off, std::uint32_t down_off, std::uint32_t in, std::uint32_t ffn,
                                      std::uint32_t out) {
    if (!ffn_available_) throw std::runtime_error("Q8MatVecPipeline fused FFN path is unavailable");
    if (!host_input || !host_output) throw std::runtime_error("Q8MatVecPipeline::run_staged_ffn received null host buffer");
    if (!in || !ffn || !out || in % 32u || ffn % 32u) {
        throw std::runtime_error("Q8 fused FFN dimensions must be non-zero and Q8 aligned");
    }
    if ((gate_off & 3u) || (up_off & 3u) || (down_off & 3u)) {
        throw std::runtime_error("Q8 fused FFN weight offsets must be 4-byte aligned");
    }
    if (gate_off + matrix_bytes(in, ffn, "Q8 fused FFN gate matrix size overflow") > weights.size() ||
        up_off + matrix_bytes(in, ffn, "Q8 fused FFN up matrix size overflow") > weights.size() ||
        down_off + matrix_bytes(ffn, out, "Q8 fused FFN down matrix size overflow") > weights.size()) {
        throw std::runtime_error("Q8 fused FFN weight buffer is too small");
    }
    const std::uint64_t ib = 4ull * in, fb = 4ull * ffn, ob = 4ull * out;
    if (ib > input.size() || ib > staging_input.size() || host_input_bytes < ib || 2 * fb + ob > workspace.size() ||
        ob > staging_output.size() || host_output_bytes < ob) {
        throw std::runtime_error("Q8 fused FFN activation/staging buffer is too small");
    }
    input.upload(host_input, ib);
    float* ws = static_cast<float*>(workspace.device_ptr());
    check(vrt_q8_ffn(context_.native(), weights.device_ptr(), weights.size(), gate_off, up_off, down_off,
                     static_cast<const float*>(input.device_ptr()), ws, ws + 2 * static_cast<std::size_t>(ffn), in, ffn,
                     out, nullptr));
    workspace.download(host_output, ob, 2 * fb);
}

namespace {

template <std::size_t N>
void packed(VulkanContext& ctx, Buffer& weights, Buffer& input, Buffer& output, Buffer& staging_input,
            Buffer& staging_output, const void* host_input, std::size_t host_input_bytes, void* host_output,
            std::size_t host_output_bytes, const std::array<std::uint32_t, N>& offs, std::uint32_t in,
            const std::array<std::uint32_t, N>& dims, const char* name, const char* kind) {
    const std::string pre = std::string("Q8 ") + kind;
    if (!host_input || !host_output) {
        throw std::runtime_error(std::string("Q8MatVecPipeline::") + name + " received null host buffer");
    }
    if (!in || in % 32u) {
        throw std::runtime_error(std::string("Q8MatVecPipeline ") + kind + " input_dim must be non-zero and divisible by 32");
    }
    const std::uint64_t ib = 4ull * in;
    if (ib > input.size() || ib > staging_input.size() || host_input_bytes < ib) {
        throw std::runtime_error(pre + " input buffer is too small");
    }
    std::uint64_t total = 0;
    std::uint64_t o64[N];
    for (std::size_t i = 0; i < N; ++i) {
        if (!dims[i]) throw std::runtime_error(pre + " output dimensions must be non-zero");
        if (offs[i] & 3u) throw std::runtime_error(pre + " weight offsets must be 4-byte aligned");
        if (offs[i] + matrix_bytes(in, dims[i], "Q8 matrix byte size overflow") > weights.size()) {
            throw std::runtime_error(pre + " weight buffer is too small");
        }
        o64[i] = offs[i];
        total += 4ull * dims[i];
    }
    if (total > output.size() || total > staging_output.size() || host_output_bytes < total) {
        throw std::runtime_error(pre + " output buffer is too small");
    }
    input.upload(host_input, ib);
    check(vrt_q8_gemv_multi(ctx.native(), weights.device_ptr(), weights.size(), o64, dims.data(), N,
                            static_cast<const float*>(input.device_ptr()), static_cast<float*>(output.device_ptr()), in,
                            nullptr));
    output.download(host_output, total);
}

}  // namespace

void Q8MatVecPipeline::run_staged_pair(Buffer& weights, Buffer& input, Buffer& output, Buffer& si, Buffer& so,
                                       const void* hi, std::size_t hib, void* ho, std::size_t hob,
                                       const std::array<std::uint32_t, 2>& offs, std::uint32_t in,
                                       const std::array<std::uint32_t, 2>& dims) {
    packed<2>(context_, weights, input, output, si, so, hi, hib, ho, hob, offs, in, dims, "run_staged_pair", "pair");
}

void Q8MatVecPipeline::run_staged_triplet(Buffer& weights, Buffer& input, Buffer& output, Buffer& si, Buffer& so,
                                          const void* hi, std::size_t hib, void* ho, std::size_t hob,
                                          const std::array<std::uint32_t, 3>& offs, std::uint32_t in,
                                          const std::array<std::uint32_t, 3>& dims) {
    packed<3>(context_, weights, input, output, si, so, hi, hib, ho, hob, offs, in, dims, "run_staged_triplet",
              "triplet");
}

ArgmaxPipeline::ArgmaxPipeline(VulkanContext& context, const std::string&) : context_(context) {}

void ArgmaxPipeline::run(Buffer& input, Buffer& output, std::uint32_t n) {
    if (n == 0) throw std::runtime_error("ArgmaxPipeline requires non-zero input");
    if (4ull * n > input.size()) throw std::runtime_error("ArgmaxPipeline input buffer is too small");
    if (sizeof(ArgmaxResult) > output.size()) throw std::runtime_error("ArgmaxPipeline output buffer is too small");
    check(vrt_argmax(context_.native(), static_cast<const float*>(input.device_ptr()), n,
                     static_cast<vrt_argmax_result*>(output.device_ptr()), nullptr));
    context_.synchronize();
}

}  // namespace vortexrt
