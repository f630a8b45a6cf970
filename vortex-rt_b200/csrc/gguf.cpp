// GGUF v2/v3 reader behind vortexrt::GgufFile (include/vortexrt/gguf.hpp).
//
// The file is memory-mapped once; parsing walks a bounds-checked cursor over
// the mapping.  Limits follow the reference loader's intent (src/gguf.cpp:
// strings <= 1 GiB, arrays <= 2^28 elements, nesting <= 8, <= 10^6 tensors
// and keys, power-of-two alignment, every tensor payload inside the file);
// all failures throw std::runtime_error.

#include "vortexrt/gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <limits>
#include <stdexcept>

namespace vortexrt {
namespace {

constexpr std::uint32_t kMagic = 0x46554747u;  // "GGUF"
constexpr std::uint64_t kStringLimit = 1ull << 30;
constexpr std::uint64_t kArrayLimit = 1ull << 28;
constexpr std::uint32_t kDepthLimit = 8;
constexpr std::uint64_t kCountLimit = 1000000ull;

struct Cursor {
    const std::uint8_t* base;
    std::uint64_t size;
    std::uint64_t at = 0;

    void need(std::uint64_t n) const {
        if (n > size - at) throw std::runtime_error("Unexpected end of GGUF file");
    }
    template <typename T>
    T take() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string text() {
        const auto n = take<std::uint64_t>();
        if (n > kStringLimit) throw std::runtime_error("GGUF string length exceeds safety limit");
        need(n);
        std::string s(reinterpret_cast<const char*>(base + at), static_cast<std::size_t>(n));
        at += n;
        return s;
    }
};

GgufValue parse_value(Cursor& c, GgufValueType type, std::uint32_t depth) {
    GgufValue v;
    v.type = type;
    switch (type) {
    case GgufValueType::UInt8: v.scalar = static_cast<std::uint64_t>(c.take<std::uint8_t>()); break;
    case GgufValueType::Int8: v.scalar = static_cast<std::int64_t>(c.take<std::int8_t>()); break;
    case GgufValueType::UInt16: v.scalar = static_cast<std::uint64_t>(c.take<std::uint16_t>()); break;
    case GgufValueType::Int16: v.scalar = static_cast<std::int64_t>(c.take<std::int16_t>()); break;
    case GgufValueType::UInt32: v.scalar = static_cast<std::uint64_t>(c.take<std::uint32_t>()); break;
    case GgufValueType::Int32: v.scalar = static_cast<std::int64_t>(c.take<std::int32_t>()); break;
    case GgufValueType::Float32: v.scalar = static_cast<double>(c.take<float>()); break;
    case GgufValueType::Bool: {
        const auto b = c.take<std::uint8_t>();
        if (b > 1) throw std::runtime_error("GGUF boolean value is not 0/1");
        v.scalar = b == 1;
        break;
    }
    case GgufValueType::String: v.scalar = c.text(); break;
    case GgufValueType::UInt64: v.scalar = c.take<std::uint64_t>(); break;
    case GgufValueType::Int64: v.scalar = c.take<std::int64_t>(); break;
    case GgufValueType::Float64: v.scalar = c.take<double>(); break;
    case GgufValueType::Array: {
        if (depth >= kDepthLimit) throw std::runtime_error("GGUF array nesting is too deep");
        const auto et = c.take<std::uint32_t>();
        if (et > static_cast<std::uint32_t>(GgufValueType::Float64)) {
            throw std::runtime_error("GGUF array has invalid element type");
        }
        const auto n = c.take<std::uint64_t>();
        if (n > kArrayLimit) throw std::runtime_error("GGUF array length exceeds safety limit");
        v.array_element_type = static_cast<GgufValueType>(et);
        v.array.reserve(static_cast<std::size_t>(n));
        for (std::uint64_t i = 0; i < n; ++i) v.array.push_back(parse_value(c, v.array_element_type, depth + 1));
        break;
    }
    default: throw std::runtime_error("GGUF metadata has invalid value type");
    }
    return v;
}

// (block elements, block bytes) of the ggml types this runtime can size.
bool type_blocks(std::uint32_t type, std::uint64_t& elems, std::uint64_t& bytes) {
    switch (type) {
    case 0: elems = 1; bytes = 4; return true;    // F32
    case 1: elems = 1; bytes = 2; return true;    // F16
    case 8: elems = 32; bytes = 34; return true;  // Q8_0
    case 24: elems = 1; bytes = 1; return true;   // I8
    case 25: elems = 1; bytes = 2; return true;   // I16
    case 26: elems = 1; bytes = 4; return true;   // I32
    case 27: elems = 1; bytes = 8; return true;   // I64
    case 28: elems = 1; bytes = 8; return true;   // F64
    case 30: elems = 1; bytes = 2; return true;   // BF16
    default: return false;
    }
}

std::optional<std::uint64_t> payload_bytes(const GgufTensorInfo& t) {
    std::uint64_t be, bb;
    if (!type_blocks(t.type, be, bb)) return std::nullopt;
    std::uint64_t n = 1;
    for (const auto d : t.dimensions) {
        if (d == 0) return std::uint64_t{0};
        if (n > std::numeric_limits<std::uint64_t>::max() / d) throw std::runtime_error("GGUF tensor element count overflow");
        n *= d;
    }
    if (n % be) throw std::runtime_error("GGUF tensor element count is not divisible by quant block size");
    if (n / be > std::numeric_limits<std::uint64_t>::max() / bb) throw std::runtime_error("GGUF tensor byte size overflow");
    return n / be * bb;
}

float half_to_float(std::uint16_t h) {
    // exact fp16 -> fp32, subnormals normalised
    const std::uint32_t sign = (h & 0x8000u) << 16;
    const std::uint32_t exp = (h >> 10) & 0x1fu;
    std::uint32_t man = h & 0x3ffu, bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        std::uint32_t e = 113;
        while (!(man & 0x400u)) {
            man <<= 1;
            --e;
        }
        bits = sign | (e << 23) | ((man & 0x3ffu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

std::optional<std::string> GgufValue::as_string() const {
    if (auto p = std::get_if<std::string>(&scalar)) return *p;
    return std::nullopt;
}
std::optional<std::uint64_t> GgufValue::as_u64() const {
    if (auto p = std::get_if<std::uint64_t>(&scalar)) return *p;
    if (auto p = std::get_if<std::int64_t>(&scalar); p && *p >= 0) return static_cast<std::uint64_t>(*p);
    return std::nullopt;
}
std::optional<std::int64_t> GgufValue::as_i64() const {
    if (auto p = std::get_if<std::int64_t>(&scalar)) return *p;
    if (auto p = std::get_if<std::uint64_t>(&scalar);
        p && *p <= static_cast<std::uint64_t>(std::numeric_limits<std::int64_t>::max())) {
        return static_cast<std::int64_t>(*p);
    }
    return std::nullopt;
}
std::optional<double> GgufValue::as_f64() const {
    if (auto p = std::get_if<double>(&scalar)) return *p;
    return std::nullopt;
}
std::optional<bool> GgufValue::as_bool() const {
    if (auto p = std::get_if<bool>(&scalar)) return *p;
    return std::nullopt;
}

GgufFile::GgufFile(const std::filesystem::path& path) : path_(path) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw std::runtime_error("Failed to open GGUF file: " + path.string());
    struct stat st {};
    if (::fstat(fd, &st) != 0) {
        ::close(fd);
        throw std::runtime_error("Failed to determine GGUF file size");
    }
    file_size_ = static_cast<std::uint64_t>(st.st_size);
    if (file_size_ == 0) {
        ::close(fd);
        throw std::runtime_error("Unexpected end of GGUF file");
    }
    void* m = ::mmap(nullptr, file_size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw std::runtime_error("Failed to map GGUF file: " + path.string());
    map_ = static_cast<const std::uint8_t*>(m);
    try {
        Cursor c{map_, file_size_};
        if (c.take<std::uint32_t>() != kMagic) throw std::runtime_error("Invalid GGUF magic");
        version_ = c.take<std::uint32_t>();
        if (version_ < 2 || version_ > 3) throw std::runtime_error("Unsupported GGUF version: " + std::to_string(version_));
        const auto n_tensors = c.take<std::uint64_t>();
        const auto n_kv = c.take<std::uint64_t>();
        if (n_tensors > kCountLimit || n_kv > kCountLimit) throw std::runtime_error("GGUF header counts exceed safety limits");
        metadata_.reserve(static_cast<std::size_t>(n_kv));
        for (std::uint64_t i = 0; i < n_kv; ++i) {
            GgufMetadata kv;
            kv.key = c.text();
            const auto t = c.take<std::uint32_t>();
            if (t > static_cast<std::uint32_t>(GgufValueType::Float64)) {
                throw std::runtime_error("GGUF metadata has invalid value type");
            }
            kv.value = parse_value(c, static_cast<GgufValueType>(t), 0);
            metadata_.push_back(std::move(kv));
            metadata_index_.emplace(metadata_.back().key, metadata_.size() - 1);
        }
        if (const auto* a = find_metadata("general.alignment")) {
            const auto v = a->as_u64();
            if (!v || *v == 0 || *v > std::numeric_limits<std::uint32_t>::max()) {
                throw std::runtime_error("Invalid general.alignment metadata");
            }
            alignment_ = static_cast<std::uint32_t>(*v);
        }
        if (alignment_ & (alignment_ - 1u)) throw std::runtime_error("GGUF alignment must be a power of two");
        tensors_.reserve(static_cast<std::size_t>(n_tensors));
        for (std::uint64_t i = 0; i < n_tensors; ++i) {
            GgufTensorInfo t;
            t.name = c.text();
            const auto nd = c.take<std::uint32_t>();
            if (nd == 0 || nd > 8) throw std::runtime_error("GGUF tensor has invalid dimension count");
            for (std::uint32_t d = 0; d < nd; ++d) t.dimensions.push_back(c.take<std::uint64_t>());
            t.type = c.take<std::uint32_t>();
            t.offset = c.take<std::uint64_t>();
            tensors_.push_back(std::move(t));
            tensor_index_.emplace(tensors_.back().name, tensors_.size() - 1);
        }
        data_offset_ = (c.at + alignment_ - 1) / alignment_ * alignment_;
        validate();
    } catch (...) {
        ::munmap(const_cast<std::uint8_t*>(map_), file_size_);
        map_ = nullptr;
        throw;
    }
}

GgufFile::~GgufFile() {
    if (map_) ::munmap(const_cast<std::uint8_t*>(map_), file_size_);
}

const GgufValue* GgufFile::find_metadata(const std::string& key) const noexcept {
    const auto it = metadata_index_.find(key);
    return it == metadata_index_.end() ? nullptr : &metadata_[it->second].value;
}

const GgufTensorInfo* GgufFile::find_tensor(const std::string& name) const noexcept {
    const auto it = tensor_index_.find(name);
    return it == tensor_index_.end() ? nullptr : &tensors_[it->second];
}

std::optional<std::string> GgufFile::metadata_string(const std::string& key) const {
    const auto* v = find_metadata(key);
    return v ? v->as_string() : std::nullopt;
}

std::optional<std::uint64_t> GgufFile::metadata_u64(const std::string& key) const {
    const auto* v = find_metadata(key);
    return v ? v->as_u64() : std::nullopt;
}

std::optional<std::uint64_t> GgufFile::tensor_byte_size(const GgufTensorInfo& tensor) const {
    return payload_bytes(tensor);
}

const std::uint8_t* GgufFile::tensor_data(const GgufTensorInfo& tensor) const {
    const auto bytes = payload_bytes(tensor);
    if (!bytes) throw std::runtime_error("Unsupported GGML tensor type for payload read: " + tensor.name);
    const std::uint64_t at = data_offset_ + tensor.offset;
    if (at > file_size_ || *bytes > file_size_ - at) {
        throw std::runtime_error("Tensor payload is outside GGUF file: " + tensor.name);
    }
    return map_ + at;
}

std::vector<std::byte> GgufFile::read_tensor_bytes(const GgufTensorInfo& tensor) const {
    const auto* p = tensor_data(tensor);
    const auto n = *payload_bytes(tensor);
    std::vector<std::byte> out(static_cast<std::size_t>(n));
    if (n) std::memcpy(out.data(), p, static_cast<std::size_t>(n));
    return out;
}

std::vector<float> GgufFile::read_f32_tensor(const GgufTensorInfo& tensor) const {
    if (tensor.type != 0) throw std::runtime_error("Expected F32 tensor: " + tensor.name);
    const auto* p = tensor_data(tensor);
    const auto n = *payload_bytes(tensor) / 4;
    std::vector<float> out(static_cast<std::size_t>(n));
    if (n) std::memcpy(out.data(), p, static_cast<std::size_t>(n) * 4);
    return out;
}

std::vector<float> GgufFile::read_q8_0_row(const GgufTensorInfo& tensor, std::uint64_t row) const {
    if (tensor.type != 8) throw std::runtime_error("Expected Q8_0 tensor: " + tensor.name);
    if (tensor.dimensions.empty() || tensor.dimensions[0] == 0 || tensor.dimensions[0] % 32) {
        throw std::runtime_error("Q8_0 tensor has unsupported row layout: " + tensor.name);
    }
    const std::uint64_t width = tensor.dimensions[0];
    std::uint64_t rows = 1;
    for (std::size_t i = 1; i < tensor.dimensions.size(); ++i) {
        const auto d = tensor.dimensions[i];
        if (d && rows > std::numeric_limits<std::uint64_t>::max() / d) {
            throw std::runtime_error("Q8_0 tensor row count overflow: " + tensor.name);
        }
        rows *= d;
    }
    if (row >= rows) throw std::runtime_error("Q8_0 row index out of range: " + tensor.name);
    const std::uint64_t row_bytes = width / 32 * 34;
    const auto* p = tensor_data(tensor) + row * row_bytes;
    std::vector<float> out(static_cast<std::size_t>(width));
    for (std::uint64_t b = 0; b < width / 32; ++b) {
        const auto* blk = p + b * 34;
        const float d = half_to_float(static_cast<std::uint16_t>(blk[0] | (blk[1] << 8)));
        for (int k = 0; k < 32; ++k) out[b * 32 + k] = d * static_cast<float>(static_cast<std::int8_t>(blk[2 + k]));
    }
    return out;
}

void GgufFile::validate() const {
    if (data_offset_ > file_size_) throw std::runtime_error("GGUF tensor data offset lies beyond end of file");
    for (const auto& t : tensors_) {
        if (t.offset % alignment_) throw std::runtime_error("GGUF tensor offset is not aligned: " + t.name);
        if (t.offset > file_size_ - data_offset_) {
            throw std::runtime_error("GGUF tensor offset lies beyond end of file: " + t.name);
        }
        if (const auto b = payload_bytes(t); b && *b > file_size_ - data_offset_ - t.offset) {
            throw std::runtime_error("GGUF tensor payload lies beyond end of file: " + t.name);
        }
    }
}

const char* gguf_value_type_name(GgufValueType type) noexcept {
    static const char* const names[] = {"uint8", "int8",  "uint16", "int16",  "uint32", "int32", "float32",
                                        "bool",  "string", "array", "uint64", "int64",  "float64"};
    const auto i = static_cast<std::uint32_t>(type);
    return i < 13 ? names[i] : "unknown";
}

const char* ggml_type_name(std::uint32_t type) noexcept {
    switch (type) {
    case 0: return "F32";
    case 1: return "F16";
    case 2: return "Q4_0";
    case 3: return "Q4_1";
    case 6: return "Q5_0";
    case 7: return "Q5_1";
    case 8: return "Q8_0";
    case 9: return "Q8_1";
    case 10: return "Q2_K";
    case 11: return "Q3_K";
    case 12: return "Q4_K";
    case 13: return "Q5_K";
    case 14: return "Q6_K";
    case 15: return "Q8_K";
    case 24: return "I8";
    case 25: return "I16";
    case 26: return "I32";
    case 27: return "I64";
    case 28: return "F64";
    case 30: return "BF16";
    default: return "UNKNOWN";
    }
}

}  // namespace vortexrt
