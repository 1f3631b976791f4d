// gguf_reader.hpp -- GGUF v3 checkpoint reader for the samq host layer, written
// against the GGUF file format itself (no GGML gguf API).
//
// Mirrors sam::internal::GgufReader (src/io/gguf_reader.hpp in the SAM.cpp
// tree): the same public shape (tensors(), read(), u32(), string(), size()),
// the same limits (<= 4096 tensors, <= 256 metadata keys, 16 MiB of metadata)
// and the same rejections: not GGUF, not version 3, alignment other than 32,
// duplicate keys, non-positive or overflowing dimensions, rows not aligned to
// their quantization block, tensor ranges that overlap, leave gaps, have
// nonzero padding or run past the file, and bytes after the last tensor.  The
// reference checks canonical encoding by re-serialising through GGML; here the
// parser requires it directly: the metadata ends, zero-padded, exactly at the
// 32-byte-aligned data section and tensors follow in file order.
//
// Supported tensor types are the ones SAM checkpoints use: F32, F16, BF16,
// Q8_0, Q4_K, Q5_K, Q6_K (GGML type ids).  load_quantized_linear() turns a
// packed weight into a samq handle (QuantizedLinear).
#pragma once

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace sam::internal::samq_io {

struct GgufTensor {
    std::string name;
    std::vector<std::int64_t> dimensions;  // GGML order: dimensions[0] is the contiguous (row) width
    std::int32_t type = 0;
    std::uint64_t offset = 0;  // absolute file offset of the data
    std::uint64_t size_bytes = 0;
};

enum class GgufValueType : std::uint32_t {
    Uint8 = 0, Int8 = 1, Uint16 = 2, Int16 = 3, Uint32 = 4, Int32 = 5, Float32 = 6, Bool = 7,
    String = 8, Array = 9, Uint64 = 10, Int64 = 11, Float64 = 12,
};

struct GgufValue {
    GgufValueType type = GgufValueType::Uint8;
    GgufValueType element_type = GgufValueType::Uint8;  // arrays
    std::uint64_t count = 0;                            // arrays
    std::vector<std::uint8_t> raw;                      // scalar bytes, array element bytes (non-string)
    std::vector<std::string> strings;                   // string value, or string array elements
};

class GgufReader {
public:
    static constexpr std::size_t metadata_limit = 16 * 1024 * 1024;
    static constexpr std::uint64_t kAlignment = 32;

    explicit GgufReader(const std::string& path) : stream_(path, std::ios::binary) {
        if (!stream_) throw std::runtime_error("cannot open SAM checkpoint: " + path);
        stream_.seekg(0, std::ios::end);
        const auto length = stream_.tellg();
        if (length < 0) throw std::runtime_error("cannot determine SAM checkpoint size");
        size_ = static_cast<std::uint64_t>(length);
        if (size_ < 24) throw std::runtime_error("truncated GGUF checkpoint header");
        const std::uint64_t budget = std::min<std::uint64_t>(size_, metadata_limit);
        meta_.resize(static_cast<std::size_t>(budget));
        read(0, reinterpret_cast<char*>(meta_.data()), meta_.size());
        if (std::memcmp(meta_.data(), "GGUF", 4) != 0)
            throw std::runtime_error("unsupported checkpoint: expected GGUF");
        cursor_ = 4;
        if (u32_at() != 3) throw std::runtime_error("SAM checkpoints require little-endian GGUF v3");
        const std::uint64_t tensor_count = u64_at(), key_count = u64_at();
        if (tensor_count == 0 || tensor_count > 4096 || key_count > 256)
            throw std::runtime_error("GGUF tensor or metadata key count exceeds checkpoint limits");
        for (std::uint64_t i = 0; i < key_count; ++i) {
            std::string key = string_at(65535);
            if (key.empty()) throw std::runtime_error("empty GGUF metadata key");
            GgufValue value = value_at(static_cast<GgufValueType>(u32_at()), 0);
            if (!values_.emplace(std::move(key), std::move(value)).second)
                throw std::runtime_error("ambiguous GGUF metadata key");
        }
        const auto align = values_.find("general.alignment");
        if (align != values_.end() &&
            (align->second.type != GgufValueType::Uint32 || scalar<std::uint32_t>(align->second) != kAlignment))
            throw std::runtime_error("SAM GGUF checkpoints require 32-byte alignment");
        std::vector<std::uint64_t> relative(static_cast<std::size_t>(tensor_count));
        std::map<std::string, bool> names;
        for (std::uint64_t i = 0; i < tensor_count; ++i) {
            GgufTensor tensor;
            tensor.name = string_at(GGUF_NAME_LIMIT);
            if (tensor.name.empty()) throw std::runtime_error("empty GGUF tensor name");
            if (!names.emplace(tensor.name, true).second)
                throw std::runtime_error("duplicate GGUF tensor name: " + tensor.name);
            const std::uint32_t dims = u32_at();
            if (dims == 0 || dims > 4) throw std::runtime_error("invalid GGUF tensor rank: " + tensor.name);
            std::uint64_t elements = 1;
            for (std::uint32_t d = 0; d < dims; ++d) {
                const std::uint64_t extent = u64_at();
                if (extent == 0 || extent > static_cast<std::uint64_t>(INT64_MAX) ||
                    elements > static_cast<std::uint64_t>(INT64_MAX) / extent)
                    throw std::runtime_error("invalid or overflowing GGUF tensor dimensions: " + tensor.name);
                elements *= extent;
                tensor.dimensions.push_back(static_cast<std::int64_t>(extent));
            }
            while (tensor.dimensions.size() > 1 && tensor.dimensions.back() == 1) tensor.dimensions.pop_back();
            tensor.type = static_cast<std::int32_t>(u32_at());
            std::uint64_t block = 0, bytes = 0;
            if (!type_geometry(tensor.type, block, bytes))
                throw std::runtime_error("unsupported GGUF tensor type " + std::to_string(tensor.type) + ": " +
                                         tensor.name);
            if (static_cast<std::uint64_t>(tensor.dimensions[0]) % block != 0)
                throw std::runtime_error("GGUF tensor row width is not quantization-block aligned: " + tensor.name);
            if (elements / block > std::numeric_limits<std::uint64_t>::max() / bytes)
                throw std::runtime_error("invalid or overflowing GGUF tensor byte count: " + tensor.name);
            tensor.size_bytes = elements / block * bytes;
            relative[static_cast<std::size_t>(i)] = u64_at();
            tensors_.push_back(std::move(tensor));
        }
        // Canonical layout: zero padding from the end of the tensor infos to the
        // aligned data section, tensors in order, each zero-padded to 32 bytes.
        data_offset_ = (cursor_ + kAlignment - 1) / kAlignment * kAlignment;
        if (data_offset_ > size_) throw std::runtime_error("truncated GGUF data section");
        check_zero(cursor_, data_offset_ - cursor_, "nonzero GGUF metadata padding");
        const std::uint64_t available = size_ - data_offset_;
        std::uint64_t expected = 0;
        for (std::size_t i = 0; i < tensors_.size(); ++i) {
            GgufTensor& tensor = tensors_[i];
            const std::uint64_t padding = (kAlignment - tensor.size_bytes % kAlignment) % kAlignment;
            if (relative[i] != expected || relative[i] > available || tensor.size_bytes > available - relative[i] ||
                padding > available - relative[i] - tensor.size_bytes)
                throw std::runtime_error("overlapping, overflowing or truncated GGUF tensor range: " + tensor.name);
            tensor.offset = data_offset_ + relative[i];
            check_zero(tensor.offset + tensor.size_bytes, padding, "nonzero GGUF tensor padding: " + tensor.name);
            expected = relative[i] + tensor.size_bytes + padding;
        }
        if (expected != available) throw std::runtime_error("unexpected data after GGUF tensor blob");
    }

    std::uint64_t size() const { return size_; }
    std::uint64_t data_offset() const { return data_offset_; }
    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    const std::map<std::string, GgufValue>& metadata() const { return values_; }

    const GgufTensor& tensor(const std::string& name) const {
        for (const GgufTensor& t : tensors_)
            if (t.name == name) return t;
        throw std::runtime_error("missing GGUF tensor: " + name);
    }

    void read(std::uint64_t offset, char* output, std::size_t bytes) {
        if (offset > size_ || bytes > size_ - offset ||
            bytes > static_cast<std::size_t>(std::numeric_limits<std::streamsize>::max()))
            throw std::runtime_error("invalid or truncated GGUF file range");
        stream_.clear();
        stream_.seekg(static_cast<std::streamoff>(offset));
        stream_.read(output, static_cast<std::streamsize>(bytes));
        if (!stream_) throw std::runtime_error("GGUF checkpoint changed or became unreadable");
    }

    std::vector<std::uint8_t> tensor_bytes(const GgufTensor& t) {
        std::vector<std::uint8_t> out(static_cast<std::size_t>(t.size_bytes));
        read(t.offset, reinterpret_cast<char*>(out.data()), out.size());
        return out;
    }

    const GgufValue& key(const std::string& name, GgufValueType type) const {
        const auto it = values_.find(name);
        if (it == values_.end() || it->second.type != type)
            throw std::runtime_error("missing or incompatible GGUF metadata: " + name);
        return it->second;
    }
    std::uint32_t u32(const std::string& name) const { return scalar<std::uint32_t>(key(name, GgufValueType::Uint32)); }
    std::string string(const std::string& name, std::size_t maximum = 2048) const {
        const std::string& s = key(name, GgufValueType::String).strings.at(0);
        if (s.empty() || s.size() > maximum) throw std::runtime_error("invalid or oversized GGUF string: " + name);
        return s;
    }
    const GgufValue& array(const std::string& name, GgufValueType type, std::size_t count) const {
        const GgufValue& v = key(name, GgufValueType::Array);
        if (v.element_type != type || v.count != count) throw std::runtime_error("incompatible GGUF array: " + name);
        return v;
    }

    // Element width / block of the GGML types SAM checkpoints hold.
    static bool type_geometry(std::int32_t type, std::uint64_t& block, std::uint64_t& bytes) {
        switch (type) {
            case 0: block = 1; bytes = 4; return true;      // F32
            case 1: block = 1; bytes = 2; return true;      // F16
            case 30: block = 1; bytes = 2; return true;     // BF16
            case 8: block = 32; bytes = 34; return true;    // Q8_0
            case 12: block = 256; bytes = 144; return true; // Q4_K
            case 13: block = 256; bytes = 176; return true; // Q5_K
            case 14: block = 256; bytes = 210; return true; // Q6_K
            default: return false;
        }
    }

private:
    static constexpr std::size_t GGUF_NAME_LIMIT = 64;  // GGML_MAX_NAME

    void need(std::uint64_t bytes) const {
        if (cursor_ > meta_.size() || bytes > meta_.size() - cursor_)
            throw std::runtime_error("invalid, truncated or oversized GGUF metadata");
    }
    std::uint64_t integer_at(std::size_t bytes) {
        need(bytes);
        std::uint64_t v = 0;
        for (std::size_t i = 0; i < bytes; ++i) v |= static_cast<std::uint64_t>(meta_[cursor_ + i]) << (8 * i);
        cursor_ += bytes;
        return v;
    }
    std::uint32_t u32_at() { return static_cast<std::uint32_t>(integer_at(4)); }
    std::uint64_t u64_at() { return integer_at(8); }
    std::string string_at(std::size_t maximum) {
        const std::uint64_t n = u64_at();
        if (n > maximum) throw std::runtime_error("invalid or oversized GGUF string");
        need(n);
        std::string s(reinterpret_cast<const char*>(meta_.data() + cursor_), static_cast<std::size_t>(n));
        cursor_ += n;
        return s;
    }
    static std::size_t scalar_width(GgufValueType t) {
        switch (t) {
            case GgufValueType::Uint8: case GgufValueType::Int8: case GgufValueType::Bool: return 1;
            case GgufValueType::Uint16: case GgufValueType::Int16: return 2;
            case GgufValueType::Uint32: case GgufValueType::Int32: case GgufValueType::Float32: return 4;
            case GgufValueType::Uint64: case GgufValueType::Int64: case GgufValueType::Float64: return 8;
            default: return 0;
        }
    }
    GgufValue value_at(GgufValueType type, int depth) {
        GgufValue v;
        v.type = type;
        if (type == GgufValueType::String) {
            v.strings.push_back(string_at(metadata_limit));
        } else if (type == GgufValueType::Array) {
            if (depth > 0) throw std::runtime_error("nested GGUF arrays are not supported");
            v.element_type = static_cast<GgufValueType>(u32_at());
            v.count = u64_at();
            if (v.element_type == GgufValueType::String) {
                if (v.count > metadata_limit / 8) throw std::runtime_error("oversized GGUF array");
                for (std::uint64_t i = 0; i < v.count; ++i) v.strings.push_back(string_at(metadata_limit));
            } else {
                const std::size_t w = scalar_width(v.element_type);
                if (w == 0) throw std::runtime_error("invalid GGUF array element type");
                if (v.count > metadata_limit / w) throw std::runtime_error("oversized GGUF array");
                need(v.count * w);
                v.raw.assign(meta_.begin() + static_cast<std::ptrdiff_t>(cursor_),
                             meta_.begin() + static_cast<std::ptrdiff_t>(cursor_ + v.count * w));
                cursor_ += v.count * w;
            }
        } else {
            const std::size_t w = scalar_width(type);
            if (w == 0) throw std::runtime_error("invalid GGUF metadata value type");
            need(w);
            v.raw.assign(meta_.begin() + static_cast<std::ptrdiff_t>(cursor_),
                         meta_.begin() + static_cast<std::ptrdiff_t>(cursor_ + w));
            cursor_ += w;
        }
        return v;
    }
    template <class T>
    static T scalar(const GgufValue& v) {
        T out{};
        if (v.raw.size() != sizeof(T)) throw std::runtime_error("GGUF scalar width mismatch");
        std::memcpy(&out, v.raw.data(), sizeof(T));
        return out;
    }
    void check_zero(std::uint64_t offset, std::uint64_t bytes, const std::string& what) {
        if (bytes == 0) return;
        std::array<char, 64> buf{};
        while (bytes > 0) {
            const std::size_t n = static_cast<std::size_t>(std::min<std::uint64_t>(bytes, buf.size()));
            read(offset, buf.data(), n);
            for (std::size_t i = 0; i < n; ++i)
                if (buf[i] != 0) throw std::runtime_error(what);
            offset += n;
            bytes -= n;
        }
    }

    std::ifstream stream_;
    std::vector<std::uint8_t> meta_;
    std::size_t cursor_ = 0;
    std::uint64_t size_ = 0, data_offset_ = 0;
    std::map<std::string, GgufValue> values_;
    std::vector<GgufTensor> tensors_;
};

}  // namespace sam::internal::samq_io
