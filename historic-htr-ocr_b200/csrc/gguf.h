// gguf.h — GGUF v2/v3 header reader (the rules of app/crates/ocr-gguf/src/lib.rs, restated in C++).
// A tensor is (file offset, byte length, ggml type, shape); its bytes are read on demand from a Source straight into
// the device upload's staging buffer — the model is never held whole in host memory (lib.rs:5-10).
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace ocr {

// TensorSource (lib.rs:27-30): random-access reads
struct Source {
    virtual ~Source() = default;
    virtual uint64_t size() const = 0;
    // fill buf with bytes [off, off + n); false + msg on failure
    virtual bool read_at(uint64_t off, void* buf, size_t n, std::string& msg) const = 0;
};

std::unique_ptr<Source> file_source(const std::string& path, std::string& msg);
std::unique_ptr<Source> memory_source(const void* bytes, size_t n);

// ggml types read here (lib.rs:100-136): F32 0, F16 1, Q8_0 8, BF16 30
enum class GType { F32, F16, BF16, Q8_0 };

struct GValue {
    int type = -1;  // GGUF value type 0..12
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<GValue> arr;
};

struct GTensor {
    std::string name;
    std::vector<uint64_t> shape;  // ggml order: shape[0] is the contiguous dimension
    GType type = GType::F32;
    uint64_t offset = 0;       // within the data section
    uint64_t file_offset = 0;  // absolute
    uint64_t n_elements() const;
    uint64_t n_bytes() const;
};

struct Gguf {
    uint32_t version = 0;
    std::map<std::string, GValue> meta;
    std::vector<GTensor> tensors;
    std::map<std::string, size_t> by_name;
    uint64_t alignment = 32, data_offset = 0;
    std::unique_ptr<Source> src;

    // Gguf::from_source (lib.rs:300-322): the header from a growing prefix; every tensor inside the file
    bool parse(std::unique_ptr<Source> s, std::string& msg);
    const GTensor* info(const std::string& name) const;
    bool has(const std::string& name) const { return by_name.count(name) != 0; }
    bool has_key(const std::string& key) const { return meta.count(key) != 0; }
    // typed accessors (lib.rs:419-447): u32 accepts U32 and I32 >= 0
    bool get_u32(const std::string& key, uint32_t& out, std::string& msg) const;
    bool get_f32(const std::string& key, float& out, std::string& msg) const;
    bool get_str(const std::string& key, std::string& out, std::string& msg) const;
};

}  // namespace ocr
