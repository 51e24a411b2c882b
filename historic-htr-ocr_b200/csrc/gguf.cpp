// gguf.cpp — GGUF v2/v3 parsing with the reference reader's checks (app/crates/ocr-gguf/src/lib.rs:300-401):
// magic, version 2–3, value types 0–12 (no nested arrays), duplicate keys/tensors refused, general.alignment a power
// of two (default 32), 1–4 dims, only F32/F16/BF16/Q8_0, offsets aligned, rows whole blocks, every tensor inside the
// file. The header is parsed from a prefix that doubles while it is too short (1 MB first, lib.rs:305-317).
#include "gguf.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <set>
#include <stdexcept>

namespace ocr {

namespace {

struct FileSource : Source {
    int fd = -1;
    uint64_t len = 0;
    ~FileSource() override {
        if (fd >= 0) close(fd);
    }
    uint64_t size() const override { return len; }
    bool read_at(uint64_t off, void* buf, size_t n, std::string& msg) const override {
        size_t done = 0;
        while (done < n) {
            const ssize_t r = pread(fd, (char*)buf + done, n - done, (off_t)(off + done));
            if (r <= 0) {
                msg = "read " + std::to_string(n) + " bytes at " + std::to_string(off) + " failed";
                return false;
            }
            done += (size_t)r;
        }
        return true;
    }
};

struct MemSource : Source {
    const uint8_t* p;
    size_t n;
    MemSource(const void* b, size_t len) : p((const uint8_t*)b), n(len) {}
    uint64_t size() const override { return n; }
    bool read_at(uint64_t off, void* buf, size_t len, std::string& msg) const override {
        if (off + len > n) {
            msg = "read past the end (" + std::to_string(off + len) + " > " + std::to_string(n) + ")";
            return false;
        }
        memcpy(buf, p + off, len);
        return true;
    }
};

// the header did not fit in the prefix read so far
struct NeedMore {};

struct Cursor {
    const uint8_t* b;
    size_t n, pos = 0;
    const uint8_t* take(size_t k) {
        if (k > n - pos) throw NeedMore{};
        const uint8_t* r = b + pos;
        pos += k;
        return r;
    }
    template <class T>
    T get() {
        T v;
        memcpy(&v, take(sizeof(T)), sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t k = get<uint64_t>();
        if (k > (uint64_t)1 << 40) throw std::runtime_error("GGUF length overflow");
        const uint8_t* s = take((size_t)k);
        return std::string((const char*)s, (size_t)k);
    }
    GValue value(uint32_t ty, int depth) {
        GValue v;
        v.type = (int)ty;
        switch (ty) {
        case 0: v.u = get<uint8_t>(); break;
        case 1: v.i = get<int8_t>(); break;
        case 2: v.u = get<uint16_t>(); break;
        case 3: v.i = get<int16_t>(); break;
        case 4: v.u = get<uint32_t>(); break;
        case 5: v.i = get<int32_t>(); break;
        case 6: v.f = get<float>(); break;
        case 7: {
            const uint8_t x = get<uint8_t>();
            if (x > 1) throw std::runtime_error("GGUF bool value " + std::to_string(x));
            v.u = x;
            break;
        }
        case 8: v.s = str(); break;
        case 9: {
            if (depth > 0) throw std::runtime_error("GGUF nested arrays are not part of the format");
            const uint32_t ety = get<uint32_t>();
            const uint64_t k = get<uint64_t>();
            v.arr.reserve((size_t)(k < (1u << 20) ? k : (1u << 20)));
            for (uint64_t i = 0; i < k; i++) v.arr.push_back(value(ety, depth + 1));
            break;
        }
        case 10: v.u = get<uint64_t>(); break;
        case 11: v.i = get<int64_t>(); break;
        case 12: v.f = get<double>(); break;
        default: throw std::runtime_error("GGUF value type " + std::to_string(ty) + " unknown");
        }
        return v;
    }
};

bool gtype(uint32_t t, GType& out) {
    switch (t) {
    case 0: out = GType::F32; return true;
    case 1: out = GType::F16; return true;
    case 8: out = GType::Q8_0; return true;
    case 30: out = GType::BF16; return true;
    default: return false;
    }
}

}  // namespace

std::unique_ptr<Source> file_source(const std::string& path, std::string& msg) {
    auto f = std::make_unique<FileSource>();
    f->fd = open(path.c_str(), O_RDONLY);
    if (f->fd < 0) {
        msg = "cannot open " + path;
        return nullptr;
    }
    struct stat st;
    if (fstat(f->fd, &st) != 0) {
        msg = "cannot stat " + path;
        return nullptr;
    }
    f->len = (uint64_t)st.st_size;
    return f;
}

std::unique_ptr<Source> memory_source(const void* bytes, size_t n) { return std::make_unique<MemSource>(bytes, n); }

uint64_t GTensor::n_elements() const {
    uint64_t n = 1;
    for (uint64_t d : shape) n *= d;
    return n;
}

uint64_t GTensor::n_bytes() const {
    switch (type) {
    case GType::F32: return n_elements() * 4;
    case GType::F16:
    case GType::BF16: return n_elements() * 2;
    case GType::Q8_0: return n_elements() / 32 * 34;
    }
    return 0;
}

static bool parse_header(Gguf& g, const uint8_t* b, size_t n, std::string& msg) {
    Cursor c{b, n};
    if (memcmp(c.take(4), "GGUF", 4) != 0) throw std::runtime_error("no GGUF magic");
    g.version = c.get<uint32_t>();
    if (g.version < 2 || g.version > 3)
        throw std::runtime_error("GGUF version " + std::to_string(g.version) + " (2 or 3 expected)");
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    g.meta.clear();
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = c.str();
        const uint32_t ty = c.get<uint32_t>();
        GValue v;
        try {
            v = c.value(ty, 0);
        } catch (const std::runtime_error& e) {
            throw std::runtime_error("metadata key " + key + ": " + e.what());
        }
        if (!g.meta.emplace(key, std::move(v)).second) throw std::runtime_error("duplicate metadata key " + key);
    }
    g.alignment = 32;
    auto it = g.meta.find("general.alignment");
    if (it != g.meta.end()) {
        if (it->second.type != 4) throw std::runtime_error("general.alignment has the wrong type");
        g.alignment = it->second.u;
    }
    if (g.alignment == 0 || (g.alignment & (g.alignment - 1)) != 0)
        throw std::runtime_error("general.alignment " + std::to_string(g.alignment) + " is not a power of two");
    g.tensors.clear();
    std::set<std::string> names;
    for (uint64_t i = 0; i < n_tensors; i++) {
        GTensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd == 0 || nd > 4) throw std::runtime_error("tensor " + t.name + ": " + std::to_string(nd) + " dimensions");
        for (uint32_t k = 0; k < nd; k++) t.shape.push_back(c.get<uint64_t>());
        const uint32_t raw = c.get<uint32_t>();
        if (!gtype(raw, t.type))
            throw std::runtime_error("tensor " + t.name + ": ggml type " + std::to_string(raw) +
                                     " is not supported (F32, F16, BF16, Q8_0 only)");
        t.offset = c.get<uint64_t>();
        if (t.offset % g.alignment != 0)
            throw std::runtime_error("tensor " + t.name + ": offset " + std::to_string(t.offset) + " not aligned to " +
                                     std::to_string(g.alignment));
        const uint64_t blk = t.type == GType::Q8_0 ? 32 : 1;
        if (t.shape[0] % blk != 0)
            throw std::runtime_error("tensor " + t.name + ": row of " + std::to_string(t.shape[0]) +
                                     " elements is not a whole number of blocks");
        if (!names.insert(t.name).second) throw std::runtime_error("duplicate tensor " + t.name);
        g.tensors.push_back(std::move(t));
    }
    g.data_offset = (c.pos + g.alignment - 1) / g.alignment * g.alignment;
    for (auto& t : g.tensors) t.file_offset = g.data_offset + t.offset;
    (void)msg;
    return true;
}

bool Gguf::parse(std::unique_ptr<Source> s, std::string& msg) {
    src = std::move(s);
    const uint64_t file_len = src->size();
    uint64_t want = 1u << 20;
    for (;;) {
        const size_t n = (size_t)(want < file_len ? want : file_len);
        std::vector<uint8_t> prefix(n);
        if (n && !src->read_at(0, prefix.data(), n, msg)) return false;
        try {
            parse_header(*this, prefix.data(), n, msg);
            break;
        } catch (const NeedMore&) {
            if (n < file_len) {
                want *= 2;
                continue;
            }
            msg = "GGUF truncated: the header runs past the end of the file";
            return false;
        } catch (const std::runtime_error& e) {
            msg = e.what();
            return false;
        }
    }
    for (const auto& t : tensors) {
        const uint64_t end = t.file_offset + t.n_bytes();
        if (end > file_len) {
            msg = "tensor " + t.name + " ends at byte " + std::to_string(end) + ", the file has " + std::to_string(file_len);
            return false;
        }
    }
    by_name.clear();
    for (size_t i = 0; i < tensors.size(); i++) by_name[tensors[i].name] = i;
    return true;
}

const GTensor* Gguf::info(const std::string& name) const {
    auto it = by_name.find(name);
    return it == by_name.end() ? nullptr : &tensors[it->second];
}

bool Gguf::get_u32(const std::string& key, uint32_t& out, std::string& msg) const {
    auto it = meta.find(key);
    if (it == meta.end()) {
        msg = "GGUF has no metadata key " + key;
        return false;
    }
    if (it->second.type == 4) out = (uint32_t)it->second.u;
    else if (it->second.type == 5 && it->second.i >= 0) out = (uint32_t)it->second.i;
    else {
        msg = key + " is not u32";
        return false;
    }
    return true;
}

bool Gguf::get_f32(const std::string& key, float& out, std::string& msg) const {
    auto it = meta.find(key);
    if (it == meta.end()) {
        msg = "GGUF has no metadata key " + key;
        return false;
    }
    if (it->second.type != 6) {
        msg = key + " is not f32";
        return false;
    }
    out = (float)it->second.f;
    return true;
}

bool Gguf::get_str(const std::string& key, std::string& out, std::string& msg) const {
    auto it = meta.find(key);
    if (it == meta.end()) {
        msg = "GGUF has no metadata key " + key;
        return false;
    }
    if (it->second.type != 8) {
        msg = key + " is not a string";
        return false;
    }
    out = it->second.s;
    return true;
}

}  // namespace ocr
