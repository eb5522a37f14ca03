// GGUF v3 reader (see gguf.h for the layout).
#include "gguf.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>

namespace pixal3d {
namespace b200 {

namespace {

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};
enum : uint32_t { kTypeF32 = 0, kTypeF16 = 1, kTypeBF16 = 30 };

bool fail(std::string *error, const std::string &msg) {
    if (error) *error = msg;
    return false;
}

struct FileCloser {
    void operator()(std::FILE *f) const {
        if (f) std::fclose(f);
    }
};

class Cursor {
public:
    explicit Cursor(std::FILE *f) : f_(f) {}
    template <typename T>
    bool pod(T &v) {
        return std::fread(&v, sizeof(T), 1, f_) == 1;
    }
    bool str(std::string &s) {
        uint64_t n = 0;
        if (!pod(n) || n > (uint64_t(1) << 30)) return false;
        s.resize(static_cast<std::size_t>(n));
        return n == 0 || std::fread(&s[0], 1, static_cast<std::size_t>(n), f_) == n;
    }
    bool skip(uint64_t bytes) { return std::fseek(f_, static_cast<long>(bytes), SEEK_CUR) == 0; }
    uint64_t tell() const { return static_cast<uint64_t>(std::ftell(f_)); }

private:
    std::FILE *f_;
};

uint64_t scalar_size(uint32_t type) {
    switch (type) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// IEEE 754 binary16 -> binary32 (exact).
float half_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);  // inf / nan
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;  // signed zero
        } else {          // subnormal: normalise
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while ((man & 0x400u) == 0);
            bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float bf16_to_float(uint16_t b) {
    const uint32_t bits = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

uint64_t GgufTensor::elements() const {
    uint64_t n = 1;
    for (uint64_t d : dims) n *= d;
    return n;
}

uint64_t GgufTensor::bytes() const {
    switch (type) {
        case kTypeF32: return 4 * elements();
        case kTypeF16:
        case kTypeBF16: return 2 * elements();
        default: return 0;
    }
}

bool GgufFile::open(const std::string &path, std::string *error) {
    path_ = path;
    kv_.clear();
    tensors_.clear();
    index_.clear();
    std::unique_ptr<std::FILE, FileCloser> f(std::fopen(path.c_str(), "rb"));
    if (!f) return fail(error, "cannot open GGUF pack: " + path);
    if (std::fseek(f.get(), 0, SEEK_END) != 0) return fail(error, "cannot size GGUF pack: " + path);
    file_size_ = static_cast<uint64_t>(std::ftell(f.get()));
    std::rewind(f.get());
    Cursor c(f.get());
    char magic[4];
    if (std::fread(magic, 1, 4, f.get()) != 4 || std::memcmp(magic, "GGUF", 4) != 0)
        return fail(error, "not a GGUF file: " + path);
    uint64_t n_tensors = 0, n_kv = 0;
    if (!c.pod(version_) || !c.pod(n_tensors) || !c.pod(n_kv)) return fail(error, "truncated GGUF header: " + path);
    if (version_ != 3) return fail(error, "unsupported GGUF version: " + std::to_string(version_));
    if (n_tensors > (uint64_t(1) << 24) || n_kv > (uint64_t(1) << 24)) return fail(error, "corrupt GGUF header");
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        Value v;
        if (!c.str(key) || !c.pod(v.type)) return fail(error, "truncated GGUF metadata");
        switch (v.type) {
            case kU8: { uint8_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.u = x; v.i = x; break; }
            case kI8: { int8_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.i = x; v.u = static_cast<uint64_t>(x); break; }
            case kU16: { uint16_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.u = x; v.i = x; break; }
            case kI16: { int16_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.i = x; v.u = static_cast<uint64_t>(x); break; }
            case kU32: { uint32_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.u = x; v.i = x; break; }
            case kI32: { int32_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.i = x; v.u = static_cast<uint64_t>(x); break; }
            case kF32: { float x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.f = x; break; }
            case kBool: { uint8_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.u = x ? 1 : 0; break; }
            case kString: if (!c.str(v.s)) return fail(error, "truncated GGUF metadata"); break;
            case kU64: { uint64_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.u = x; v.i = static_cast<int64_t>(x); break; }
            case kI64: { int64_t x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.i = x; v.u = static_cast<uint64_t>(x); break; }
            case kF64: { double x; if (!c.pod(x)) return fail(error, "truncated GGUF metadata"); v.f = x; break; }
            case kArray: {
                uint32_t et = 0;
                uint64_t n = 0;
                if (!c.pod(et) || !c.pod(n)) return fail(error, "truncated GGUF metadata");
                if (et == kString) {
                    for (uint64_t j = 0; j < n; ++j) {
                        std::string s;
                        if (!c.str(s)) return fail(error, "truncated GGUF metadata");
                    }
                } else {
                    const uint64_t sz = scalar_size(et);
                    if (sz == 0 || !c.skip(sz * n)) return fail(error, "bad GGUF metadata array: " + key);
                }
                break;
            }
            default: return fail(error, "unknown GGUF metadata type for " + key);
        }
        kv_[key] = v;
    }
    auto al = kv_.find("general.alignment");
    if (al != kv_.end() && (al->second.type == kU32 || al->second.type == kU64 || al->second.type == kI32)) {
        alignment_ = al->second.u;
        if (alignment_ == 0 || (alignment_ & (alignment_ - 1)) != 0) return fail(error, "bad GGUF alignment");
    }
    tensors_.reserve(static_cast<std::size_t>(n_tensors));
    for (uint64_t i = 0; i < n_tensors; ++i) {
        GgufTensor t;
        uint32_t nd = 0;
        if (!c.str(t.name) || !c.pod(nd) || nd > 8) return fail(error, "truncated GGUF tensor info");
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; ++d)
            if (!c.pod(t.dims[d])) return fail(error, "truncated GGUF tensor info");
        if (!c.pod(t.type) || !c.pod(t.offset)) return fail(error, "truncated GGUF tensor info");
        if (t.name.empty() || index_.count(t.name)) return fail(error, "GGUF tensor names must be non-empty and unique");
        index_[t.name] = tensors_.size();
        tensors_.push_back(std::move(t));
    }
    const uint64_t pos = c.tell();
    data_offset_ = (pos + alignment_ - 1) / alignment_ * alignment_;
    for (const GgufTensor &t : tensors_) {
        if (t.offset % alignment_ != 0) return fail(error, "GGUF tensor offset is not aligned: " + t.name);
        const uint64_t b = t.bytes();
        if (b != 0 && (data_offset_ + t.offset > file_size_ || b > file_size_ - data_offset_ - t.offset))
            return fail(error, "GGUF tensor payload is outside the file: " + t.name);
    }
    return true;
}

const GgufTensor *GgufFile::find(const std::string &name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

bool GgufFile::get_string(const std::string &key, std::string &out, bool required, std::string *error) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return required ? fail(error, "missing GGUF metadata: " + key) : true;
    if (it->second.type != kString) return fail(error, "GGUF metadata is not a string: " + key);
    out = it->second.s;
    return true;
}

bool GgufFile::get_u32(const std::string &key, uint32_t &out, bool required, std::string *error) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return required ? fail(error, "missing GGUF metadata: " + key) : true;
    const Value &v = it->second;
    switch (v.type) {
        case kU8: case kU16: case kU32: case kU64:
            if (v.u > 0xffffffffull) return fail(error, "GGUF metadata out of range: " + key);
            out = static_cast<uint32_t>(v.u);
            return true;
        case kI8: case kI16: case kI32: case kI64:
            if (v.i < 0 || v.i > 0xffffffffll) return fail(error, "GGUF metadata out of range: " + key);
            out = static_cast<uint32_t>(v.i);
            return true;
        default: return fail(error, "GGUF metadata is not an integer: " + key);
    }
}

bool GgufFile::get_f32(const std::string &key, float &out, bool required, std::string *error) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return required ? fail(error, "missing GGUF metadata: " + key) : true;
    const Value &v = it->second;
    if (v.type == kF32 || v.type == kF64) out = static_cast<float>(v.f);
    else if (v.type == kU8 || v.type == kU16 || v.type == kU32 || v.type == kU64) out = static_cast<float>(v.u);
    else if (v.type == kI8 || v.type == kI16 || v.type == kI32 || v.type == kI64) out = static_cast<float>(v.i);
    else return fail(error, "GGUF metadata is not a number: " + key);
    return true;
}

bool GgufFile::get_bool(const std::string &key, bool &out, bool required, std::string *error) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return required ? fail(error, "missing GGUF metadata: " + key) : true;
    const Value &v = it->second;
    if (v.type == kBool || v.type == kU8 || v.type == kU32 || v.type == kI32) out = v.u != 0;
    else return fail(error, "GGUF metadata is not a bool: " + key);
    return true;
}

bool GgufFile::read_f32(const GgufTensor &t, std::vector<float> &out, std::string *error) const {
    const uint64_t bytes = t.bytes();
    if (bytes == 0 && t.elements() != 0) return fail(error, "unsupported GGUF tensor type for " + t.name);
    std::unique_ptr<std::FILE, FileCloser> f(std::fopen(path_.c_str(), "rb"));
    if (!f) return fail(error, "cannot open GGUF pack: " + path_);
    if (std::fseek(f.get(), static_cast<long>(data_offset_ + t.offset), SEEK_SET) != 0)
        return fail(error, "cannot seek GGUF tensor: " + t.name);
    const uint64_t n = t.elements();
    out.resize(static_cast<std::size_t>(n));
    if (t.type == kTypeF32) {
        if (std::fread(out.data(), 4, static_cast<std::size_t>(n), f.get()) != n)
            return fail(error, "truncated GGUF tensor: " + t.name);
    } else {
        std::vector<uint16_t> raw(static_cast<std::size_t>(n));
        if (std::fread(raw.data(), 2, static_cast<std::size_t>(n), f.get()) != n)
            return fail(error, "truncated GGUF tensor: " + t.name);
        for (uint64_t i = 0; i < n; ++i) out[i] = t.type == kTypeF16 ? half_to_float(raw[i]) : bf16_to_float(raw[i]);
    }
    for (float v : out)
        if (!std::isfinite(v)) return fail(error, "SLat flow tensor contains a non-finite value: " + t.name);
    return true;
}

}  // namespace b200
}  // namespace pixal3d
