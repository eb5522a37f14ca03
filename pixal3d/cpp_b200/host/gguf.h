// Minimal reader of GGUF v3 weight packs (the format of the reference's
// Pixal3D packs, read there through ggml's gguf library: src/pack.cpp:127-260).
// Written from the published GGUF layout:
//   header   magic "GGUF", u32 version, u64 tensor count, u64 metadata count
//   metadata key (u64 length + bytes), u32 value type, value
//            (u8 i8 u16 i16 u32 i32 f32 bool string array u64 i64 f64;
//             array = u32 element type, u64 count, elements)
//   tensors  name, u32 n_dims, u64 dims[n_dims] (dims[0] innermost),
//            u32 ggml type, u64 offset from the data section
//   data     starts at the next multiple of general.alignment (default 32)
// Only F32, F16 and BF16 tensors are converted (the types the SLat flow packs
// use, src/slat_flow.cpp:360-395).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace pixal3d {
namespace b200 {

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;  // dims[0] innermost
    uint32_t type = 0;           // ggml type id
    uint64_t offset = 0;         // from the data section
    uint64_t elements() const;
    uint64_t bytes() const;      // 0 for unsupported types
};

class GgufFile {
public:
    bool open(const std::string &path, std::string *error);

    uint32_t version() const { return version_; }
    uint64_t alignment() const { return alignment_; }
    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    const GgufTensor *find(const std::string &name) const;

    bool has_key(const std::string &key) const { return kv_.count(key) != 0; }
    // Typed metadata; `required` false leaves `out` untouched when absent.
    bool get_string(const std::string &key, std::string &out, bool required, std::string *error) const;
    bool get_u32(const std::string &key, uint32_t &out, bool required, std::string *error) const;
    bool get_f32(const std::string &key, float &out, bool required, std::string *error) const;
    bool get_bool(const std::string &key, bool &out, bool required, std::string *error) const;

    // Tensor payload as f32 (F32 copied, F16 / BF16 widened); every value
    // must be finite.
    bool read_f32(const GgufTensor &t, std::vector<float> &out, std::string *error) const;

private:
    struct Value {
        uint32_t type = 0;
        uint64_t u = 0;  // unsigned / bool payload
        int64_t i = 0;   // signed payload
        double f = 0;    // float payload
        std::string s;   // string payload
    };
    std::string path_;
    uint32_t version_ = 0;
    uint64_t alignment_ = 32;
    uint64_t data_offset_ = 0;
    uint64_t file_size_ = 0;
    std::map<std::string, Value> kv_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, std::size_t> index_;
};

}  // namespace b200
}  // namespace pixal3d
