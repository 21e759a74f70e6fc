// GGUF reader for the engine's model loader.
//
// Reads the format the reference reads (src/gguf.h:113-195 in
// py-ai-dev/wav2vec2.cpp): header magic/version/counts, KV metadata (scalars,
// strings, arrays of u32 and strings), tensor infos (dims innermost first,
// type id, offset) and a 32-byte aligned data section.  Instead of copying the
// whole file into host vectors it memory-maps the file and hands out views,
// so weights go from the page cache straight into pinned staging for the
// device upload.  Every read is bounds-checked; a malformed file raises
// std::runtime_error with the reference's messages where they exist.
#pragma once
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace w2v {

enum GgufType : uint32_t { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8 };

// Raw byte size of n elements (src/gguf.h:46-64).
inline size_t gguf_nbytes(uint32_t t, uint64_t n) {
    switch (t) {
        case GT_F32: return n * 4;
        case GT_F16: return n * 2;
        case GT_Q4_0: return n / 32 * 18;
        case 3: return n / 32 * 20;
        case 6: return n / 32 * 22;
        case 7: return n / 32 * 24;
        case GT_Q8_0: return n / 32 * 34;
        case 9: return n / 32 * 36;
        default: return n * 4;
    }
}

struct GgufTensorView {
    std::vector<uint64_t> shape;   // innermost first
    uint64_t n = 0;
    uint32_t type = 0;
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
};

struct GgufValue {
    uint32_t type = 0;
    uint64_t u64 = 0;
    std::string str;
    std::vector<uint32_t> arr_u32;
    std::vector<std::string> arr_str;
};

class GgufFile {
public:
    explicit GgufFile(const std::string& path);
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    bool has_kv(const std::string& k) const { return kv_.count(k) != 0; }
    uint32_t u32(const std::string& k) const;
    const std::string& str(const std::string& k) const;
    const std::vector<uint32_t>& arr_u32(const std::string& k) const;
    const std::vector<std::string>& arr_str(const std::string& k) const;

    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const GgufTensorView& tensor(const std::string& name) const;
    // F32 or F16 tensor widened to fp32 (src/gguf.h:183-190).
    std::vector<float> floats(const std::string& name) const;

private:
    const GgufValue& get(const std::string& k) const;
    void parse();
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
    int fd_ = -1;
    std::unordered_map<std::string, GgufValue> kv_;
    std::unordered_map<std::string, GgufTensorView> tensors_;
};

float f16_to_f32(uint16_t h);

}  // namespace w2v
