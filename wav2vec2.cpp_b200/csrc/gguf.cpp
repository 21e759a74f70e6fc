#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace w2v {

float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        float f = (float)m * (1.0f / 16777216.0f);
        memcpy(&bits, &f, 4);
        bits |= s;
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

namespace {
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    void need(size_t n) {
        if ((size_t)(end - p) < n) throw std::runtime_error("gguf: truncated file");
    }
    template <typename T>
    T get() {
        need(sizeof(T));
        T v;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        need(n);
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

// Scalar KV value (src/gguf.h:95-111).
void read_scalar(Reader& r, uint32_t t, GgufValue& v) {
    switch (t) {
        case 0: v.u64 = r.get<uint8_t>(); break;
        case 1: v.u64 = (uint64_t)(int64_t)r.get<int8_t>(); break;
        case 2: v.u64 = r.get<uint16_t>(); break;
        case 3: v.u64 = (uint64_t)(int64_t)r.get<int16_t>(); break;
        case 4: v.u64 = r.get<uint32_t>(); break;
        case 5: v.u64 = (uint64_t)(int64_t)r.get<int32_t>(); break;
        case 6: r.get<float>(); break;
        case 7: v.u64 = r.get<uint8_t>(); break;
        case 8: v.str = r.str(); break;
        case 10: v.u64 = r.get<uint64_t>(); break;
        case 11: v.u64 = (uint64_t)r.get<int64_t>(); break;
        case 12: r.get<double>(); break;
        default: throw std::runtime_error("gguf: unsupported scalar type " + std::to_string(t));
    }
}
}  // namespace

GgufFile::GgufFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("Cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0 || st.st_size < 24) {
        ::close(fd_);
        fd_ = -1;
        throw std::runtime_error("Not GGUF");
    }
    size_ = (size_t)st.st_size;
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        ::close(fd_);
        fd_ = -1;
        throw std::runtime_error("Cannot map " + path);
    }
    base_ = static_cast<const uint8_t*>(m);
    try {
        parse();
    } catch (...) {
        munmap(const_cast<uint8_t*>(base_), size_);
        ::close(fd_);
        base_ = nullptr;
        fd_ = -1;
        throw;
    }
}

GgufFile::~GgufFile() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    if (fd_ >= 0) ::close(fd_);
}

void GgufFile::parse() {
    Reader r{base_, base_ + size_};
    if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("Not GGUF");
    r.get<uint32_t>();  // version
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) throw std::runtime_error("gguf: implausible header counts");
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = r.str();
        GgufValue v;
        v.type = r.get<uint32_t>();
        if (v.type == 9) {  // array (src/gguf.h:130-138)
            const uint32_t et = r.get<uint32_t>();
            const uint64_t an = r.get<uint64_t>();
            if (an > size_) throw std::runtime_error("gguf: implausible array length");
            for (uint64_t j = 0; j < an; j++) {
                if (et == 8) v.arr_str.push_back(r.str());
                else if (et == 4) v.arr_u32.push_back(r.get<uint32_t>());
                else { GgufValue tmp; read_scalar(r, et, tmp); }
            }
        } else {
            read_scalar(r, v.type, v);
        }
        kv_[key] = std::move(v);
    }
    struct Info { std::string name; std::vector<uint64_t> shape; uint32_t type; uint64_t off; };
    std::vector<Info> infos(n_tensors);
    for (auto& ti : infos) {
        ti.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd > 4) throw std::runtime_error("gguf: tensor rank > 4: " + ti.name);
        ti.shape.resize(nd);
        for (auto& d : ti.shape) d = r.get<uint64_t>();
        ti.type = r.get<uint32_t>();
        ti.off = r.get<uint64_t>();
    }
    const uint64_t data_start = ((uint64_t)(r.p - base_) + 31u) & ~31ull;  // src/gguf.h:162-165
    for (auto& ti : infos) {
        GgufTensorView t;
        t.shape = ti.shape;
        t.n = 1;
        for (auto d : ti.shape) t.n *= d;
        t.type = ti.type;
        t.nbytes = gguf_nbytes(ti.type, t.n);
        if (data_start + ti.off > size_ || t.nbytes > size_ - (data_start + ti.off))
            throw std::runtime_error("gguf: tensor data out of file bounds: " + ti.name);
        t.data = base_ + data_start + ti.off;
        tensors_[ti.name] = std::move(t);
    }
}

const GgufValue& GgufFile::get(const std::string& k) const {
    auto it = kv_.find(k);
    if (it == kv_.end()) throw std::runtime_error("Missing key: " + k);
    return it->second;
}
uint32_t GgufFile::u32(const std::string& k) const { return (uint32_t)get(k).u64; }
const std::string& GgufFile::str(const std::string& k) const { return get(k).str; }
const std::vector<uint32_t>& GgufFile::arr_u32(const std::string& k) const { return get(k).arr_u32; }
const std::vector<std::string>& GgufFile::arr_str(const std::string& k) const { return get(k).arr_str; }

const GgufTensorView& GgufFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("Missing tensor: " + name);
    return it->second;
}

std::vector<float> GgufFile::floats(const std::string& name) const {
    const auto& t = tensor(name);
    std::vector<float> out(t.n);
    if (t.type == GT_F32) {
        memcpy(out.data(), t.data, t.n * 4);
    } else if (t.type == GT_F16) {
        for (uint64_t i = 0; i < t.n; i++) {
            uint16_t h;
            memcpy(&h, t.data + 2 * i, 2);
            out[i] = f16_to_f32(h);
        }
    } else {
        throw std::runtime_error("Tensor " + name + " is quantized — expected F32/F16");
    }
    return out;
}

}  // namespace w2v
