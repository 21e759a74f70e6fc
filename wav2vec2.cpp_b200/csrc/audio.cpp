// WAV ingestion: restates the reference CLI's reader
// (examples/main/main.cpp:20-82 in py-ai-dev/wav2vec2.cpp) over an in-memory
// file image with bounds checks.
//
// Same results as the reference for every file it reads correctly:
//  * chunks are walked from offset 12 as (id, size) pairs with no RIFF pad
//    byte, stopping at the first "data" chunk; "fmt " is read as 16 bytes
//    from its start whatever its declared size (main.cpp:37-51);
//  * a sample is the float sum over channels, in channel order, of
//    s/32768 (PCM16), s/2^31 (PCM32) or s (float32), divided by the channel
//    count (main.cpp:55-66);
//  * resampling: out_n = n*target/sr; position i*sr/target in double, lower
//    neighbour by truncation, upper clamped to the last sample, weight
//    (float)(pos - lo) (main.cpp:70-80).
// The reference is released with -O3 -ffast-math -mfma (CMakeLists.txt:12-25),
// under which its channel mean is evaluated as sum * (1/n_ch) and its
// interpolation lo*(1-w) + hi*w as fma(lo, 1-w, hi*w); both are written out
// here in that form, which reproduces the reference build bit for bit
// (checked against it on PCM16/PCM32/float files of 1-3 channels at
// 8-48 kHz).
// Where the reference's behaviour is undefined this reader is defined: a
// zero channel count or bit depth is "Malformed WAV" (the reference divides
// by zero), and a data chunk that runs past the end of the file yields only
// the complete sample frames present (the reference reads indeterminate
// values there).
#include "audio.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>

namespace w2v {
namespace {

uint32_t le32(const unsigned char* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint16_t le16(const unsigned char* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

}  // namespace

std::vector<float> decode_wav(const unsigned char* data, size_t size, int target_sr) {
    // Reads past the end of the image return zero bytes, as the reference's
    // fread into zero-initialised values does.
    auto rd = [&](size_t off, size_t n, unsigned char* out) {
        for (size_t i = 0; i < n; i++) out[i] = off + i < size ? data[off + i] : 0;
    };
    unsigned char b[16];
    rd(0, 4, b);
    if (le32(b) != 0x46464952u) throw std::runtime_error("Not a RIFF file");
    rd(8, 4, b);
    if (le32(b) != 0x45564157u) throw std::runtime_error("Not a WAVE file");

    uint16_t fmt = 0, n_ch = 0, bits = 0;
    uint32_t sr = 0, data_size = 0;
    size_t data_off = 0;
    bool have_fmt = false, have_data = false;
    size_t pos = 12;
    while (pos < size) {
        rd(pos, 8, b);
        const uint32_t id = le32(b), sz = le32(b + 4);
        pos += 8;
        if (id == 0x20746d66u) {            // "fmt "
            rd(pos, 16, b);
            fmt = le16(b);
            n_ch = le16(b + 2);
            sr = le32(b + 4);
            bits = le16(b + 14);
            pos += sz > 16 ? sz : 16;
            have_fmt = true;
        } else if (id == 0x61746164u) {     // "data"
            data_size = sz;
            data_off = pos;
            have_data = true;
            break;
        } else {
            pos += sz;
        }
    }
    if (!have_fmt || !have_data) throw std::runtime_error("Malformed WAV");
    if (fmt != 1 && fmt != 3) throw std::runtime_error("Only PCM/float WAV");
    const uint32_t bytes = bits / 8u;
    if (n_ch == 0 || bytes == 0) throw std::runtime_error("Malformed WAV");
    uint32_t n = data_size / ((uint32_t)n_ch * bytes);
    if (n == 0) return {};
    const bool pcm16 = fmt == 1 && bits == 16, pcm32 = fmt == 1 && bits == 32, f32 = fmt == 3 && bits == 32;
    if (!pcm16 && !pcm32 && !f32) throw std::runtime_error("Unsupported bit depth");
    const size_t frame = (size_t)n_ch * bytes;
    const size_t avail = data_off < size ? (size - data_off) / frame : 0;
    if (avail < n) n = (uint32_t)avail;

    std::vector<float> mono(n);
    const unsigned char* p = data + data_off;
    for (uint32_t i = 0; i < n; i++) {
        float sum = 0.f;
        for (uint16_t c = 0; c < n_ch; c++, p += bytes) {
            if (pcm16) {
                sum += (float)(int16_t)le16(p) / 32768.f;
            } else if (pcm32) {
                sum += (float)(int32_t)le32(p) / 2147483648.f;
            } else {
                float v;
                std::memcpy(&v, p, 4);
                sum += v;
            }
        }
        mono[i] = sum * (1.f / (float)n_ch);
    }
    if ((int)sr == target_sr || n == 0) return mono;
    if (sr == 0 || target_sr <= 0) throw std::runtime_error("Malformed WAV");

    const uint32_t out_n = (uint32_t)((uint64_t)n * (uint64_t)target_sr / sr);
    std::vector<float> out(out_n);
    for (uint32_t i = 0; i < out_n; i++) {
        const double at = (double)i * sr / target_sr;
        const uint32_t lo = (uint32_t)at;
        const uint32_t hi = std::min(lo + 1u, n - 1u);
        const float w = (float)(at - lo);
        out[i] = std::fma(mono[lo], 1.f - w, mono[hi] * w);
    }
    return out;
}

std::vector<float> load_wav(const char* path, int target_sr) {
    FILE* f = path ? std::fopen(path, "rb") : nullptr;
    if (!f) throw std::runtime_error(std::string("Cannot open WAV: ") + (path ? path : "(null)"));
    std::vector<unsigned char> buf;
    unsigned char chunk[1 << 16];
    size_t got;
    while ((got = std::fread(chunk, 1, sizeof(chunk), f)) > 0) buf.insert(buf.end(), chunk, chunk + got);
    std::fclose(f);
    return decode_wav(buf.data(), buf.size(), target_sr);
}

}  // namespace w2v
