// WAV ingestion for the command-line and batch callers.
#pragma once
#include <vector>

namespace w2v {

// Decode a RIFF/WAVE file (PCM 16-bit, PCM 32-bit or IEEE float 32-bit; any
// channel count and sample rate), average the channels to mono and resample
// to target_sr by linear interpolation.  Throws std::runtime_error with the
// reference reader's messages on failure.
std::vector<float> load_wav(const char* path, int target_sr);

// The same, from an in-memory file image.
std::vector<float> decode_wav(const unsigned char* data, size_t size, int target_sr);

}  // namespace w2v
