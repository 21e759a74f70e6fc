// Internal interface of the tensor-core conv layer 0 (conv0_tc.cu), used by
// w2v_conv0 in extractor.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace w2v {

struct Conv0TcArgs {
    const float* audio; const long long* off; const int* frames;
    const float* stats;            // per utterance (mean, 1/std) of the waveform
    const float* w0; const float* b0; int C; int norm;
    const float* gw; const float* gb;
    const float2* gnf;             // norm == 1: per (utterance, channel) (scale, shift) of bias + GroupNorm
    __half* out; long long rows_max; int n_utt; int n_fb; int* err;
};

bool conv0_tc_supported(int C, int k0, int s0, int norm, const void* out);
int launch_conv0_tc(const Conv0TcArgs& a, cudaStream_t st);

}  // namespace w2v
