// Bandwidth-bound kernels around the GEMMs: weight expansion at load time,
// waveform statistics, conv layer 0 with its norm + GELU, row LayerNorm and
// the greedy CTC decoder.
#include <mutex>

#include "common.cuh"
#include "conv0_tc.cuh"
#include "w2v_kernels.h"

namespace w2v {

// ── weight expansion (GGUF blocks -> fp16 rows) ─────────────────────────────
// Q8_0: 34-byte blocks {fp16 d, int8 q[32]}, w = d*q.  Q4_0: 18-byte blocks
// {fp16 d, 16 bytes}, byte j = elem j (low nibble) | elem j+16 (high), w =
// d*(q-8)  (scripts/convert_to_gguf.py:63-97).  d*q is exact in fp32 and
// rounded once to fp16.
__global__ void dequant_q_kernel(const uint8_t* __restrict__ raw, int type, long long n_blocks,
                                 __half* __restrict__ out) {
    const long long blk = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n_blocks) return;
    float v[32];
    if (type == 8) {
        const uint8_t* b = raw + blk * 34;
        const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = d * (float)(int8_t)b[2 + j];
    } else {
        const uint8_t* b = raw + blk * 18;
        const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
#pragma unroll
        for (int j = 0; j < 16; j++) {
            v[j] = d * (float)((int)(b[2 + j] & 0xF) - 8);
            v[j + 16] = d * (float)((int)(b[2 + j] >> 4) - 8);
        }
    }
    uint4* o = reinterpret_cast<uint4*>(out + blk * 32);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint4 u;
        u.x = pack_half2(v[8 * j + 0], v[8 * j + 1]);
        u.y = pack_half2(v[8 * j + 2], v[8 * j + 3]);
        u.z = pack_half2(v[8 * j + 4], v[8 * j + 5]);
        u.w = pack_half2(v[8 * j + 6], v[8 * j + 7]);
        o[j] = u;
    }
}

// GGUF Q8_0 / Q4_0 blocks of rows [N, K] -> the fused GEMM's planes (layout
// in qgemm_tc.cu): codes[n][k] int8 (Q8_0) or, per eight weights 8g..8g+7, a
// 32-bit word holding weight 8g+2j in bits 4j..4j+3 and weight 8g+2j+1 in
// bits 16+4j..19+4j, as the unsigned 4-bit code (Q4_0); scales[k/32][n] =
// the block's fp16 scale bits.  One thread per block.
__global__ void repack_q_kernel(const uint8_t* __restrict__ raw, int type, long long n_rows, long long K,
                                uint8_t* __restrict__ codes, uint16_t* __restrict__ scales, long long ld_s) {
    const long long nbr = K / 32;
    const long long blk = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n_rows * nbr) return;
    const long long n = blk / nbr, j = blk - n * nbr;
    if (type == 8) {
        const uint8_t* b = raw + blk * 34;
        scales[j * ld_s + n] = (uint16_t)(b[0] | (b[1] << 8));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            w[i] = (uint32_t)b[2 + 4 * i] | ((uint32_t)b[3 + 4 * i] << 8) | ((uint32_t)b[4 + 4 * i] << 16) |
                   ((uint32_t)b[5 + 4 * i] << 24);
        uint4* dst = reinterpret_cast<uint4*>(codes + n * K + j * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
        const uint8_t* b = raw + blk * 18;
        scales[j * ld_s + n] = (uint16_t)(b[0] | (b[1] << 8));
        uint32_t e[32];
#pragma unroll
        for (int t = 0; t < 16; t++) {
            e[t] = b[2 + t] & 0xFu;
            e[t + 16] = b[2 + t] >> 4;
        }
        uint32_t w[4];
#pragma unroll
        for (int g = 0; g < 4; g++) {
            uint32_t v = 0;
#pragma unroll
            for (int jj = 0; jj < 4; jj++) v |= (e[8 * g + 2 * jj] << (4 * jj)) | (e[8 * g + 2 * jj + 1] << (16 + 4 * jj));
            w[g] = v;
        }
        *reinterpret_cast<uint4*>(codes + n * (K / 2) + j * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, long long n, __half* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}

// ── waveform statistics (src/wav2vec2.cpp:262-271) ──────────────────────────
template <typename T>
W2V_DEV T block_sum(T v, T* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    T s = 0;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

// One block per utterance, one pass: sum and sum of squares in fp64 (four
// independent accumulators per thread, 16-byte loads on the aligned body).
// var = E[x^2] - mean^2 in fp64 equals the reference's two-pass fp32
// population variance to well below fp32 resolution for audio-range values.
__global__ void __launch_bounds__(1024) wave_stats_kernel(const float* __restrict__ audio,
                                                          const long long* __restrict__ off,
                                                          const int* __restrict__ len, float* __restrict__ stats) {
    __shared__ double red[32];
    const int u = blockIdx.x;
    const float* x = audio + off[u];
    const int n = len[u];
    if (n <= 0) {
        if (threadIdx.x == 0) { stats[2 * u] = 0.f; stats[2 * u + 1] = 1.f / sqrtf(1e-7f); }
        return;
    }
    // scalar head up to a 16-byte boundary, float4 body, scalar tail
    const int head = min(n, (int)(((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) / 4));
    const int nv = (n - head) / 4;
    const float4* xv = reinterpret_cast<const float4*>(x + head);
    double s0 = 0, s1 = 0, q0 = 0, q1 = 0;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
        const float4 v = __ldg(xv + i);
        s0 += (double)v.x + (double)v.y;
        s1 += (double)v.z + (double)v.w;
        q0 = fma((double)v.x, (double)v.x, fma((double)v.y, (double)v.y, q0));
        q1 = fma((double)v.z, (double)v.z, fma((double)v.w, (double)v.w, q1));
    }
    for (int i = threadIdx.x; i < head; i += blockDim.x) { const double v = x[i]; s0 += v; q0 = fma(v, v, q0); }
    for (int i = head + 4 * nv + threadIdx.x; i < n; i += blockDim.x) {
        const double v = x[i];
        s1 += v;
        q1 = fma(v, v, q1);
    }
    const double S = block_sum(s0 + s1, red);
    const double Q = block_sum(q0 + q1, red);
    if (threadIdx.x == 0) {
        const double mean = S / n;
        const float var = (float)fmax(Q / n - mean * mean, 0.0);
        stats[2 * u] = (float)mean;
        stats[2 * u + 1] = 1.f / sqrtf(var + 1e-7f);
    }
}

// ── conv layer 0 GroupNorm statistics from window moments ───────────────────
// For the published first layer (kernel 10, stride 5) with GroupNorm (one
// group per channel, statistics over all frames; src/ops.h:39-50) the mean
// and variance of y[f,c] = b[c] + sum_k w[c,k] xn[5f+k] over the F frames
// follow exactly from the moments of the normalised windows xn = (x - mu) r:
//   sum_f y   = F b + w.S
//   sum_f y^2 = F b^2 + 2 b w.S + w^T G w,
//   S_k = sum_f xn[5f+k],  G_kl = sum_f xn[5f+k] xn[5f+l].
// S and G are accumulated in fp64 from the raw samples (a product of two
// floats is exact in fp64) and normalised afterwards with the utterance's
// (mu, r): 65 fp64 FMAs per frame instead of a second evaluation of the
// 5120-FMA convolution.  Per-chunk partials are reduced in a fixed order, so
// an utterance's statistics do not depend on the rest of its batch.
constexpr int kGramK = 10, kGramS = 5, kGramN = kGramK + kGramK * (kGramK + 1) / 2;   // 65
constexpr int kGramThreads = 256;

W2V_DEV int gram_index(int k, int l) {   // k <= l
    return kGramK + k * kGramK - k * (k - 1) / 2 + (l - k);
}

__global__ void __launch_bounds__(kGramThreads) conv0_gram_kernel(const float* __restrict__ audio,
                                                                  const long long* __restrict__ off,
                                                                  const int* __restrict__ frames, int chunks,
                                                                  double* __restrict__ part) {
    __shared__ double red[kGramThreads / 32][kGramN];
    const int u = blockIdx.y, ch = blockIdx.x;
    const int F = frames[u];
    const int per = (F + chunks - 1) / chunks;
    const int f0 = ch * per, f1 = min(F, f0 + per);
    const float* x = audio + off[u];
    double acc[kGramN];
#pragma unroll
    for (int i = 0; i < kGramN; i++) acc[i] = 0.0;
    for (int f = f0 + (int)threadIdx.x; f < f1; f += kGramThreads) {
        double v[kGramK];
#pragma unroll
        for (int k = 0; k < kGramK; k++) v[k] = (double)__ldg(x + (long long)f * kGramS + k);
#pragma unroll
        for (int k = 0; k < kGramK; k++) {
            acc[k] += v[k];
#pragma unroll
            for (int l = k; l < kGramK; l++) acc[gram_index(k, l)] = fma(v[k], v[l], acc[gram_index(k, l)]);
        }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < kGramN; i++) {
        double a = acc[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) red[w][i] = a;
    }
    __syncthreads();
    if (threadIdx.x < kGramN) {
        double t = 0.0;
#pragma unroll
        for (int i = 0; i < kGramThreads / 32; i++) t += red[i][threadIdx.x];
        part[((long long)u * chunks + ch) * kGramN + threadIdx.x] = t;
    }
}

// Per (utterance, channel) GroupNorm mean and 1/sqrt(var + 1e-5) from the
// window moments; `stats` holds the (mu, r) the conv kernel normalises with.
// With gw/gb given, writes the channel's full affine instead: (scale, shift)
// with GroupNorm(b + conv) = conv * scale + shift.
__global__ void conv0_gram_finalize_kernel(const double* __restrict__ part, int chunks,
                                           const float* __restrict__ stats, const int* __restrict__ frames,
                                           const float* __restrict__ w0, const float* __restrict__ b0, int C,
                                           const float* __restrict__ gw, const float* __restrict__ gb,
                                           float2* __restrict__ gnf) {
    __shared__ double m[kGramN];
    __shared__ double Sn[kGramK];
    __shared__ double Gn[kGramK][kGramK];
    const int u = blockIdx.x;
    if (threadIdx.x < kGramN) {
        double t = 0.0;
        for (int c = 0; c < chunks; c++) t += part[((long long)u * chunks + c) * kGramN + threadIdx.x];
        m[threadIdx.x] = t;
    }
    __syncthreads();
    const int F = frames[u];
    const double Fd = (double)F, mu = (double)stats[2 * u], r = (double)stats[2 * u + 1];
    if (threadIdx.x < kGramK) Sn[threadIdx.x] = r * (m[threadIdx.x] - Fd * mu);
    if (threadIdx.x < kGramK * kGramK) {
        const int k = threadIdx.x / kGramK, l = threadIdx.x % kGramK;
        const double P = m[gram_index(min(k, l), max(k, l))];
        Gn[k][l] = r * r * (P - mu * (m[k] + m[l]) + Fd * mu * mu);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float2 o = make_float2(0.f, 1.f / sqrtf(1e-5f));
        if (F > 0) {
            double wv[kGramK];
#pragma unroll
            for (int k = 0; k < kGramK; k++) wv[k] = (double)__ldg(w0 + c * kGramK + k);
            const double b = b0 ? (double)__ldg(b0 + c) : 0.0;
            double ws = 0.0, wgw = 0.0;
#pragma unroll
            for (int k = 0; k < kGramK; k++) {
                ws = fma(wv[k], Sn[k], ws);
                double g = 0.0;
#pragma unroll
                for (int l = 0; l < kGramK; l++) g = fma(wv[l], Gn[k][l], g);
                wgw = fma(wv[k], g, wgw);
            }
            const double mean = (Fd * b + ws) / Fd;
            const double ey2 = (Fd * b * b + 2.0 * b * ws + wgw) / Fd;
            const float var = (float)fmax(ey2 - mean * mean, 0.0);
            o = make_float2((float)mean, 1.f / sqrtf(var + 1e-5f));
        }
        if (gw) {
            const float sc = o.y * __ldg(gw + c);
            const float bc = b0 ? __ldg(b0 + c) : 0.f;
            o = make_float2(sc, __ldg(gb + c) + (bc - o.x) * sc);
        }
        gnf[(long long)u * C + c] = o;
    }
}

// ── conv layer 0 + norm + GELU (src/wav2vec2.cpp:273-287) ────────────────────
// Block: 256 threads, thread t owns channels (2t, 2t+1) (C <= 512, even) and
// keeps their K0 taps in registers; the normalised samples the block needs
// are staged once in shared memory and read as broadcasts.  Frames are
// processed in register groups of 32.  K0 is 10 for every published model;
// other first-layer kernels (<= 16) run the K0 = 16 instance with zero taps.
constexpr int kC0Group = 32;        // frames per register group
constexpr int kC0ApplyFrames = 256; // frames per apply block
constexpr int kC0StatFrames = 1024; // frames per statistics block
constexpr int kC0MaxK = 16;
constexpr int kC0K = 10, kC0S = 5, kC0Sub = 8, kC0Win = (kC0Sub - 1) * kC0S + kC0K;   // 45

struct Conv0Args {
    const float* audio; const long long* off; const int* len; const int* frames;
    const float* stats; const float* w0; const float* b0; int C, k0, s0, norm;
    const float* gw; const float* gb; double* gn; __half* out; long long rows_max;
    const float2* gnf;   // GroupNorm (mean, 1/std) per (utterance, channel), when precomputed
};

// Stage normalised samples for frames f0 .. f0+nf-1 (zero-padded by kC0MaxK).
W2V_DEV void conv0_stage(const Conv0Args& a, int u, int f0, int nf, float* xs) {
    const float mean = a.stats[2 * u], inv = a.stats[2 * u + 1];
    const float* x = a.audio + a.off[u];
    const int ns = (nf - 1) * a.s0 + a.k0;
    for (int i = threadIdx.x; i < ns + kC0MaxK + kC0Win; i += blockDim.x)
        xs[i] = i < ns ? (x[(long long)f0 * a.s0 + i] - mean) * inv : 0.f;
}

template <int K0>
W2V_DEV void conv0_load_w(const Conv0Args& a, int c, float (&w)[2][K0], float& b0, float& b1) {
#pragma unroll
    for (int k = 0; k < K0; k++) {
        w[0][k] = k < a.k0 ? __ldg(a.w0 + c * a.k0 + k) : 0.f;
        w[1][k] = k < a.k0 ? __ldg(a.w0 + (c + 1) * a.k0 + k) : 0.f;
    }
    b0 = a.b0 ? __ldg(a.b0 + c) : 0.f;
    b1 = a.b0 ? __ldg(a.b0 + c + 1) : 0.f;
}

template <int K0>
W2V_DEV void conv0_group(const float* xs, int g0, int s0, const float (&w)[2][K0], float b0, float b1,
                         float (&y)[kC0Group][2]) {
#pragma unroll
    for (int f = 0; f < kC0Group; f++) {
        const float* x = xs + (g0 + f) * s0;
        float y0 = b0, y1 = b1;
#pragma unroll
        for (int k = 0; k < K0; k++) {
            const float v = x[k];
            y0 = fmaf(v, w[0][k], y0);
            y1 = fmaf(v, w[1][k], y1);
        }
        y[f][0] = y0;
        y[f][1] = y1;
    }
}

// Statistics pass (GroupNorm only): per-channel sum and sum of squares over
// the utterance's frames, accumulated in fp64.
template <int K0>
__global__ void __launch_bounds__(256) conv0_gn_stats_kernel(Conv0Args a) {
    extern __shared__ float xs[];
    const int u = blockIdx.y;
    const int F = a.frames[u];
    const int f0 = blockIdx.x * kC0StatFrames;
    if (f0 >= F) return;
    const int nf = min(kC0StatFrames, F - f0);
    conv0_stage(a, u, f0, nf, xs);
    __syncthreads();
    const int c = 2 * threadIdx.x;
    if (c >= a.C) return;
    float w[2][K0], b0, b1;
    conv0_load_w<K0>(a, c, w, b0, b1);
    double s0 = 0, s1 = 0, q0 = 0, q1 = 0;
    for (int g0 = 0; g0 < nf; g0 += kC0Group) {
        float y[kC0Group][2];
        conv0_group<K0>(xs, g0, a.s0, w, b0, b1, y);
        float ps0 = 0.f, ps1 = 0.f, pq0 = 0.f, pq1 = 0.f;   // fp32 within a group of <= 32 frames
#pragma unroll
        for (int f = 0; f < kC0Group; f++) {
            if (g0 + f < nf) {
                ps0 += y[f][0]; ps1 += y[f][1];
                pq0 = fmaf(y[f][0], y[f][0], pq0); pq1 = fmaf(y[f][1], y[f][1], pq1);
            }
        }
        s0 += ps0; s1 += ps1; q0 += pq0; q1 += pq1;
    }
    double* g = a.gn + ((long long)u * a.C + c) * 2;
    atomicAdd(g + 0, s0); atomicAdd(g + 1, q0);
    atomicAdd(g + 2, s1); atomicAdd(g + 3, q1);
}

template <int K0>
__global__ void __launch_bounds__(256) conv0_apply_kernel(Conv0Args a) {
    extern __shared__ float xs[];
    __shared__ float red[8][kC0Group];
    __shared__ float rowstat[2][kC0Group];
    const int u = blockIdx.y;
    const int F = a.frames[u];
    const int f0 = blockIdx.x * kC0ApplyFrames;
    if (f0 >= F) return;
    const int nf = min(kC0ApplyFrames, F - f0);
    conv0_stage(a, u, f0, nf, xs);
    __syncthreads();
    const int c = 2 * threadIdx.x;
    const bool active = c < a.C;
    float w[2][K0], b0 = 0.f, b1 = 0.f;
    float m[2] = {0.f, 0.f}, iv[2] = {1.f, 1.f}, ga[2] = {1.f, 1.f}, be[2] = {0.f, 0.f};
    if (active) {
        conv0_load_w<K0>(a, c, w, b0, b1);
        if (a.norm) {
            ga[0] = a.gw[c]; ga[1] = a.gw[c + 1];
            be[0] = a.gb[c]; be[1] = a.gb[c + 1];
        }
        if (a.norm == 1) {
            // GroupNorm (one group per channel) over all frames of the
            // utterance (src/ops.h:39-50), statistics from the stats pass
            const double* g = a.gn + ((long long)u * a.C + c) * 2;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const double mu = g[2 * j] / F;
                const float var = (float)fmax(g[2 * j + 1] / F - mu * mu, 0.0);
                m[j] = (float)mu;
                iv[j] = 1.f / sqrtf(var + 1e-5f);
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < K0; k++) w[0][k] = w[1][k] = 0.f;
    }
    const int wi = threadIdx.x >> 5, l = threadIdx.x & 31;
    for (int g0 = 0; g0 < nf; g0 += kC0Group) {
        float y[kC0Group][2];
        conv0_group<K0>(xs, g0, a.s0, w, b0, b1, y);
        if (a.norm == 2) {
            // LayerNorm over channels per frame (src/ops.h:24-36), two-pass
            for (int pass = 0; pass < 2; pass++) {
#pragma unroll
                for (int f = 0; f < kC0Group; f++) {
                    float v = 0.f;
                    if (active) {
                        if (pass == 0) v = y[f][0] + y[f][1];
                        else {
                            const float d0 = y[f][0] - rowstat[0][f], d1 = y[f][1] - rowstat[0][f];
                            v = d0 * d0 + d1 * d1;
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (l == 0) red[wi][f] = v;
                }
                __syncthreads();
                if (threadIdx.x < kC0Group) {
                    float sum = 0.f;
                    for (int i = 0; i < (int)(blockDim.x >> 5); i++) sum += red[i][threadIdx.x];
                    if (pass == 0) rowstat[0][threadIdx.x] = sum / a.C;
                    else rowstat[1][threadIdx.x] = 1.f / sqrtf(sum / a.C + 1e-5f);
                }
                __syncthreads();
            }
        }
        if (active) {
#pragma unroll
            for (int f = 0; f < kC0Group; f++) {
                if (g0 + f < nf) {
                    float v0 = y[f][0], v1 = y[f][1];
                    if (a.norm == 1) {
                        v0 = (v0 - m[0]) * iv[0] * ga[0] + be[0];
                        v1 = (v1 - m[1]) * iv[1] * ga[1] + be[1];
                    } else if (a.norm == 2) {
                        v0 = (v0 - rowstat[0][f]) * rowstat[1][f] * ga[0] + be[0];
                        v1 = (v1 - rowstat[0][f]) * rowstat[1][f] * ga[1] + be[1];
                    }
                    *reinterpret_cast<__half2*>(a.out + ((long long)u * a.rows_max + f0 + g0 + f) * a.C + c) =
                        __floats2half2_rn(gelu_tanh(v0), gelu_tanh(v1));
                }
            }
        }
        if (a.norm == 2) __syncthreads();   // rowstat is rewritten by the next group
    }
}

// ── row LayerNorm (src/ops.h:24-36), warp per row ───────────────────────────
template <int MAXV>
__global__ void layer_norm_kernel(const void* __restrict__ in, int in_f16, long long ld_in, long long in_batch_rows,
                                  const int* __restrict__ rows, const long long* __restrict__ out_off,
                                  int n_batch, int n_rows, int D, const float* __restrict__ w,
                                  const float* __restrict__ b, int gelu, float* __restrict__ out32,
                                  __half* __restrict__ out16, long long ld_out) {
    const int warps = blockDim.x >> 5;
    const long long gw = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const long long rows_per_b = rows ? in_batch_rows : n_rows;
    const long long bi = gw / rows_per_b, r = gw % rows_per_b;
    if (bi >= n_batch) return;
    if (r >= (rows ? rows[bi] : n_rows)) return;
    const long long irow = bi * in_batch_rows + r;
    const long long orow = out_off ? out_off[bi] + r : irow;
    float v[MAXV];
    const int per = D / 32;   // D % 32 == 0, per <= MAXV
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; i++) {
        if (i < per) {
            const int col = lane + 32 * i;
            v[i] = in_f16 ? __half2float(reinterpret_cast<const __half*>(in)[irow * ld_in + col])
                          : reinterpret_cast<const float*>(in)[irow * ld_in + col];
            s += v[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; i++)
        if (i < per) { const float d = v[i] - mean; q += d * d; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.f / sqrtf(q / D + 1e-5f);
#pragma unroll
    for (int i = 0; i < MAXV; i++) {
        if (i < per) {
            const int col = lane + 32 * i;
            float y = (v[i] - mean) * inv * w[col] + b[col];
            if (gelu) y = gelu_tanh(y);
            if (out32) out32[orow * ld_out + col] = y;
            if (out16) out16[orow * ld_out + col] = __float2half_rn(y);
        }
    }
}

// Specialised conv 0 for the published extractor shape (kernel 10, stride 5):
// 128 threads, thread t owns channels 4t..4t+3 (40 taps in registers) and
// computes 8 frames at a time from a 45-sample window held in registers, so a
// broadcast shared-memory load feeds 32 FMAs instead of 2.  Same arithmetic
// order per output as conv0_group (bias, then taps 0..K-1).

W2V_DEV void conv0x4_sub(const float* xs, int f, const float (&w)[4][kC0K], const float (&bb)[4],
                         float (&y)[kC0Sub][4]) {
    float xr[kC0Win];
#pragma unroll
    for (int i = 0; i < kC0Win; i++) xr[i] = xs[f * kC0S + i];
#pragma unroll
    for (int fr = 0; fr < kC0Sub; fr++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float acc = bb[c];
#pragma unroll
            for (int k = 0; k < kC0K; k++) acc = fmaf(xr[fr * kC0S + k], w[c][k], acc);
            y[fr][c] = acc;
        }
}

W2V_DEV void conv0x4_load(const Conv0Args& a, int c0, float (&w)[4][kC0K], float (&bb)[4]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int k = 0; k < kC0K; k++) w[c][k] = __ldg(a.w0 + (c0 + c) * kC0K + k);
        bb[c] = a.b0 ? __ldg(a.b0 + c0 + c) : 0.f;
    }
}

__global__ void __launch_bounds__(128) conv0x4_gn_stats_kernel(Conv0Args a) {
    extern __shared__ float xs[];
    const int u = blockIdx.y;
    const int F = a.frames[u];
    const int f0 = blockIdx.x * kC0StatFrames;
    if (f0 >= F) return;
    const int nf = min(kC0StatFrames, F - f0);
    conv0_stage(a, u, f0, nf, xs);
    __syncthreads();
    const int c0 = 4 * threadIdx.x;
    if (c0 >= a.C) return;
    float w[4][kC0K], bb[4];
    conv0x4_load(a, c0, w, bb);
    double s[4] = {0, 0, 0, 0}, q[4] = {0, 0, 0, 0};
    for (int g = 0; g < nf; g += 32) {
        float ps[4] = {0, 0, 0, 0}, pq[4] = {0, 0, 0, 0};     // fp32 within <= 32 frames
#pragma unroll 1
        for (int f = g; f < g + 32; f += kC0Sub) {
            float y[kC0Sub][4];
            conv0x4_sub(xs, f, w, bb, y);
#pragma unroll
            for (int fr = 0; fr < kC0Sub; fr++)
                if (f + fr < nf)
#pragma unroll
                    for (int c = 0; c < 4; c++) { ps[c] += y[fr][c]; pq[c] = fmaf(y[fr][c], y[fr][c], pq[c]); }
        }
#pragma unroll
        for (int c = 0; c < 4; c++) { s[c] += ps[c]; q[c] += pq[c]; }
    }
    double* gp = a.gn + ((long long)u * a.C + c0) * 2;
#pragma unroll
    for (int c = 0; c < 4; c++) { atomicAdd(gp + 2 * c, s[c]); atomicAdd(gp + 2 * c + 1, q[c]); }
}

__global__ void __launch_bounds__(128) conv0x4_apply_kernel(Conv0Args a) {
    extern __shared__ float xs[];
    __shared__ float red[4][kC0Sub];
    __shared__ float rowstat[2][kC0Sub];
    const int u = blockIdx.y;
    const int F = a.frames[u];
    const int f0 = blockIdx.x * kC0ApplyFrames;
    if (f0 >= F) return;
    const int nf = min(kC0ApplyFrames, F - f0);
    conv0_stage(a, u, f0, nf, xs);
    __syncthreads();
    const int c0 = 4 * threadIdx.x;
    const bool active = c0 < a.C;
    float w[4][kC0K], bb[4];
    float m[4], iv[4], ga[4], be[4];
#pragma unroll
    for (int c = 0; c < 4; c++) { m[c] = 0.f; iv[c] = 1.f; ga[c] = 1.f; be[c] = 0.f; bb[c] = 0.f; }
    if (active) {
        conv0x4_load(a, c0, w, bb);
        if (a.norm) {
#pragma unroll
            for (int c = 0; c < 4; c++) { ga[c] = a.gw[c0 + c]; be[c] = a.gb[c0 + c]; }
        }
        if (a.norm == 1 && a.gnf) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float2 g = a.gnf[(long long)u * a.C + c0 + c];
                m[c] = g.x;
                iv[c] = g.y;
            }
        } else if (a.norm == 1) {
            const double* gp = a.gn + ((long long)u * a.C + c0) * 2;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const double mu = gp[2 * c] / F;
                const float var = (float)fmax(gp[2 * c + 1] / F - mu * mu, 0.0);
                m[c] = (float)mu;
                iv[c] = 1.f / sqrtf(var + 1e-5f);
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
            for (int k = 0; k < kC0K; k++) w[c][k] = 0.f;
    }
    const int wi = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll 1
    for (int f = 0; f < nf; f += kC0Sub) {
        float y[kC0Sub][4];
        conv0x4_sub(xs, f, w, bb, y);
        if (a.norm == 2) {
            // LayerNorm over channels per frame (src/ops.h:24-36), two-pass
            for (int pass = 0; pass < 2; pass++) {
#pragma unroll
                for (int fr = 0; fr < kC0Sub; fr++) {
                    float v = 0.f;
                    if (active) {
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const float d = pass == 0 ? y[fr][c] : y[fr][c] - rowstat[0][fr];
                            v += pass == 0 ? d : d * d;
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (l == 0) red[wi][fr] = v;
                }
                __syncthreads();
                if (threadIdx.x < kC0Sub) {
                    float sum = 0.f;
                    for (int i = 0; i < (int)(blockDim.x >> 5); i++) sum += red[i][threadIdx.x];
                    if (pass == 0) rowstat[0][threadIdx.x] = sum / a.C;
                    else rowstat[1][threadIdx.x] = 1.f / sqrtf(sum / a.C + 1e-5f);
                }
                __syncthreads();
            }
        }
        if (active) {
#pragma unroll
            for (int fr = 0; fr < kC0Sub; fr++) {
                if (f + fr < nf) {
                    float v[4];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        v[c] = y[fr][c];
                        if (a.norm == 1) v[c] = (v[c] - m[c]) * iv[c] * ga[c] + be[c];
                        else if (a.norm == 2) v[c] = (v[c] - rowstat[0][fr]) * rowstat[1][fr] * ga[c] + be[c];
                        v[c] = gelu_tanh(v[c]);
                    }
                    uint2 pk;
                    pk.x = pack_half2(v[0], v[1]);
                    pk.y = pack_half2(v[2], v[3]);
                    *reinterpret_cast<uint2*>(a.out + ((long long)u * a.rows_max + f0 + f + fr) * a.C + c0) = pk;
                }
            }
        }
        if (a.norm == 2) __syncthreads();
    }
}

// Conv layer 0 + LayerNorm over its 512 channels + GELU, for the LayerNorm
// feature extractor (wav2vec2-large / XLS-R: src/wav2vec2.cpp:273-287 with
// src/ops.h:24-36) at the published shape (10 taps, stride 5, 512 channels).
// A warp owns whole frames, so the per-frame LayerNorm needs only warp
// shuffles: lane l holds channel pairs p = l + 32 j (channels 2p, 2p+1,
// j = 0..7) of kLnF = 4 frames at a time.  The 10 x 512 weights and the bias
// sit in shared memory as pairs (one conflict-free 8-byte read serves 4
// frames x 2 channels), the samples of the block's frames are staged once
// normalised, and the convolution runs as packed fp32-pair FMAs.  Two-pass
// statistics in fp32 as the reference; GELU on fp16 pairs (gelu_f16x2) as the
// tensor-core conv 0 does, since the output is fp16.
constexpr int kLnF = 4;                   // frames per register group
constexpr int kLnThreads = 128;           // 4 warps
constexpr int kLnBlockFrames = 512;       // frames per block: 128 per warp
constexpr int kLnC = 512;
constexpr int kLnSamples = (kLnBlockFrames - 1) * kC0S + kC0K;   // 2565

__global__ void __launch_bounds__(kLnThreads, 3) conv0_ln_kernel(Conv0Args a) {
    __shared__ uint64_t ws[kC0K][kLnC / 2];   // (w[2p][k], w[2p+1][k])
    __shared__ uint64_t wb[kLnC / 2];         // (b[2p], b[2p+1])
    __shared__ float xs[kLnSamples + kLnF * kC0S];
    const int u = blockIdx.y;
    const int F = a.frames[u];
    const int f0 = blockIdx.x * kLnBlockFrames;
    if (f0 >= F) return;
    const int nf = min(kLnBlockFrames, F - f0);
    {
        const float mean = a.stats[2 * u], inv = a.stats[2 * u + 1];
        const float* x = a.audio + a.off[u] + (long long)f0 * kC0S;
        const int ns = (nf - 1) * kC0S + kC0K;
        for (int i = threadIdx.x; i < kLnSamples + kLnF * kC0S; i += kLnThreads)
            xs[i] = i < ns ? (x[i] - mean) * inv : 0.f;
        for (int i = threadIdx.x; i < kC0K * kLnC / 2; i += kLnThreads) {
            const int k = i / (kLnC / 2), p = i % (kLnC / 2);
            ws[k][p] = f32x2(__ldg(a.w0 + (2 * p) * kC0K + k), __ldg(a.w0 + (2 * p + 1) * kC0K + k));
        }
        for (int p = threadIdx.x; p < kLnC / 2; p += kLnThreads)
            wb[p] = a.b0 ? f32x2(__ldg(a.b0 + 2 * p), __ldg(a.b0 + 2 * p + 1)) : 0ull;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t g2[8], b2[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int c = 2 * (lane + 32 * j);
        g2[j] = f32x2(__ldg(a.gw + c), __ldg(a.gw + c + 1));
        b2[j] = f32x2(__ldg(a.gb + c), __ldg(a.gb + c + 1));
    }
    constexpr float kInvC = 1.f / kLnC;
    const int wf0 = warp * (kLnBlockFrames / 4);
    __half* orow = a.out + ((long long)u * a.rows_max + f0) * kLnC;
#pragma unroll 1
    for (int g = wf0; g < wf0 + kLnBlockFrames / 4 && g < nf; g += kLnF) {
        uint64_t acc[kLnF][8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint64_t b = wb[lane + 32 * j];
#pragma unroll
            for (int f = 0; f < kLnF; f++) acc[f][j] = b;
        }
#pragma unroll 1
        for (int k = 0; k < kC0K; k++) {
            uint64_t xk[kLnF];
#pragma unroll
            for (int f = 0; f < kLnF; f++) {
                const float v = xs[(g + f) * kC0S + k];
                xk[f] = f32x2(v, v);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint64_t w = ws[k][lane + 32 * j];
#pragma unroll
                for (int f = 0; f < kLnF; f++) acc[f][j] = fma_f32x2(xk[f], w, acc[f][j]);
            }
        }
        // the four frames' reductions interleaved (independent shuffle chains);
        // frames past the block's last are computed on zeros and not stored
        float mean[kLnF], r[kLnF];
#pragma unroll
        for (int f = 0; f < kLnF; f++) {
            uint64_t s2 = acc[f][0];
#pragma unroll
            for (int j = 1; j < 8; j++) s2 = add_f32x2(s2, acc[f][j]);
            float lo, hi;
            f32x2_split(s2, lo, hi);
            mean[f] = lo + hi;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int f = 0; f < kLnF; f++) mean[f] += __shfl_xor_sync(0xffffffffu, mean[f], o);
#pragma unroll
        for (int f = 0; f < kLnF; f++) {
            mean[f] *= kInvC;
            const uint64_t nm2 = f32x2(-mean[f], -mean[f]);
            uint64_t q2 = 0ull;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                acc[f][j] = add_f32x2(acc[f][j], nm2);   // centred in place
                q2 = fma_f32x2(acc[f][j], acc[f][j], q2);
            }
            float lo, hi;
            f32x2_split(q2, lo, hi);
            r[f] = lo + hi;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int f = 0; f < kLnF; f++) r[f] += __shfl_xor_sync(0xffffffffu, r[f], o);
#pragma unroll
        for (int f = 0; f < kLnF; f++) {
            if (g + f >= nf) break;
            const float rf = 1.f / sqrtf(r[f] * kInvC + 1e-5f);
            const uint64_t r2 = f32x2(rf, rf);
            uint32_t* dst = reinterpret_cast<uint32_t*>(orow + (long long)(g + f) * kLnC) + lane;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint64_t y2 = fma_f32x2(fma_f32x2(acc[f][j], r2, 0ull), g2[j], b2[j]);
                float lo, hi;
                f32x2_split(y2, lo, hi);
                dst[32 * j] = gelu_half2(lo, hi);
            }
        }
    }
}

static bool conv0_ln_supported(int C, int k0, int s0, int norm, const void* out) {
    return norm == 2 && C == kLnC && k0 == kC0K && s0 == kC0S && (reinterpret_cast<uintptr_t>(out) & 3) == 0;
}

// Vectorised row LayerNorm: warp per row, each lane holds NV groups of 4
// consecutive columns (D = 128 * NV); 16-byte fp32 / 8-byte fp16 accesses.
template <int NV>
__global__ void __launch_bounds__(256)
layer_norm_vec_kernel(const void* __restrict__ in, int in_f16, long long ld_in, long long in_batch_rows,
                      const int* __restrict__ rows, const long long* __restrict__ out_off, int n_batch, int n_rows,
                      const float* __restrict__ w, const float* __restrict__ b, int gelu, float* __restrict__ out32,
                      __half* __restrict__ out16, long long ld_out, float2* __restrict__ stats) {
    constexpr int D = 128 * NV;
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const long long rows_per_b = rows ? in_batch_rows : n_rows;
    const long long bi = gw / rows_per_b, r = gw % rows_per_b;
    if (bi >= n_batch) return;
    if (r >= (rows ? rows[bi] : n_rows)) return;
    const long long irow = bi * in_batch_rows + r;
    const long long orow = out_off ? out_off[bi] + r : irow;
    float v[NV][4];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int col = 4 * (lane + 32 * i);
        if (in_f16) {
            const uint2 p = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(in) + irow * ld_in + col);
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&p.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&p.y));
            v[i][0] = lo.x; v[i][1] = lo.y; v[i][2] = hi.x; v[i][3] = hi.y;
        } else {
            const float4 p = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in) + irow * ld_in + col);
            v[i][0] = p.x; v[i][1] = p.y; v[i][2] = p.z; v[i][3] = p.w;
        }
        s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) { const float d = v[i][j] - mean; q = fmaf(d, d, q); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.f / sqrtf(q / D + 1e-5f);
    if (stats && lane == 0) stats[orow] = make_float2(mean, inv);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int col = 4 * (lane + 32 * i);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + col));
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b + col));
        float y[4] = {(v[i][0] - mean) * inv * wv.x + bv.x, (v[i][1] - mean) * inv * wv.y + bv.y,
                      (v[i][2] - mean) * inv * wv.z + bv.z, (v[i][3] - mean) * inv * wv.w + bv.w};
        if (gelu) {
#pragma unroll
            for (int j = 0; j < 4; j++) y[j] = gelu_tanh(y[j]);
        }
        if (out32) *reinterpret_cast<float4*>(out32 + orow * ld_out + col) = make_float4(y[0], y[1], y[2], y[3]);
        if (out16) {
            uint2 p;
            p.x = pack_half2(y[0], y[1]);
            p.y = pack_half2(y[2], y[3]);
            *reinterpret_cast<uint2*>(out16 + orow * ld_out + col) = p;
        }
    }
}

// Post-LN statistics pass: fp32 rows [M, D] in; fp16 normalised rows and
// (mean, rstd) per row out.  Each warp owns RPW rows and issues all their
// loads (read-only path) before the first reduction, with the same two-pass
// arithmetic per row as layer_norm_vec_kernel: 5.5 TB/s at 31936 x 768.
template <int NV, int RPW>
__global__ void __launch_bounds__(256)
ln_stats_rows_kernel(const float* __restrict__ in, long long M, const float* __restrict__ w,
                     const float* __restrict__ b, __half* __restrict__ out16, float2* __restrict__ stats) {
    constexpr int D = 128 * NV;
    const long long row0 = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
    const int lane = threadIdx.x & 31;
    if (row0 >= M) return;
    float4 v[RPW][NV];
#pragma unroll
    for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int i = 0; i < NV; i++)
            v[r][i] = row0 + r < M ? __ldg(reinterpret_cast<const float4*>(in + (row0 + r) * D) + lane + 32 * i)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    float mean[RPW], inv[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) s += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
        mean[r] = s;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < RPW; r++) mean[r] += __shfl_xor_sync(0xffffffffu, mean[r], o);
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        mean[r] = mean[r] / D;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            float d = v[r][i].x - mean[r];
            q = fmaf(d, d, q);
            d = v[r][i].y - mean[r];
            q = fmaf(d, d, q);
            d = v[r][i].z - mean[r];
            q = fmaf(d, d, q);
            d = v[r][i].w - mean[r];
            q = fmaf(d, d, q);
        }
        inv[r] = q;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < RPW; r++) inv[r] += __shfl_xor_sync(0xffffffffu, inv[r], o);
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        inv[r] = 1.f / sqrtf(inv[r] / D + 1e-5f);
        if (lane == 0 && row0 + r < M) stats[row0 + r] = make_float2(mean[r], inv[r]);
    }
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int col = 4 * (lane + 32 * i);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + col));
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b + col));
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            if (row0 + r >= M) continue;
            uint2 p;
            p.x = pack_half2((v[r][i].x - mean[r]) * inv[r] * wv.x + bv.x, (v[r][i].y - mean[r]) * inv[r] * wv.y + bv.y);
            p.y = pack_half2((v[r][i].z - mean[r]) * inv[r] * wv.z + bv.z, (v[r][i].w - mean[r]) * inv[r] * wv.w + bv.w);
            *reinterpret_cast<uint2*>(out16 + (row0 + r) * D + col) = p;
        }
    }
}

// ── greedy CTC (src/ops.h:132-149) ───────────────────────────────────────────
// One block per utterance: per-frame argmax (strict >, first max wins), then a
// block-wide scan over run starts to emit spans {id, t_start, t_end}.
__global__ void ctc_greedy_kernel(const float* __restrict__ logits, const long long* __restrict__ off,
                                  const int* __restrict__ Tn, int V, int* __restrict__ ids,
                                  int* __restrict__ spans, int* __restrict__ n_spans) {
    __shared__ int warp_tot[32];
    __shared__ int carry_s;
    const int u = blockIdx.x;
    const int T = Tn[u];
    const long long base = off[u];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    // pass 1: argmax per frame
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float* row = logits + (base + t) * V;
        int best = 0;
        float bv = row[0];
        for (int v = 1; v < V; v++) {
            const float x = row[v];
            if (x > bv) { bv = x; best = v; }
        }
        ids[base + t] = best;
    }
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    // pass 2: run starts -> span index by exclusive scan
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        const int flag = (t < T) && (t == 0 || ids[base + t] != ids[base + t - 1]);
        int incl = flag;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) warp_tot[w] = incl;
        __syncthreads();
        int wbase = 0;
        for (int i = 0; i < w; i++) wbase += warp_tot[i];
        const int carry = carry_s;
        if (flag) {
            const int si = carry + wbase + incl - 1;
            spans[3 * (base + si)] = ids[base + t];
            spans[3 * (base + si) + 1] = t;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int tot = 0;
            for (int i = 0; i < nw; i++) tot += warp_tot[i];
            carry_s = carry + tot;
        }
        __syncthreads();
    }
    const int ns = carry_s;
    // pass 3: span ends = next span start (or T)
    for (int i = threadIdx.x; i < ns; i += blockDim.x)
        spans[3 * (base + i) + 2] = (i + 1 < ns) ? spans[3 * (base + i + 1) + 1] : T;
    if (threadIdx.x == 0) n_spans[u] = ns;
}

}  // namespace w2v

using namespace w2v;

static cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
static int launch_rc() { return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH; }

extern "C" int w2v_dequant_f16(const void* raw, int type, long long n_rows, long long K, void* out, void* stream) {
    if (n_rows <= 0 || K <= 0) return W2V_ERR_ARGS;
    const long long n = n_rows * K;
    if (type == 1) {
        return cudaMemcpyAsync(out, raw, n * 2, cudaMemcpyDeviceToDevice, S(stream)) == cudaSuccess ? W2V_OK
                                                                                                    : W2V_ERR_LAUNCH;
    }
    if (type == 0) {
        f32_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, S(stream)>>>((const float*)raw, n, (__half*)out);
        return launch_rc();
    }
    if ((type != 2 && type != 8) || K % 32) return W2V_ERR_ARGS;
    const long long nb = n / 32;
    dequant_q_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, S(stream)>>>((const uint8_t*)raw, type, nb,
                                                                          (__half*)out);
    return launch_rc();
}

extern "C" int w2v_repack_q(const void* raw, int type, long long n_rows, long long K, void* codes, void* scales,
                            long long ld_s, void* stream) {
    if ((type != 2 && type != 8) || n_rows <= 0 || K <= 0 || K % 64 || ld_s < n_rows ||
        (reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(scales) & 1))
        return W2V_ERR_ARGS;
    const long long nb = n_rows * (K / 32);
    repack_q_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, S(stream)>>>((const uint8_t*)raw, type, n_rows, K,
                                                                         (uint8_t*)codes, (uint16_t*)scales, ld_s);
    return launch_rc();
}

extern "C" int w2v_wave_stats(const float* audio, const long long* off, const int* len, int n_utt, float* stats,
                              void* stream) {
    if (n_utt <= 0) return W2V_OK;
    wave_stats_kernel<<<n_utt, 1024, 0, S(stream)>>>(audio, off, len, stats);
    return launch_rc();
}

extern "C" int w2v_conv0(const float* audio, const long long* off, const int* len, const int* frames, int n_utt,
                         const float* stats, const float* w0, const float* b0, int C, int k0, int s0, int norm,
                         const float* gw, const float* gb, double* gn_sums, void* out, long long rows_max,
                         int max_frames, int* err, void* stream) {
    if (C <= 0 || C > 512 || C % 2 || k0 > kC0MaxK || k0 <= 0 || s0 <= 0 || norm < 0 || norm > 2)
        return W2V_ERR_ARGS;
    if ((norm == 1 && !gn_sums) || (norm && (!gw || !gb))) return W2V_ERR_ARGS;
    if (n_utt <= 0 || max_frames <= 0) return W2V_OK;
    Conv0Args a{audio, off, len, frames, stats, w0, b0, C, k0, s0, norm, gw, gb, gn_sums, (__half*)out, rows_max,
                nullptr};
    const bool k10 = k0 == 10;
    if (conv0_ln_supported(C, k0, s0, norm, out)) {
        dim3 g((max_frames + kLnBlockFrames - 1) / kLnBlockFrames, n_utt);
        conv0_ln_kernel<<<g, kLnThreads, 0, S(stream)>>>(a);
        return launch_rc();
    }
    if (k0 == kC0K && s0 == kC0S && C % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0) {
        // published shape: 4 channels per thread, 8-frame register windows
        if (norm == 1) {
            // GroupNorm statistics from fp64 window moments.  gn_sums
            // ([n_utt][C][2] doubles) holds the (mean, 1/std) floats in its
            // first half and the per-chunk moment partials in its second.
            const int chunks = C / kGramN < 8 ? C / kGramN : 8;
            if (chunks >= 1) {
                float2* gnf = reinterpret_cast<float2*>(gn_sums);
                double* part = gn_sums + (size_t)n_utt * C;
                conv0_gram_kernel<<<dim3(chunks, n_utt), kGramThreads, 0, S(stream)>>>(audio, off, frames, chunks,
                                                                                        part);
                int rc = launch_rc();
                if (rc) return rc;
                const bool tc = conv0_tc_supported(C, k0, s0, norm, out);
                conv0_gram_finalize_kernel<<<n_utt, 512, 0, S(stream)>>>(part, chunks, stats, frames, w0, b0, C,
                                                                         tc ? gw : nullptr, tc ? gb : nullptr, gnf);
                rc = launch_rc();
                if (rc) return rc;
                a.gnf = gnf;
                if (tc) {
                    // tensor-core conv + GroupNorm affine + GELU
                    Conv0TcArgs t{audio, off, frames, stats, w0, b0, C, norm, gw, gb, gnf, (__half*)out, rows_max,
                                  n_utt, (max_frames + 127) / 128, err};
                    return launch_conv0_tc(t, S(stream));
                }
            } else {
                if (cudaMemsetAsync(gn_sums, 0, sizeof(double) * 2 * C * (size_t)n_utt, S(stream)) != cudaSuccess)
                    return W2V_ERR_LAUNCH;
                const size_t sh = (size_t)((kC0StatFrames - 1) * s0 + k0 + kC0MaxK + kC0Win) * sizeof(float);
                dim3 g((max_frames + kC0StatFrames - 1) / kC0StatFrames, n_utt);
                conv0x4_gn_stats_kernel<<<g, 128, sh, S(stream)>>>(a);
                int rc = launch_rc();
                if (rc) return rc;
            }
        }
        const size_t sh = (size_t)((kC0ApplyFrames - 1) * s0 + k0 + kC0MaxK + kC0Win) * sizeof(float);
        dim3 g((max_frames + kC0ApplyFrames - 1) / kC0ApplyFrames, n_utt);
        conv0x4_apply_kernel<<<g, 128, sh, S(stream)>>>(a);
        return launch_rc();
    }
    if (norm == 1) {
        if (cudaMemsetAsync(gn_sums, 0, sizeof(double) * 2 * C * (size_t)n_utt, S(stream)) != cudaSuccess)
            return W2V_ERR_LAUNCH;
        const size_t sh = (size_t)((kC0StatFrames - 1) * s0 + k0 + kC0MaxK + kC0Win) * sizeof(float);
        dim3 g((max_frames + kC0StatFrames - 1) / kC0StatFrames, n_utt);
        if (k10) conv0_gn_stats_kernel<10><<<g, 256, sh, S(stream)>>>(a);
        else conv0_gn_stats_kernel<kC0MaxK><<<g, 256, sh, S(stream)>>>(a);
        int rc = launch_rc();
        if (rc) return rc;
    }
    const size_t sh = (size_t)((kC0ApplyFrames - 1) * s0 + k0 + kC0MaxK + kC0Win) * sizeof(float);
    dim3 g((max_frames + kC0ApplyFrames - 1) / kC0ApplyFrames, n_utt);
    if (k10) conv0_apply_kernel<10><<<g, 256, sh, S(stream)>>>(a);
    else conv0_apply_kernel<kC0MaxK><<<g, 256, sh, S(stream)>>>(a);
    return launch_rc();
}

extern "C" int w2v_layer_norm(const void* in, int in_f16, long long ld_in, long long in_batch_rows, const int* rows,
                              const long long* out_off, int n_batch, int n_rows, int D, const float* w,
                              const float* b, int gelu, float* out32, void* out16, long long ld_out,
                              void* stream) {
    if (D % 32 || D > 64 * 32 || D <= 0) return W2V_ERR_ARGS;
    const long long total = rows ? (long long)n_batch * in_batch_rows : (long long)n_rows;
    if (total <= 0) return W2V_OK;
    const int warps = 8;
    const unsigned grid = (unsigned)((total + warps - 1) / warps);
    const int nb = rows ? n_batch : 1;
    const uintptr_t align = reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(w) |
                            reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out32) |
                            reinterpret_cast<uintptr_t>(out16);
    const bool vec_ok = D % 128 == 0 && (align % 16) == 0 && ld_in % 4 == 0 && ld_out % 4 == 0;
#define W2V_LN_VEC(NV)                                                                                          \
    case NV:                                                                                                    \
        layer_norm_vec_kernel<NV><<<grid, warps * 32, 0, S(stream)>>>(in, in_f16, ld_in, in_batch_rows, rows,    \
                                                                      out_off, nb, n_rows, w, b, gelu, out32,   \
                                                                      (__half*)out16, ld_out, nullptr);         \
        return launch_rc();
    if (vec_ok) {
        switch (D / 128) {
            W2V_LN_VEC(1) W2V_LN_VEC(2) W2V_LN_VEC(3) W2V_LN_VEC(4) W2V_LN_VEC(5) W2V_LN_VEC(6) W2V_LN_VEC(8)
            W2V_LN_VEC(10) W2V_LN_VEC(12) W2V_LN_VEC(16)
            default: break;
        }
    }
#undef W2V_LN_VEC
    if (D <= 16 * 32)
        layer_norm_kernel<16><<<grid, warps * 32, 0, S(stream)>>>(in, in_f16, ld_in, in_batch_rows, rows, out_off,
                                                                  nb, n_rows, D, w, b, gelu, out32,
                                                                  (__half*)out16, ld_out);
    else
        layer_norm_kernel<64><<<grid, warps * 32, 0, S(stream)>>>(in, in_f16, ld_in, in_batch_rows, rows, out_off,
                                                                  nb, n_rows, D, w, b, gelu, out32,
                                                                  (__half*)out16, ld_out);
    return launch_rc();
}

extern "C" int w2v_layer_norm_stats(const float* in, long long M, int D, const float* w, const float* b,
                                    void* out16, float* stats, void* stream) {
    if (D % 128 || D > 16 * 128 || D <= 0 || M < 0 || !in || !w || !b || !out16 || !stats) return W2V_ERR_ARGS;
    const uintptr_t align = reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(w) |
                            reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out16) |
                            reinterpret_cast<uintptr_t>(stats);
    if (align % 16) return W2V_ERR_ARGS;
    if (M == 0) return W2V_OK;
    const int warps = 8;
    constexpr int RPW = 1;   // measured at 31936 x 768: 26.7 us (1 row per warp), 27.8 us (2 rows)
    const unsigned grid = (unsigned)((M + warps * RPW - 1) / (warps * RPW));
    float2* st2 = reinterpret_cast<float2*>(stats);
#define W2V_LN_ST(NV)                                                                                           \
    case NV:                                                                                                    \
        ln_stats_rows_kernel<NV, RPW><<<grid, warps * 32, 0, S(stream)>>>(in, M, w, b, (__half*)out16, st2);    \
        return launch_rc();
    switch (D / 128) {
        W2V_LN_ST(1) W2V_LN_ST(2) W2V_LN_ST(3) W2V_LN_ST(4) W2V_LN_ST(5) W2V_LN_ST(6) W2V_LN_ST(8)
        W2V_LN_ST(10) W2V_LN_ST(12) W2V_LN_ST(16)
        default: return W2V_ERR_ARGS;
    }
#undef W2V_LN_ST
}

extern "C" int w2v_ctc_greedy(const float* logits, const long long* off, const int* T, int n_utt, int V, int* ids,
                              int* spans, int* n_spans, int max_T, void* stream) {
    if (V <= 0) return W2V_ERR_ARGS;
    if (n_utt <= 0) return W2V_OK;
    (void)max_T;
    ctc_greedy_kernel<<<n_utt, 256, 0, S(stream)>>>(logits, off, T, V, ids, spans, n_spans);
    return launch_rc();
}

// ── conv layer 0 for callers that cannot allocate device memory ─────────────
// Some hosts cannot call cudaMalloc once they are running: e.g. a process
// whose device memory is owned by another allocator, or a real-time audio
// thread that must not make a call that can block on the device.  For those
// callers this variant of w2v_conv0 keeps the GroupNorm statistics (its only
// scratch memory) in a fixed buffer compiled into this library instead of a
// caller-provided one.  The buffer is a file-scope __device__ array: every GPU
// that loads the library holds it (512 KiB) until the process exits.
namespace {
constexpr int kNoAllocMaxUtt = 64;        // utterances per call (GroupNorm models)
constexpr int kNoAllocMaxChannels = 512;  // conv channels
constexpr int kNoAllocMaxDevices = 64;
__device__ __align__(256) double g_conv0_gn_scratch[kNoAllocMaxUtt * kNoAllocMaxChannels * 2];

std::mutex g_scratch_mu;
double* g_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device (with that device current) and cached.
int scratch_address(double** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return W2V_ERR_LAUNCH;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_conv0_gn_scratch) != cudaSuccess || !p) return W2V_ERR_LAUNCH;
        g_scratch_addr[dev] = static_cast<double*>(p);
    }
    *out = g_scratch_addr[dev];
    return W2V_OK;
}
}  // namespace

extern "C" int w2v_conv0_noalloc(const float* audio, const long long* off, const int* len, const int* frames,
                                 int n_utt, const float* stats, const float* w0, const float* b0, int C, int k0,
                                 int s0, int norm, const float* gw, const float* gb, void* out, long long rows_max,
                                 int max_frames, int* err, void* stream) {
    double* gn = nullptr;
    if (C <= 0) return W2V_ERR_ARGS;
    if (norm == 1) {
        if (n_utt > kNoAllocMaxUtt || C > kNoAllocMaxChannels) return W2V_ERR_CAPACITY;
        const int rc = scratch_address(&gn);
        if (rc != W2V_OK) return rc;
    }
    // w2v_conv0 zeroes the statistics before accumulating into them.
    return w2v_conv0(audio, off, len, frames, n_utt, stats, w0, b0, C, k0, s0, norm, gw, gb, gn, out, rows_max,
                     max_frames, err, stream);
}
