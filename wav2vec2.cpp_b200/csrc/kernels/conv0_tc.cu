// Feature-extractor conv layer 0 on tcgen05 (src/wav2vec2.cpp:273-287 with
// src/ops.h:76-99 and, for GroupNorm models, src/ops.h:39-50; GELU
// src/ops.h:18-21), for the published first layer: kernel 10, stride 5,
// C in {256, 512} channels.
//
// y[f, c] = b[c] + sum_k w[c, k] xn[5f + k], xn = (x - mu) r the normalised
// waveform, as a GEMM with M = frames, N = channels, K = 10 taps (padded to
// 16).  fp32 accuracy from fp16 tensor-core operands: each operand is split
// into a high and a low fp16 part (v = hi + lo, |lo| <= 2^-11 |v|) and three
// K = 16 MMAs accumulate x_hi w_hi + x_lo w_hi + x_hi w_lo in fp32; the
// dropped x_lo w_lo term is below 2^-22 relative.
//
// Persistent CTAs walk tiles (utterance, 128-frame block, 256-channel half):
//   warps 0..3   build the A tile: one frame per thread, its 10 samples
//                normalised, split and written as two 8-tap chunks (K-major,
//                no swizzle, 16-byte rows); two tiles in flight
//   warp 4       one thread issues the MMAs into one of two TMEM accumulators
//   warps 5..20  epilogue (four warps per TMEM lane quarter, 64 channels
//                each): acc * scale + shift (bias and GroupNorm folded into
//                one per-channel affine by the statistics kernel) -> GELU ->
//                fp16, through the per-warp staging buffer so that stores
//                cover 4 frames x 64 bytes per instruction.
// The hi/lo weight operand (32 KB) is built in shared memory once per CTA.
// Every mbarrier wait is bounded.
#include "common.cuh"
#include "conv0_tc.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kC0tM = 128;                       // frames per tile
constexpr int kC0tN = 256;                       // channels per tile
constexpr int kC0tK = 10, kC0tS = 5;
constexpr int kC0tBuildWarps = 4, kC0tEpiWarps = 16;
constexpr int kC0tMmaWarp = kC0tBuildWarps;
constexpr int kC0tEpiWarp0 = kC0tBuildWarps + 1;
constexpr int kC0tThreads = 32 * (kC0tBuildWarps + 1 + kC0tEpiWarps);   // 672
constexpr int kC0tStages = 2;
constexpr int kC0tChunkA = kC0tM * 16;           // one 8-tap chunk of 128 rows: 2 KB
constexpr int kC0tABytes = 4 * kC0tChunkA;       // hi/lo x 2 chunks: 8 KB
constexpr int kC0tMaxC = 512;
constexpr int kC0tChunkB = kC0tMaxC * 16;        // one 8-tap chunk of 512 channels: 8 KB
constexpr int kC0tBBytes = 4 * kC0tChunkB;       // hi/lo x 2 chunks: 32 KB
constexpr int kC0tStageBytes = kC0tEpiWarps * 32 * 32 * 4;
constexpr int kC0tSmemUsed = kC0tBBytes + kC0tStages * kC0tABytes + kC0tStageBytes + 1024 + 128;
// Requested above half an SM's shared memory so no two CTAs share an SM:
// each allocates all 512 TMEM columns.
constexpr int kC0tSmem = kC0tSmemUsed > 120 * 1024 ? kC0tSmemUsed : 120 * 1024;

W2V_DEV void split_half(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

__global__ void __launch_bounds__(kC0tThreads, 1) conv0_tc_kernel(Conv0TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sB = smem;
    uint8_t* sA = sB + kC0tBBytes;
    float* stage_buf = reinterpret_cast<float*>(sA + kC0tStages * kC0tABytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kC0tStages * kC0tABytes + kC0tStageBytes);
    uint64_t* a_full = bars;                 // [kC0tStages]
    uint64_t* a_empty = bars + 2;            // [kC0tStages]
    uint64_t* t_full = bars + 4;             // [2]
    uint64_t* t_empty = bars + 6;            // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nh = a.C / kC0tN;
    const int total = a.n_utt * a.n_fb * nh;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kC0tStages; s++) { mbar_init(&a_full[s], kC0tBuildWarps); mbar_init(&a_empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&t_full[b], 1); mbar_init(&t_empty[b], kC0tEpiWarps); }
        fence_mbar_init();
    }
    // weights, split hi/lo: [hi|lo][tap chunk][channel][8 taps] (taps 10..15 zero)
    for (int i = threadIdx.x; i < a.C * 2; i += blockDim.x) {
        const int c = i >> 1, ch = i & 1;
        __half hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int k = ch * 8 + j;
            split_half(k < kC0tK ? __ldg(a.w0 + c * kC0tK + k) : 0.f, hi[j], lo[j]);
        }
        *reinterpret_cast<uint4*>(sB + (0 * 2 + ch) * kC0tChunkB + c * 16) = *reinterpret_cast<uint4*>(hi);
        *reinterpret_cast<uint4*>(sB + (1 * 2 + ch) * kC0tChunkB + c * 16) = *reinterpret_cast<uint4*>(lo);
    }
    fence_async_smem();
    if (warp == kC0tMmaWarp) { tmem_alloc(tmem_slot, 2 * kC0tN); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kC0tBuildWarps) {
        const int row = threadIdx.x;                       // 0..127
        int stage = 0;
        uint32_t phase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            const int rest = t / nh, fb = rest % a.n_fb, u = rest / a.n_fb;
            const int F = a.frames[u];
            if (fb * kC0tM >= F) continue;
            if (!mbar_wait(&a_empty[stage], phase ^ 1u, a.err)) break;
            const int f = fb * kC0tM + row;
            __half hi[16], lo[16];
#pragma unroll
            for (int k = 0; k < 16; k++) hi[k] = lo[k] = __float2half_rn(0.f);
            if (f < F) {
                const float mu = a.stats[2 * u], r = a.stats[2 * u + 1];
                const float* x = a.audio + a.off[u] + (long long)f * kC0tS;
#pragma unroll
                for (int k = 0; k < kC0tK; k++) split_half((__ldg(x + k) - mu) * r, hi[k], lo[k]);
            }
            uint8_t* dst = sA + stage * kC0tABytes + row * 16;
            *reinterpret_cast<uint4*>(dst + 0 * kC0tChunkA) = *reinterpret_cast<uint4*>(hi);
            *reinterpret_cast<uint4*>(dst + 1 * kC0tChunkA) = *reinterpret_cast<uint4*>(hi + 8);
            *reinterpret_cast<uint4*>(dst + 2 * kC0tChunkA) = *reinterpret_cast<uint4*>(lo);
            *reinterpret_cast<uint4*>(dst + 3 * kC0tChunkA) = *reinterpret_cast<uint4*>(lo + 8);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[stage]);
            if (++stage == kC0tStages) { stage = 0; phase ^= 1u; }
        }
    } else if (warp == kC0tMmaWarp) {
        if (elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(kC0tM, kC0tN);
            int stage = 0, it = 0;
            uint32_t phase = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                const int h = t % nh, rest = t / nh, fb = rest % a.n_fb, u = rest / a.n_fb;
                if (fb * kC0tM >= a.frames[u]) continue;
                const int ab = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&a_full[stage], phase, a.err)) break;
                if (!mbar_wait(&t_empty[ab], aph ^ 1u, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * kC0tN);
                const uint32_t a_hi = smem_u32(sA + stage * kC0tABytes), a_lo = a_hi + 2 * kC0tChunkA;
                const uint32_t b_hi = smem_u32(sB) + h * kC0tN * 16, b_lo = b_hi + 2 * kC0tChunkB;
                umma_f16(d, umma_desc_noswz(a_hi, kC0tChunkA, 128), umma_desc_noswz(b_hi, kC0tChunkB, 128), idesc, 0);
                umma_f16(d, umma_desc_noswz(a_lo, kC0tChunkA, 128), umma_desc_noswz(b_hi, kC0tChunkB, 128), idesc, 1);
                umma_f16(d, umma_desc_noswz(a_hi, kC0tChunkA, 128), umma_desc_noswz(b_lo, kC0tChunkB, 128), idesc, 1);
                umma_commit(&a_empty[stage]);
                umma_commit(&t_full[ab]);
                if (++stage == kC0tStages) { stage = 0; phase ^= 1u; }
                it++;
            }
            // no MMA may still be writing TMEM when it is freed
            if (it > 0) mbar_wait(&t_full[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, a.err);
        }
        __syncwarp();
    } else {
        const int ew = warp - kC0tEpiWarp0;                // 0..15
        const int q = warp & 3;                            // TMEM lane quarter
        const int cq = ew >> 2;                            // which 64 of the tile's 256 channels
        float* stg = stage_buf + ew * 32 * 32;
        const int cg = lane & 7, rs = lane >> 3;
        int it = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            const int h = t % nh, rest = t / nh, fb = rest % a.n_fb, u = rest / a.n_fb;
            const int F = a.frames[u];
            if (fb * kC0tM >= F) continue;
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            it++;
            if (!mbar_wait(&t_full[ab], aph, a.err)) break;
            tc_fence_after();
            const int f0 = fb * kC0tM + q * 32;            // frame of lane 0 / staged row 0
            __half* orow0 = a.out + ((long long)u * a.rows_max + f0) * a.C;
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                const int col = cq * 64 + c * 32;         // within the tile
                float v[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * kC0tN + col), v);
                __syncwarp();
                stage_put(stg, v);
                __syncwarp();
                // this thread's 4 channels: conv * scale + shift
                const int ch = h * kC0tN + col + 4 * cg;
                float sc[4], sh[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (a.norm == 1) {
                        const float2 g = __ldg(a.gnf + (long long)u * a.C + ch + j);
                        sc[j] = g.x;
                        sh[j] = g.y;
                    } else {
                        sc[j] = 1.f;
                        sh[j] = a.b0 ? __ldg(a.b0 + ch + j) : 0.f;
                    }
                }
                float4 xs[8];
#pragma unroll
                for (int i = 0; i < 8; i++) xs[i] = stage_get(stg, rs + 4 * i, cg);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int r = rs + 4 * i;
                    if (f0 + r < F) {
                        uint2 pk;
                        pk.x = gelu_half2(fmaf(xs[i].x, sc[0], sh[0]), fmaf(xs[i].y, sc[1], sh[1]));
                        pk.y = gelu_half2(fmaf(xs[i].z, sc[2], sh[2]), fmaf(xs[i].w, sc[3], sh[3]));
                        *reinterpret_cast<uint2*>(orow0 + (long long)r * a.C + ch) = pk;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_empty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kC0tMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * kC0tN);
    }
}

bool conv0_tc_supported(int C, int k0, int s0, int norm, const void* out) {
    return k0 == kC0tK && s0 == kC0tS && (C == 256 || C == 512) && (norm == 0 || norm == 1) &&
           (reinterpret_cast<uintptr_t>(out) & 7) == 0;
}

int launch_conv0_tc(const Conv0TcArgs& a, cudaStream_t st) {
    static bool attr[64] = {};
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(conv0_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kC0tSmem) !=
            cudaSuccess)
            return W2V_ERR_LAUNCH;
        cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
        if (sms[dev & 63] <= 0) sms[dev & 63] = 148;
        attr[dev & 63] = true;
    }
    const long long total = (long long)a.n_utt * a.n_fb * (a.C / kC0tN);
    const int grid = (int)(total < sms[dev & 63] ? total : sms[dev & 63]);
    if (grid <= 0) return W2V_OK;
    conv0_tc_kernel<<<grid, kC0tThreads, kC0tSmem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

}  // namespace w2v
