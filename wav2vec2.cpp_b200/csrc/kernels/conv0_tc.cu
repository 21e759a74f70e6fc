// Feature-extractor conv layer 0 on tcgen05 (src/wav2vec2.cpp:273-287 with
// src/ops.h:76-99 and, for GroupNorm models, src/ops.h:39-50; GELU
// src/ops.h:18-21), for the published first layer: kernel 10, stride 5,
// C in {256, 512} channels.
//
// z[f, c] = s[u, c] sum_k w[c, k] xn[5f + k] + t[u, c], xn = (x - mu) r the
// normalised waveform of utterance u, s and t the per-(utterance, channel)
// scale and shift into which the statistics kernel folds the conv bias and
// the GroupNorm (s = 1, t = bias without a norm).  The scale and shift are
// folded into the weights: the GEMM has M = frames, N = channels and K = 16
// taps, taps 0..9 = (w s, xn), tap 10 = (t, 1), taps 11..15 zero, so the
// accumulator already holds z and the epilogue is GELU alone.
// fp32 accuracy from fp16 tensor-core operands: each operand is split into a
// high and a low fp16 part (v = hi + lo, |lo| <= 2^-11 |v|) and three K = 16
// MMAs accumulate x_hi w_hi + x_lo w_hi + x_hi w_lo in fp32; the dropped
// x_lo w_lo term is below 2^-22 relative.
//
// Each CTA walks a contiguous range of tiles (utterance, 256-channel half,
// 128-frame block), frame blocks fastest, so the folded weights change only
// when the (utterance, half) group does:
//   warps 0..3   fold the weights of each new group into one of two shared
//                buffers; build the A tile: one frame per thread, its 10
//                samples normalised, split and written as two 8-tap chunks
//                (K-major, no swizzle, 16-byte rows); two tiles in flight
//   warp 4       one thread issues the MMAs into one of two TMEM accumulators
//   warps 5..20  epilogue, four warps per TMEM lane quarter and 64 channels
//                each: GELU -> fp16 into a 32-frame x 64-channel box in
//                shared memory (128-byte swizzle) -> TMA tile store.  The
//                box that crosses an utterance's last frame is stored row by
//                row instead, so no frame past the end is written.
// Every mbarrier wait is bounded.
#include "common.cuh"
#include "conv0_tc.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kC0tM = 128;                       // frames per tile
constexpr int kC0tN = 256;                       // channels per tile
constexpr int kC0tK = 10, kC0tS = 5;
constexpr int kC0tShiftTap = kC0tK;              // tap carrying the shift (A = 1)
constexpr int kC0tBuildWarps = 4, kC0tEpiWarps = 16;
constexpr int kC0tMmaWarp = kC0tBuildWarps;
constexpr int kC0tEpiWarp0 = kC0tBuildWarps + 1;
constexpr int kC0tThreads = 32 * (kC0tBuildWarps + 1 + kC0tEpiWarps);   // 672
constexpr int kC0tStages = 2;
constexpr int kC0tChunkA = kC0tM * 16;           // one 8-tap chunk of 128 frames: 2 KB
constexpr int kC0tABytes = 4 * kC0tChunkA;       // hi/lo x 2 chunks: 8 KB
constexpr int kC0tChunkB = kC0tN * 16;           // one 8-tap chunk of 256 channels: 4 KB
constexpr int kC0tBBytes = 4 * kC0tChunkB;       // hi/lo x 2 chunks: 16 KB per group
constexpr int kC0tBoxBytes = 32 * 128;           // 32 frames x 64 channels fp16
constexpr int kC0tOutBytes = kC0tEpiWarps * 2 * kC0tBoxBytes;            // two boxes per warp: 128 KB
constexpr int kC0tSmem = kC0tOutBytes + 2 * kC0tBBytes + kC0tStages * kC0tABytes + 1024 + 256;

W2V_DEV void split_half(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// Position in a CTA's tile range: group (utterance u, channel half h), frame
// block fb < nfb = ceil(frames[u] / 128); `left` tiles remain.
struct C0Walk {
    int u, h, fb, nfb, left;
};

W2V_DEV int c0_blocks(const Conv0TcArgs& a, int u) { return (a.frames[u] + kC0tM - 1) / kC0tM; }

// The tiles of CTA b: [b total / G, (b + 1) total / G) of the tiles of all
// utterances in the order (u, h, fb).
W2V_DEV C0Walk c0_walk_begin(const Conv0TcArgs& a, int nh) {
    long long total = 0;
    for (int u = 0; u < a.n_utt; u++) total += (long long)nh * c0_blocks(a, u);
    const long long s = total * blockIdx.x / gridDim.x, e = total * (blockIdx.x + 1) / gridDim.x;
    C0Walk w{a.n_utt, 0, 0, 0, (int)(e - s)};
    long long r = s;
    for (int u = 0; u < a.n_utt && w.left > 0; u++) {
        const int nfb = c0_blocks(a, u);
        if (r < (long long)nh * nfb) {
            w.u = u;
            w.h = (int)(r / nfb);
            w.fb = (int)(r % nfb);
            w.nfb = nfb;
            break;
        }
        r -= (long long)nh * nfb;
    }
    return w;
}

// Advance to the next tile; returns true if it starts a new group.
W2V_DEV bool c0_walk_next(const Conv0TcArgs& a, int nh, C0Walk& w) {
    w.left--;
    if (++w.fb < w.nfb) return false;
    w.fb = 0;
    if (++w.h < nh) return true;
    w.h = 0;
    do {
        w.u++;
    } while (w.u < a.n_utt && (w.nfb = c0_blocks(a, w.u)) == 0);
    return true;
}

__global__ void __launch_bounds__(kC0tThreads, 1)
conv0_tc_kernel(const __grid_constant__ CUtensorMap tmo, Conv0TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sOut = smem;                                  // 1024-aligned boxes
    uint8_t* sB = sOut + kC0tOutBytes;                     // [2 groups][hi|lo][tap chunk][channel][8 taps]
    uint8_t* sA = sB + 2 * kC0tBBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kC0tStages * kC0tABytes);
    uint64_t* a_full = bars;                 // [kC0tStages]
    uint64_t* a_empty = bars + 2;            // [kC0tStages]
    uint64_t* t_full = bars + 4;             // [2]
    uint64_t* t_empty = bars + 6;            // [2]
    uint64_t* b_free = bars + 8;             // [2] the MMAs reading a weight buffer are done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nh = a.C / kC0tN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kC0tStages; s++) { mbar_init(&a_full[s], kC0tBuildWarps); mbar_init(&a_empty[s], 1); }
        for (int b = 0; b < 2; b++) {
            mbar_init(&t_full[b], 1);
            mbar_init(&t_empty[b], kC0tEpiWarps);
            mbar_init(&b_free[b], 1);
        }
        fence_mbar_init();
        tma_prefetch_desc(&tmo);
    }
    if (warp == kC0tMmaWarp) { tmem_alloc(tmem_slot, 2 * kC0tN); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kC0tBuildWarps) {
        const int row = threadIdx.x;                       // 0..127
        int stage = 0, group = -1;
        uint32_t phase = 0;
        C0Walk w = c0_walk_begin(a, nh);
        bool new_group = true;
        while (w.left > 0) {
            if (new_group) {
                // fold (scale, shift) of the new group into its weight buffer,
                // once the MMAs of the group that last used the buffer are done
                group++;
                if (group >= 2 && !mbar_wait(&b_free[group & 1], (uint32_t)((group >> 1) - 1) & 1u, a.err)) break;
                uint8_t* bdst = sB + (group & 1) * kC0tBBytes;
#pragma unroll 1
                for (int cl = row; cl < kC0tN; cl += kC0tBuildWarps * 32) {
                    const int c = w.h * kC0tN + cl;
                    float sc = 1.f, sh = a.b0 ? __ldg(a.b0 + c) : 0.f;
                    if (a.norm == 1) {
                        const float2 g = __ldg(a.gnf + (long long)w.u * a.C + c);
                        sc = g.x;
                        sh = g.y;
                    }
                    __half hi[16], lo[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        const float v = k < kC0tK ? __ldg(a.w0 + c * kC0tK + k) * sc : (k == kC0tShiftTap ? sh : 0.f);
                        split_half(v, hi[k], lo[k]);
                    }
                    uint8_t* d = bdst + cl * 16;
                    *reinterpret_cast<uint4*>(d + 0 * kC0tChunkB) = *reinterpret_cast<uint4*>(hi);
                    *reinterpret_cast<uint4*>(d + 1 * kC0tChunkB) = *reinterpret_cast<uint4*>(hi + 8);
                    *reinterpret_cast<uint4*>(d + 2 * kC0tChunkB) = *reinterpret_cast<uint4*>(lo);
                    *reinterpret_cast<uint4*>(d + 3 * kC0tChunkB) = *reinterpret_cast<uint4*>(lo + 8);
                }
            }
            if (!mbar_wait(&a_empty[stage], phase ^ 1u, a.err)) break;
            const int F = a.frames[w.u];
            const int f = w.fb * kC0tM + row;
            __half hi[16], lo[16];
#pragma unroll
            for (int k = 0; k < 16; k++) hi[k] = lo[k] = __float2half_rn(0.f);
            hi[kC0tShiftTap] = __float2half_rn(1.f);
            if (f < F) {
                const float mu = a.stats[2 * w.u], r = a.stats[2 * w.u + 1];
                const float* x = a.audio + a.off[w.u] + (long long)f * kC0tS;
#pragma unroll
                for (int k = 0; k < kC0tK; k++) split_half((__ldg(x + k) - mu) * r, hi[k], lo[k]);
            }
            uint8_t* dst = sA + stage * kC0tABytes + row * 16;
            *reinterpret_cast<uint4*>(dst + 0 * kC0tChunkA) = *reinterpret_cast<uint4*>(hi);
            *reinterpret_cast<uint4*>(dst + 1 * kC0tChunkA) = *reinterpret_cast<uint4*>(hi + 8);
            *reinterpret_cast<uint4*>(dst + 2 * kC0tChunkA) = *reinterpret_cast<uint4*>(lo);
            *reinterpret_cast<uint4*>(dst + 3 * kC0tChunkA) = *reinterpret_cast<uint4*>(lo + 8);
            fence_async_smem();   // A and any new weights, before the MMA reads them
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[stage]);
            if (++stage == kC0tStages) { stage = 0; phase ^= 1u; }
            new_group = c0_walk_next(a, nh, w);
        }
    } else if (warp == kC0tMmaWarp) {
        if (elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(kC0tM, kC0tN);
            int stage = 0, it = 0, group = 0;
            uint32_t phase = 0;
            C0Walk w = c0_walk_begin(a, nh);
            while (w.left > 0) {
                const int ab = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&a_full[stage], phase, a.err)) break;
                if (!mbar_wait(&t_empty[ab], aph ^ 1u, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * kC0tN);
                const uint32_t a_hi = smem_u32(sA + stage * kC0tABytes), a_lo = a_hi + 2 * kC0tChunkA;
                const uint32_t b_hi = smem_u32(sB + (group & 1) * kC0tBBytes), b_lo = b_hi + 2 * kC0tChunkB;
                umma_f16(d, umma_desc_noswz(a_hi, kC0tChunkA, 128), umma_desc_noswz(b_hi, kC0tChunkB, 128), idesc, 0);
                umma_f16(d, umma_desc_noswz(a_lo, kC0tChunkA, 128), umma_desc_noswz(b_hi, kC0tChunkB, 128), idesc, 1);
                umma_f16(d, umma_desc_noswz(a_hi, kC0tChunkA, 128), umma_desc_noswz(b_lo, kC0tChunkB, 128), idesc, 1);
                umma_commit(&a_empty[stage]);
                umma_commit(&t_full[ab]);
                if (++stage == kC0tStages) { stage = 0; phase ^= 1u; }
                it++;
                if (c0_walk_next(a, nh, w)) {
                    umma_commit(&b_free[group & 1]);   // this group's weights are read for the last time
                    group++;
                }
            }
            // no MMA may still be writing TMEM when it is freed
            if (it > 0) mbar_wait(&t_full[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, a.err);
        }
        __syncwarp();
    } else {
        const int ew = warp - kC0tEpiWarp0;                // 0..15
        const int q = warp & 3;                            // TMEM lane quarter
        const int cq = ew >> 2;                            // which 64 of the tile's 256 channels
        uint8_t* box0 = sOut + ew * 2 * kC0tBoxBytes;
        const int r = lane;                                // frame within the box
        int it = 0;
        C0Walk w = c0_walk_begin(a, nh);
        for (; w.left > 0; c0_walk_next(a, nh, w)) {
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            uint8_t* box = box0 + ab * kC0tBoxBytes;
            it++;
            const int F = a.frames[w.u];
            const int f0 = w.fb * kC0tM + q * 32;          // frame of box row 0
            // the store issued from this box two tiles ago has finished reading it
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            if (!mbar_wait(&t_full[ab], aph, a.err)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                float v[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * kC0tN + cq * 64 + c * 32), v);
                if (c == 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&t_empty[ab]);
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint4 pk;
                    pk.x = gelu_half2(v[8 * j + 0], v[8 * j + 1]);
                    pk.y = gelu_half2(v[8 * j + 2], v[8 * j + 3]);
                    pk.z = gelu_half2(v[8 * j + 4], v[8 * j + 5]);
                    pk.w = gelu_half2(v[8 * j + 6], v[8 * j + 7]);
                    const int chunk = c * 4 + j;           // 16-byte chunk of the 128-byte row
                    *reinterpret_cast<uint4*>(box + r * 128 + ((chunk ^ (r & 7)) << 4)) = pk;
                }
            }
            const int col = w.h * kC0tN + cq * 64;
            if (f0 + 32 <= F) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tmo, box, col, f0, w.u);
                    bulk_commit_group();
                }
            } else {
                __syncwarp();
                if (f0 + r < F) {
                    uint4* dst = reinterpret_cast<uint4*>(a.out + ((long long)w.u * a.rows_max + f0 + r) * a.C + col);
#pragma unroll
                    for (int chunk = 0; chunk < 8; chunk++)
                        dst[chunk] = *reinterpret_cast<const uint4*>(box + r * 128 + ((chunk ^ (r & 7)) << 4));
                }
            }
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
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
           (reinterpret_cast<uintptr_t>(out) & 15) == 0;
}

static PFN_cuTensorMapEncodeTiled_v12000 c0_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
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
    const long long total = (long long)a.n_utt * a.n_fb * (a.C / kC0tN);   // upper bound on the tiles
    const int grid = (int)(total < sms[dev & 63] ? total : sms[dev & 63]);
    if (grid <= 0) return W2V_OK;
    // the output [n_utt][rows_max][C] fp16 as boxes of 64 channels x 32 frames
    auto enc = c0_encode_fn();
    if (!enc) return W2V_ERR_DRIVER;
    CUtensorMap tmo;
    const uint64_t dims[3] = {(uint64_t)a.C, (uint64_t)a.rows_max, (uint64_t)a.n_utt};
    const uint64_t strides[2] = {(uint64_t)a.C * 2, (uint64_t)a.rows_max * a.C * 2};
    const uint32_t box[3] = {64, 32, 1}, es[3] = {1, 1, 1};
    if (enc(&tmo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, a.out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return W2V_ERR_TENSOR_MAP;
    conv0_tc_kernel<<<grid, kC0tThreads, kC0tSmem, st>>>(tmo, a);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

}  // namespace w2v
