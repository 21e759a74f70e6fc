// Positional convolution embedding: grouped conv1d over time (kernel Kp,
// padding Kp/2, G groups, first T of the T+1 outputs), GELU, residual add
// (src/wav2vec2.cpp:349-356; conv src/ops.h:76-99).
//
// tcgen05 implicit GEMM.  One CTA per (utterance, group, 128 * kTiles - 1
// output frames): kTiles 128-frame tiles, each a TMEM accumulator of 2 Cg fp32
// columns (M = 128, N = 2 Cg, K = Kp/2 tap pairs x Cg).  The CTA's fp16 input
// window (128 kTiles + Kp frames x Cg channels, zero outside the utterance) is
// staged once in shared memory in the K-major no-swizzle layout with a
// 16-byte row pitch:
//   [Cg/8 channel chunks][window rows][8 channels]
// Core matrices (8 rows x 16 B) are then contiguous at ANY row offset, so
// the A operand of tap k for tile r is the same window addressed k rows
// further on: no im2col and no reload per tap.
// Two taps share each MMA: B stacks the weights of taps 2p and 2p+1 along N,
// laid out at load time as [G][Kp/2][Cg/8][2 Cg (tap 2p's co, then tap
// 2p+1's)][8 (ci)] fp16, and A is the window at tap 2p.  The first Cg columns
// of a tile then hold sum_p win[i + 2p] W_2p and the second Cg
// sum_p win[i + 2p] W_2p+1, which is tap 2p+1's contribution to frame i - 1:
//   out[i] = acc_even[i] + acc_odd[i + 1].
// Each MMA reads its 128-row A slice once for twice the columns, halving the
// shared-memory reads per flop that bound the one-tap form (N = Cg).  The
// last accumulator row only feeds the row before it, so a CTA outputs
// 128 kTiles - 1 frames.  The weights stream through a shared-memory ring, one
// tap pair per bulk copy.
// Roles (192 threads): warp 0 bulk-copies weights; warp 1 issues the MMAs;
// warps 2..5 stage the input window, then drain the accumulators:
// out = xin + gelu(acc + bias); the row-shifted odd sums move down one lane
// by shuffle, and across warps and tiles through shared memory.  fp16
// operands, fp32 accumulation.  Every mbarrier wait is bounded.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kPcTaps = 2;                  // taps per weight stage (one stacked pair)
constexpr int kPcMaxKp = 128;

template <int CG>
struct PcCfg {
    // Two 128-frame tiles per CTA and two CTAs per SM where TMEM (2 x 2 CG
    // columns) and shared memory allow, so one CTA's window staging and
    // epilogue overlap the other's MMAs; three tiles and one CTA otherwise.
    static constexpr int kTiles = CG <= 64 ? 2 : 3;           // 128-frame accumulator tiles of 2 CG columns
    static constexpr int kMinBlocks = CG <= 64 ? 2 : 1;
    static constexpr int kFrames = 128 * kTiles - 1;          // output frames per CTA
    static constexpr int kChunks = CG / 8;                    // 16-byte channel chunks
    static constexpr int kWinRows = 128 * kTiles + kPcMaxKp;  // staged rows (the last one or two unused)
    static constexpr int kChunkA = kWinRows * 16;             // bytes per window chunk
    static constexpr int kABytes = kChunks * kChunkA;
    static constexpr int kPairBytes = 2 * CG * CG * 2;        // one tap pair, stacked along N
    static constexpr int kChunkB = 2 * CG * 16;               // one 8-channel chunk of a pair
    static constexpr int kStageBytes = (kPcTaps / 2) * kPairBytes;
    static constexpr int kEdgeBytes = kTiles * 4 * CG * 4;    // odd sums of each warp's first row, per tile
    static constexpr int kBudget = (kMinBlocks == 2 ? 115712 : 232448) - kABytes - kEdgeBytes - 1024 - 128;
    static constexpr int kStages = kBudget / kStageBytes >= 4 ? 4 : kBudget / kStageBytes;
    static constexpr int kSmem = kABytes + kStages * kStageBytes + kEdgeBytes + 1024 + 128;
    static constexpr int kTmemCols = kTiles * 2 * CG <= 128 ? 128 : kTiles * 2 * CG <= 256 ? 256 : 512;
    static_assert(kTiles * 2 * CG <= 512 && (kMinBlocks == 1 || kTmemCols <= 256), "TMEM");
    static_assert(kStages >= 2, "shared memory");
};

struct PosConvArgs {
    float* out; const float* xin; const long long* off; const int* Tn;
    int H, Kp, G; const __half* wt; const float* bias; int* err;
};

W2V_DEV void epi_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }   // the four epilogue warps

template <int CG>
__global__ void __launch_bounds__(192, PcCfg<CG>::kMinBlocks) pos_conv_tc_kernel(PosConvArgs a) {
    using Cfg = PcCfg<CG>;
    const int u = blockIdx.z, g = blockIdx.y;
    const int T = a.Tn[u];
    const int t0 = blockIdx.x * Cfg::kFrames;
    if (t0 >= T) return;
    const int n_out = min(Cfg::kFrames, T - t0);          // frames this CTA writes
    const int n_tiles = (n_out + 1 + 127) / 128;          // accumulator rows 0 .. n_out (the last feeds n_out - 1)
    const int Kp = a.Kp, half = Kp / 2;
    const long long base = a.off[u];
    const int n_stages_total = Kp / kPcTaps;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sA = smem;
    uint8_t* sB = smem + Cfg::kABytes;
    float* edge = reinterpret_cast<float*>(sB + Cfg::kStages * Cfg::kStageBytes);   // [tile][quarter][CG]
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(edge) + Cfg::kEdgeBytes);
    uint64_t* full = bars;                          // [kStages]
    uint64_t* empty = bars + Cfg::kStages;          // [kStages]
    uint64_t* a_ready = bars + 2 * Cfg::kStages;
    uint64_t* acc_full = a_ready + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(a_ready, 4);
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            const uint8_t* wg = reinterpret_cast<const uint8_t*>(a.wt) + (size_t)g * (Kp / 2) * Cfg::kPairBytes;
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            for (int i = 0; i < n_stages_total; i++) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, a.err)) break;
                mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
                bulk_load(sB + stage * Cfg::kStageBytes, wg + (size_t)i * Cfg::kStageBytes, Cfg::kStageBytes,
                          &full[stage]);
                issued |= 1u << stage;
                last_par = (last_par & ~(1u << stage)) | (phase << stage);
                if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
            }
            for (int s = 0; s < Cfg::kStages; s++)
                if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, a.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(128, 2 * CG);
            // Descriptors are built once and advanced by adding (byte offset >> 4)
            // to their start-address field (shared memory < 256 KB: no carry out of
            // the field), keeping the single issuing thread's work per MMA to an add.
            const uint64_t a_desc0 = umma_desc_noswz(smem_u32(sA), Cfg::kChunkA, 128);
            const uint64_t b_desc0 = umma_desc_noswz(smem_u32(sB), Cfg::kChunkB, 128);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = mbar_wait(a_ready, 0, a.err);
            for (int i = 0; i < n_stages_total && ok; i++) {
                if (!mbar_wait(&full[stage], phase, a.err)) break;
                tc_fence_after();
                const uint64_t b_stage = b_desc0 + (uint64_t)((stage * Cfg::kStageBytes) >> 4);
#pragma unroll
                for (int pp = 0; pp < kPcTaps / 2; pp++) {
                    const int p = i * (kPcTaps / 2) + pp;               // tap pair: taps 2p, 2p + 1
                    const uint64_t a_tap = a_desc0 + (uint64_t)(2 * p);  // window rows from tap 2p (16 B each)
#pragma unroll
                    for (int s = 0; s < CG / 16; s++) {
                        const uint64_t bd =
                            b_stage + (uint64_t)((pp * Cfg::kPairBytes + 2 * s * Cfg::kChunkB) >> 4);
                        const uint32_t acc = (p | s) != 0;
#pragma unroll
                        for (int r = 0; r < Cfg::kTiles; r++)
                            if (r < n_tiles)
                                umma_f16(tmem_base + (uint32_t)(r * 2 * CG),
                                         a_tap + (uint64_t)((2 * s * Cfg::kChunkA + r * 128 * 16) >> 4), bd, idesc,
                                         acc);
                    }
                }
                umma_commit(&empty[stage]);
                if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
            }
            umma_commit(acc_full);   // also on error: completes once the issued MMAs have
        }
        __syncwarp();
    } else {
        // stage the input window: row w is frame t0 - Kp/2 + w, zero outside [0, T)
        const int et = threadIdx.x - 64;                       // 0..127
        const int rows = 128 * Cfg::kTiles + Kp;
        const int n_items = rows * Cfg::kChunks;
        constexpr int kBatch = 6;                              // loads in flight per thread
        for (int i0 = et; i0 < n_items; i0 += 128 * kBatch) {
            float4 v[kBatch][2];
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                const int i = i0 + j * 128;
                const int w = i % rows, c = i / rows;
                const int t = t0 - half + w;
                v[j][0] = v[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < n_items && t >= 0 && t < T) {
                    const float4* src = reinterpret_cast<const float4*>(a.xin + (base + t) * a.H + g * CG + c * 8);
                    v[j][0] = __ldg(src);
                    v[j][1] = __ldg(src + 1);
                }
            }
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                const int i = i0 + j * 128;
                if (i < n_items) {
                    const int w = i % rows, c = i / rows;
                    uint4 p;
                    p.x = pack_half2(v[j][0].x, v[j][0].y);
                    p.y = pack_half2(v[j][0].z, v[j][0].w);
                    p.z = pack_half2(v[j][1].x, v[j][1].y);
                    p.w = pack_half2(v[j][1].z, v[j][1].w);
                    *reinterpret_cast<uint4*>(sA + c * Cfg::kChunkA + w * 16) = p;
                }
            }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_ready);

        // epilogue: out[i] = xin[i] + gelu(acc_even[i] + acc_odd[i + 1] + bias) for frames < T
        const int q = warp & 3;
        const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16);
        const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, a.err));   // warp-uniform for the shuffles
        if (ok) {
            tc_fence_after();
            // the odd sums of each warp's first row, for the lane above it (previous warp or tile)
            for (int r = 0; r < n_tiles; r++) {
#pragma unroll
                for (int c = 0; c < CG / 16; c++) {
                    float v[16];
                    tmem_ld16(tq + (uint32_t)(r * 2 * CG + CG + c * 16), v);
                    if (lane == 0) {
#pragma unroll
                        for (int i = 0; i < 16; i++) edge[(r * 4 + q) * CG + c * 16 + i] = v[i];
                    }
                }
            }
        }
        epi_barrier();
        if (ok) {
            const float* bias = a.bias + g * CG;
            for (int r = 0; r < n_tiles; r++) {
                const int i_row = r * 128 + q * 32 + lane;             // row within the CTA
                const int t = t0 + i_row;
                const long long idx = (base + t) * a.H + g * CG;
                // lane 31's next row: the first row of the next warp's quarter, or of the next tile
                const bool has_nx = q < 3 || r + 1 < n_tiles;
                const float* nx = edge + (has_nx ? (q < 3 ? r * 4 + q + 1 : (r + 1) * 4) : 0) * CG;
#pragma unroll
                for (int c = 0; c < CG / 16; c++) {
                    float ve[16], vo[16];
                    tmem_ld16(tq + (uint32_t)(r * 2 * CG + c * 16), ve);
                    tmem_ld16(tq + (uint32_t)(r * 2 * CG + CG + c * 16), vo);
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float dn = __shfl_down_sync(0xffffffffu, vo[i], 1);
                        ve[i] += lane < 31 ? dn : (has_nx ? nx[c * 16 + i] : 0.f);
                    }
                    if (i_row < n_out) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 x = *reinterpret_cast<const float4*>(a.xin + idx + c * 16 + j);
                            const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c * 16 + j));
                            float4 o;
                            o.x = x.x + gelu_tanh(ve[j] + b.x);
                            o.y = x.y + gelu_tanh(ve[j + 1] + b.y);
                            o.z = x.z + gelu_tanh(ve[j + 2] + b.z);
                            o.w = x.w + gelu_tanh(ve[j + 3] + b.w);
                            *reinterpret_cast<float4*>(a.out + idx + c * 16 + j) = o;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

template <int CG>
static int launch_pc(const PosConvArgs& a, int n_utt, int max_T, cudaStream_t st) {
    using Cfg = PcCfg<CG>;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(pos_conv_tc_kernel<CG>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) !=
            cudaSuccess)
            return W2V_ERR_LAUNCH;
        attr[dev & 63] = true;
    }
    dim3 grid((max_T + Cfg::kFrames - 1) / Cfg::kFrames, a.G, n_utt);
    pos_conv_tc_kernel<CG><<<grid, 192, Cfg::kSmem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

}  // namespace w2v

extern "C" int w2v_pos_conv(float* x, const float* xin, const long long* off, const int* T, int n_utt, int H,
                            int Kp, int G, const void* wt, const float* bias, int max_T, int* err, void* stream) {
    if (G <= 0 || H % G || Kp <= 0 || Kp % w2v::kPcTaps || Kp > w2v::kPcMaxKp || x == xin) return W2V_ERR_ARGS;
    if ((reinterpret_cast<uintptr_t>(wt) & 15) || (reinterpret_cast<uintptr_t>(xin) & 15) ||
        (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(bias) & 15))
        return W2V_ERR_ARGS;
    if (n_utt <= 0 || max_T <= 0) return W2V_OK;
    w2v::PosConvArgs a{x, xin, off, T, H, Kp, G, (const __half*)wt, bias, err};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (H / G) {
        case 32: return w2v::launch_pc<32>(a, n_utt, max_T, st);
        case 48: return w2v::launch_pc<48>(a, n_utt, max_T, st);
        case 64: return w2v::launch_pc<64>(a, n_utt, max_T, st);
        case 80: return w2v::launch_pc<80>(a, n_utt, max_T, st);
        default: return W2V_ERR_ARGS;
    }
}
