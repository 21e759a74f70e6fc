// Positional convolution embedding: grouped conv1d over time (kernel Kp,
// padding Kp/2, G groups, first T of the T+1 outputs), GELU, residual add
// (src/wav2vec2.cpp:349-356; conv src/ops.h:76-99).
//
// Implicit GEMM per (utterance, group, 128-frame tile): for every tap the A
// operand is the fp16 input window shifted by one row, read straight out of a
// shared-memory copy of the 128+Kp input rows with per-lane ldmatrix row
// addresses (no im2col); the B operand is that tap's [co][ci] weight slice,
// streamed through a double-buffered shared-memory ring.  fp16 operands,
// fp32 accumulation.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kPcRows = 128;   // output frames per block (8 warps x 16)

struct PosConvArgs {
    float* out; const float* xin; const long long* off; const int* Tn;
    int H, Kp, G, Cg, TC; const __half* wt; const float* bias;
};

template <int CG>
__global__ void __launch_bounds__(256)
pos_conv_kernel(PosConvArgs a) {
    constexpr int LDS = CG + 8;           // conflict-free ldmatrix row stride (halves)
    constexpr int NT = CG / 8, KS = CG / 16;
    extern __shared__ __align__(16) __half sm[];
    const int u = blockIdx.z, g = blockIdx.y;
    const int T = a.Tn[u];
    const int t0 = blockIdx.x * kPcRows;
    if (t0 >= T) return;
    const int Kp = a.Kp, TC = a.TC, half = Kp / 2;
    const int xrows = kPcRows + Kp;
    __half* sX = sm;
    __half* sW = sm + xrows * LDS;        // 2 chunks of TC*CG rows
    const int chunk_elems = TC * CG * LDS;
    const long long base = a.off[u];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    auto load_w = [&](int chunk, int buf) {
        const __half* src = a.wt + ((long long)g * Kp + (long long)chunk * TC) * CG * CG;
        __half* dst = sW + buf * chunk_elems;
        constexpr int CPR = CG / 8;      // 16-byte chunks per row
        for (int i = threadIdx.x; i < TC * CG * CPR; i += blockDim.x) {
            const int r = i / CPR, c = i % CPR;
            cp_async16(smem_u32(dst + r * LDS + c * 8), src + (long long)r * CG + c * 8);
        }
    };
    load_w(0, 0);
    cp_async_commit();

    // input window rows t0-half .. t0+kPcRows+half-1 (zero outside [0, T))
    for (int i = threadIdx.x; i < xrows * (CG / 4); i += blockDim.x) {
        const int r = i / (CG / 4), c4 = i % (CG / 4);
        const int t = t0 - half + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t >= 0 && t < T) v = *reinterpret_cast<const float4*>(a.xin + (base + t) * a.H + g * CG + c4 * 4);
        uint2 p;
        p.x = pack_half2(v.x, v.y);
        p.y = pack_half2(v.z, v.w);
        *reinterpret_cast<uint2*>(sX + r * LDS + c4 * 4) = p;
    }

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    const int n_chunks = Kp / TC;
    for (int ch = 0; ch < n_chunks; ch++) {
        cp_async_wait<0>();
        __syncthreads();
        if (ch + 1 < n_chunks) load_w(ch + 1, (ch + 1) & 1);
        cp_async_commit();
        const __half* cw = sW + (ch & 1) * chunk_elems;
        for (int tt = 0; tt < TC; tt++) {
            const int tap = ch * TC + tt;
            const __half* wtap = cw + tt * CG * LDS;
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
                uint32_t a0, a1, a2, a3;
                const int xr = warp * 16 + (lane & 15) + tap;
                ldsm_x4(smem_u32(sX + xr * LDS + ks * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < NT / 2; np++) {
                    const int co = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                    const int ci = ks * 16 + ((lane >> 3) & 1) * 8;
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(smem_u32(wtap + co * LDS + ci), b0, b1, b2, b3);
                    mma_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            }
        }
    }
    // epilogue: out = x + gelu(conv + bias), rows < T
    const int r0 = t0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int co = g * CG + nt * 8 + (lane & 3) * 2;
        const float b0 = a.bias[co], b1 = a.bias[co + 1];
        if (r0 < T) {
            const long long idx = (base + r0) * a.H + co;
            const float2 x = *reinterpret_cast<const float2*>(a.xin + idx);
            *reinterpret_cast<float2*>(a.out + idx) =
                make_float2(x.x + gelu_tanh(acc[nt][0] + b0), x.y + gelu_tanh(acc[nt][1] + b1));
        }
        if (r1 < T) {
            const long long idx = (base + r1) * a.H + co;
            const float2 x = *reinterpret_cast<const float2*>(a.xin + idx);
            *reinterpret_cast<float2*>(a.out + idx) =
                make_float2(x.x + gelu_tanh(acc[nt][2] + b0), x.y + gelu_tanh(acc[nt][3] + b1));
        }
    }
}

template <int CG>
static int launch_pc(PosConvArgs a, int n_utt, int max_T, cudaStream_t st) {
    // taps per weight chunk: a power of two dividing Kp, chunk <= 48 KB
    int tc = 1;
    while (tc * 2 <= a.Kp && a.Kp % (tc * 2) == 0 && (tc * 2) * CG * (CG + 8) * 2 <= 49152) tc *= 2;
    a.TC = tc;
    const size_t smem = ((size_t)(kPcRows + a.Kp) * (CG + 8) + 2 * (size_t)tc * CG * (CG + 8)) * 2;
    if (smem > 227 * 1024) return W2V_ERR_ARGS;
    if (cudaFuncSetAttribute(pos_conv_kernel<CG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return W2V_ERR_LAUNCH;
    dim3 grid((max_T + kPcRows - 1) / kPcRows, a.G, n_utt);
    pos_conv_kernel<CG><<<grid, 256, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

}  // namespace w2v

extern "C" int w2v_pos_conv(float* x, const float* xin, const long long* off, const int* T, int n_utt, int H,
                            int Kp, int G, const void* wt, const float* bias, int max_T, void* stream) {
    if (G <= 0 || H % G || Kp <= 0 || Kp % 2 || x == xin) return W2V_ERR_ARGS;
    if (n_utt <= 0 || max_T <= 0) return W2V_OK;
    w2v::PosConvArgs a{x, xin, off, T, H, Kp, G, H / G, 1, (const __half*)wt, bias};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (H / G) {
        case 32: return w2v::launch_pc<32>(a, n_utt, max_T, st);
        case 48: return w2v::launch_pc<48>(a, n_utt, max_T, st);
        case 64: return w2v::launch_pc<64>(a, n_utt, max_T, st);
        case 80: return w2v::launch_pc<80>(a, n_utt, max_T, st);
        default: return W2V_ERR_ARGS;
    }
}
