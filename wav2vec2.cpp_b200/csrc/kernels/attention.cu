// Bidirectional multi-head self-attention, flash-style (online softmax, the
// T x T score matrix never leaves registers).  Replaces the reference's
// per-head scores/softmax/PV triple loops (src/wav2vec2.cpp:304-334,
// softmax src/ops.h:101-106).  Ragged batches: each query attends only to the
// keys of its own utterance; rows outside [0, T_u) are zero-filled in shared
// memory and masked with -inf in the scores, which reproduces the reference's
// unpadded single-utterance computation.
//
// fp16 Q/K/V/P operands with fp32 accumulation and fp32 softmax statistics.
// Tile: 64 queries x 64 keys per step, 4 warps x 16 query rows, K/V double
// buffered with cp.async.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {

template <int D>
struct AttnCfg {
    static constexpr int kLds = D + 8;                 // smem row stride (halves), conflict-free ldmatrix
    static constexpr int kTile = 64 * kLds;            // halves per 64-row tile
    static constexpr int kSmem = 5 * kTile * 2;        // Q + 2 K + 2 V
};

template <int D>
W2V_DEV void load_tile(__half* s, const __half* g, long long ld, int row0, int T) {
    constexpr int kChunks = D / 8;                     // 16-byte chunks per row
    for (int i = threadIdx.x; i < 64 * kChunks; i += blockDim.x) {
        const int r = i / kChunks, c = i % kChunks;
        __half* dst = s + r * AttnCfg<D>::kLds + c * 8;
        if (row0 + r < T) cp_async16(smem_u32(dst), g + (long long)(row0 + r) * ld + c * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
}

template <int D>
__global__ void __launch_bounds__(128)
attn_kernel(const __half* __restrict__ qkv, __half* __restrict__ out, const long long* __restrict__ off,
            const int* __restrict__ Tn, int H, float scale_log2) {
    using Cfg = AttnCfg<D>;
    extern __shared__ __align__(16) __half sm[];
    __half* sQ = sm;
    __half* sK = sm + Cfg::kTile;          // 2 buffers
    __half* sV = sm + 3 * Cfg::kTile;      // 2 buffers
    const int u = blockIdx.z, h = blockIdx.y;
    const int T = Tn[u];
    const int q0 = blockIdx.x * 64;
    if (q0 >= T) return;
    const long long base = off[u];
    const long long ld = 3LL * H;
    const __half* Qg = qkv + base * ld + (long long)h * D;
    const __half* Kg = Qg + H;
    const __half* Vg = Qg + 2 * H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    load_tile<D>(sQ, Qg, ld, q0, T);
    load_tile<D>(sK, Kg, ld, 0, T);
    load_tile<D>(sV, Vg, ld, 0, T);
    cp_async_commit();

    constexpr int KS = D / 16;     // k16 steps over the head dim
    constexpr int NT = D / 8;      // n8 output tiles over the head dim
    uint32_t qa[KS][4];
    float o[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    const int n_kv = (T + 63) / 64;
    for (int j = 0; j < n_kv; j++) {
        cp_async_wait<0>();
        __syncthreads();
        if (j + 1 < n_kv) {
            const int nb = (j + 1) & 1;
            load_tile<D>(sK + nb * Cfg::kTile, Kg, ld, (j + 1) * 64, T);
            load_tile<D>(sV + nb * Cfg::kTile, Vg, ld, (j + 1) * 64, T);
        }
        cp_async_commit();
        if (j == 0) {
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
                const int r = warp * 16 + (lane & 15), c = ks * 16 + (lane >> 4) * 8;
                ldsm_x4(smem_u32(sQ + r * Cfg::kLds + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
            }
        }
        const __half* cK = sK + (j & 1) * Cfg::kTile;
        const __half* cV = sV + (j & 1) * Cfg::kTile;

        // S = Q K^T for 16 rows x 64 keys
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int c = ks * 16 + ((lane >> 3) & 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(cK + key * Cfg::kLds + c), b0, b1, b2, b3);
                mma_16816(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
                mma_16816(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
            }
        }
        // mask keys beyond the utterance
        const int kbase = j * 64;
        if (kbase + 64 > T) {
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                const int k = kbase + nt * 8 + (lane & 3) * 2;
                if (k >= T) { s[nt][0] = -INFINITY; s[nt][2] = -INFINITY; }
                if (k + 1 >= T) { s[nt][1] = -INFINITY; s[nt][3] = -INFINITY; }
            }
        }
        // online softmax (rows r0 = lane/4, r1 = lane/4 + 8 of this warp's 16)
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
            mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
        }
#pragma unroll
        for (int o2 = 1; o2 < 4; o2 <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o2));
        }
        const float c0 = exp2f((m0 - mx0) * scale_log2), c1 = exp2f((m1 - mx1) * scale_log2);
        m0 = mx0; m1 = mx1;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            s[nt][0] = exp2f((s[nt][0] - mx0) * scale_log2);
            s[nt][1] = exp2f((s[nt][1] - mx0) * scale_log2);
            s[nt][2] = exp2f((s[nt][2] - mx1) * scale_log2);
            s[nt][3] = exp2f((s[nt][3] - mx1) * scale_log2);
            rs0 += s[nt][0] + s[nt][1];
            rs1 += s[nt][2] + s[nt][3];
        }
        l0 = l0 * c0 + rs0;
        l1 = l1 * c1 + rs1;
#pragma unroll
        for (int i = 0; i < NT; i++) { o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1; }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint32_t a0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);
            const uint32_t a1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            const uint32_t a2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            const uint32_t a3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < NT / 2; dp++) {
                const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int c = dp * 16 + (lane >> 4) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_u32(cV + key * Cfg::kLds + c), b0, b1, b2, b3);
                mma_16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
                mma_16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
            }
        }
    }
    // finalise: full row sums across the quad, normalise, store fp16
#pragma unroll
    for (int o2 = 1; o2 < 4; o2 <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
    }
    const float i0 = 1.f / l0, i1 = 1.f / l1;
    const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
    __half* O = out + base * (long long)H + (long long)h * D;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int c = nt * 8 + (lane & 3) * 2;
        if (r0 < T) *reinterpret_cast<__half2*>(O + (long long)r0 * H + c) = __floats2half2_rn(o[nt][0] * i0, o[nt][1] * i0);
        if (r1 < T) *reinterpret_cast<__half2*>(O + (long long)r1 * H + c) = __floats2half2_rn(o[nt][2] * i1, o[nt][3] * i1);
    }
}

template <int D>
static int launch_attn(const void* qkv, void* out, const long long* off, const int* T, int n_utt, int H,
                       int n_heads, int max_T, cudaStream_t st) {
    using Cfg = AttnCfg<D>;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) !=
            cudaSuccess)
            return W2V_ERR_LAUNCH;
        attr[dev & 63] = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    dim3 grid((max_T + 63) / 64, n_heads, n_utt);
    attn_kernel<D><<<grid, 128, Cfg::kSmem, st>>>((const __half*)qkv, (__half*)out, off, T, H, scale_log2);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

}  // namespace w2v

extern "C" int w2v_attention(const void* qkv, void* out, const long long* off, const int* T, int n_utt, int H,
                             int n_heads, int max_T, void* stream) {
    if (n_heads <= 0 || H % n_heads) return W2V_ERR_ARGS;
    if (n_utt <= 0 || max_T <= 0) return W2V_OK;
    const int d = H / n_heads;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (d) {
        case 64: return w2v::launch_attn<64>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        case 80: return w2v::launch_attn<80>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        case 128: return w2v::launch_attn<128>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        default: return W2V_ERR_ARGS;
    }
}
