// Persistent warp-specialised tcgen05 GEMM for sm_100a:  C = epi(A . B^T).
//
// Replaces every linear of the reference (ggml_mul_mat through
// GgmlScratch::linear, src/ggml_backend.h:78-120; call sites
// src/wav2vec2.cpp:300-302,336,347,368-370,386-388,489) and, through a
// strided 3-D view of A, the stride-s convolutions 1..6 of the feature
// extractor (src/ops.h:76-99 via src/wav2vec2.cpp:273-287) as implicit GEMMs.
//
//   A  fp16, K-major, read through a 4-D TMA view (channel, phase, row group,
//      batch) of a [rows][Cin] activation: K index = tap*Cin + ci of output
//      row t is input row t*s + tap = s*(t + tap/s) + tap%s, i.e. view
//      coordinate (ci, tap%s, t + tap/s, b).  Plain GEMMs use taps = s = 1.
//      The conv windows are therefore read in place (no im2col).
//   B  fp16 [N, K] row-major (weights, dequantized once at load time).
//   D  fp32 accumulators in TMEM, two buffers so the epilogue of tile i
//      overlaps the MMAs of tile i+1.
//
// Roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: STAGES-deep smem ring, mbarrier full/empty.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2..9  epilogue: tcgen05.ld -> bias / GELU / residual -> global;
//               two warps per TMEM lane quarter, each taking half the columns.
// Every mbarrier wait is bounded (common.cuh); on expiry the kernel records
// an error code and returns.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kBM = 128;       // tile rows (UMMA M)
constexpr int kBK = 64;        // K per stage (128 B of fp16: one swizzle row)
constexpr int kUmmaK = 16;     // K per tcgen05.mma kind::f16
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;

struct GemmParams {
    int vec;              // 16-byte vector stores/loads are aligned for this C / resid
    int kb_per_tap;       // Cin / 64
    int conv_stride;      // s (1 for plain GEMMs)
    int m_valid;          // valid rows per batch
    int m_tiles;          // tiles per batch along rows
    int n_batch;
    int N;
    int n_tiles;
    int k_blocks;
    void* C;
    long long ldc;        // elements
    long long c_batch_rows;
    const float* bias;
    const float* resid;
    long long ldr;
    int* err;
};

template <int BN>
struct GemmCfg {
    static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int kSmem = kStages * (kABytes + kBBytes) + 1024 + 256;
};

template <int EPI>
W2V_DEV void epilogue_chunk(const GemmParams& p, long long out_row, long long res_row, int col0, float (&v)[32]) {
    const int ncol = p.vec ? min(32, p.N - col0) : -1;   // -1: scalar path
    if (p.bias) {
        if (ncol == 32) {
            const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 b = __ldg(b4 + j);
                v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
            }
        } else {
            
#pragma unroll
            for (int j = 0; j < 32; j++) if (col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
        }
    }
    if (EPI == W2V_EPI_F16_GELU) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = gelu_tanh(v[j]);
    }
    if (EPI == W2V_EPI_F32_RESID) {
        const float* r = p.resid + res_row * p.ldr + col0;
        if (ncol == 32) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 x = *reinterpret_cast<const float4*>(r + 4 * j);
                v[4 * j] += x.x; v[4 * j + 1] += x.y; v[4 * j + 2] += x.z; v[4 * j + 3] += x.w;
            }
        } else {
            
#pragma unroll
            for (int j = 0; j < 32; j++) if (col0 + j < p.N) v[j] += r[j];
        }
    }
    if (EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU) {
        __half* c = reinterpret_cast<__half*>(p.C) + out_row * p.ldc + col0;
        if (ncol == 32) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint4 u;
                u.x = pack_half2(v[8 * j + 0], v[8 * j + 1]);
                u.y = pack_half2(v[8 * j + 2], v[8 * j + 3]);
                u.z = pack_half2(v[8 * j + 4], v[8 * j + 5]);
                u.w = pack_half2(v[8 * j + 6], v[8 * j + 7]);
                reinterpret_cast<uint4*>(c)[j] = u;
            }
        } else {
            
#pragma unroll
            for (int j = 0; j < 32; j++) if (col0 + j < p.N) c[j] = __float2half_rn(v[j]);
        }
    } else {
        float* c = reinterpret_cast<float*>(p.C) + out_row * p.ldc + col0;
        if (ncol == 32) {
#pragma unroll
            for (int j = 0; j < 8; j++)
                reinterpret_cast<float4*>(c)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
            
#pragma unroll
            for (int j = 0; j < 32; j++) if (col0 + j < p.N) c[j] = v[j];
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = bars + 2 * S + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.n_batch * p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], kEpiWarps); }
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const int ni = tile % p.n_tiles;
                const int rest = tile / p.n_tiles;
                const int mi = rest % p.m_tiles, b = rest / p.m_tiles;
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[stage], Cfg::kABytes + Cfg::kBBytes);
                    const int tap = kb / p.kb_per_tap, cb = kb - tap * p.kb_per_tap;
                    tma_load_4d(sA + stage * Cfg::kABytes, &tmA, &full[stage], cb * kBK, tap % p.conv_stride,
                                mi * kBM + tap / p.conv_stride, b);
                    tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, &full[stage], kb * kBK, ni * BN);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
            }
            // Never leave the CTA with a bulk copy still writing its smem.
            for (int s = 0; s < S; s++)
                if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, p.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(kBM, BN);
            int stage = 0, it = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, it++) {
                const int ab = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&tempty[ab], aph ^ 1u, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * BN);
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * Cfg::kABytes);
                    const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; kk++) {
                        umma_f16(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                                 (kb | kk) != 0);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
                if (ok) umma_commit(&tfull[ab]);
            }
        }
        __syncwarp();
    } else {
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;       // which half of the tile's columns
        constexpr int kChunks = BN / 32 / 2;    // 32-column chunks per warp
        const int r_in_tile = q * 32 + lane;
        int it = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, it++) {
            const int ni = tile % p.n_tiles;
            const int rest = tile / p.n_tiles;
            const int mi = rest % p.m_tiles, b = rest / p.m_tiles;
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            if (!mbar_wait(&tfull[ab], aph, p.err)) break;
            tc_fence_after();
            const int row = mi * kBM + r_in_tile;
            const bool valid = row < p.m_valid;
            const long long out_row = (long long)b * p.c_batch_rows + row;
#pragma unroll 1
            for (int c = half * kChunks; c < (half + 1) * kChunks; c++) {
                float v[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN + c * 32), v);
                const int col0 = ni * BN + c * 32;
                if (valid && col0 < p.N) epilogue_chunk<EPI>(p, out_row, out_row, col0, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// Self-test of the bounded wait: one thread waits on an mbarrier that nothing
// ever arrives on; the wait expires after limit_ns, records the error code and
// the kernel returns normally (no trap), leaving the context usable.
__global__ void wait_selftest_kernel(int* err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait_for(&bar, 0, err, limit_ns);
}

// ── host side ───────────────────────────────────────────────────────────────

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// fp16 tensor map, 128-byte swizzle, innermost box of 64 elements.
static int make_map_f16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box) {
    auto enc = get_encode();
    if (!enc) return W2V_ERR_DRIVER;
    uint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), dims, strides_bytes, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? W2V_OK : W2V_ERR_TENSOR_MAP;
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int BN, int EPI>
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    using Cfg = GemmCfg<BN>;
    auto kern = gemm_tc_kernel<BN, EPI>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) != cudaSuccess)
            return W2V_ERR_LAUNCH;
        attr_set[dev & 63] = true;
    }
    const int total = p.n_batch * p.m_tiles * p.n_tiles;
    const int grid = total < sm_count() ? total : sm_count();
    kern<<<grid, kThreads, Cfg::kSmem, st>>>(ta, tb, p);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

template <int EPI>
static int launch_epi(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    switch (bn) {
        case 256: return launch_bn<256, EPI>(ta, tb, p, st);
        case 128: return launch_bn<128, EPI>(ta, tb, p, st);
        default: return launch_bn<64, EPI>(ta, tb, p, st);
    }
}

// Pick the N tile: the widest of 256/128/64 dividing N (64 covers small or
// ragged N through TMA zero fill), preferring fewer wasted wave slots.
static int pick_bn(int N, long long m_tiles_total) {
    const int sms = sm_count();
    int best = 64;
    double best_cost = 1e30;
    for (int bn : {256, 128, 64}) {
        if (N % bn != 0 && bn != 64) continue;
        const long long tiles = m_tiles_total * ((N + bn - 1) / bn);
        const long long waves = (tiles + sms - 1) / sms;
        // time ~ waves * per-tile time (proportional to bn), plus a small
        // penalty for narrower tiles (more A re-reads, less MMA efficiency)
        const double cost = (double)waves * bn * (bn == 64 ? 1.15 : (bn == 128 ? 1.05 : 1.0));
        if (cost < best_cost) { best_cost = cost; best = bn; }
    }
    return best;
}

}  // namespace w2v

using namespace w2v;

extern "C" int w2v_selftest_wait_timeout(int* err, int limit_ms, void* stream) {
    if (!err || limit_ms <= 0 || limit_ms > 2000) return W2V_ERR_ARGS;
    wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        err, (unsigned long long)limit_ms * 1000000ull);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

extern "C" int w2v_gemm_f16(const void* A, long long a_cin, int a_taps, int a_stride, long long a_row_stride,
                            long long a_rows_in, long long a_batches, long long a_batch_stride, const void* B,
                            int N, void* C, long long ldc, long long c_batch_rows, int m_valid, const float* bias,
                            const float* resid, long long ldr, int epilogue, int block_n, int* err,
                            void* stream) {
    if (a_cin % kBK != 0 || a_cin <= 0 || a_taps <= 0 || a_stride <= 0 || N <= 0 || a_rows_in <= 0 ||
        a_batches <= 0 || m_valid < 0 || a_row_stride < a_cin)
        return W2V_ERR_ARGS;
    if ((a_row_stride * 2) % 16 || (a_batch_stride * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15) ||
        (reinterpret_cast<uintptr_t>(B) & 15) || a_rows_in % a_stride)
        return W2V_ERR_ARGS;
    if (a_batches > 1 && a_batch_stride < a_rows_in * a_row_stride) return W2V_ERR_ARGS;
    if (m_valid == 0) return W2V_OK;
    // every row an output row < m_valid needs must exist in the view
    if ((long long)(m_valid - 1) * a_stride + a_taps - 1 >= a_rows_in) return W2V_ERR_ARGS;
    CUtensorMap ta, tb;
    const long long groups = a_rows_in / a_stride;
    const long long bstride = a_batches > 1 ? a_batch_stride : a_rows_in * a_row_stride;
    const uint64_t adims[4] = {(uint64_t)a_cin, (uint64_t)a_stride, (uint64_t)groups, (uint64_t)a_batches};
    const uint64_t astr[3] = {(uint64_t)a_row_stride * 2, (uint64_t)a_row_stride * a_stride * 2,
                              (uint64_t)bstride * 2};
    const uint32_t abox[4] = {kBK, 1, kBM, 1};
    int rc = make_map_f16(&ta, A, 4, adims, astr, abox);
    if (rc) return rc;
    const long long K = a_cin * a_taps;
    GemmParams p;
    p.kb_per_tap = (int)(a_cin / kBK);
    p.conv_stride = a_stride;
    p.m_valid = m_valid;
    p.m_tiles = (int)((m_valid + kBM - 1) / kBM);
    p.n_batch = (int)a_batches;
    p.N = N;
    int bn = block_n ? block_n : pick_bn(N, (long long)p.m_tiles * p.n_batch);
    if (bn != 256 && bn != 128 && bn != 64) return W2V_ERR_ARGS;
    p.n_tiles = (N + bn - 1) / bn;
    p.k_blocks = (int)(K / kBK);
    p.C = C;
    p.ldc = ldc;
    p.c_batch_rows = c_batch_rows;
    p.bias = bias;
    p.resid = resid;
    p.ldr = ldr;
    p.err = err;
    {
        const bool f16 = epilogue == W2V_EPI_F16 || epilogue == W2V_EPI_F16_GELU;
        const uintptr_t cb = reinterpret_cast<uintptr_t>(C), rb = reinterpret_cast<uintptr_t>(resid),
                        bb = reinterpret_cast<uintptr_t>(bias);
        p.vec = (ldc % (f16 ? 8 : 4) == 0) && (cb % 16 == 0) && (!resid || (ldr % 4 == 0 && rb % 16 == 0)) &&
                (!bias || bb % 16 == 0);
    }
    const uint64_t bdims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t bstr[1] = {(uint64_t)K * 2};
    const uint32_t bbox[2] = {kBK, (uint32_t)bn};
    rc = make_map_f16(&tb, B, 2, bdims, bstr, bbox);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (epilogue) {
        case W2V_EPI_F16: return launch_epi<W2V_EPI_F16>(bn, ta, tb, p, st);
        case W2V_EPI_F16_GELU: return launch_epi<W2V_EPI_F16_GELU>(bn, ta, tb, p, st);
        case W2V_EPI_F32: return launch_epi<W2V_EPI_F32>(bn, ta, tb, p, st);
        case W2V_EPI_F32_RESID:
            if (!resid) return W2V_ERR_ARGS;
            return launch_epi<W2V_EPI_F32_RESID>(bn, ta, tb, p, st);
        default: return W2V_ERR_ARGS;
    }
}
