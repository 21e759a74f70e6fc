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
// Roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: STAGES-deep smem ring, mbarrier full/empty.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2..9  epilogue: tcgen05.ld -> bias / GELU / residual -> global (fp16
//               C through per-warp TMA tile stores where its layout allows,
//               fp32 C through the staged coalesced stores below); two
//               warps per TMEM lane quarter, each taking half of the tile's
//               columns.
// Every mbarrier wait is bounded (common.cuh); on expiry the kernel records
// an error code and returns.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {

constexpr int kBM = 128;       // tile rows (UMMA M)
constexpr int kBK = 64;        // K per stage (128 B of fp16: one swizzle row)
constexpr int kUmmaK = 16;     // K per tcgen05.mma kind::f16
// Epilogue warps: 8 (two per TMEM lane quarter) for every epilogue.  The
// fp16 ones (TMA tile stores, GELU on fp16 pairs) are short enough that more
// warps buy nothing, while the 4 KB of staging a warp holds is shared memory
// the TMA ring can use: at 8 warps a CTA pair with 256-wide tiles keeps six
// stages in flight instead of five (QKV 96.2 -> 93.7 us at 31936 rows).
__host__ __device__ constexpr int epi_warps(int) { return 8; }
__host__ __device__ constexpr int gemm_threads(int epi) { return 64 + 32 * epi_warps(epi); }
constexpr int kSmemCap = 232448;        // opt-in dynamic shared memory per block on sm_100
__host__ __device__ constexpr int fit_stages(int want, int stage_bytes, int fixed_bytes) {
    return (kSmemCap - fixed_bytes) / stage_bytes < want ? (kSmemCap - fixed_bytes) / stage_bytes : want;
}

struct GemmParams {
    int vec;              // 16-byte vector stores/loads are aligned for this C / resid
    int tma_c;            // fp16 C is written by TMA tile stores (tensor map tmC)
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
    const float2* ln_stats;   // W2V_EPI_F32_RESID_LN: per resid row (mean, rstd)
    const float* ln_w;
    const float* ln_b;
};

template <int BN, int NE>
struct GemmCfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = NE * 32 * 32 * 4;   // epilogue staging, 4 KB per warp
    static constexpr int kStages = fit_stages(BN == 256 ? 4 : BN == 192 ? 4 : BN == 128 ? 6 : 8, kABytes + kBBytes,
                                              kStageBytes + 1024 + 256);
    // two accumulators; TMEM is allocated in powers of two columns
    static constexpr int kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static constexpr int kSmem = kStages * (kABytes + kBBytes) + kStageBytes + 1024 + 256;
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

// ── coalesced epilogue (fp32 outputs, and fp16 ones TMA cannot store) ──────
// tcgen05.ld 32x32b gives a thread one row; storing that directly makes each
// warp instruction touch 32 rows.  Instead each epilogue warp stages its
// 32 x 32 fp32 chunk in a private 4 KB shared buffer (float4 groups XOR-
// swizzled by row, so the row-per-thread writes and the 8-threads-per-row
// reads are both bank-conflict free) and then works on 4 rows x 32 columns
// per instruction: thread t owns column group t%8 of rows t/8 + 4i.

// Residual of this thread's 8 (row, 4-column) cells of a chunk; rows past
// m_valid and columns past N read as zero.
template <int EPI>
W2V_DEV void load_resid_t(const GemmParams& p, long long out_row0, int row0, int col0, float4 (&res)[8]) {
    const int lane = threadIdx.x & 31, cg = lane & 7, rs = lane >> 3;
    const int col = col0 + 4 * cg;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = rs + 4 * i;
        res[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row0 + r < p.m_valid) {
            const float* src = p.resid + (out_row0 + r) * p.ldr + col;
            if (col + 3 < p.N) res[i] = *reinterpret_cast<const float4*>(src);
            else {
                if (col < p.N) res[i].x = src[0];
                if (col + 1 < p.N) res[i].y = src[1];
                if (col + 2 < p.N) res[i].z = src[2];
            }
        }
    }
}

// W2V_EPI_F32_RESID_LN: the (mean, rstd) of this thread's 8 rows of the tile
// (rows t/8 + 4i of the warp's 32), fetched once per tile.
W2V_DEV void load_ln_stats_t(const GemmParams& p, long long out_row0, int row0, float2 (&st)[8]) {
    const int rs = (threadIdx.x & 31) >> 3;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = rs + 4 * i;
        st[i] = row0 + r < p.m_valid ? p.ln_stats[out_row0 + r] : make_float2(0.f, 0.f);
    }
}

template <int EPI>
W2V_DEV void epilogue_chunk_t(const GemmParams& p, const float* stg, long long out_row0, int row0, int col0,
                              const float4 (&res)[8], const float2 (&st)[8]) {
    const int lane = threadIdx.x & 31, cg = lane & 7, rs = lane >> 3;
    const int col = col0 + 4 * cg;
    if (col >= p.N) return;
    const bool full4 = col + 3 < p.N;
    float4 lw = make_float4(0.f, 0.f, 0.f, 0.f), lb = lw;
    if (EPI == W2V_EPI_F32_RESID_LN) {
        if (full4) {
            lw = __ldg(reinterpret_cast<const float4*>(p.ln_w + col));
            lb = __ldg(reinterpret_cast<const float4*>(p.ln_b + col));
        } else {
            lw.x = __ldg(p.ln_w + col); lb.x = __ldg(p.ln_b + col);
            if (col + 1 < p.N) { lw.y = __ldg(p.ln_w + col + 1); lb.y = __ldg(p.ln_b + col + 1); }
            if (col + 2 < p.N) { lw.z = __ldg(p.ln_w + col + 2); lb.z = __ldg(p.ln_b + col + 2); }
        }
    }
    float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.bias) {
        if (full4) b = __ldg(reinterpret_cast<const float4*>(p.bias + col));
        else {
            b.x = __ldg(p.bias + col);
            if (col + 1 < p.N) b.y = __ldg(p.bias + col + 1);
            if (col + 2 < p.N) b.z = __ldg(p.bias + col + 2);
        }
    }
    // all shared-memory reads before any global store (which the compiler
    // cannot prove disjoint from them), so the 32 cells compute in parallel
    float4 xs[8];
#pragma unroll
    for (int i = 0; i < 8; i++) xs[i] = stage_get(stg, rs + 4 * i, cg);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4& x = xs[i];
        x.x += b.x; x.y += b.y; x.z += b.z; x.w += b.w;
        if (EPI == W2V_EPI_F32_RESID) {
            x.x += res[i].x; x.y += res[i].y; x.z += res[i].z; x.w += res[i].w;
        }
        if (EPI == W2V_EPI_F32_RESID_LN) {
            // the LayerNorm this raw residual row stands for (same expression as the row LayerNorm kernel)
            x.x += (res[i].x - st[i].x) * st[i].y * lw.x + lb.x;
            x.y += (res[i].y - st[i].x) * st[i].y * lw.y + lb.y;
            x.z += (res[i].z - st[i].x) * st[i].y * lw.z + lb.z;
            x.w += (res[i].w - st[i].x) * st[i].y * lw.w + lb.w;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = rs + 4 * i;
        if (row0 + r >= p.m_valid) continue;
        const float4 x = xs[i];
        const long long orow = out_row0 + r;
        if (EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU) {
            __half* c = reinterpret_cast<__half*>(p.C) + orow * p.ldc + col;
            if (full4) {
                uint2 u;
                if (EPI == W2V_EPI_F16_GELU) {
                    u.x = gelu_half2(x.x, x.y);
                    u.y = gelu_half2(x.z, x.w);
                } else {
                    u.x = pack_half2(x.x, x.y);
                    u.y = pack_half2(x.z, x.w);
                }
                *reinterpret_cast<uint2*>(c) = u;
            } else {
                const bool g = EPI == W2V_EPI_F16_GELU;
                c[0] = __float2half_rn(g ? gelu_tanh(x.x) : x.x);
                if (col + 1 < p.N) c[1] = __float2half_rn(g ? gelu_tanh(x.y) : x.y);
                if (col + 2 < p.N) c[2] = __float2half_rn(g ? gelu_tanh(x.z) : x.z);
            }
        } else {
            float* c = reinterpret_cast<float*>(p.C) + orow * p.ldc + col;
            if (full4) *reinterpret_cast<float4*>(c) = x;
            else {
                c[0] = x.x;
                if (col + 1 < p.N) c[1] = x.y;
                if (col + 2 < p.N) c[2] = x.z;
            }
        }
    }
}

// One epilogue warp's share of an accumulator: TMEM lane quarter q (rows
// row0 .. row0+31 of the batch), 32-column chunks c0 .. c1-1.
template <int EPI>
W2V_DEV void epilogue_warp(const GemmParams& p, uint32_t tmem_row, float* stg, long long out_row0, int row0,
                           int col_base, int c0, int c1, float4 (&res)[8], const float2 (&st)[8]) {
    const int lane = threadIdx.x & 31;
    if (!p.vec) {
        // unaligned C or residual: row-per-thread scalar path
        const bool valid = row0 + lane < p.m_valid;
#pragma unroll 1
        for (int c = c0; c < c1; c++) {
            float v[32];
            tmem_ld32(tmem_row + (uint32_t)(c * 32), v);
            const int col0 = col_base + c * 32;
            if (valid && col0 < p.N) epilogue_chunk<EPI>(p, out_row0 + lane, out_row0 + lane, col0, v);
        }
        return;
    }
#pragma unroll 1
    for (int c = c0; c < c1; c++) {
        float v[32];
        tmem_ld32(tmem_row + (uint32_t)(c * 32), v);
        const int col0 = col_base + c * 32;
        float4 cur[8];
#pragma unroll
        for (int i = 0; i < 8; i++) cur[i] = res[i];
        // next chunk's residual loads are in flight while this chunk is stored
        if ((EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN) && c + 1 < c1 && col0 + 32 < p.N)
            load_resid_t<EPI>(p, out_row0, row0, col0 + 32, res);
        __syncwarp();
        stage_put(stg, v);
        __syncwarp();
        epilogue_chunk_t<EPI>(p, stg, out_row0, row0, col0, cur, st);
    }
    __syncwarp();
}

// fp16 epilogues with a TMA-store-able C: each 32 x 32 chunk goes, as fp16,
// into one of the warp's two 2 KB boxes (32 rows of 64 bytes, 64-byte swizzle:
// 16-byte group j of row r at j ^ ((r >> 1) & 3), so the row-per-thread
// writes are bank-conflict free) and leaves by one TMA tile store.  The
// tensor map's bounds (N columns, m_valid rows per batch) clip the rows and
// columns of a box that starts inside the tensor; a box that would start past
// the last row (lane quarters beyond m_valid in the last row tile) is never
// stored.  nst counts this warp's stores (box parity); a box is rewritten
// only after the store issued from it two stores earlier has read it.
template <int EPI>
W2V_DEV void epilogue_warp_tma(const GemmParams& p, const CUtensorMap* tmC, uint32_t tmem_row, uint8_t* box0,
                               int row0, int b, int col_base, int c0, int c1, uint32_t& nst) {
    const int lane = threadIdx.x & 31;
    if (row0 >= p.m_valid) return;   // every row of this warp's quarter is past the end
#pragma unroll 1
    for (int c = c0; c < c1; c++) {
        const int col0 = col_base + c * 32;
        if (col0 >= p.N) break;
        float v[32];
        tmem_ld32(tmem_row + (uint32_t)(c * 32), v);
        if (p.bias) {
            if (col0 + 32 <= p.N) {
                const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 bb = __ldg(b4 + j);
                    v[4 * j] += bb.x; v[4 * j + 1] += bb.y; v[4 * j + 2] += bb.z; v[4 * j + 3] += bb.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) if (col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
            }
        }
        uint8_t* box = box0 + (nst & 1u) * 2048;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint4 pk;
            if (EPI == W2V_EPI_F16_GELU) {
                pk.x = gelu_half2(v[8 * j + 0], v[8 * j + 1]);
                pk.y = gelu_half2(v[8 * j + 2], v[8 * j + 3]);
                pk.z = gelu_half2(v[8 * j + 4], v[8 * j + 5]);
                pk.w = gelu_half2(v[8 * j + 6], v[8 * j + 7]);
            } else {
                pk.x = pack_half2(v[8 * j + 0], v[8 * j + 1]);
                pk.y = pack_half2(v[8 * j + 2], v[8 * j + 3]);
                pk.z = pack_half2(v[8 * j + 4], v[8 * j + 5]);
                pk.w = pack_half2(v[8 * j + 6], v[8 * j + 7]);
            }
            *reinterpret_cast<uint4*>(box + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = pk;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_3d(tmC, box, col0, row0, b);
            bulk_commit_group();
        }
        nst++;
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, GemmParams p) {
    constexpr int NE = epi_warps(EPI);
    using Cfg = GemmCfg<BN, NE>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    float* stage_buf = reinterpret_cast<float*>(sB + S * Cfg::kBBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes + Cfg::kStageBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = bars + 2 * S + 2;
    uint64_t* done = bars + 2 * S + 4;    // every MMA this CTA issued has completed (teardown)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.n_batch * p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], NE); }
        mbar_init(done, 1);
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
            // no MMA may still be writing TMEM when it is freed (also after an expired wait)
            umma_commit(done);
            mbar_wait(done, 0, p.err);
        }
        __syncwarp();
    } else {
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        // NE/4 warps per TMEM lane quarter, each taking a contiguous share of the 32-column chunks
        const int part = (warp - 2) >> 2;
        constexpr int kNch = BN / 32, kParts = NE / 4;
        const int cb = part * kNch / kParts, ce = (part + 1) * kNch / kParts;
        float* stg = stage_buf + (warp - 2) * 32 * 32;
        constexpr bool kF16 = EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU;
        uint32_t nst = 0;   // TMA stores issued by this warp
        int it = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, it++) {
            const int ni = tile % p.n_tiles;
            const int rest = tile / p.n_tiles;
            const int mi = rest % p.m_tiles, b = rest / p.m_tiles;
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            const int row0 = mi * kBM + q * 32;
            const long long out_row0 = (long long)b * p.c_batch_rows + row0;
            const int c0 = cb;
            float4 res[8];
            float2 lst[8];
            // the residual does not depend on the MMA: fetch it while the MMA runs
            if ((EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN) && p.vec && c0 < ce && ni * BN + c0 * 32 < p.N)
                load_resid_t<EPI>(p, out_row0, row0, ni * BN + c0 * 32, res);
            if (EPI == W2V_EPI_F32_RESID_LN) load_ln_stats_t(p, out_row0, row0, lst);
            if (!mbar_wait(&tfull[ab], aph, p.err)) break;
            tc_fence_after();
            const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
            if constexpr (kF16) {
                if (p.tma_c)
                    epilogue_warp_tma<EPI>(p, &tmC, trow, reinterpret_cast<uint8_t*>(stg), row0, b, ni * BN, c0, ce,
                                           nst);
                else
                    epilogue_warp<EPI>(p, trow, stg, out_row0, row0, ni * BN, c0, ce, res, lst);
            } else {
                epilogue_warp<EPI>(p, trow, stg, out_row0, row0, ni * BN, c0, ce, res, lst);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);
        }
        if (kF16 && p.tma_c) {   // the stores are complete before the CTA exits
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ── CTA-pair variant (tcgen05 cta_group::2) ─────────────────────────────────
// A cluster of two CTAs computes a 256 x BN output tile.  Each CTA stages its
// own 128 rows of A and BN/2 rows of B; the even CTA (the leader) issues
// tcgen05.mma with M = 256, which reads the operands from both CTAs' shared
// memory and writes rows 0..127 of the accumulator into the leader's TMEM and
// rows 128..255 into the peer's.  Per SM this stages BN/2 instead of BN rows
// of B for the same MMA work, cutting L2->SM operand traffic by a third at
// BN = 256.
//   full[s]   leader only: armed by the leader with both CTAs' bytes; both
//             CTAs' TMA loads complete on it (peer through a cluster address)
//   empty[s]  each CTA: the leader's MMA commit arrives on both
//   tfull[b]  each CTA: accumulator b of this CTA's rows is ready
//   tempty[b] leader: the epilogue warps of both CTAs have drained accumulator b
//   done      leader: every MMA the leader issued has completed (teardown)
template <int BN, int NE>
struct Gemm2Cfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = (BN / 2) * kBK * 2;
    static constexpr int kStageBytes = NE * 32 * 32 * 4;
    static constexpr int kStages = fit_stages(BN == 256 ? 6 : BN == 192 ? 6 : 8, kABytes + kBBytes,
                                              kStageBytes + 1024 + 256);
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
    static constexpr int kSmem = kStages * (kABytes + kBBytes) + kStageBytes + 1024 + 256;
};

template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm_threads(EPI), 1)
gemm2_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, GemmParams p) {
    constexpr int NE = epi_warps(EPI);
    using Cfg = Gemm2Cfg<BN, NE>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    // identical offset in both CTAs: the MMA addresses the peer's operands
    // at the leader's shared-memory offsets
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    float* stage_buf = reinterpret_cast<float*>(sB + S * Cfg::kBBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes + Cfg::kStageBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = bars + 2 * S + 2;
    uint64_t* done = bars + 2 * S + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int total = p.n_batch * p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 2 * NE); }
        mbar_init(done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) { tmem_alloc_pair(tmem_slot, Cfg::kTmemCols); tmem_relinquish_pair(); }
    tc_fence_before();
    cluster_sync_all();    // barriers of both CTAs initialised before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            for (int tile = pair; tile < total && ok; tile += n_pairs) {
                const int ni = tile % p.n_tiles;
                const int rest = tile / p.n_tiles;
                const int mi = rest % p.m_tiles, b = rest / p.m_tiles;
                const int row0 = (mi * 2 + (int)rank) * kBM;
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) { ok = false; break; }
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::kABytes + Cfg::kBBytes));
                    const int tap = kb / p.kb_per_tap, cb = kb - tap * p.kb_per_tap;
                    const uint32_t fb = full_lead + (uint32_t)(stage * 8);
                    tma_load_4d_pair(sA + stage * Cfg::kABytes, &tmA, fb, cb * kBK, tap % p.conv_stride,
                                     row0 + tap / p.conv_stride, b);
                    tma_load_2d_pair(sB + stage * Cfg::kBBytes, &tmB, fb, kb * kBK, ni * BN + (int)rank * (BN / 2));
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
            }
            // The leader's full barriers count both CTAs' bytes: once they
            // have completed no bulk copy of the pair is still writing.  The
            // peer leaves only after the closing cluster barrier, i.e. after
            // this drain.
            if (rank == 0)
                for (int s = 0; s < S; s++)
                    if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, p.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(2 * kBM, BN);
            const uint32_t empty_peer = mapa_shared(smem_u32(empty), 1);
            const uint32_t tfull_peer = mapa_shared(smem_u32(tfull), 1);
            int stage = 0, it = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total && ok; tile += n_pairs, it++) {
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
                        umma_f16_pair(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                                      (kb | kk) != 0);
                    }
                    umma_commit_pair(smem_u32(&empty[stage]));
                    umma_commit_pair(empty_peer + (uint32_t)(stage * 8));
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
                if (ok) {
                    umma_commit_pair(smem_u32(&tfull[ab]));
                    umma_commit_pair(tfull_peer + (uint32_t)(ab * 8));
                }
            }
            // no MMA may still be writing either CTA's TMEM at deallocation
            umma_commit_pair(smem_u32(done));
            mbar_wait(done, 0, p.err);
        }
        __syncwarp();
    } else {
        const int q = warp & 3;
        const int part = (warp - 2) >> 2;
        constexpr int kNch = BN / 32, kParts = NE / 4;
        const int cb = part * kNch / kParts, ce = (part + 1) * kNch / kParts;
        const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);
        float* stg = stage_buf + (warp - 2) * 32 * 32;
        constexpr bool kF16 = EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU;
        uint32_t nst = 0;   // TMA stores issued by this warp
        int it = 0;
        for (int tile = pair; tile < total; tile += n_pairs, it++) {
            const int ni = tile % p.n_tiles;
            const int rest = tile / p.n_tiles;
            const int mi = rest % p.m_tiles, b = rest / p.m_tiles;
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            const int row0 = mi * 2 * kBM + (int)rank * kBM + q * 32;
            const long long out_row0 = (long long)b * p.c_batch_rows + row0;
            const int c0 = cb;
            float4 res[8];
            float2 lst[8];
            if ((EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN) && p.vec && c0 < ce && ni * BN + c0 * 32 < p.N)
                load_resid_t<EPI>(p, out_row0, row0, ni * BN + c0 * 32, res);
            if (EPI == W2V_EPI_F32_RESID_LN) load_ln_stats_t(p, out_row0, row0, lst);
            if (!mbar_wait(&tfull[ab], aph, p.err)) break;
            tc_fence_after();
            const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
            if constexpr (kF16) {
                if (p.tma_c)
                    epilogue_warp_tma<EPI>(p, &tmC, trow, reinterpret_cast<uint8_t*>(stg), row0, b, ni * BN, c0, ce,
                                           nst);
                else
                    epilogue_warp<EPI>(p, trow, stg, out_row0, row0, ni * BN, c0, ce, res, lst);
            } else {
                epilogue_warp<EPI>(p, trow, stg, out_row0, row0, ni * BN, c0, ce, res, lst);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty_lead + (uint32_t)(ab * 8));
        }
        if (kF16 && p.tma_c) {   // the stores are complete before the CTA exits
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        }
    }

    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
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
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p,
                     cudaStream_t st) {
    using Cfg = GemmCfg<BN, epi_warps(EPI)>;
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
    kern<<<grid, gemm_threads(EPI), Cfg::kSmem, st>>>(ta, tb, tc, p);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

// Clusters of two that can be resident at once (a GPC may leave an SM unpaired).
template <int BN, int EPI>
static int max_pairs(int dev) {
    static int n[64] = {};
    if (!n[dev & 63]) {
        using Cfg = Gemm2Cfg<BN, epi_warps(EPI)>;
        auto kern = gemm2_tc_kernel<BN, EPI>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) != cudaSuccess)
            return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
        cfg.blockDim = dim3(gemm_threads(EPI), 1, 1);
        cfg.dynamicSmemBytes = Cfg::kSmem;
        int c = 0;
        if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess || c <= 0) {
            cudaGetLastError();
            c = sm_count() / 2;
        }
        n[dev & 63] = c;
    }
    return n[dev & 63];
}

template <int BN, int EPI>
static int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p,
                       cudaStream_t st) {
    using Cfg = Gemm2Cfg<BN, epi_warps(EPI)>;
    int dev = 0;
    cudaGetDevice(&dev);
    const int mp = max_pairs<BN, EPI>(dev);
    if (mp <= 0) return W2V_ERR_LAUNCH;
    const int total = p.n_batch * p.m_tiles * p.n_tiles;
    const int pairs = total < mp ? total : mp;
    gemm2_tc_kernel<BN, EPI><<<2 * pairs, gemm_threads(EPI), Cfg::kSmem, st>>>(ta, tb, tc, p);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

template <int EPI>
static int launch_epi(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                      const GemmParams& p, cudaStream_t st) {
    switch (bn) {
        case 256: return launch_bn<256, EPI>(ta, tb, tc, p, st);
        case 192: return launch_bn<192, EPI>(ta, tb, tc, p, st);
        case 128: return launch_bn<128, EPI>(ta, tb, tc, p, st);
        case -256: return launch_pair<256, EPI>(ta, tb, tc, p, st);
        case -192: return launch_pair<192, EPI>(ta, tb, tc, p, st);
        case -128: return launch_pair<128, EPI>(ta, tb, tc, p, st);
        default: return launch_bn<64, EPI>(ta, tb, tc, p, st);
    }
}

// Pick the tile: single-CTA 128 x {256,128,64} (64 covers small or ragged N
// through TMA zero fill) or CTA-pair 256 x {256,128} (returned negated).
// Estimated time = waves x tile width x (K x m + E x e):
//   m  MMA time per unit of K relative to 128 x 256 tiles (narrow tiles stage
//      more operand bytes per MAC; pairs stage half of B per SM);
//   E  epilogue work per output in the same units (fp16 store < fp32 store <
//      GELU < fp32 residual), only partly hidden behind the next tile's MMAs;
//   e  pairs wait for both CTAs' epilogues before reusing an accumulator.
// Constants fitted on B200 to the encoder GEMMs (M = 31936, K = 768/3072,
// N = 768/2304/3072, every epilogue, every tile): the model picks the
// measured-fastest tile for each of them.
static int pick_bn(int N, int m_valid, int n_batch, long long K, int epilogue) {
    const int sms = sm_count();
    const long long mt1 = (long long)((m_valid + kBM - 1) / kBM) * n_batch;
    const long long mt2 = (long long)((m_valid + 2 * kBM - 1) / (2 * kBM)) * n_batch;
    const double E = epilogue == W2V_EPI_F16 ? 293 : epilogue == W2V_EPI_F16_GELU ? 442
                   : epilogue == W2V_EPI_F32 ? 450 : epilogue == W2V_EPI_F32_RESID ? 932 : 1000;
    int best = 64;
    double best_cost = 1e300;
    for (int bn : {256, 192, 128, 64, -256, -192, -128}) {
        const int w = bn < 0 ? -bn : bn;
        if (N % w != 0 && bn != 64) continue;
        const long long tiles = (bn < 0 ? mt2 : mt1) * ((N + w - 1) / w);
        const long long slots = bn < 0 ? sms / 2 : sms;
        const long long waves = (tiles + slots - 1) / slots;
        const double m = bn == 256 ? 1.0 : bn == 192 ? 1.15 : bn == 128 ? 1.3 : bn == 64 ? 1.6
                       : bn == -256 ? 0.78 : bn == -192 ? 1.0 : 1.3;
        const double e = bn < 0 ? 1.34 : 1.0;
        const double cost = (double)waves * w * ((double)K * m + E * e);
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

static int gemm_impl(const void* A, long long a_cin, int a_taps, int a_stride, long long a_row_stride,
                     long long a_rows_in, long long a_batches, long long a_batch_stride, const void* B, int N,
                     void* C, long long ldc, long long c_batch_rows, int m_valid, const float* bias,
                     const float* resid, long long ldr, int epilogue, const float* ln_stats, const float* ln_w,
                     const float* ln_b, int block_n, int* err, void* stream) {
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
    p.n_batch = (int)a_batches;
    p.N = N;
    const int bn = block_n ? block_n : pick_bn(N, m_valid, p.n_batch, K, epilogue);
    if (bn != 256 && bn != 192 && bn != 128 && bn != 64 && bn != -256 && bn != -192 && bn != -128)
        return W2V_ERR_ARGS;
    const int tile_rows = bn < 0 ? 2 * kBM : kBM, tile_cols = bn < 0 ? -bn : bn;
    p.m_tiles = (int)((m_valid + tile_rows - 1) / tile_rows);
    p.n_tiles = (N + tile_cols - 1) / tile_cols;
    p.k_blocks = (int)(K / kBK);
    p.C = C;
    p.ldc = ldc;
    p.c_batch_rows = c_batch_rows;
    p.bias = bias;
    p.resid = resid;
    p.ldr = ldr;
    p.err = err;
    p.ln_stats = reinterpret_cast<const float2*>(ln_stats);
    p.ln_w = ln_w;
    p.ln_b = ln_b;
    {
        const bool f16 = epilogue == W2V_EPI_F16 || epilogue == W2V_EPI_F16_GELU;
        const uintptr_t cb = reinterpret_cast<uintptr_t>(C), rb = reinterpret_cast<uintptr_t>(resid),
                        bb = reinterpret_cast<uintptr_t>(bias);
        p.vec = (ldc % (f16 ? 8 : 4) == 0) && (cb % 16 == 0) && (!resid || (ldr % 4 == 0 && rb % 16 == 0)) &&
                (!bias || bb % 16 == 0);
    }
    const uint64_t bdims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t bstr[1] = {(uint64_t)K * 2};
    const uint32_t bbox[2] = {kBK, (uint32_t)(bn < 0 ? -bn / 2 : bn)};
    rc = make_map_f16(&tb, B, 2, bdims, bstr, bbox);
    if (rc) return rc;
    // fp16 C by TMA tile stores: [n_batch][c_batch_rows][ldc], rows m_valid and
    // columns N in bounds, boxes of 32 x 32 (64-byte swizzle).  A store clips
    // the innermost dimension at 16-byte granularity only (a partly covered
    // 16-byte group is written whole), so N must be a multiple of 8.
    CUtensorMap tc = tb;
    p.tma_c = 0;
    if ((epilogue == W2V_EPI_F16 || epilogue == W2V_EPI_F16_GELU) && p.vec && ldc % 8 == 0 && N % 8 == 0 &&
        (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
        auto enc = get_encode();
        if (!enc) return W2V_ERR_DRIVER;
        const uint64_t cdims[3] = {(uint64_t)N, (uint64_t)m_valid, (uint64_t)a_batches};
        const uint64_t cstr[2] = {(uint64_t)ldc * 2, (uint64_t)c_batch_rows * ldc * 2};
        const uint32_t cbox[3] = {32, 32, 1}, ces[3] = {1, 1, 1};
        if (enc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, C, cdims, cstr, cbox, ces, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return W2V_ERR_TENSOR_MAP;
        p.tma_c = 1;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (epilogue) {
        case W2V_EPI_F16: return launch_epi<W2V_EPI_F16>(bn, ta, tb, tc, p, st);
        case W2V_EPI_F16_GELU: return launch_epi<W2V_EPI_F16_GELU>(bn, ta, tb, tc, p, st);
        case W2V_EPI_F32: return launch_epi<W2V_EPI_F32>(bn, ta, tb, tc, p, st);
        case W2V_EPI_F32_RESID:
            if (!resid) return W2V_ERR_ARGS;
            return launch_epi<W2V_EPI_F32_RESID>(bn, ta, tb, tc, p, st);
        case W2V_EPI_F32_RESID_LN:
            if (!resid || !ln_stats || !ln_w || !ln_b || !p.vec ||
                ((reinterpret_cast<uintptr_t>(ln_stats) | reinterpret_cast<uintptr_t>(ln_w) |
                  reinterpret_cast<uintptr_t>(ln_b)) & 15))
                return W2V_ERR_ARGS;
            return launch_epi<W2V_EPI_F32_RESID_LN>(bn, ta, tb, tc, p, st);
        default: return W2V_ERR_ARGS;
    }
}

extern "C" int w2v_gemm_f16(const void* A, long long a_cin, int a_taps, int a_stride, long long a_row_stride,
                            long long a_rows_in, long long a_batches, long long a_batch_stride, const void* B,
                            int N, void* C, long long ldc, long long c_batch_rows, int m_valid, const float* bias,
                            const float* resid, long long ldr, int epilogue, int block_n, int* err,
                            void* stream) {
    if (epilogue == W2V_EPI_F32_RESID_LN) return W2V_ERR_ARGS;   // needs the statistics: w2v_gemm_f16_ln_resid
    return gemm_impl(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches, a_batch_stride, B, N, C, ldc,
                     c_batch_rows, m_valid, bias, resid, ldr, epilogue, nullptr, nullptr, nullptr, block_n, err,
                     stream);
}

extern "C" int w2v_gemm_f16_ln_resid(const void* A, long long a_cin, int a_taps, int a_stride,
                                     long long a_row_stride, long long a_rows_in, long long a_batches,
                                     long long a_batch_stride, const void* B, int N, void* C, long long ldc,
                                     long long c_batch_rows, int m_valid, const float* bias, const float* resid,
                                     long long ldr, const float* ln_stats, const float* ln_w, const float* ln_b,
                                     int block_n, int* err, void* stream) {
    return gemm_impl(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches, a_batch_stride, B, N, C, ldc,
                     c_batch_rows, m_valid, bias, resid, ldr, W2V_EPI_F32_RESID_LN, ln_stats, ln_w, ln_b, block_n,
                     err, stream);
}
