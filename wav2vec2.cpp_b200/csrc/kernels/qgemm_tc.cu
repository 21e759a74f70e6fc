// Dequant-fused tcgen05 GEMM for GGUF Q8_0 / Q4_0 weights (sm_100a):
//   C[r][n] = epi( sum_k A[r][k] * W[n][k] ),  W dequantised on the fly.
//
// Replaces ggml_mul_mat on quantised weights (GgmlScratch::linear,
// src/ggml_backend.h:78-120), which the reference runs on the raw blocks it
// keeps resident (src/ggml_backend.h:43-50).  Here the blocks stay resident
// too, repacked once at load (w2v_repack_q) into
//   codes   Q8_0: [N][K] int8;  Q4_0: [N][K/8] 32-bit words, weight 8g+2j in
//           bits 4j..4j+3 and weight 8g+2j+1 in bits 16+4j.. (unsigned codes)
//   scales  [K/32][ld_s] fp16, one per block of 32 weights along K.
//
// The weights are the MMA's A operand and live in TENSOR MEMORY: per 64-deep
// k-block each converter thread owns one weight row, reads its 64 codes and
// 2 scales from shared memory (TMA-loaded, swizzled so the row-per-thread
// reads are free of bank conflicts), expands them to 32 fp16 pairs and writes
// them with one tcgen05.st (lane = weight row, 32-bit column c = weights 2c,
// 2c+1).  The activations are the B operand: [rows][K] fp16 tiles in shared
// memory by TMA (128-byte swizzle, K-major).  The accumulator is therefore
// transposed, D[n][r] (TMEM lane = output feature, column = activation row),
// and the epilogue stores it with each lane writing one feature: every store
// instruction covers 32 consecutive features of one row.
// Expansion: a code byte u in the mantissa of 1024.0 reads as 1024 + u, one
// fp16 subtraction leaves the integer (q for Q8_0, q - 8 for Q4_0) exactly, and
// one fp16 multiplication by the scale is the single rounding of d * q -- the
// values the load-time expansion (w2v_dequant_f16) produces.
//
// Tiles: one CTA per 128 weight rows x BN activation rows, or a CTA pair
// (tcgen05 cta_group::2) per 256 weight rows x BN activation rows in which
// each CTA expands its own 128 weight rows into its own TMEM and stages BN/2
// activation rows; the leader issues the MMA.  TMEM per CTA: two BN-column
// accumulators plus up to four 32-column weight tiles (512 columns).
// Roles (320 threads): warp 0 TMA producer; warp 1 TMEM allocation + MMA
// issue; warps 2..5 epilogue; warps 6..9 converters.  Warp w may access
// TMEM lanes 32 (w % 4) .. +31, so both the epilogue and the converter warps
// cover the four lane quarters once.  Every mbarrier wait is bounded.
#include "common.cuh"
#include "w2v_kernels.h"

namespace w2v {
namespace qg {

constexpr int kBK = 64;             // K per k-block (128 bytes of fp16)
constexpr int kRows = 128;          // weight rows per CTA (TMEM lanes)
constexpr int kNC = 4;              // converter warps (epilogue warps: QCfg::kNE)
constexpr int kSmemCap = 232448;
enum : int { kQ8 = 1, kQ4 = 2 };
__host__ __device__ constexpr int code_row_bytes(int wq) { return wq == kQ8 ? 64 : 32; }
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }

struct QParams {
    int m_valid;         // activation rows
    int N;               // weight rows = output features
    int f_tiles, r_tiles, k_blocks;
    int tma;             // epilogue through shared-memory boxes and TMA (tmC, tmR); else direct stores
    void* C;
    long long ldc;
    const float* bias;
    const float* resid;
    long long ldr;
    const float2* ln_stats;
    const float* ln_w;
    const float* ln_b;
    int* err;
};

template <int BN, int WQ, bool PAIR, int EPI, int EH = 1>
struct QCfg {
    // EH epilogue warps per TMEM lane quarter (they take alternate 32-row chunks)
    static constexpr int kNE = 4 * EH;
    static constexpr int kThreads = 64 + 32 * (kNE + kNC);
    static constexpr int kXRows = PAIR ? BN / 2 : BN;          // activation rows one CTA stages
    static constexpr int kXBytes = kXRows * kBK * 2;
    static constexpr int kCodeBytes = kRows * code_row_bytes(WQ);
    static constexpr int kScaleBytes = 2 * kRows * 2;
    static constexpr int kPer = kXBytes + kCodeBytes + kScaleBytes;
    // Staged epilogue, per epilogue warp: two 32 x 32 output boxes (fp16 or fp32),
    // and for the residual epilogues a ring of kResBoxes fp32 residual boxes
    // (fetched kResBoxes - 1 chunks ahead: the residual does not depend on the
    // MMA, and one box ahead left every chunk waiting on a DRAM round trip);
    // then per warp the current chunk's row statistics (256 B).
    static constexpr bool kRes = EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN;
    static constexpr int kOutBox = (EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU) ? 2048 : 4096;
    static constexpr int kResBoxes = kRes ? (EH == 2 ? 2 : 4) : 0;
    static constexpr int kEpiWarp = 2 * kOutBox + kResBoxes * 4096;
    static constexpr int kEpiBytes = kNE * (kEpiWarp + 256);
    static constexpr int kStages = cmin(8, (kSmemCap - 1024 - 512 - kEpiBytes) / kPer);
    static constexpr int kOffCode = kStages * kXBytes;
    static constexpr int kOffScale = kOffCode + kStages * kCodeBytes;
    static constexpr int kOffEpi = kOffScale + kStages * kScaleBytes;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kSmem = kOffBar + 512 + 1024;
    static constexpr int kSB = cmin(4, (512 - 2 * BN) / 32);   // weight tiles in TMEM
    static constexpr int kACol = 2 * BN;                        // first weight-tile column
    static_assert(kStages >= 2 && kSB >= 2, "plan");
    static_assert(kXBytes % 1024 == 0 && kCodeBytes % 1024 == 0, "alignment");
    static_assert((3 * kStages + 2 * kSB + 5 + kNE * (kResBoxes > 1 ? kResBoxes : 1)) * 8 + 4 <= 512, "barriers");
};

// ── tcgen05 forms used only here ────────────────────────────────────────────
W2V_DEV void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
// D (256 rows over the CTA pair) (+)= A[tmem of both CTAs] . B[smem of both CTAs]^T
W2V_DEV void umma_f16_pair_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                  uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

W2V_DEV void tma_store_2d(const CUtensorMap* m, const void* smem_src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
                 : "memory");
}

W2V_DEV uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
W2V_DEV uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// four int8 codes (one word) -> two fp16 pairs times the scale pair dd
W2V_DEV void q8_word(uint32_t w, uint32_t dd, uint32_t& lo, uint32_t& hi) {
    const uint32_t x = w ^ 0x80808080u;
    lo = hmul2_u32(hsub2_u32(__byte_perm(x, 0x64646464u, 0x4140), 0x64806480u), dd);
    hi = hmul2_u32(hsub2_u32(__byte_perm(x, 0x64646464u, 0x4342), 0x64806480u), dd);
}
// eight 4-bit codes (one word) -> four fp16 pairs times dd
W2V_DEV void q4_word(uint32_t w, uint32_t dd, uint32_t* o) {
#pragma unroll
    for (int j = 0; j < 4; j++)
        o[j] = hmul2_u32(hsub2_u32(((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u, 0x64086408u), dd);
}

template <int BN, int EPI, int WQ, bool PAIR, int EH>
__global__ void __launch_bounds__(QCfg<BN, WQ, PAIR, EPI, EH>::kThreads, 1)
qgemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmQ,
             const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmC,
             const __grid_constant__ CUtensorMap tmR, QParams p) {
    using Cfg = QCfg<BN, WQ, PAIR, EPI, EH>;
    constexpr int S = Cfg::kStages, SB = Cfg::kSB, CT = PAIR ? 2 : 1, kNE = Cfg::kNE;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sX = smem;
    uint8_t* sQ = smem + Cfg::kOffCode;
    uint8_t* sS = smem + Cfg::kOffScale;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;                 // activation tile of stage s landed (pair: leader, both CTAs' bytes)
    uint64_t* cfull = bars + S;            // codes + scales of stage s landed (local)
    uint64_t* empty = bars + 2 * S;        // stage s consumed by the MMA (each CTA)
    uint64_t* afull = bars + 3 * S;        // weight tile f in TMEM (pair: leader, both CTAs' converters)
    uint64_t* aempty = afull + SB;         // weight tile f consumed by the MMA (each CTA)
    uint64_t* tfull = aempty + SB;         // accumulator b ready (each CTA)
    uint64_t* tempty = tfull + 2;          // accumulator b drained (pair: leader, both CTAs' epilogues)
    uint64_t* done = tempty + 2;
    constexpr int RB = Cfg::kResBoxes > 0 ? Cfg::kResBoxes : 1;
    uint64_t* rbar = done + 1;             // residual box b of epilogue warp w landed: rbar[RB w + b]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + RB * kNE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int total = p.f_tiles * p.r_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&cfull[s], 1); mbar_init(&empty[s], 1); }
        for (int f = 0; f < SB; f++) { mbar_init(&afull[f], kNC * CT); mbar_init(&aempty[f], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], kNE * CT); }
        mbar_init(done, 1);
        for (int i = 0; i < RB * kNE; i++) mbar_init(&rbar[i], 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmS);
    }
    if (warp == 1) {
        if (PAIR) { tmem_alloc_pair(tmem_slot, 512); tmem_relinquish_pair(); }
        else { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    }
    tc_fence_before();
    if (PAIR) cluster_sync_all(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            const uint32_t full_lead = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            for (int tile = unit; tile < total && ok; tile += n_units) {
                const int fi = tile % p.f_tiles, ri = tile / p.f_tiles;
                const int frow = fi * kRows * CT + (int)rank * kRows;
                const int xrow = ri * BN + (int)rank * Cfg::kXRows;
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) { ok = false; break; }
                    if constexpr (PAIR) {
                        if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kXBytes);
                        tma_load_2d_pair(sX + stage * Cfg::kXBytes, &tmX, full_lead + (uint32_t)(stage * 8), kb * kBK,
                                         xrow);
                    } else {
                        mbar_arrive_expect_tx(&full[stage], Cfg::kXBytes);
                        tma_load_2d(sX + stage * Cfg::kXBytes, &tmX, &full[stage], kb * kBK, xrow);
                    }
                    mbar_arrive_expect_tx(&cfull[stage], Cfg::kCodeBytes + Cfg::kScaleBytes);
                    tma_load_2d(sQ + stage * Cfg::kCodeBytes, &tmQ, &cfull[stage], kb * code_row_bytes(WQ), frow);
                    tma_load_2d(sS + stage * Cfg::kScaleBytes, &tmS, &cfull[stage], frow, 2 * kb);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
            }
            // no bulk copy may still be writing this CTA's shared memory when it exits
            for (int s = 0; s < S; s++)
                if (issued & (1u << s)) {
                    if (!PAIR || rank == 0) mbar_wait(&full[s], (last_par >> s) & 1u, p.err);
                    mbar_wait(&cfull[s], (last_par >> s) & 1u, p.err);
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = umma_idesc_f16(kRows * CT, BN);
            const uint32_t empty_peer = PAIR ? mapa_shared(smem_u32(empty), 1) : 0u;
            const uint32_t aempty_peer = PAIR ? mapa_shared(smem_u32(aempty), 1) : 0u;
            const uint32_t tfull_peer = PAIR ? mapa_shared(smem_u32(tfull), 1) : 0u;
            int stage = 0, it = 0, kq = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = unit; tile < total && ok; tile += n_units, it++) {
                const int ab = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&tempty[ab], aph ^ 1u, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * BN);
                for (int kb = 0; kb < p.k_blocks; kb++, kq++) {
                    const int f = kq % SB;
                    if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
                    const bool aok = PAIR ? mbar_wait_cluster(&afull[f], (uint32_t)(kq / SB) & 1u, p.err)
                                          : mbar_wait(&afull[f], (uint32_t)(kq / SB) & 1u, p.err);
                    if (!aok) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = tmem_base + (uint32_t)(Cfg::kACol + f * 32);
                    const uint32_t b0 = smem_u32(sX + stage * Cfg::kXBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; kk++) {
                        if constexpr (PAIR)
                            umma_f16_pair_tmem_a(d, a0 + (uint32_t)(kk * 8), umma_desc_sw128(b0 + kk * 32), idesc,
                                                 (kb | kk) != 0);
                        else
                            umma_f16_tmem_a(d, a0 + (uint32_t)(kk * 8), umma_desc_sw128(b0 + kk * 32), idesc,
                                            (kb | kk) != 0);
                    }
                    if constexpr (PAIR) {
                        umma_commit_pair(smem_u32(&empty[stage]));
                        umma_commit_pair(empty_peer + (uint32_t)(stage * 8));
                        umma_commit_pair(smem_u32(&aempty[f]));
                        umma_commit_pair(aempty_peer + (uint32_t)(f * 8));
                    } else {
                        umma_commit(&empty[stage]);
                        umma_commit(&aempty[f]);
                    }
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
                if (ok) {
                    if constexpr (PAIR) {
                        umma_commit_pair(smem_u32(&tfull[ab]));
                        umma_commit_pair(tfull_peer + (uint32_t)(ab * 8));
                    } else {
                        umma_commit(&tfull[ab]);
                    }
                }
            }
            // no MMA may still be using TMEM when it is freed (also after an expired wait)
            if constexpr (PAIR) umma_commit_pair(smem_u32(done)); else umma_commit(done);
            mbar_wait(done, 0, p.err);
        }
        __syncwarp();
    } else if (warp >= 2 + kNE) {
        // converters: weight row fl of this CTA -> its TMEM lane, one k-block at a time
        const int q = warp & 3;
        const int fl = 32 * q + lane;
        const uint32_t afull_lead = PAIR ? mapa_shared(smem_u32(afull), 0) : 0u;
        const uint32_t trow = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)Cfg::kACol;
        int kq = 0;
        bool ok = true;
        for (int tile = unit; tile < total && ok; tile += n_units) {
            for (int kb = 0; kb < p.k_blocks; kb++, kq++) {
                const int s = kq % S, f = kq % SB;
                if (!mbar_wait(&cfull[s], (uint32_t)(kq / S) & 1u, p.err)) {
                    ok = false;
                    break;
                }
                // expand first, then wait for the MMA to release weight tile f: only the
                // TMEM store stays between that release and the next k-block's MMA
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(sS + s * Cfg::kScaleBytes);
                const uint32_t d0 = sc[fl], d1 = sc[kRows + fl];
                const uint32_t dd0 = d0 | (d0 << 16), dd1 = d1 | (d1 << 16);
                const uint8_t* row = sQ + s * Cfg::kCodeBytes + fl * code_row_bytes(WQ);
                uint32_t v[32];
                if constexpr (WQ == kQ8) {
                    // 64-byte rows, 64-byte swizzle: 16-byte group j at j ^ ((row >> 1) & 3)
                    uint4 c[4];
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        c[j] = *reinterpret_cast<const uint4*>(row + ((j ^ ((fl >> 1) & 3)) << 4));
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint32_t dd = j < 2 ? dd0 : dd1;    // weights 16j..16j+15: block j / 2
                        q8_word(c[j].x, dd, v[8 * j + 0], v[8 * j + 1]);
                        q8_word(c[j].y, dd, v[8 * j + 2], v[8 * j + 3]);
                        q8_word(c[j].z, dd, v[8 * j + 4], v[8 * j + 5]);
                        q8_word(c[j].w, dd, v[8 * j + 6], v[8 * j + 7]);
                    }
                } else {
                    // 32-byte rows, 32-byte swizzle: 16-byte group j at j ^ ((row >> 2) & 1)
                    uint4 c[2];
#pragma unroll
                    for (int j = 0; j < 2; j++)
                        c[j] = *reinterpret_cast<const uint4*>(row + ((j ^ ((fl >> 2) & 1)) << 4));
                    q4_word(c[0].x, dd0, v + 0);
                    q4_word(c[0].y, dd0, v + 4);
                    q4_word(c[0].z, dd0, v + 8);
                    q4_word(c[0].w, dd0, v + 12);
                    q4_word(c[1].x, dd1, v + 16);
                    q4_word(c[1].y, dd1, v + 20);
                    q4_word(c[1].z, dd1, v + 24);
                    q4_word(c[1].w, dd1, v + 28);
                }
                if (!mbar_wait(&aempty[f], ((uint32_t)(kq / SB) & 1u) ^ 1u, p.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();   // the MMA that read weight tile f has completed
                tmem_st32u(trow + (uint32_t)(f * 32), v);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR) mbar_arrive_remote(afull_lead + (uint32_t)(f * 8));
                    else mbar_arrive(&afull[f]);
                }
            }
        }
    } else {
        // epilogue: lane = output feature, the 32 registers of a chunk = 32 activation rows;
        // with EH = 2 two warps share a lane quarter and take alternate chunks (eh, eh + 2, ...)
        const int q = warp & 3;
        const int eh = (warp - 2) / 4;
        if (p.tma) {
            // Staged: per 32 x 32 chunk, the residual box arrives by TMA R - 1 chunks
            // ahead (a ring of R boxes per warp, the first R - 1 requested before the
            // accumulator is ready), and the results go through one of two output
            // boxes and a TMA tile store.  Register j of lane f is row j,
            // feature f of the box: each shared-memory access of the warp touches
            // one contiguous 64- or 128-byte box row, so none conflicts on a bank.
            constexpr bool kRes = EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN;
            constexpr bool kF16 = EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU;
            constexpr int kNch = BN / 32;
            constexpr uint32_t R = RB;             // residual boxes per warp (residual epilogues)
            uint8_t* ebase = smem + Cfg::kOffEpi + (warp - 2) * Cfg::kEpiWarp;
            float* rbox = reinterpret_cast<float*>(ebase + 2 * Cfg::kOutBox);
            // rows 2i, 2i+1 of the chunk: (mean, rstd, mean, rstd)
            float4* sst = reinterpret_cast<float4*>(smem + Cfg::kOffEpi + kNE * Cfg::kEpiWarp + (warp - 2) * 256);
            uint64_t* rb = rbar + RB * (warp - 2);
            const uint32_t tempty_lead = PAIR ? mapa_shared(smem_u32(tempty), 0) : 0u;
            uint32_t nst = 0, nrl = 0, nrw = 0;   // output boxes stored, residual boxes requested / awaited
            int it = 0;
            for (int tile = unit; tile < total; tile += n_units, it++) {
                const int fi = tile % p.f_tiles, ri = tile / p.f_tiles;
                const int ab = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                const int fcol0 = fi * kRows * CT + (int)rank * kRows + 32 * q;
                const int fcol = fcol0 + lane;
                const bool fv = fcol < p.N;
                const float bias = (p.bias && fv) ? __ldg(p.bias + fcol) : 0.f;
                float lw = 0.f, lb = 0.f;
                if (EPI == W2V_EPI_F32_RESID_LN && fv) { lw = __ldg(p.ln_w + fcol); lb = __ldg(p.ln_b + fcol); }
                if (fcol0 >= p.N) {
                    // every feature of this warp's quarter is past the last one: nothing to
                    // load or store, only the accumulator to hand back
                    if (!mbar_wait(&tfull[ab], aph, p.err)) break;
                    tc_fence_after();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (PAIR) mbar_arrive_remote(tempty_lead + (uint32_t)(ab * 8));
                        else mbar_arrive(&tempty[ab]);
                    }
                    continue;
                }
                auto request = [&](int c) {          // residual box of chunk c (lane 0)
                    const uint32_t b = nrl % R;
                    fence_async_smem();              // earlier reads of this box precede the TMA write
                    mbar_arrive_expect_tx(&rb[b], 32 * 32 * 4);
                    tma_load_2d(rbox + b * 1024, &tmR, &rb[b], fcol0, ri * BN + c * 32);
                };
                const uint32_t rfirst = nrl;
                // this warp's chunks: eh, eh + EH, ...; the residual of its k-th chunk goes
                // to ring slot (rfirst + k) % R
                int nreq = 0;                        // of this warp's chunks in this tile, residuals requested
                auto chunk_ok = [&](int k) { return eh + k * EH < kNch && ri * BN + (eh + k * EH) * 32 < p.m_valid; };
                if constexpr (kRes) {
                    // the first R-1 before the accumulator is ready; chunk k + R - 1 at chunk k
                    for (; nreq < (int)R - 1 && chunk_ok(nreq); nreq++) {
                        if (lane == 0) request(eh + nreq * EH);
                        nrl++;
                    }
                }
                float2 stn = make_float2(0.f, 0.f);
                if (EPI == W2V_EPI_F32_RESID_LN && ri * BN + eh * 32 + lane < p.m_valid)
                    stn = p.ln_stats[ri * BN + eh * 32 + lane];
                if (!mbar_wait(&tfull[ab], aph, p.err)) break;
                tc_fence_after();
                const uint32_t tacc = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * BN);
                bool ok = true;
#pragma unroll 1
                for (int c = eh, k = 0; c < kNch; c += EH, k++) {
                    float v[32];
                    tmem_ld32(tacc + (uint32_t)(c * 32), v);
                    if (c + EH >= kNch) {
                        // this warp's last chunk is in registers: its share of the accumulator is free
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if constexpr (PAIR) mbar_arrive_remote(tempty_lead + (uint32_t)(ab * 8));
                            else mbar_arrive(&tempty[ab]);
                        }
                    }
                    const int r0 = ri * BN + c * 32;
                    if (r0 >= p.m_valid) continue;
                    const float2 st = stn;
                    if (EPI == W2V_EPI_F32_RESID_LN && c + EH < kNch)
                        stn = r0 + 32 * EH + lane < p.m_valid ? p.ln_stats[r0 + 32 * EH + lane] : make_float2(0.f, 0.f);
                    const float* rcur = rbox;
                    if constexpr (kRes) {
                        const uint32_t idx = rfirst + (uint32_t)k;
                        if (chunk_ok(nreq)) {
                            __syncwarp();            // every lane is done with the box chunk nreq reuses (chunk k - 1's)
                            if (lane == 0) request(eh + nreq * EH);
                            nrl++;
                            nreq++;
                        }
                        if (!mbar_wait(&rb[idx % R], (idx / R) & 1u, p.err)) { ok = false; break; }
                        nrw = idx + 1;
                        rcur = rbox + (idx % R) * 1024;
                    }
                    uint8_t* ob = ebase + (nst & 1u) * Cfg::kOutBox;
                    if (lane == 0) bulk_wait_group_read<1>();   // the store issued from this box two boxes ago has read it
                    if (EPI == W2V_EPI_F32_RESID_LN) {
                        // the chunk's row statistics, read back by every lane as a broadcast
                        // (the previous chunk's reads precede this store: __syncwarp above)
                        reinterpret_cast<float2*>(sst)[lane] = st;
                    }
                    __syncwarp();
                    if constexpr (kF16) {
                        __half* oh = reinterpret_cast<__half*>(ob);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            const float a = v[j] + bias, b = v[j + 1] + bias;
                            const uint32_t h = EPI == W2V_EPI_F16_GELU ? gelu_half2(a, b) : pack_half2(a, b);
                            reinterpret_cast<uint16_t*>(oh)[j * 32 + lane] = (uint16_t)(h & 0xFFFFu);
                            reinterpret_cast<uint16_t*>(oh)[(j + 1) * 32 + lane] = (uint16_t)(h >> 16);
                        }
                    } else {
                        float* of = reinterpret_cast<float*>(ob);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float a0 = v[j] + bias, a1 = v[j + 1] + bias;
                            if (EPI == W2V_EPI_F32_RESID) {
                                a0 += rcur[j * 32 + lane];
                                a1 += rcur[(j + 1) * 32 + lane];
                            }
                            if (EPI == W2V_EPI_F32_RESID_LN) {
                                const float4 s2 = sst[j / 2];
                                a0 += (rcur[j * 32 + lane] - s2.x) * s2.y * lw + lb;
                                a1 += (rcur[(j + 1) * 32 + lane] - s2.z) * s2.w * lw + lb;
                            }
                            of[j * 32 + lane] = a0;
                            of[(j + 1) * 32 + lane] = a1;
                        }
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, ob, fcol0, r0);
                        bulk_commit_group();
                    }
                    nst++;
                }
                if (!ok) break;
            }
            // the stores have completed and no residual box is still being written
            // (after an expired wait boxes may have been requested and not awaited)
            if constexpr (kRes)
                for (uint32_t idx = nrw; idx < nrl; idx++) mbar_wait(&rb[idx % R], (idx / R) & 1u, p.err);
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        } else {
        const uint32_t tempty_lead = PAIR ? mapa_shared(smem_u32(tempty), 0) : 0u;
        constexpr bool kRes = EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN;
        constexpr int kNch = BN / 32;
        int it = 0;
        for (int tile = unit; tile < total; tile += n_units, it++) {
            const int fi = tile % p.f_tiles, ri = tile / p.f_tiles;
            const int ab = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            const int fcol = fi * kRows * CT + (int)rank * kRows + 32 * q + lane;
            const bool fv = fcol < p.N;
            const float bias = (p.bias && fv) ? __ldg(p.bias + fcol) : 0.f;
            float lw = 0.f, lb = 0.f;
            if (EPI == W2V_EPI_F32_RESID_LN && fv) { lw = __ldg(p.ln_w + fcol); lb = __ldg(p.ln_b + fcol); }
            // The residual does not depend on the MMA: chunk c+1's residual (and its
            // rows' LayerNorm statistics) is in flight while chunk c is computed, and
            // chunk 0's while the accumulator is awaited.  Chunks cover distinct rows,
            // so reading ahead never crosses the in-place stores.
            float rn[32];
            float2 stn = make_float2(0.f, 0.f);
            auto fetch = [&](int c) {
                const int r0 = ri * BN + c * 32;
                if constexpr (kRes) {
                    const float* rp = p.resid + (long long)r0 * p.ldr + fcol;
#pragma unroll
                    for (int j = 0; j < 32; j++) rn[j] = (fv && r0 + j < p.m_valid) ? rp[(long long)j * p.ldr] : 0.f;
                }
                if (EPI == W2V_EPI_F32_RESID_LN) stn = r0 + lane < p.m_valid ? p.ln_stats[r0 + lane] : make_float2(0.f, 0.f);
            };
            if (kRes) fetch(eh);
            if (!mbar_wait(&tfull[ab], aph, p.err)) break;
            tc_fence_after();
            const uint32_t tacc = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * BN);
#pragma unroll 1
            for (int c = eh; c < kNch; c += EH) {
                float v[32];
                tmem_ld32(tacc + (uint32_t)(c * 32), v);
                if (c + EH >= kNch) {
                    // the accumulator is in registers: hand it back to the MMA
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (PAIR) mbar_arrive_remote(tempty_lead + (uint32_t)(ab * 8));
                        else mbar_arrive(&tempty[ab]);
                    }
                }
                const int r0 = ri * BN + c * 32;
                float rv[32];
                float2 st = stn;
                if constexpr (kRes) {
#pragma unroll
                    for (int j = 0; j < 32; j++) rv[j] = rn[j];
                    if (c + EH < kNch && r0 + 32 * EH < p.m_valid) fetch(c + EH);
                }
                if (r0 >= p.m_valid) continue;
                if (EPI == W2V_EPI_F16 || EPI == W2V_EPI_F16_GELU) {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const int r = r0 + j;
                        const float a = v[j] + bias, b = v[j + 1] + bias;
                        const uint32_t h = EPI == W2V_EPI_F16_GELU ? gelu_half2(a, b) : pack_half2(a, b);
                        __half* cp = reinterpret_cast<__half*>(p.C) + (long long)r * p.ldc + fcol;
                        if (fv && r < p.m_valid) *reinterpret_cast<uint16_t*>(cp) = (uint16_t)(h & 0xFFFFu);
                        if (fv && r + 1 < p.m_valid) *reinterpret_cast<uint16_t*>(cp + p.ldc) = (uint16_t)(h >> 16);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        float a = v[j] + bias;
                        if (EPI == W2V_EPI_F32_RESID) a += rv[j];
                        if (EPI == W2V_EPI_F32_RESID_LN) {
                            const float m = __shfl_sync(0xffffffffu, st.x, j), sd = __shfl_sync(0xffffffffu, st.y, j);
                            a += (rv[j] - m) * sd * lw + lb;
                        }
                        v[j] = a;
                    }
                    float* cp = reinterpret_cast<float*>(p.C) + (long long)r0 * p.ldc + fcol;
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (fv && r0 + j < p.m_valid) cp[(long long)j * p.ldc] = v[j];
                }
            }
        }
    }

    }

    tc_fence_before();
    if (PAIR) cluster_sync_all(); else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, 512); else tmem_dealloc(tmem_base, 512);
    }
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

static int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int BN, int EPI, int WQ, bool PAIR, int EH = 1>
static int launch(const CUtensorMap& tx, const CUtensorMap& tq, const CUtensorMap& ts, const CUtensorMap& tc,
                  const CUtensorMap& tr, const QParams& p, cudaStream_t st) {
    using Cfg = QCfg<BN, WQ, PAIR, EPI, EH>;
    auto kern = qgemm_kernel<BN, EPI, WQ, PAIR, EH>;
    static int max_units[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = PAIR ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = PAIR ? 1 : 0;
    if (!max_units[dev & 63]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) != cudaSuccess)
            return W2V_ERR_LAUNCH;
        int units = PAIR ? sm_count() / 2 : sm_count();
        if (PAIR) {
            // clusters of two that can be resident at once (a GPC may leave an SM unpaired)
            cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
            int c = 0;
            if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) == cudaSuccess && c > 0) units = c;
            cudaGetLastError();
        }
        max_units[dev & 63] = units;
    }
    const int total = p.f_tiles * p.r_tiles;
    const int units = total < max_units[dev & 63] ? total : max_units[dev & 63];
    cfg.gridDim = dim3((unsigned)(units * (PAIR ? 2 : 1)), 1, 1);
    if (cudaLaunchKernelEx(&cfg, kern, tx, tq, ts, tc, tr, p) != cudaSuccess) return W2V_ERR_LAUNCH;
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
}

template <int EPI, int WQ, int EH>
static int launch_tile(int bn, const CUtensorMap& tx, const CUtensorMap& tq, const CUtensorMap& ts,
                       const CUtensorMap& tc, const CUtensorMap& tr, const QParams& p, cudaStream_t st) {
    switch (bn) {
        case -224: return launch<224, EPI, WQ, true, EH>(tx, tq, ts, tc, tr, p, st);
        case 224: return launch<224, EPI, WQ, false, EH>(tx, tq, ts, tc, tr, p, st);
        case -192: return launch<192, EPI, WQ, true, EH>(tx, tq, ts, tc, tr, p, st);
        case -128: return launch<128, EPI, WQ, true, EH>(tx, tq, ts, tc, tr, p, st);
        case 192: return launch<192, EPI, WQ, false, EH>(tx, tq, ts, tc, tr, p, st);
        case 128: return launch<128, EPI, WQ, false, EH>(tx, tq, ts, tc, tr, p, st);
        case 64: return launch<64, EPI, WQ, false, EH>(tx, tq, ts, tc, tr, p, st);
        default: return W2V_ERR_ARGS;
    }
}

// eh = 2: two epilogue warps per lane quarter for the heavier epilogues (the
// fp32 residual ones and fp16 + GELU).  Measured at 31936 rows: the
// out-projection's LayerNorm residual 580 -> 688 TFLOP/s (its tiles finish
// their MMAs, K = 768, before one warp per quarter drains them), FFN-up + GELU
// 1013 -> 1040, FFN-down 1022 -> 1030; plain fp16 (QKV) unchanged, so it
// keeps one.
template <int EPI>
static int launch_w(int wq, int bn, int eh, const CUtensorMap& tx, const CUtensorMap& tq, const CUtensorMap& ts,
                    const CUtensorMap& tc, const CUtensorMap& tr, const QParams& p, cudaStream_t st) {
    if constexpr (EPI == W2V_EPI_F32_RESID || EPI == W2V_EPI_F32_RESID_LN || EPI == W2V_EPI_F16_GELU) {
        if (eh == 2)
            return wq == kQ8 ? launch_tile<EPI, kQ8, 2>(bn, tx, tq, ts, tc, tr, p, st)
                             : launch_tile<EPI, kQ4, 2>(bn, tx, tq, ts, tc, tr, p, st);
    }
    return wq == kQ8 ? launch_tile<EPI, kQ8, 1>(bn, tx, tq, ts, tc, tr, p, st)
                     : launch_tile<EPI, kQ4, 1>(bn, tx, tq, ts, tc, tr, p, st);
}

// Tile: CTA pairs (256 weight rows per tile) or single CTAs (128), each over
// 224, 192 or 128 activation rows, or single CTAs over 64 rows for short
// batches.  Each SM computes 128 weight rows x BN rows per tile either way.
// Estimated time = waves of tiles over the SMs x tile width x the measured
// time per activation row of that tile (B200, the base encoder linears at
// 31936 rows: wider tiles stage fewer operand bytes per MAC -- 224 rows 5 %
// and 192 rows 36 % faster per row than 128 -- and pairs stage half the
// activation bytes of single CTAs; 64 rows expand each weight k-block for
// half as many rows as 128).  Short batches (one utterance: 499 rows) fill
// more SMs with 64-row tiles.
static double tile_row_cost(int bn) {
    switch (bn) {
        case -224: return 0.95;
        case 224: return 0.96;
        case -192: return 1.0;
        case 192: return 1.03;
        case -128: return 1.36;
        case 128: return 1.39;
        default: return 2.2;
    }
}

static int pick_tile(int N, int m_valid) {
    const int sms = sm_count();
    int best = 128;
    double best_cost = 1e300;
    for (int bn : {-224, -192, -128, 224, 192, 128, 64}) {
        const bool pair = bn < 0;
        const int w = pair ? -bn : bn;
        const long long ft = (N + kRows * (pair ? 2 : 1) - 1) / (kRows * (pair ? 2 : 1));
        const long long rt = (m_valid + w - 1) / w;
        const long long slots = pair ? sms / 2 : sms;
        const long long waves = (ft * rt + slots - 1) / slots;
        const double cost = (double)waves * w * tile_row_cost(bn);
        if (cost < best_cost) { best_cost = cost; best = bn; }
    }
    return best;
}

static int qgemm_impl(const void* A, long long K, long long M, const void* Bq, const void* Bs, long long ld_s,
                      int gguf_type, int N, void* C, long long ldc, const float* bias, const float* resid,
                      long long ldr, int epilogue, const float* ln_stats, const float* ln_w, const float* ln_b,
                      int block_n, int* err, void* stream) {
    const int wq = gguf_type == 8 ? kQ8 : gguf_type == 2 ? kQ4 : 0;
    if (!wq || K <= 0 || K % kBK || M < 0 || M > 0x7fffffffLL || N <= 0 || !A || !Bq || !Bs || !C ||
        ld_s < N || ld_s % 8 || ldc < N)
        return W2V_ERR_ARGS;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Bq) | reinterpret_cast<uintptr_t>(Bs)) & 15)
        return W2V_ERR_ARGS;
    if ((epilogue == W2V_EPI_F32_RESID || epilogue == W2V_EPI_F32_RESID_LN) && (!resid || ldr < N)) return W2V_ERR_ARGS;
    if (epilogue == W2V_EPI_F32_RESID_LN && (!ln_stats || !ln_w || !ln_b)) return W2V_ERR_ARGS;
    if (epilogue < W2V_EPI_F16 || epilogue > W2V_EPI_F32_RESID_LN) return W2V_ERR_ARGS;
    if (M == 0) return W2V_OK;
    const int bn = block_n ? block_n : pick_tile(N, (int)M);
    if (bn != 224 && bn != 192 && bn != 128 && bn != 64 && bn != -224 && bn != -192 && bn != -128) return W2V_ERR_ARGS;
    const bool pair = bn < 0;
    const int w = pair ? -bn : bn;
    auto enc = get_encode();
    if (!enc) return W2V_ERR_DRIVER;
    CUtensorMap tx, tq, ts;
    const uint32_t es[2] = {1, 1};
    {   // activations [M][K] fp16, boxes of 64 x (rows one CTA stages), 128-byte swizzle
        const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
        const uint64_t str[1] = {(uint64_t)K * 2};
        const uint32_t box[2] = {kBK, (uint32_t)(pair ? w / 2 : w)};
        if (enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(A), dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return W2V_ERR_TENSOR_MAP;
    }
    {   // codes: [N][row bytes], one k-block of 128 rows per box, swizzled for row-per-thread reads
        const uint64_t rowb = (uint64_t)K * code_row_bytes(wq) / kBK;
        const uint64_t dims[2] = {rowb, (uint64_t)N};
        const uint64_t str[1] = {rowb};
        const uint32_t box[2] = {(uint32_t)code_row_bytes(wq), (uint32_t)kRows};
        if (enc(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(Bq), dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, wq == kQ8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return W2V_ERR_TENSOR_MAP;
    }
    {   // scales: [K/32][ld_s] fp16, the k-block's two scale rows for 128 weight rows per box
        const uint64_t dims[2] = {(uint64_t)N, (uint64_t)(K / 32)};
        const uint64_t str[1] = {(uint64_t)ld_s * 2};
        const uint32_t box[2] = {(uint32_t)kRows, 2};
        if (enc(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(Bs), dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return W2V_ERR_TENSOR_MAP;
    }
    // C and the residual as 32 x 32 boxes for the staged epilogue: fp16 C needs N
    // and ldc multiples of 8, fp32 C and the residual multiples of 4 (a store
    // clips the innermost dimension at 16-byte granularity only)
    const bool f16 = epilogue == W2V_EPI_F16 || epilogue == W2V_EPI_F16_GELU;
    const bool res = epilogue == W2V_EPI_F32_RESID || epilogue == W2V_EPI_F32_RESID_LN;
    bool tma = (reinterpret_cast<uintptr_t>(C) & 15) == 0 && (f16 ? (N % 8 == 0 && ldc % 8 == 0) : (N % 4 == 0 && ldc % 4 == 0));
    if (res) tma = tma && (reinterpret_cast<uintptr_t>(resid) & 15) == 0 && ldr % 4 == 0;
    CUtensorMap tc = tx, tr = tx;
    if (tma) {
        const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
        const uint64_t str[1] = {(uint64_t)ldc * (f16 ? 2 : 4)};
        const uint32_t box[2] = {32, 32};
        if (enc(&tc, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return W2V_ERR_TENSOR_MAP;
        if (res) {
            const uint64_t rstr[1] = {(uint64_t)ldr * 4};
            if (enc(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(resid), dims, rstr, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return W2V_ERR_TENSOR_MAP;
        }
    }
    QParams p;
    p.tma = tma ? 1 : 0;
    p.m_valid = (int)M;
    p.N = N;
    p.f_tiles = (N + kRows * (pair ? 2 : 1) - 1) / (kRows * (pair ? 2 : 1));
    p.r_tiles = (int)((M + w - 1) / w);
    p.k_blocks = (int)(K / kBK);
    p.C = C;
    p.ldc = ldc;
    p.bias = bias;
    p.resid = resid;
    p.ldr = ldr;
    p.ln_stats = reinterpret_cast<const float2*>(ln_stats);
    p.ln_w = ln_w;
    p.ln_b = ln_b;
    p.err = err;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int eh = tma ? 2 : 1;   // used by the residual and GELU epilogues (launch_w)
    switch (epilogue) {
        case W2V_EPI_F16: return launch_w<W2V_EPI_F16>(wq, bn, 1, tx, tq, ts, tc, tr, p, st);
        case W2V_EPI_F16_GELU: return launch_w<W2V_EPI_F16_GELU>(wq, bn, eh, tx, tq, ts, tc, tr, p, st);
        case W2V_EPI_F32: return launch_w<W2V_EPI_F32>(wq, bn, 1, tx, tq, ts, tc, tr, p, st);
        case W2V_EPI_F32_RESID: return launch_w<W2V_EPI_F32_RESID>(wq, bn, eh, tx, tq, ts, tc, tr, p, st);
        default: return launch_w<W2V_EPI_F32_RESID_LN>(wq, bn, eh, tx, tq, ts, tc, tr, p, st);
    }
}

}  // namespace qg
}  // namespace w2v

extern "C" int w2v_gemm_q(const void* A, long long K, long long M, const void* Bq, const void* Bs, long long ld_s,
                          int gguf_type, int N, void* C, long long ldc, const float* bias, const float* resid,
                          long long ldr, int epilogue, int block_n, int* err, void* stream) {
    if (epilogue == W2V_EPI_F32_RESID_LN) return W2V_ERR_ARGS;   // needs the statistics: w2v_gemm_q_ln_resid
    return w2v::qg::qgemm_impl(A, K, M, Bq, Bs, ld_s, gguf_type, N, C, ldc, bias, resid, ldr, epilogue, nullptr,
                               nullptr, nullptr, block_n, err, stream);
}

extern "C" int w2v_gemm_q_ln_resid(const void* A, long long K, long long M, const void* Bq, const void* Bs,
                                   long long ld_s, int gguf_type, int N, void* C, long long ldc, const float* bias,
                                   const float* resid, long long ldr, const float* ln_stats, const float* ln_w,
                                   const float* ln_b, int block_n, int* err, void* stream) {
    return w2v::qg::qgemm_impl(A, K, M, Bq, Bs, ld_s, gguf_type, N, C, ldc, bias, resid, ldr, W2V_EPI_F32_RESID_LN,
                               ln_stats, ln_w, ln_b, block_n, err, stream);
}
