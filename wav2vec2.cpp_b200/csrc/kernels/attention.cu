// Bidirectional multi-head self-attention, flash-style (online softmax, the
// T x T score matrix never leaves registers).  Replaces the reference's
// per-head scores/softmax/PV triple loops (src/wav2vec2.cpp:304-334,
// softmax src/ops.h:101-106).  Ragged batches: each query attends only to the
// keys of its own utterance; rows outside [0, T_u) are zero-filled in shared
// memory and masked with -inf in the scores, which reproduces the reference's
// unpadded single-utterance computation.
//
// fp16 Q/K/V/P operands with fp32 accumulation and fp32 softmax statistics.
// The tcgen05 kernel below (attn_tc_kernel) runs every published head dim:
// 64 and 128 with 128-byte-swizzled tiles, 80 (XLS-R-1B) with no-swizzle
// core-matrix tiles.  The warp-level mma.sync kernel (attn_kernel: 64 queries
// x 64 keys per step, K/V double buffered with cp.async) remains only for a
// qkv buffer that TMA cannot address (not 16-byte aligned).
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

// ── tcgen05 flash attention (head dim 64 or 128) ────────────────────────────
// One CTA per (utterance, head, 128-query tile); 192 threads:
//   warp 0      TMA: Q once, then K/V tiles of KV keys through a kStages ring
//   warp 1      one thread issues tcgen05.mma: S = Q K^T into one of two TMEM
//               S buffers, then O += P V with P read from TMEM (A operand)
//               and V straight from its TMA tile as an MN-major operand
//   warps 2..5  softmax, one query row per thread (its TMEM lane), in two
//               passes over S (row max, then 2^x and P) so only 32 scores
//               are live in registers; P is packed to fp16 over the first
//               KV/2 columns of its S buffer (each 32-score chunk is read
//               before the 16 columns it overwrites).
// The running max used as the exponent reference is only raised when the
// row max exceeds it by more than 2^8 (in the exp2 domain): P then stays
// <= 256 (exact in fp16 range) and the O rescale in TMEM is rare.  The sum
// and O use the same reference, so the result is unchanged.
// Pipeline: S(j+1) is computed into the other buffer while the softmax works
// on S(j).  The single MMA thread issues, in order, S(0), then per tile j:
// S(j+1), [wait for P(j)], PV(j).  PV(j) reads P(j) from buffer j & 1 before
// S(j+2) overwrites it (in-order execution); S(j) completing implies PV(j-2)
// has.  A softmax that must rescale O at tile j first waits for PV(j-1)
// (pv_done), so O then holds PV(0..j-1).  P(j) is published on p_full[j & 1]:
// S(j+1) is ready before PV(j) is issued, so a softmax warp can finish tile
// j+1 while another is still on tile j, and with one barrier its second
// arrival would complete tile j's phase early.  With one P barrier per S
// buffer a warp is at most one tile ahead (S(j+2) waits for PV(j), which
// waits for every warp's P(j)), and every arrival, s_full and pv_done phase
// is at most one phase from the one its waiter expects.  Handoffs use
// mbarriers with bounded waits.
// TMEM: S buffers at columns 0..KV-1 and KV..2KV-1, O at 2KV..2KV+D-1: 256
// columns, so two CTAs share an SM; the K/V ring is as deep as that allows.
template <int D, int KV, bool NS = false>
struct AttnTc {
    static constexpr int kAtoms = NS ? 1 : D / 64;      // 64-column swizzle atoms per row
    static constexpr int kTileQ = 128 * D * 2;
    static constexpr int kTileKV = KV * D * 2;          // one K or V tile
    static constexpr int kAtomQ = 128 * 128;            // 128 rows x 128 B
    static constexpr int kAtomKV = KV * 128;
    static constexpr int kColO = 2 * KV;
    static constexpr int kTmemCols = 2 * KV + D <= 128 ? 128 : 2 * KV + D <= 256 ? 256 : 512;
    static constexpr int kMinBlocks = kTmemCols <= 128 ? 4 : kTmemCols <= 256 ? 2 : 1;
    // K/V stages: as many as kMinBlocks CTAs per SM leave room for, 2..4
    static constexpr int kFit = ((228 * 1024) / kMinBlocks - 1024 - kTileQ - 1024 - 128) / (2 * kTileKV);
    static constexpr int kStages = kFit > 4 ? 4 : kFit < 2 ? 2 : kFit;
    static constexpr int kSmem = kTileQ + kStages * 2 * kTileKV + 1024 + 128;
};

constexpr float kLazyRescaleLog2 = 8.f;

// NS (head dims that are not a multiple of 64, e.g. 80): Q, K and V tiles are
// loaded through a 3-D view (8 columns, rows, column chunks of 8) into the
// no-swizzle core-matrix layout [chunk][row][16 bytes]; Q and K are read as
// K-major operands (LBO = chunk stride, SBO = 8 rows), V as the MN-major
// operand (SBO = chunk stride, LBO = 8 keys).
template <int D, int KV, bool NS>
__global__ void __launch_bounds__(192, AttnTc<D, KV, NS>::kMinBlocks)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
               __half* __restrict__ out, const long long* __restrict__ off, const int* __restrict__ Tn, int H,
               float scale_log2, int* err) {
    using Cfg = AttnTc<D, KV, NS>;
    constexpr int kChunks = KV / 32;
    const int u = blockIdx.z, h = blockIdx.y;
    const int T = Tn[u];
    const int q0 = blockIdx.x * 128;
    if (q0 >= T) return;
    const long long base = off[u];
    const int n_kv = (T + KV - 1) / KV;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* sQ = smem;
    uint8_t* sKV = sQ + Cfg::kTileQ;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + Cfg::kStages * 2 * Cfg::kTileKV);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;                     // [kStages]
    uint64_t* kv_empty = bars + 1 + Cfg::kStages;     // [kStages]
    uint64_t* s_full = bars + 1 + 2 * Cfg::kStages;   // [2] one per S buffer
    uint64_t* p_full = s_full + 2;                    // [2] one per S buffer
    uint64_t* pv_done = s_full + 4;
    uint64_t* o_full = s_full + 5;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 6);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < Cfg::kStages; s++) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(&p_full[0], 4);
        mbar_init(&p_full[1], 4);
        mbar_init(pv_done, 1);
        mbar_init(o_full, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmq);
        tma_prefetch_desc(&tmkv);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t tO = tmem_base + Cfg::kColO;
    const int colQ = h * D, colK = H + h * D, colV = 2 * H + h * D;

    if (warp == 0) {
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, Cfg::kTileQ);
            if constexpr (NS) {
                tma_load_3d(sQ, &tmq, q_full, 0, (int)(base + q0), colQ / 8);
            } else {
#pragma unroll
                for (int a = 0; a < Cfg::kAtoms; a++)
                    tma_load_2d(sQ + a * Cfg::kAtomQ, &tmq, q_full, colQ + 64 * a, (int)(base + q0));
            }
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            for (int j = 0; j < n_kv; j++) {
                if (!mbar_wait(&kv_empty[stage], phase ^ 1u, err)) break;
                mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::kTileKV);
                uint8_t* sK = sKV + stage * 2 * Cfg::kTileKV;
                uint8_t* sV = sK + Cfg::kTileKV;
                if constexpr (NS) {
                    tma_load_3d(sK, &tmkv, &kv_full[stage], 0, (int)(base + j * KV), colK / 8);
                    tma_load_3d(sV, &tmkv, &kv_full[stage], 0, (int)(base + j * KV), colV / 8);
                } else {
#pragma unroll
                    for (int a = 0; a < Cfg::kAtoms; a++) {
                        tma_load_2d(sK + a * Cfg::kAtomKV, &tmkv, &kv_full[stage], colK + 64 * a,
                                    (int)(base + j * KV));
                        tma_load_2d(sV + a * Cfg::kAtomKV, &tmkv, &kv_full[stage], colV + 64 * a,
                                    (int)(base + j * KV));
                    }
                }
                issued |= 1u << stage;
                last_par = (last_par & ~(1u << stage)) | (phase << stage);
                if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
            }
            // never leave with a bulk copy still writing shared memory
            mbar_wait(q_full, 0, err);
            for (int s = 0; s < Cfg::kStages; s++)
                if (issued & (1u << s)) mbar_wait(&kv_full[s], (last_par >> s) & 1u, err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc_s = umma_idesc_f16(128, KV);
            constexpr uint32_t idesc_o = umma_idesc_f16_bmn(128, D);
            // descriptors built once, advanced by (byte offset >> 4) in their
            // start-address field (shared memory < 256 KB: no carry out of it)
            // K-step advance per 16 columns / 16 keys, in 16-byte units (no-swizzle layout)
            constexpr uint32_t kQStep = 2 * 128, kKStep = 2 * KV, kVStep = NS ? 16 : 128;
            const uint64_t q_desc = NS ? umma_desc_noswz(smem_u32(sQ), 128 * 16, 128) : umma_desc_sw128(smem_u32(sQ));
            const uint64_t k_desc0 =
                NS ? umma_desc_noswz(smem_u32(sKV), KV * 16, 128) : umma_desc_sw128(smem_u32(sKV));
            const uint64_t v_desc0 = NS ? umma_desc_noswz(smem_u32(sKV + Cfg::kTileKV), 128, KV * 16)
                                        : umma_desc_sw128_mn(smem_u32(sKV + Cfg::kTileKV), Cfg::kAtomKV);
            // S(i) = Q K(i)^T into S buffer i & 1, from K/V stage i % kStages
            auto issue_s = [&](int i) {
                const uint64_t so = (uint64_t)(((i % Cfg::kStages) * 2 * Cfg::kTileKV) >> 4);
                const uint32_t tSi = tmem_base + (uint32_t)((i & 1) * KV);
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t oq = NS ? kk * kQStep : ((kk / 4) * Cfg::kAtomQ + (kk % 4) * 32) >> 4;
                    const uint32_t ok_ = NS ? kk * kKStep : ((kk / 4) * Cfg::kAtomKV + (kk % 4) * 32) >> 4;
                    umma_f16(tSi, q_desc + oq, k_desc0 + so + ok_, idesc_s, kk > 0);
                }
                umma_commit(&s_full[i & 1]);
            };
            bool ok = mbar_wait(q_full, 0, err) && mbar_wait(&kv_full[0], 0, err);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < n_kv && ok; j++) {
                if (j + 1 < n_kv) {
                    if (!mbar_wait(&kv_full[(j + 1) % Cfg::kStages], (uint32_t)((j + 1) / Cfg::kStages) & 1u, err))
                        break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(&p_full[j & 1], (uint32_t)(j >> 1) & 1u, err)) break;
                tc_fence_after();
                const int sj = j % Cfg::kStages;
                const uint64_t so = (uint64_t)((sj * 2 * Cfg::kTileKV) >> 4);
                const uint32_t tSj = tmem_base + (uint32_t)((j & 1) * KV);
#pragma unroll
                for (int kk = 0; kk < KV / 16; kk++)
                    umma_f16_tmem_a(tO, tSj + (uint32_t)(kk * 8), v_desc0 + so + (uint64_t)(kk * kVStep), idesc_o,
                                    (j > 0 || kk > 0));
                umma_commit(pv_done);
                umma_commit(&kv_empty[sj]);
            }
            umma_commit(o_full);   // also reached on error: completes once the issued MMAs have
        }
        __syncwarp();
    } else {
        const int qd = warp & 3;                       // TMEM lane quarter
        const int row = qd * 32 + lane;
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        float m = -INFINITY, l = 0.f;                  // exponent reference (raw score units) and row sum
        bool ok = true;
        for (int j = 0; j < n_kv && ok; j++) {
            const uint32_t tS = tmem_base + (uint32_t)((j & 1) * KV);   // this tile's S buffer
            if (!mbar_wait(&s_full[j & 1], (uint32_t)(j >> 1) & 1u, err)) { ok = false; break; }
            tc_fence_after();
            const int nvalid = T - j * KV < KV ? T - j * KV : KV;   // keys of this tile inside the utterance
            const bool full = nvalid == KV;
            // pass 1: row max (a single 32-score chunk stays in registers for pass 2)
            float mx = -INFINITY;
            float t1[32];
#pragma unroll
            for (int c = 0; c < kChunks; c++) {
                float t[32];
                tmem_ld32(tS + lane_off + c * 32, t);
                if constexpr (kChunks == 1) {
#pragma unroll
                    for (int i = 0; i < 32; i++) t1[i] = t[i];
                }
                if (full) {
                    float m0 = mx, m1 = t[0];
#pragma unroll
                    for (int i = 1; i < 29; i += 4) {   // t[1] .. t[28]
                        m0 = max3f(m0, t[i], t[i + 1]);
                        m1 = max3f(m1, t[i + 2], t[i + 3]);
                    }
                    mx = max3f(max3f(m0, m1, t[29]), t[30], t[31]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (c * 32 + i < nvalid) mx = fmaxf(mx, t[i]);
                }
            }
            const bool raise = (mx - m) * scale_log2 > kLazyRescaleLog2;   // always at j == 0
            float o_scale = 1.f;
            if (raise) {
                o_scale = ex2_sfu((m - mx) * scale_log2);      // 0 at j == 0
                l *= o_scale;
                m = mx;
            }
            // rescale O once it holds PV(0..j-1)
            if (j > 0 && __any_sync(0xffffffffu, raise)) {
                if (!mbar_wait(pv_done, (uint32_t)(j - 1) & 1u, err)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int a = 0; a < D / 16; a++) {        // 16-column steps: D = 80 is not a multiple of 32
                    float t[16];
                    tmem_ld16(tO + lane_off + a * 16, t);
                    uint32_t u[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) u[i] = __float_as_uint(t[i] * o_scale);
                    tmem_st16(tO + lane_off + a * 16, u);
                }
                tmem_wait_st();
            }
            // pass 2: P = 2^(s*scale - m*scale) in fp16 over S's first KV/2 columns
            const float ms = m * scale_log2;
            float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
            for (int c = 0; c < kChunks; c++) {
                float t[32];
                if constexpr (kChunks == 1) {
#pragma unroll
                    for (int i = 0; i < 32; i++) t[i] = t1[i];
                } else {
                    tmem_ld32(tS + lane_off + c * 32, t);
                }
                uint32_t pk[16];
                if (full) {
                    // pairs: (s * scale - m * scale) and the running sums two at a time
                    const uint64_t sc2 = f32x2(scale_log2, scale_log2), nm2 = f32x2(-ms, -ms);
                    uint64_t s2 = f32x2(sum0, sum1);
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float y0, y1;
                        f32x2_split(fma_f32x2(f32x2(t[i], t[i + 1]), sc2, nm2), y0, y1);
                        const float p0 = ex2_sfu(y0), p1 = ex2_sfu(y1);
                        s2 = add_f32x2(s2, f32x2(p0, p1));
                        pk[i / 2] = pack_half2(p0, p1);
                    }
                    f32x2_split(s2, sum0, sum1);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float p0 = c * 32 + i < nvalid ? ex2_sfu(fmaf(t[i], scale_log2, -ms)) : 0.f;
                        const float p1 = c * 32 + i + 1 < nvalid ? ex2_sfu(fmaf(t[i + 1], scale_log2, -ms)) : 0.f;
                        sum0 += p0;
                        sum1 += p1;
                        pk[i / 2] = pack_half2(p0, p1);
                    }
                }
                tmem_st16(tS + lane_off + c * 16, pk);
            }
            l += sum0 + sum1;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[j & 1]);
        }
        // o_full is committed on every path once the issued MMAs complete: wait
        // for it even after an expired wait, so TMEM is never freed under an MMA
        if (mbar_wait(o_full, 0, err) && ok) {
            tc_fence_after();
            const float inv = __fdividef(1.f, l);
            const bool valid = q0 + row < T;
            __half* o = out + (base + q0 + row) * (long long)H + (long long)h * D;
#pragma unroll
            for (int a = 0; a < D / 16; a++) {
                float t[16];
                tmem_ld16(tO + lane_off + a * 16, t);
                if (valid) {
#pragma unroll
                    for (int v = 0; v < 2; v++) {
                        uint4 pk;
                        pk.x = pack_half2(t[8 * v + 0] * inv, t[8 * v + 1] * inv);
                        pk.y = pack_half2(t[8 * v + 2] * inv, t[8 * v + 3] * inv);
                        pk.z = pack_half2(t[8 * v + 4] * inv, t[8 * v + 5] * inv);
                        pk.w = pack_half2(t[8 * v + 6] * inv, t[8 * v + 7] * inv);
                        *reinterpret_cast<uint4*>(o + a * 16 + v * 8) = pk;
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

static PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
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

template <int D, int KV, bool NS>
static int launch_attn_tc(const void* qkv, void* out, const long long* off, const int* T, int n_utt, int H,
                          int n_heads, int max_T, long long M, int* err, cudaStream_t st) {
    using Cfg = AttnTc<D, KV, NS>;
    auto enc = attn_encode_fn();
    if (!enc) return W2V_ERR_DRIVER;
    // two views of qkv [M][3H]: 128-row boxes for Q, KV-row boxes for K and V
    CUtensorMap tmq, tmkv;
    CUresult r1, r2;
    if constexpr (NS) {
        // (8 columns, rows, 8-column chunks): boxes land as [chunk][row][16 B]
        const uint64_t dims[3] = {8, (uint64_t)M, (uint64_t)3 * H / 8};
        const uint64_t strides[2] = {(uint64_t)3 * H * 2, 16};
        const uint32_t es[3] = {1, 1, 1};
        const uint32_t boxq[3] = {8, 128, D / 8}, boxkv[3] = {8, (uint32_t)KV, D / 8};
        r1 = enc(&tmq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(qkv), dims, strides, boxq, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        r2 = enc(&tmkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(qkv), dims, strides, boxkv, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const uint64_t dims[2] = {(uint64_t)3 * H, (uint64_t)M};
        const uint64_t strides[1] = {(uint64_t)3 * H * 2};
        const uint32_t es[2] = {1, 1};
        const uint32_t boxq[2] = {64, 128}, boxkv[2] = {64, (uint32_t)KV};
        r1 = enc(&tmq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(qkv), dims, strides, boxq, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        r2 = enc(&tmkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(qkv), dims, strides, boxkv, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) return W2V_ERR_TENSOR_MAP;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(attn_tc_kernel<D, KV, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cfg::kSmem) != cudaSuccess)
            return W2V_ERR_LAUNCH;
        attr[dev & 63] = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    dim3 grid((max_T + 127) / 128, n_heads, n_utt);
    attn_tc_kernel<D, KV, NS><<<grid, 192, Cfg::kSmem, st>>>(tmq, tmkv, (__half*)out, off, T, H, scale_log2, err);
    return cudaPeekAtLastError() == cudaSuccess ? W2V_OK : W2V_ERR_LAUNCH;
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
                             int n_heads, int max_T, long long M, int* err, void* stream) {
    if (n_heads <= 0 || H % n_heads || M < 0) return W2V_ERR_ARGS;
    if (n_utt <= 0 || max_T <= 0 || M == 0) return W2V_OK;
    const int d = H / n_heads;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool tma_ok = (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && H % 64 == 0;
    switch (d) {
        case 64:
            if (tma_ok) return w2v::launch_attn_tc<64, 32, false>(qkv, out, off, T, n_utt, H, n_heads, max_T, M, err, st);
            return w2v::launch_attn<64>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        case 80:
            if ((reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && H % 8 == 0)
                return w2v::launch_attn_tc<80, 32, true>(qkv, out, off, T, n_utt, H, n_heads, max_T, M, err, st);
            return w2v::launch_attn<80>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        case 128:
            if (tma_ok) return w2v::launch_attn_tc<128, 32, false>(qkv, out, off, T, n_utt, H, n_heads, max_T, M, err, st);
            return w2v::launch_attn<128>(qkv, out, off, T, n_utt, H, n_heads, max_T, st);
        default: return W2V_ERR_ARGS;
    }
}
