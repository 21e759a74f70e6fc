// Shared device helpers for the sm_100a kernels: mbarriers with bounded
// waits, TMA (cp.async.bulk.tensor) loads, tcgen05 (UMMA / TMEM) wrappers,
// fp16 packing and the reference's tanh-form GELU.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define W2V_DEV __device__ __forceinline__

namespace w2v {

// Error codes written to the engine's device error word (first writer wins).
enum : int {
    kErrNone = 0,
    kErrBarrierTimeout = 1,   // an mbarrier wait exceeded its time limit
    kErrBadArgs = 2,
};

// Upper bound for any mbarrier wait (ns).  Kernels normally wait microseconds;
// on expiry the waiting thread records kErrBarrierTimeout and abandons the
// pipeline so that the launch ends instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

W2V_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

W2V_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

W2V_DEV void report_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ── mbarrier ────────────────────────────────────────────────────────────────
W2V_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
W2V_DEV void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
W2V_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
                 : "memory");
}
W2V_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
W2V_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity.  Returns false (and
// records the error) if the limit expired.
W2V_DEV bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 255u) == 0 && globaltimer() - t0 > limit_ns) {
            report_error(err, kErrBarrierTimeout);
            return false;
        }
    }
    return true;
}
W2V_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    return mbar_wait_for(bar, parity, err, kWaitLimitNs);
}
// Bounded wait with cluster-scope acquire: for phases completed by arrivals
// from the other CTA of a pair whose writes the waiter relies on.
W2V_DEV bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
W2V_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (!mbar_try_wait_cluster(bar, parity)) {
        if ((++spins & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
            report_error(err, kErrBarrierTimeout);
            return false;
        }
    }
    return true;
}

// ── TMA ────────────────────────────────────────────────────────────────────
W2V_DEV void tma_prefetch_desc(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
W2V_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
W2V_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
W2V_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// Tile store shared -> global (one destination); completion tracked per thread
// through bulk async-groups.  Coordinates must be non-negative and the
// innermost one a multiple of 16 bytes.
W2V_DEV void tma_store_3d(const CUtensorMap* m, const void* smem_src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
W2V_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed groups still read shared memory.
template <int N>
W2V_DEV void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's committed groups are incomplete.
template <int N>
W2V_DEV void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ── tcgen05 (5th-gen tensor cores, accumulators in TMEM) ────────────────────
W2V_DEV void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
W2V_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
W2V_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
W2V_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
W2V_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16/bf16 in, fp32 accumulate).
W2V_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
W2V_DEV void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Instruction descriptor for kind::f16: fp16 A/B (K-major), fp32 accumulator.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4)                          // D format: f32
           | (0u << 7) | (0u << 10)           // A, B format: f16
           | (0u << 15) | (0u << 16)          // A, B K-major
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B,
// 8-row atoms of 1024 B (SBO), tile base 1024-byte aligned.
W2V_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);      // start address
    d |= (uint64_t)1 << 16;                        // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;              // SBO
    d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
    return d;
}
// K-major, no swizzle ("interleaved" core matrices of 8 rows x 16 B):
// LBO = byte distance between core matrices adjacent in K,
// SBO = byte distance between core matrices adjacent in M/N.
W2V_DEV uint64_t umma_desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// 32 lanes x 32 consecutive fp32 columns of TMEM -> 32 registers per thread.
W2V_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

W2V_DEV bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n .reg .pred p;\n .reg .b32 r;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(pred));
    return pred != 0;
}

// ── numerics ────────────────────────────────────────────────────────────────
// The reference's tanh-approximation GELU (ops.h:18-21),
//   0.5 x (1 + tanh(u)),  u = 0.7978845608 (x + 0.044715 x^3),
// evaluated through 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)) with the
// constants folded into the exponent: -2 u log2(e) = x (A + B x^2),
// A = -2 sqrt(2/pi) log2(e), B = 0.044715 A.  Five FMA-pipe operations plus
// ex2 and rcp on the special-function unit; within 1e-6 of the tanh form
// (well below the fp16 rounding of every output it feeds).  x -> -inf gives
// -0 (the power overflows to inf), x -> +inf gives x.
W2V_DEV float gelu_tanh(float x) {
    const float z = x * fmaf(x * x, -0.10294324f, -2.3022082f);
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(z));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return x * r;
}

// Three-input max and packed fp32-pair arithmetic (sm_100): one instruction
// for two lanes' worth of FMA / add; a pair is a 64-bit register (lo, hi).
W2V_DEV float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
W2V_DEV uint64_t f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
W2V_DEV void f32x2_split(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
W2V_DEV uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
W2V_DEV uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

W2V_DEV uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// gelu_tanh of two values, rounded to a packed fp16 pair: the tanh form
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) evaluated entirely on fp16
// pairs once x is rounded to fp16, six pair instructions and one of them on
// the special-function unit.  The reference evaluates the same formula with
// fp32 tanhf (src/ops.h:18-21); this is a deliberate precision trade for
// outputs that are stored as fp16 anyway: error within 2e-3 (1 + |gelu(x)|),
// about twice the fp16 rounding of the result.  Large |x|: x^2 and the tanh
// argument saturate to +-inf (tanh -> +-1), giving x or 0.
W2V_DEV uint32_t gelu_f16x2(uint32_t x) {
    const uint32_t c0 = 0x3a623a62u;   // sqrt(2/pi) in fp16, both halves
    const uint32_t c1 = 0x28912891u;   // 0.044715 sqrt(2/pi)
    const uint32_t half = 0x38003800u; // 0.5
    uint32_t x2, p, u, t, h, o;
    asm("mul.rn.f16x2 %0, %1, %1;" : "=r"(x2) : "r"(x));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p) : "r"(x2), "r"(c1), "r"(c0));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(u) : "r"(x), "r"(p));
    asm("tanh.approx.f16x2 %0, %1;" : "=r"(t) : "r"(u));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h) : "r"(x), "r"(half));
    asm("fma.rn.f16x2 %0, %1, %2, %1;" : "=r"(o) : "r"(h), "r"(t));
    return o;
}

W2V_DEV uint32_t gelu_half2(float a, float b) { return gelu_f16x2(pack_half2(a, b)); }

}  // namespace w2v

namespace w2v {
// ── warp-level fp16 MMA (used by the attention and positional-conv kernels) ──
W2V_DEV void ldsm_x4(uint32_t saddr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(saddr));
}
W2V_DEV void ldsm_x4_t(uint32_t saddr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(saddr));
}
// D(16x8 fp32) += A(16x16 fp16, row) * B(16x8 fp16, col)
W2V_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
W2V_DEV void cp_async16(uint32_t saddr, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
W2V_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
W2V_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
}  // namespace w2v

namespace w2v {
// ── more tcgen05 helpers (attention) ────────────────────────────────────────
// 32 lanes x 32 consecutive 32-bit TMEM columns <- 32 registers per thread.
W2V_DEV void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Instruction descriptor for kind::f16 with A K-major and B MN-major
// (B element (n, k) at n contiguous: e.g. V stored [key][d]).
__host__ __device__ constexpr uint32_t umma_idesc_f16_bmn(int M, int N) {
    return umma_idesc_f16(M, N) | (1u << 16);
}

// MN-major, 128-byte swizzle: rows along K of 128 B (64 fp16 along MN), 8-row
// atoms of 1024 B (SBO); lbo = byte distance between 64-wide MN atoms.
W2V_DEV uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

W2V_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
}  // namespace w2v

namespace w2v {
// ── CTA-pair (cluster of 2) helpers for cta_group::2 ────────────────────────
W2V_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
W2V_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same smem location in CTA `rank` of the cluster
W2V_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
W2V_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrive on an mbarrier of either CTA of the pair with the default (CTA-scope)
// release.  For hand-offs whose payload is tensor-memory state ordered by
// tcgen05.fence::before_thread_sync: a cluster-scope release would also make
// the arriving thread wait until all of its earlier global stores are
// performed, which stalls an epilogue that has just issued thousands.
W2V_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
W2V_DEV void mbar_arrive_expect_tx_addr(uint32_t saddr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr), "r"(bytes) : "memory");
}
// TMA load whose completion is signalled on an mbarrier that may live in the
// peer CTA of the pair (cluster address).
W2V_DEV void tma_load_4d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster, int c0, int c1, int c2,
                              int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
W2V_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}
W2V_DEV void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
W2V_DEV void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
W2V_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (256 rows over the CTA pair) (+)= A . B^T, issued by the pair's leader.
W2V_DEV void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier (shared::cluster address: this CTA's or the peer's)
// once every tcgen05 operation this thread issued before has completed.
W2V_DEV void umma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}
}  // namespace w2v

namespace w2v {
// D (+)= A . B^T with A (M x K, 16-bit, K-major) read from TMEM: lane m holds
// row m, 32-bit column c holds elements (2c, 2c+1), the lower index in the
// low half.
W2V_DEV void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                             uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes <- registers.
W2V_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
W2V_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 2^x on the SFU (ex2.approx.ftz.f32): relative error about 2^-22, 0 for -inf.
W2V_DEV float ex2_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
}  // namespace w2v


namespace w2v {
// Bulk (non-tensor) global -> shared copy completing on an mbarrier; both
// addresses 16-byte aligned, bytes a multiple of 16.
W2V_DEV void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// 32 lanes x 16 consecutive fp32 TMEM columns -> registers (waits for completion).
W2V_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
}  // namespace w2v

namespace w2v {
// Per-warp 32 x 32 fp32 transpose through a private 4 KB shared buffer:
// stage_put writes a row per lane (float4 groups XOR-swizzled by row, so
// both this and the reads below are bank-conflict free); stage_get then reads
// row r, column group cg (4 floats), letting a warp work on 4 rows x 32
// columns per instruction (thread t: column group t%8 of rows t/8 + 4i).
W2V_DEV void stage_put(float* stg, const float (&v)[32]) {
    const int lane = threadIdx.x & 31;
    float4* row = reinterpret_cast<float4*>(stg + lane * 32);
#pragma unroll
    for (int j = 0; j < 8; j++) row[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
W2V_DEV float4 stage_get(const float* stg, int r, int cg) {
    return reinterpret_cast<const float4*>(stg + r * 32)[cg ^ (r & 7)];
}
}  // namespace w2v
