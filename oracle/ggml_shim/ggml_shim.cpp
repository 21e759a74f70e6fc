// Oracle-only ggml-API shim: just enough of ggml for the reference's
// src/ggml_backend.h to build and run on the CPU.  Test infrastructure; the
// product never links it.
//
// ggml (github.com/ggerganov/ggml) is absent from the reference checkout and
// unpinned (.gitmodules:1-3, empty third_party/ggml).  The matmul arithmetic
// below restates ggml's published CPU algorithm for `ggml_mul_mat(W, x)`:
//
//   * W in Q8_0 or Q4_0: each activation row is first quantized to Q8_0
//     blocks (32 values, d = amax/127 stored as fp16, q = round(x/d)), then
//     y[m][n] = sum_b (int dot of block b) * d_w[b] * d_x[b], in fp32.
//   * W in F16: activations are rounded to fp16, products summed in double.
//   * W in F32: fp32 products summed in double.
//
// Mode "exact" (env W2V_ORACLE_LINEAR=exact) instead keeps fp32 activations
// and sums fp32(x) * fp32(dequant(W)) in double -- the ideal fp32 linear.
// Which of the two ggml really does cannot be checked here; "ggml" mode is the
// assumed default.
#include "ggml.h"
#include "ggml-cpu.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>
#include <stdexcept>

namespace {

struct Graph {
    int n_nodes = 0;
    ggml_tensor * nodes[64];
};

constexpr size_t kAlign = 32;

size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

uint16_t fp32_to_fp16_rne(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) {                       // inf / nan
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf
    if (absx < 0x38800000u) {                        // result subnormal or zero
        // value = absx as float; fp16 subnormal unit = 2^-24
        float a; memcpy(&a, &absx, 4);
        float scaled = a * 16777216.0f;              // exact (power of two)
        // round half to even on the integer part
        float r = nearbyintf(scaled);
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t mant = absx & 0x7fffffu;
    uint32_t exp = (absx >> 23) - 127 + 15;
    uint32_t h = (exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // may carry into exponent: correct
    return (uint16_t)(sign | h);
}

float fp16_to_fp32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) { bits = s; }
        else {
            float f = (float)m * (1.0f / 16777216.0f);
            memcpy(&bits, &f, 4); bits |= s;
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}

bool exact_mode() {
    const char * m = getenv("W2V_ORACLE_LINEAR");
    return m && std::string(m) == "exact";
}

size_t row_bytes(ggml_type t, int64_t ne0) {
    switch (t) {
        case GGML_TYPE_F32:  return (size_t)ne0 * 4;
        case GGML_TYPE_F16:  return (size_t)ne0 * 2;
        case GGML_TYPE_Q4_0: return (size_t)(ne0 / 32) * 18;
        case GGML_TYPE_Q8_0: return (size_t)(ne0 / 32) * 34;
        default: throw std::runtime_error("ggml shim: unsupported tensor type " + std::to_string((int)t));
    }
}

// One activation row quantized to Q8_0: K/32 scales and K int8 values.
struct Q8Row { std::vector<float> d; std::vector<int8_t> q; };

void quantize_row_q8_0(const float * x, int64_t K, float * d_out, int8_t * q_out) {
    for (int64_t b = 0; b < K / 32; b++) {
        const float * xb = x + b * 32;
        float amax = 0.f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        d_out[b] = fp16_to_fp32(fp32_to_fp16_rne(d));
        for (int j = 0; j < 32; j++) q_out[b * 32 + j] = (int8_t)roundf(xb[j] * id);
    }
}

inline int32_t dot32_i8(const int8_t * a, const int8_t * b) {
    int32_t s = 0;
    for (int j = 0; j < 32; j++) s += (int32_t)a[j] * (int32_t)b[j];
    return s;
}

void dequant_row(const uint8_t * src, ggml_type t, int64_t K, float * out) {
    if (t == GGML_TYPE_F32) { memcpy(out, src, (size_t)K * 4); return; }
    if (t == GGML_TYPE_F16) {
        const uint16_t * h = (const uint16_t *)src;
        for (int64_t i = 0; i < K; i++) out[i] = fp16_to_fp32(h[i]);
        return;
    }
    for (int64_t b = 0; b < K / 32; b++) {
        if (t == GGML_TYPE_Q8_0) {
            const uint8_t * blk = src + b * 34;
            uint16_t dh; memcpy(&dh, blk, 2);
            const float d = fp16_to_fp32(dh);
            const int8_t * q = (const int8_t *)(blk + 2);
            for (int j = 0; j < 32; j++) out[b * 32 + j] = d * (float)q[j];
        } else {
            const uint8_t * blk = src + b * 18;
            uint16_t dh; memcpy(&dh, blk, 2);
            const float d = fp16_to_fp32(dh);
            for (int j = 0; j < 16; j++) {
                out[b * 32 + j]      = d * (float)((int)(blk[2 + j] & 0xf) - 8);
                out[b * 32 + j + 16] = d * (float)((int)(blk[2 + j] >> 4) - 8);
            }
        }
    }
}

// y[M][N] = x[M][K] . W[N][K]^T with ggml's per-type vec_dot semantics.
void mul_mat(const ggml_tensor * W, const ggml_tensor * X, ggml_tensor * Y, int n_threads) {
    const int64_t K = W->ne[0], N = W->ne[1], M = X->ne[1];
    if (X->ne[0] != K) throw std::runtime_error("ggml shim: mul_mat K mismatch");
    const float * x = (const float *)X->data;
    float * y = (float *)Y->data;
    const uint8_t * w = (const uint8_t *)W->data;
    const size_t wrow = row_bytes(W->type, K);
    const bool exact = exact_mode();
    const ggml_type wt = W->type;
    const bool quant = (wt == GGML_TYPE_Q8_0 || wt == GGML_TYPE_Q4_0);

    // Activation conversion to the vec_dot type (done once, shared by threads).
    std::vector<float> xd;            // Q8_0 scales per block
    std::vector<int8_t> xq;           // Q8_0 values
    std::vector<float> xh;            // fp16-rounded activations (as fp32)
    if (!exact) {
        if (quant) {
            xd.resize((size_t)M * (K / 32)); xq.resize((size_t)M * K);
            for (int64_t m = 0; m < M; m++)
                quantize_row_q8_0(x + m * K, K, &xd[m * (K / 32)], &xq[m * K]);
        } else if (wt == GGML_TYPE_F16) {
            xh.resize((size_t)M * K);
            for (int64_t i = 0; i < M * K; i++) xh[i] = fp16_to_fp32(fp32_to_fp16_rne(x[i]));
        }
    }

    auto work = [&](int64_t n0, int64_t n1) {
        std::vector<float> wf(K);
        std::vector<int8_t> wq(K);
        std::vector<float> wd(K / 32);
        for (int64_t n = n0; n < n1; n++) {
            const uint8_t * wr = w + n * wrow;
            if (!exact && quant) {
                // Unpack the weight row's blocks once: int values + scales.
                for (int64_t b = 0; b < K / 32; b++) {
                    if (wt == GGML_TYPE_Q8_0) {
                        const uint8_t * blk = wr + b * 34;
                        uint16_t dh; memcpy(&dh, blk, 2);
                        wd[b] = fp16_to_fp32(dh);
                        memcpy(&wq[b * 32], blk + 2, 32);
                    } else {
                        const uint8_t * blk = wr + b * 18;
                        uint16_t dh; memcpy(&dh, blk, 2);
                        wd[b] = fp16_to_fp32(dh);
                        for (int j = 0; j < 16; j++) {
                            wq[b * 32 + j]      = (int8_t)((int)(blk[2 + j] & 0xf) - 8);
                            wq[b * 32 + j + 16] = (int8_t)((int)(blk[2 + j] >> 4) - 8);
                        }
                    }
                }
                for (int64_t m = 0; m < M; m++) {
                    const int8_t * q = &xq[m * K];
                    const float * d = &xd[m * (K / 32)];
                    float sumf = 0.f;
                    if (wt == GGML_TYPE_Q8_0) {
                        for (int64_t b = 0; b < K / 32; b++)
                            sumf += (float)dot32_i8(&wq[b * 32], q + b * 32) * (wd[b] * d[b]);
                    } else {
                        for (int64_t b = 0; b < K / 32; b++)
                            sumf += (float)dot32_i8(&wq[b * 32], q + b * 32) * wd[b] * d[b];
                    }
                    y[m * N + n] = sumf;
                }
            } else {
                dequant_row(wr, wt, K, wf.data());
                const float * xs = (!exact && wt == GGML_TYPE_F16) ? xh.data() : x;
                for (int64_t m = 0; m < M; m++) {
                    const float * xr = xs + m * K;
                    double acc = 0.0;
                    for (int64_t k = 0; k < K; k++) acc += (double)(wf[k] * xr[k]);
                    y[m * N + n] = (float)acc;
                }
            }
        }
    };

    int nt = n_threads < 1 ? 1 : n_threads;
    if (nt > N) nt = (int)N;
    if (nt == 1) { work(0, N); return; }
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; t++) {
        int64_t n0 = N * t / nt, n1 = N * (t + 1) / nt;
        pool.emplace_back(work, n0, n1);
    }
    for (auto & th : pool) th.join();
}

}  // namespace

struct ggml_context {
    uint8_t * buf = nullptr;
    size_t size = 0;
    size_t used = 0;
    bool owned = false;
    bool no_alloc = false;

    void * alloc(size_t n) {
        size_t off = align_up(used);
        if (off + n > size) throw std::runtime_error("ggml shim: context out of memory");
        used = off + n;
        return buf + off;
    }
};

extern "C" {

struct ggml_context * ggml_init(struct ggml_init_params params) {
    auto * ctx = new ggml_context();
    ctx->size = params.mem_size;
    ctx->no_alloc = params.no_alloc;
    if (params.mem_buffer) {
        ctx->buf = (uint8_t *)params.mem_buffer;
    } else {
        ctx->buf = (uint8_t *)aligned_alloc(kAlign, align_up(params.mem_size ? params.mem_size : kAlign));
        ctx->owned = true;
        if (!ctx->buf) { delete ctx; return nullptr; }
    }
    return ctx;
}

void ggml_free(struct ggml_context * ctx) {
    if (!ctx) return;
    if (ctx->owned) free(ctx->buf);
    delete ctx;
}

size_t ggml_tensor_overhead(void) { return align_up(sizeof(ggml_tensor)) + kAlign; }
size_t ggml_graph_overhead(void) { return align_up(sizeof(Graph)) + kAlign; }

size_t ggml_nbytes(const struct ggml_tensor * t) {
    return row_bytes(t->type, t->ne[0]) * (size_t)t->ne[1] * (size_t)t->ne[2] * (size_t)t->ne[3];
}

struct ggml_tensor * ggml_new_tensor_2d(struct ggml_context * ctx, enum ggml_type type,
                                        int64_t ne0, int64_t ne1) {
    auto * t = (ggml_tensor *)ctx->alloc(sizeof(ggml_tensor));
    memset(t, 0, sizeof(*t));
    t->type = type;
    t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = 1; t->ne[3] = 1;
    t->nb[0] = (type == GGML_TYPE_F32) ? 4 : (type == GGML_TYPE_F16 ? 2 : 1);
    t->nb[1] = row_bytes(type, ne0);
    t->nb[2] = t->nb[1] * ne1; t->nb[3] = t->nb[2];
    t->op = GGML_OP_NONE;
    t->data = ctx->no_alloc ? nullptr : ctx->alloc(ggml_nbytes(t));
    return t;
}

struct ggml_tensor * ggml_mul_mat(struct ggml_context * ctx,
                                  struct ggml_tensor * a, struct ggml_tensor * b) {
    auto * r = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, a->ne[1], b->ne[1]);
    r->op = GGML_OP_MUL_MAT;
    r->src[0] = a; r->src[1] = b;
    return r;
}

struct ggml_cgraph * ggml_new_graph(struct ggml_context * ctx) {
    auto * g = (Graph *)ctx->alloc(sizeof(Graph));
    g->n_nodes = 0;
    return (ggml_cgraph *)g;
}

void ggml_build_forward_expand(struct ggml_cgraph * gf, struct ggml_tensor * t) {
    auto * g = (Graph *)gf;
    // Depth-first: sources before the node (only MUL_MAT nodes carry work).
    for (int i = 0; i < 2; i++)
        if (t->src[i] && t->src[i]->op != GGML_OP_NONE) ggml_build_forward_expand(gf, t->src[i]);
    for (int i = 0; i < g->n_nodes; i++) if (g->nodes[i] == t) return;
    if (g->n_nodes >= 64) throw std::runtime_error("ggml shim: graph too large");
    g->nodes[g->n_nodes++] = t;
}

int ggml_graph_compute_with_ctx(struct ggml_context * ctx, struct ggml_cgraph * gf, int n_threads) {
    (void)ctx;
    auto * g = (Graph *)gf;
    for (int i = 0; i < g->n_nodes; i++) {
        ggml_tensor * t = g->nodes[i];
        if (t->op == GGML_OP_MUL_MAT) mul_mat(t->src[0], t->src[1], t, n_threads);
    }
    return 0;
}

}  // extern "C"
