/* CPU oracle for the wav2vec2 CTC forward pass -- TEST INFRASTRUCTURE ONLY.
 * See w2v_oracle.h for scope.  Every function cites the reference code it
 * restates (paths relative to the py-ai-dev/wav2vec2.cpp checkout).
 * Summation orders differ from the reference where noted; results agree with
 * the reference within fp32 rounding (checked by tests/test_oracle.py). */
#define _GNU_SOURCE
#include "w2v_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ── fp16 helpers ──────────────────────────────────────────────────────── */

/* fp16 -> fp32 widening (src/gguf.h:14-22). */
static float h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1fu, mnt = h & 0x3ffu, bits;
    if (e == 0) {
        float f = (float)mnt * (1.0f / 16777216.0f);
        memcpy(&bits, &f, 4); bits |= s;
    } else if (e == 31) {
        bits = s | 0x7f800000u | (mnt << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (mnt << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}

/* fp32 -> fp16, round to nearest even. */
static uint16_t f2h(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) {
        float af; memcpy(&af, &a, 4);
        return (uint16_t)(sign | (uint32_t)nearbyintf(af * 16777216.0f));
    }
    uint32_t h = (((a >> 23) - 112u) << 10) | ((a & 0x7fffffu) >> 13), rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* ── GGUF reader (src/gguf.h:113-195) ──────────────────────────────────── */

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8 };

typedef struct {
    char * name;
    int ndim;
    uint64_t shape[4];
    uint32_t type;
    uint64_t n;
    uint8_t * raw;      /* raw bytes (all types) */
    float * f;          /* fp32 data (F32/F16 only), as the reference's .data */
} tensor_t;

typedef struct {
    char * key;
    uint64_t u64;
    char * str;
    int n_u32, n_str;
    uint32_t * arr_u32;
    char ** arr_str;
} kv_t;

struct wvo_model {
    int n_kv, n_tensors;
    kv_t * kv;
    tensor_t * t;
    /* hyper-parameters (src/wav2vec2.cpp:133-156) */
    int n_conv, conv_dim, n_layers, n_heads, hidden, ffn, vocab, pad_id, pos_k, pos_g;
    int group_norm, stable;
    int conv_k[16], conv_s[16];
};

typedef struct { const uint8_t * p; const uint8_t * end; int bad; } rd_t;

static int rd(rd_t * r, void * dst, size_t n) {
    if (r->bad || (size_t)(r->end - r->p) < n) { r->bad = 1; memset(dst, 0, n); return 0; }
    memcpy(dst, r->p, n); r->p += n; return 1;
}
static uint32_t rd32(rd_t * r) { uint32_t v; rd(r, &v, 4); return v; }
static uint64_t rd64(rd_t * r) { uint64_t v; rd(r, &v, 8); return v; }
static char * rdstr(rd_t * r) {
    uint64_t len = rd64(r);
    if (r->bad || len > (uint64_t)(r->end - r->p)) { r->bad = 1; return calloc(1, 1); }
    char * s = malloc(len + 1); memcpy(s, r->p, len); s[len] = 0; r->p += len; return s;
}
/* Scalar KV values (src/gguf.h:95-111). */
static void read_scalar(rd_t * r, uint32_t t, kv_t * kv) {
    switch (t) {
        case 0: case 1: case 7: { uint8_t v; rd(r, &v, 1); kv->u64 = v; break; }
        case 2: case 3: { uint16_t v; rd(r, &v, 2); kv->u64 = v; break; }
        case 4: case 5: { uint32_t v; rd(r, &v, 4); kv->u64 = v; break; }
        case 6: { float v; rd(r, &v, 4); break; }
        case 8: { char * s = rdstr(r); free(kv->str); kv->str = s; break; }
        case 10: case 11: case 12: { uint64_t v; rd(r, &v, 8); kv->u64 = v; break; }
        default: r->bad = 1;
    }
}

/* Raw bytes per tensor type (src/gguf.h:46-64). */
static size_t type_nbytes(uint32_t t, uint64_t n) {
    switch (t) {
        case T_F32: return n * 4;
        case T_F16: return n * 2;
        case T_Q4_0: return n / 32 * 18;
        case 3: return n / 32 * 20;
        case 6: return n / 32 * 22;
        case 7: return n / 32 * 24;
        case T_Q8_0: return n / 32 * 34;
        case 9: return n / 32 * 36;
        default: return n * 4;
    }
}

static const kv_t * find_kv(const wvo_model * m, const char * k) {
    for (int i = 0; i < m->n_kv; i++) if (!strcmp(m->kv[i].key, k)) return &m->kv[i];
    return NULL;
}
static const tensor_t * find_t(const wvo_model * m, const char * n) {
    for (int i = 0; i < m->n_tensors; i++) if (!strcmp(m->t[i].name, n)) return &m->t[i];
    return NULL;
}
static const float * tf(const wvo_model * m, const char * n) {
    const tensor_t * t = find_t(m, n);
    return t ? t->f : NULL;
}

void wvo_free(wvo_model * m) {
    if (!m) return;
    for (int i = 0; i < m->n_kv; i++) {
        free(m->kv[i].key); free(m->kv[i].str); free(m->kv[i].arr_u32);
        for (int j = 0; j < m->kv[i].n_str; j++) free(m->kv[i].arr_str[j]);
        free(m->kv[i].arr_str);
    }
    free(m->kv);
    for (int i = 0; i < m->n_tensors; i++) { free(m->t[i].name); free(m->t[i].raw); free(m->t[i].f); }
    free(m->t);
    free(m);
}

static int need_u32(wvo_model * m, const char * k, int * dst, char * err, int errlen) {
    const kv_t * kv = find_kv(m, k);
    if (!kv) { snprintf(err, errlen, "Missing key: %s", k); return 0; }
    *dst = (int)(uint32_t)kv->u64;
    return 1;
}

wvo_model * wvo_load(const char * path, char * err, int errlen) {
    char dummy[8]; if (!err) { err = dummy; errlen = sizeof dummy; }
    FILE * fp = fopen(path, "rb");
    if (!fp) { snprintf(err, errlen, "Cannot open %s", path); return NULL; }
    fseek(fp, 0, SEEK_END); long sz = ftell(fp); fseek(fp, 0, SEEK_SET);
    uint8_t * buf = malloc(sz > 0 ? sz : 1);
    if (fread(buf, 1, sz, fp) != (size_t)sz) { fclose(fp); free(buf); snprintf(err, errlen, "read failed"); return NULL; }
    fclose(fp);
    rd_t r = { buf, buf + sz, 0 };
    wvo_model * m = calloc(1, sizeof *m);
    if (rd32(&r) != 0x46554747u) { free(buf); free(m); snprintf(err, errlen, "Not GGUF"); return NULL; }
    rd32(&r);
    uint64_t n_t = rd64(&r), n_kv = rd64(&r);
    if (r.bad || n_kv > 1000000 || n_t > 1000000) { free(buf); free(m); snprintf(err, errlen, "Truncated GGUF header"); return NULL; }
    m->kv = calloc(n_kv ? n_kv : 1, sizeof(kv_t)); m->n_kv = (int)n_kv;
    for (uint64_t i = 0; i < n_kv && !r.bad; i++) {
        kv_t * kv = &m->kv[i];
        kv->key = rdstr(&r);
        uint32_t vt = rd32(&r);
        if (vt == 9) {  /* array (src/gguf.h:130-138) */
            uint32_t et = rd32(&r); uint64_t an = rd64(&r);
            if (an > (uint64_t)(r.end - r.p)) { r.bad = 1; break; }
            for (uint64_t j = 0; j < an && !r.bad; j++) {
                if (et == 8) {
                    kv->arr_str = realloc(kv->arr_str, (kv->n_str + 1) * sizeof(char *));
                    kv->arr_str[kv->n_str++] = rdstr(&r);
                } else if (et == 4) {
                    kv->arr_u32 = realloc(kv->arr_u32, (kv->n_u32 + 1) * sizeof(uint32_t));
                    kv->arr_u32[kv->n_u32++] = rd32(&r);
                } else {
                    kv_t tmp = {0}; read_scalar(&r, et, &tmp); free(tmp.str);
                }
            }
        } else {
            read_scalar(&r, vt, kv);
        }
    }
    typedef struct { char * name; int nd; uint64_t shape[4]; uint32_t type; uint64_t off; } ti_t;
    ti_t * ti = calloc(n_t ? n_t : 1, sizeof(ti_t));
    for (uint64_t i = 0; i < n_t && !r.bad; i++) {
        ti[i].name = rdstr(&r);
        uint32_t nd = rd32(&r);
        if (nd > 4) { r.bad = 1; break; }
        ti[i].nd = (int)nd;
        for (uint32_t d = 0; d < nd; d++) ti[i].shape[d] = rd64(&r);
        ti[i].type = rd32(&r);
        ti[i].off = rd64(&r);
    }
    if (r.bad) {
        for (uint64_t i = 0; i < n_t; i++) free(ti[i].name);
        free(ti); free(buf); wvo_free(m); snprintf(err, errlen, "Truncated GGUF metadata"); return NULL;
    }
    uint64_t data_start = ((uint64_t)(r.p - buf) + 31u) & ~31ull;   /* src/gguf.h:162-165 */
    m->t = calloc(n_t ? n_t : 1, sizeof(tensor_t)); m->n_tensors = (int)n_t;
    for (uint64_t i = 0; i < n_t; i++) {
        tensor_t * t = &m->t[i];
        t->name = ti[i].name; t->ndim = ti[i].nd; t->type = ti[i].type;
        t->n = 1;
        for (int d = 0; d < t->ndim; d++) { t->shape[d] = ti[i].shape[d]; t->n *= ti[i].shape[d]; }
        size_t nb = type_nbytes(t->type, t->n);
        if (data_start + ti[i].off + nb > (uint64_t)sz) {
            free(ti); free(buf); snprintf(err, errlen, "Tensor %s extends past end of file", t->name);
            m->n_tensors = (int)i + 1; wvo_free(m); return NULL;
        }
        t->raw = malloc(nb ? nb : 1);
        memcpy(t->raw, buf + data_start + ti[i].off, nb);
        if (t->type == T_F32) {
            t->f = malloc(t->n * 4); memcpy(t->f, t->raw, t->n * 4);
        } else if (t->type == T_F16) {          /* F16 widened on load (src/gguf.h:186-190) */
            t->f = malloc(t->n * 4);
            const uint16_t * s = (const uint16_t *)t->raw;
            for (uint64_t j = 0; j < t->n; j++) t->f[j] = h2f(s[j]);
        }
    }
    free(ti); free(buf);

    /* hyper-parameters (src/wav2vec2.cpp:133-156) */
    if (!need_u32(m, "wav2vec2.n_conv_layers", &m->n_conv, err, errlen) ||
        !need_u32(m, "wav2vec2.conv_dim", &m->conv_dim, err, errlen) ||
        !need_u32(m, "wav2vec2.n_encoder_layers", &m->n_layers, err, errlen) ||
        !need_u32(m, "wav2vec2.n_heads", &m->n_heads, err, errlen) ||
        !need_u32(m, "wav2vec2.hidden_size", &m->hidden, err, errlen) ||
        !need_u32(m, "wav2vec2.intermediate_size", &m->ffn, err, errlen) ||
        !need_u32(m, "wav2vec2.vocab_size", &m->vocab, err, errlen) ||
        !need_u32(m, "wav2vec2.pad_token_id", &m->pad_id, err, errlen) ||
        !need_u32(m, "wav2vec2.pos_conv_kernel", &m->pos_k, err, errlen) ||
        !need_u32(m, "wav2vec2.pos_conv_groups", &m->pos_g, err, errlen)) { wvo_free(m); return NULL; }
    const kv_t * fn = find_kv(m, "wav2vec2.feat_extract_norm");
    const kv_t * ck = find_kv(m, "wav2vec2.conv_kernel");
    const kv_t * cs = find_kv(m, "wav2vec2.conv_stride");
    const kv_t * tok = find_kv(m, "tokenizer.ggml.tokens");
    if (!fn || !ck || !cs || !tok) { snprintf(err, errlen, "Missing key"); wvo_free(m); return NULL; }
    m->group_norm = fn->str && !strcmp(fn->str, "group");
    m->vocab = tok->n_str;                               /* src/wav2vec2.cpp:150-151 */
    const kv_t * st = find_kv(m, "wav2vec2.stable_layer_norm");
    m->stable = st && st->u64 != 0;
    if (m->n_conv > 16 || ck->n_u32 < m->n_conv || cs->n_u32 < m->n_conv) {
        snprintf(err, errlen, "bad conv arrays"); wvo_free(m); return NULL;
    }
    for (int i = 0; i < m->n_conv; i++) { m->conv_k[i] = (int)ck->arr_u32[i]; m->conv_s[i] = (int)cs->arr_u32[i]; }
    return m;
}

int wvo_info(const wvo_model * m, int * out) {
    out[0] = m->conv_dim; out[1] = m->hidden; out[2] = m->n_layers; out[3] = m->n_heads;
    out[4] = m->ffn; out[5] = m->vocab; out[6] = m->pad_id; out[7] = m->stable;
    out[8] = m->n_conv; out[9] = m->group_norm;
    return 0;
}

/* ── primitives (src/ops.h) ────────────────────────────────────────────── */

/* tanh-approximation GELU (src/ops.h:18-21). */
float wvo_gelu(float x) {
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

/* Row LayerNorm, eps 1e-5, population variance (src/ops.h:24-36);
 * sums in double here. */
void wvo_layer_norm(float * x, const float * w, const float * b, int T, int D) {
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        float * row = x + (size_t)t * D;
        double s = 0; for (int i = 0; i < D; i++) s += row[i];
        float mean = (float)(s / D);
        double v = 0; for (int i = 0; i < D; i++) { double d = row[i] - mean; v += d * d; }
        float inv = 1.f / sqrtf((float)(v / D) + 1e-5f);
        for (int i = 0; i < D; i++) row[i] = (row[i] - mean) * inv * w[i] + b[i];
    }
}

/* Per-channel GroupNorm over time, eps 1e-5 (src/ops.h:39-50). */
void wvo_group_norm(float * x, const float * w, const float * b, int T, int C) {
    #pragma omp parallel for schedule(static)
    for (int c = 0; c < C; c++) {
        double s = 0; for (int t = 0; t < T; t++) s += x[(size_t)t * C + c];
        float mean = (float)(s / T);
        double v = 0; for (int t = 0; t < T; t++) { double d = x[(size_t)t * C + c] - mean; v += d * d; }
        float inv = 1.f / sqrtf((float)(v / T) + 1e-5f);
        for (int t = 0; t < T; t++) x[(size_t)t * C + c] = (x[(size_t)t * C + c] - mean) * inv * w[c] + b[c];
    }
}

/* Softmax with max subtraction (src/ops.h:101-106). */
void wvo_softmax(float * x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float s = 0.f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= s;
}

/* Grouped strided conv1d, x [L, Cin] time-major, w [Cout, Cin/g, K]
 * (src/ops.h:76-99).  Weights are transposed to [Cout][K][Cin/g] so the inner
 * sum runs over contiguous channels; the sum is in fp32 (vectorised order). */
int wvo_conv1d(const float * x, const float * w, const float * b, int L, int Cin, int Cout,
               int K, int stride, int pad, int groups, float * out) {
    const int Cig = Cin / groups, Cog = Cout / groups;
    const int Lout = (L + 2 * pad - K) / stride + 1;
    if (Lout <= 0) return 0;
    float * wt = malloc((size_t)Cout * K * Cig * sizeof(float));
    for (int co = 0; co < Cout; co++)
        for (int ci = 0; ci < Cig; ci++)
            for (int k = 0; k < K; k++)
                wt[((size_t)co * K + k) * Cig + ci] = w[((size_t)co * Cig + ci) * K + k];
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < Lout; t++) {
        for (int co = 0; co < Cout; co++) {
            const int g = co / Cog;
            float s = b ? b[co] : 0.f;
            for (int k = 0; k < K; k++) {
                const int src = t * stride + k - pad;
                if (src < 0 || src >= L) continue;
                const float * xr = x + (size_t)src * Cin + (size_t)g * Cig;
                const float * wr = wt + ((size_t)co * K + k) * Cig;
                float acc = 0.f;
                #pragma omp simd reduction(+:acc)
                for (int ci = 0; ci < Cig; ci++) acc += xr[ci] * wr[ci];
                s += acc;
            }
            out[(size_t)t * Cout + co] = s;
        }
    }
    free(wt);
    return Lout;
}

/* Greedy CTC spans: first max wins (strict >), runs collapsed, blanks kept
 * (src/ops.h:132-149). */
int wvo_ctc_greedy_spans(const float * logits, int T, int V, int * out3, int cap) {
    int n = 0, prev = -1, start = 0;
    for (int t = 0; t < T; t++) {
        int best = 0; float bv = logits[(size_t)t * V];
        for (int v = 1; v < V; v++) if (logits[(size_t)t * V + v] > bv) { bv = logits[(size_t)t * V + v]; best = v; }
        if (best != prev) {
            if (prev != -1) { if (n >= cap) return -1; out3[3*n] = prev; out3[3*n+1] = start; out3[3*n+2] = t; n++; }
            prev = best; start = t;
        }
    }
    if (prev != -1) { if (n >= cap) return -1; out3[3*n] = prev; out3[3*n+1] = start; out3[3*n+2] = T; n++; }
    return n;
}

/* ggml's Q8_0 row quantization (published quantize_row_q8_0 reference rule):
 * d = amax/127 stored as fp16, q = roundf(x * (1/d)). */
void wvo_quantize_q8_0_row(const float * x, int K, float * out) {
    for (int b = 0; b < K / 32; b++) {
        const float * xb = x + b * 32;
        float amax = 0.f;
        for (int j = 0; j < 32; j++) { float a = fabsf(xb[j]); if (a > amax) amax = a; }
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        const float dh = h2f(f2h(d));
        for (int j = 0; j < 32; j++) out[b * 32 + j] = roundf(xb[j] * id) * dh;
    }
}

/* ── linear layers (src/ggml_backend.h:78-120) ─────────────────────────── */

static void dequant_row(const tensor_t * t, int64_t n, int64_t K, float * out) {
    if (t->type == T_F32) { memcpy(out, t->f + n * K, K * 4); return; }
    if (t->type == T_F16) { memcpy(out, t->f + n * K, K * 4); return; }
    for (int64_t b = 0; b < K / 32; b++) {
        if (t->type == T_Q8_0) {
            const uint8_t * blk = t->raw + (n * (K / 32) + b) * 34;
            uint16_t dh; memcpy(&dh, blk, 2); const float d = h2f(dh);
            for (int j = 0; j < 32; j++) out[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
        } else {
            const uint8_t * blk = t->raw + (n * (K / 32) + b) * 18;
            uint16_t dh; memcpy(&dh, blk, 2); const float d = h2f(dh);
            for (int j = 0; j < 16; j++) {
                out[b * 32 + j] = d * (float)((int)(blk[2 + j] & 0xf) - 8);
                out[b * 32 + j + 16] = d * (float)((int)(blk[2 + j] >> 4) - 8);
            }
        }
    }
}

/* y[M][N] = x[M][K] . W[N][K]^T + b.  W is GGUF [K, N] (ne0 = K). */
static int linear_t(const tensor_t * W, const float * bias, const float * x, int M, int mode, float * y) {
    const int64_t K = (int64_t)W->shape[0], N = W->ndim > 1 ? (int64_t)W->shape[1] : 1;
    const int quant = (W->type == T_Q8_0 || W->type == T_Q4_0);
    float * xs = NULL;
    if (mode == WVO_LINEAR_GGML) {
        xs = malloc((size_t)M * K * sizeof(float));
        if (quant) {
            #pragma omp parallel for schedule(static)
            for (int m = 0; m < M; m++) wvo_quantize_q8_0_row(x + (size_t)m * K, (int)K, xs + (size_t)m * K);
        } else if (W->type == T_F16) {
            for (int64_t i = 0; i < (int64_t)M * K; i++) xs[i] = h2f(f2h(x[i]));
        } else {
            memcpy(xs, x, (size_t)M * K * sizeof(float));
        }
    }
    #pragma omp parallel
    {
        float * wf = malloc(K * sizeof(float));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            dequant_row(W, n, K, wf);
            const float bn = bias ? bias[n] : 0.f;
            for (int m = 0; m < M; m++) {
                if (mode == WVO_LINEAR_GGML && quant) {
                    /* block-wise: exact block sums (products of fp16-scaled
                     * ints are exact in double), accumulated in fp32 */
                    const float * xr = xs + (size_t)m * K;
                    float sumf = 0.f;
                    for (int64_t b = 0; b < K / 32; b++) {
                        double s = 0;
                        for (int j = 0; j < 32; j++) s += (double)xr[b * 32 + j] * wf[b * 32 + j];
                        sumf += (float)s;
                    }
                    y[(size_t)m * N + n] = sumf + bn;
                } else {
                    const float * xr = (mode == WVO_LINEAR_GGML ? xs : x) + (size_t)m * K;
                    double acc = 0;
                    #pragma omp simd reduction(+:acc)
                    for (int64_t k = 0; k < K; k++) acc += (double)xr[k] * wf[k];
                    y[(size_t)m * N + n] = (float)acc + bn;
                }
            }
        }
        free(wf);
    }
    free(xs);
    return 0;
}

int wvo_linear(const wvo_model * m, const char * name, const float * x, int M, int mode, float * y) {
    char wn[256], bn[256];
    snprintf(wn, sizeof wn, "%s.weight", name);
    snprintf(bn, sizeof bn, "%s.bias", name);
    const tensor_t * W = find_t(m, wn);
    if (!W) return -1;
    return linear_t(W, tf(m, bn), x, M, mode, y);
}

long wvo_weight(const wvo_model * m, const char * name, float * out, long cap) {
    char wn[256]; snprintf(wn, sizeof wn, "%s.weight", name);
    const tensor_t * W = find_t(m, wn);
    if (!W) return -1;
    const int64_t K = (int64_t)W->shape[0], N = W->ndim > 1 ? (int64_t)W->shape[1] : 1;
    if (N * K > cap) return -1;
    for (int64_t n = 0; n < N; n++) dequant_row(W, n, K, out + n * K);
    return (long)(N * K);
}

/* ── forward pass ──────────────────────────────────────────────────────── */

/* Feature extractor (src/wav2vec2.cpp:257-289): waveform mean/var
 * normalisation (eps 1e-7), then conv -> [norm] -> GELU per layer. */
int wvo_features(const wvo_model * m, const float * samples, int n, float * out, long cap) {
    if (n <= 0) return -1;
    float * cur = malloc((size_t)n * sizeof(float));
    double s = 0; for (int i = 0; i < n; i++) s += samples[i];
    float mean = (float)(s / n);
    double v = 0; for (int i = 0; i < n; i++) { double d = samples[i] - mean; v += d * d; }
    float inv = 1.f / sqrtf((float)(v / n) + 1e-7f);
    for (int i = 0; i < n; i++) cur[i] = (samples[i] - mean) * inv;
    int L = n, cin = 1;
    for (int i = 0; i < m->n_conv; i++) {
        char p[128];
        snprintf(p, sizeof p, "feature_extractor.conv_layers.%d.conv.weight", i);
        const float * w = tf(m, p);
        snprintf(p, sizeof p, "feature_extractor.conv_layers.%d.conv.bias", i);
        const float * b = tf(m, p);
        if (!w) { free(cur); return -1; }
        const int K = m->conv_k[i], S = m->conv_s[i];
        const int Lout = (L - K) / S + 1;
        if (Lout <= 0) { free(cur); return -1; }
        float * nx = malloc((size_t)Lout * m->conv_dim * sizeof(float));
        wvo_conv1d(cur, w, b, L, cin, m->conv_dim, K, S, 0, 1, nx);
        snprintf(p, sizeof p, "feature_extractor.conv_layers.%d.layer_norm.weight", i);
        const float * lw = tf(m, p);
        snprintf(p, sizeof p, "feature_extractor.conv_layers.%d.layer_norm.bias", i);
        const float * lb = tf(m, p);
        if (lw && lb) {
            if (m->group_norm) wvo_group_norm(nx, lw, lb, Lout, m->conv_dim);
            else wvo_layer_norm(nx, lw, lb, Lout, m->conv_dim);
        }
        for (long j = 0; j < (long)Lout * m->conv_dim; j++) nx[j] = wvo_gelu(nx[j]);
        free(cur); cur = nx; L = Lout; cin = m->conv_dim;
    }
    if ((long)L * m->conv_dim > cap) { free(cur); return -1; }
    memcpy(out, cur, (size_t)L * m->conv_dim * sizeof(float));
    free(cur);
    return L;
}

/* Multi-head self-attention (src/wav2vec2.cpp:293-338): separate Q/K/V
 * linears, per-head softmax(QK^T / sqrt(d)) V, output linear. */
static int attention(const wvo_model * m, int layer, const float * xin, int T, int mode, float * xout) {
    const int H = m->hidden, nh = m->n_heads, d = H / nh;
    const float scale = 1.f / sqrtf((float)d);
    char p[160];
    float * Q = malloc((size_t)T * H * 4), * Kt = malloc((size_t)T * H * 4), * Vt = malloc((size_t)T * H * 4);
    float * O = calloc((size_t)T * H, 4);
    snprintf(p, sizeof p, "encoder.layers.%d.attention.q_proj", layer); wvo_linear(m, p, xin, T, mode, Q);
    snprintf(p, sizeof p, "encoder.layers.%d.attention.k_proj", layer); wvo_linear(m, p, xin, T, mode, Kt);
    snprintf(p, sizeof p, "encoder.layers.%d.attention.v_proj", layer); wvo_linear(m, p, xin, T, mode, Vt);
    #pragma omp parallel
    {
        float * sc = malloc((size_t)T * sizeof(float));
        float * acc = malloc((size_t)d * sizeof(float));
        #pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < nh; h++) {
            for (int i = 0; i < T; i++) {
                const float * q = Q + (size_t)i * H + h * d;
                for (int j = 0; j < T; j++) {
                    const float * k = Kt + (size_t)j * H + h * d;
                    float s = 0.f;
                    for (int e = 0; e < d; e++) s += q[e] * k[e];
                    sc[j] = s * scale;
                }
                wvo_softmax(sc, T);
                for (int e = 0; e < d; e++) acc[e] = 0.f;
                for (int j = 0; j < T; j++) {
                    const float * vv = Vt + (size_t)j * H + h * d;
                    const float pj = sc[j];
                    for (int e = 0; e < d; e++) acc[e] += pj * vv[e];
                }
                for (int e = 0; e < d; e++) O[(size_t)i * H + h * d + e] = acc[e];
            }
        }
        free(sc); free(acc);
    }
    snprintf(p, sizeof p, "encoder.layers.%d.attention.out_proj", layer);
    wvo_linear(m, p, O, T, mode, xout);
    free(Q); free(Kt); free(Vt); free(O);
    return 0;
}

static void gelu_inplace(float * x, long n) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++) x[i] = wvo_gelu(x[i]);
}

/* Encoder (src/wav2vec2.cpp:340-394). */
int wvo_encode_stages(const wvo_model * m, const float * feat, int T, int mode, float * out) {
    const int H = m->hidden, C = m->conv_dim, F = m->ffn;
    const size_t blk = (size_t)T * H;
    float * fn = malloc((size_t)T * C * 4);
    memcpy(fn, feat, (size_t)T * C * 4);
    wvo_layer_norm(fn, tf(m, "feature_projection.layer_norm.weight"), tf(m, "feature_projection.layer_norm.bias"), T, C);
    float * x = malloc(blk * 4);
    wvo_linear(m, "feature_projection.projection", fn, T, mode, x);
    free(fn);
    memcpy(out, x, blk * 4);
    /* positional conv: grouped, pad K/2, keep the first T of T+1 outputs, GELU, add */
    const int pk = m->pos_k, pg = m->pos_g;
    const int Lp = (T + 2 * (pk / 2) - pk) / 1 + 1;
    float * pos = malloc((size_t)Lp * H * 4);
    wvo_conv1d(x, tf(m, "encoder.pos_conv_embed.conv.weight"), tf(m, "encoder.pos_conv_embed.conv.bias"),
               T, H, H, pk, 1, pk / 2, pg, pos);
    const int useT = T < Lp ? T : Lp;
    for (size_t i = 0; i < (size_t)useT * H; i++) x[i] += wvo_gelu(pos[i]);
    free(pos);
    float * a = malloc(blk * 4), * lnb = malloc(blk * 4);
    float * f1 = malloc((size_t)T * F * 4), * f2 = malloc(blk * 4);
    char p[160], q[160];
    if (!m->stable) {
        wvo_layer_norm(x, tf(m, "encoder.layer_norm.weight"), tf(m, "encoder.layer_norm.bias"), T, H);
        memcpy(out + blk, x, blk * 4);
        for (int l = 0; l < m->n_layers; l++) {
            attention(m, l, x, T, mode, a);
            for (size_t i = 0; i < blk; i++) x[i] += a[i];
            snprintf(p, sizeof p, "encoder.layers.%d.layer_norm.weight", l);
            snprintf(q, sizeof q, "encoder.layers.%d.layer_norm.bias", l);
            wvo_layer_norm(x, tf(m, p), tf(m, q), T, H);
            snprintf(p, sizeof p, "encoder.layers.%d.feed_forward.intermediate_dense", l);
            wvo_linear(m, p, x, T, mode, f1);
            gelu_inplace(f1, (long)T * F);
            snprintf(p, sizeof p, "encoder.layers.%d.feed_forward.output_dense", l);
            wvo_linear(m, p, f1, T, mode, f2);
            for (size_t i = 0; i < blk; i++) x[i] += f2[i];
            snprintf(p, sizeof p, "encoder.layers.%d.final_layer_norm.weight", l);
            snprintf(q, sizeof q, "encoder.layers.%d.final_layer_norm.bias", l);
            wvo_layer_norm(x, tf(m, p), tf(m, q), T, H);
            memcpy(out + (2 + l) * blk, x, blk * 4);
        }
    } else {
        memcpy(out + blk, x, blk * 4);
        for (int l = 0; l < m->n_layers; l++) {
            memcpy(lnb, x, blk * 4);
            snprintf(p, sizeof p, "encoder.layers.%d.layer_norm.weight", l);
            snprintf(q, sizeof q, "encoder.layers.%d.layer_norm.bias", l);
            wvo_layer_norm(lnb, tf(m, p), tf(m, q), T, H);
            attention(m, l, lnb, T, mode, a);
            for (size_t i = 0; i < blk; i++) x[i] += a[i];
            memcpy(lnb, x, blk * 4);
            snprintf(p, sizeof p, "encoder.layers.%d.final_layer_norm.weight", l);
            snprintf(q, sizeof q, "encoder.layers.%d.final_layer_norm.bias", l);
            wvo_layer_norm(lnb, tf(m, p), tf(m, q), T, H);
            snprintf(p, sizeof p, "encoder.layers.%d.feed_forward.intermediate_dense", l);
            wvo_linear(m, p, lnb, T, mode, f1);
            gelu_inplace(f1, (long)T * F);
            snprintf(p, sizeof p, "encoder.layers.%d.feed_forward.output_dense", l);
            wvo_linear(m, p, f1, T, mode, f2);
            for (size_t i = 0; i < blk; i++) x[i] += f2[i];
            if (l == m->n_layers - 1) {
                /* the final encoder LN belongs to the last stage block */
                wvo_layer_norm(x, tf(m, "encoder.layer_norm.weight"), tf(m, "encoder.layer_norm.bias"), T, H);
            }
            memcpy(out + (2 + l) * blk, x, blk * 4);
        }
        if (m->n_layers == 0)
            wvo_layer_norm(out + blk, tf(m, "encoder.layer_norm.weight"), tf(m, "encoder.layer_norm.bias"), T, H);
    }
    free(x); free(a); free(lnb); free(f1); free(f2);
    return T;
}

int wvo_lm_head(const wvo_model * m, const float * enc, int T, int mode, float * out) {
    return wvo_linear(m, "lm_head", enc, T, mode, out) == 0 ? T : -1;
}

/* Audio -> logits (src/wav2vec2.cpp:485-489). */
int wvo_logits(const wvo_model * m, const float * samples, int n, int mode, float * out, long cap) {
    int T0 = n;
    for (int i = 0; i < m->n_conv; i++) T0 = (T0 - m->conv_k[i]) / m->conv_s[i] + 1;
    if (T0 <= 0 || (long)T0 * m->vocab > cap) return -1;
    float * feat = malloc((size_t)T0 * m->conv_dim * 4);
    int T = wvo_features(m, samples, n, feat, (long)T0 * m->conv_dim);
    if (T <= 0) { free(feat); return -1; }
    float * st = malloc((size_t)(m->n_layers + 2) * T * m->hidden * 4);
    wvo_encode_stages(m, feat, T, mode, st);
    wvo_lm_head(m, st + (size_t)(m->n_layers + 1) * T * m->hidden, T, mode, out);
    free(feat); free(st);
    return T;
}
