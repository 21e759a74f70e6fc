/* CPU oracle for the wav2vec2 CTC forward pass -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's algorithm (py-ai-dev/wav2vec2.cpp,
 * src/wav2vec2.cpp:257-506, src/ops.h:18-149, src/gguf.h:113-195) used by the
 * tests, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the
 * checker.  The product (libwav2vec2_b200.so) never links or calls it.
 *
 * Linear layers (the reference's ggml_mul_mat, src/ggml_backend.h:78-120) have
 * two modes:
 *   WVO_LINEAR_EXACT: y = x . dequant(W)^T + b with fp32 inputs, double sums.
 *   WVO_LINEAR_GGML : ggml's published CPU algorithm: activations quantized to
 *                     Q8_0 for Q8_0/Q4_0 weights (rounded to fp16 for F16
 *                     weights), integer block dots, fp32 block accumulation.
 * ggml itself is absent and unpinned in the reference checkout, so
 * WVO_LINEAR_GGML is a restatement of its published algorithm, not pinned to
 * ggml's code; it is pinned to the reference's wav2vec2.cpp built against the
 * oracle's ggml-API shim (oracle/ggml_shim), which implements the same rule.
 */
#ifndef W2V_ORACLE_H
#define W2V_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { WVO_LINEAR_EXACT = 0, WVO_LINEAR_GGML = 1 };

typedef struct wvo_model wvo_model;

wvo_model * wvo_load(const char * path, char * err, int errlen);
void        wvo_free(wvo_model * m);

/* out[0..9] = conv_dim, hidden, n_layers, n_heads, intermediate, vocab,
 *             pad_id, stable_layer_norm, n_conv_layers, feat_norm_is_group */
int wvo_info(const wvo_model * m, int * out);

/* Feature extractor output [T, conv_dim]; returns T or -1. */
int wvo_features(const wvo_model * m, const float * samples, int n, float * out, long cap);

/* Encoder activations by stage ((n_layers + 2) blocks of [T, hidden]):
 * block 0 = feature projection output, block 1 = after positional conv
 * (+ encoder LN when post-LN), block 2 + l = after layer l. */
int wvo_encode_stages(const wvo_model * m, const float * feat, int T, int mode, float * out);

/* CTC logits [T, vocab] from audio; returns T or -1. */
int wvo_logits(const wvo_model * m, const float * samples, int n, int mode, float * out, long cap);

/* CTC logits from an encoder output [T, hidden] (lm_head linear). */
int wvo_lm_head(const wvo_model * m, const float * enc, int T, int mode, float * out);

/* Linear layer by GGUF weight name (without ".weight"), bias included. */
int wvo_linear(const wvo_model * m, const char * name, const float * x, int M, int mode, float * y);

/* Dequantized weight [N, K] of a named linear (fp32). Returns N*K or -1. */
long wvo_weight(const wvo_model * m, const char * name, float * out, long cap);

/* Primitives (reference src/ops.h). */
float wvo_gelu(float x);
void  wvo_layer_norm(float * x, const float * w, const float * b, int T, int D);
void  wvo_group_norm(float * x, const float * w, const float * b, int T, int C);
void  wvo_softmax(float * x, int n);
int   wvo_conv1d(const float * x, const float * w, const float * b, int L, int Cin, int Cout,
                 int K, int stride, int pad, int groups, float * out);
/* Greedy CTC spans (id, t_start, t_end) incl. blank runs; returns count. */
int   wvo_ctc_greedy_spans(const float * logits, int T, int V, int * out3, int cap);
/* ggml Q8_0 activation quantization of one row (K % 32 == 0): values written
 * back dequantized (fp16 scale * int8). */
void  wvo_quantize_q8_0_row(const float * x, int K, float * out);

#ifdef __cplusplus
}
#endif
#endif
