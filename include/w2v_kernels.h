/* Internal C-ABI kernel layer of the wav2vec2-b200 engine (sm_100a).
 *
 * Plain extern "C" launchers: device pointers, sizes and a cudaStream_t
 * passed as void*; they return a W2V_* status and never throw.  The C++ host
 * engine (wav2vec2.cpp_b200/csrc/engine.cpp) calls these; so do the GPU
 * parity tests, through ctypes.  Each entry names the reference code whose
 * computation it replaces (paths inside py-ai-dev/wav2vec2.cpp).
 *
 * Layouts: packed encoder rows are [M = sum of frames, width] row-major.  Conv
 * activations are padded per utterance: [n_utt][rows_max][C] fp16.  `err` is
 * a device int that kernels set (first writer wins) when a bounded wait
 * expires; it may be NULL.
 */
#ifndef W2V_KERNELS_H
#define W2V_KERNELS_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    W2V_OK = 0,
    W2V_ERR_ARGS = 1,        /* invalid sizes, strides or alignment */
    W2V_ERR_LAUNCH = 2,      /* CUDA launch/config error */
    W2V_ERR_DRIVER = 3,      /* driver entry point unavailable */
    W2V_ERR_TENSOR_MAP = 4,  /* cuTensorMapEncodeTiled rejected the view */
    W2V_ERR_DEVICE = 5,      /* kernel reported a device-side error */
    W2V_ERR_CAPACITY = 6,    /* request exceeds a fixed, built-in buffer */
};

/* GEMM epilogues. */
enum {
    W2V_EPI_F16 = 0,        /* C(fp16) = acc + bias              */
    W2V_EPI_F16_GELU = 1,   /* C(fp16) = gelu_tanh(acc + bias)   */
    W2V_EPI_F32 = 2,        /* C(fp32) = acc + bias              */
    W2V_EPI_F32_RESID = 3,  /* C(fp32) = acc + bias + resid      */
    W2V_EPI_F32_RESID_LN = 4, /* C(fp32) = acc + bias + LayerNorm(resid) (w2v_gemm_f16_ln_resid) */
};

/* tcgen05 GEMM, C = epi(A . B^T).  Replaces ggml_mul_mat in
 * GgmlScratch::linear (src/ggml_backend.h:78-120) and the strided conv1d of
 * the extractor (src/ops.h:76-99) as an implicit GEMM.
 *   A: fp16 activation rows; batch b, input row i at
 *      A + b*a_batch_stride + i*a_row_stride (a_rows_in rows per batch, a
 *      multiple of a_stride).  Output row r of batch b reads, for each of
 *      a_taps taps, input row r*a_stride + tap, columns 0..a_cin-1
 *      (a_cin % 64 == 0): K = a_taps * a_cin, ordered tap-major.
 *      Plain GEMM: a_taps = a_stride = a_batches = 1, a_rows_in = M.
 *   B: fp16 [N, K] row-major.
 *   C: row (b, r) at C + (b*c_batch_rows + r)*ldc, written for r < m_valid.
 *   bias: fp32 [N] or NULL; resid: fp32 rows like C (ldr), may alias C.
 *   block_n: 0 = automatic; 64/128/192/256 = one CTA per 128 x block_n tile;
 *            -128/-192/-256 = a CTA pair (tcgen05 cta_group::2) per 256 x -block_n tile. */
int w2v_gemm_f16(const void* A, long long a_cin, int a_taps, int a_stride, long long a_row_stride,
                 long long a_rows_in, long long a_batches, long long a_batch_stride, const void* B,
                 int N, void* C, long long ldc, long long c_batch_rows, int m_valid, const float* bias,
                 const float* resid, long long ldr, int epilogue, int block_n, int* err,
                 void* stream);

/* w2v_gemm_f16 with the W2V_EPI_F32_RESID_LN epilogue: the residual rows are
 * the raw input of a LayerNorm (src/ops.h:24-36) and are normalised on the
 * fly, C = acc + bias + (resid - mean_r) * rstd_r * ln_w + ln_b, with
 * ln_stats[2r], ln_stats[2r+1] = (mean_r, rstd_r) of row r as written by
 * w2v_layer_norm_stats.  resid may alias C.  C, resid, bias, ln_w, ln_b and
 * ln_stats 16-byte aligned, ldc and ldr multiples of 4. */
int w2v_gemm_f16_ln_resid(const void* A, long long a_cin, int a_taps, int a_stride, long long a_row_stride,
                          long long a_rows_in, long long a_batches, long long a_batch_stride, const void* B,
                          int N, void* C, long long ldc, long long c_batch_rows, int m_valid, const float* bias,
                          const float* resid, long long ldr, const float* ln_stats, const float* ln_w,
                          const float* ln_b, int block_n, int* err, void* stream);

/* Dequant-fused tcgen05 GEMM on quantised weights: C = epi(A . W^T) with W
 * the [N, K] rows of a GGUF Q8_0 (gguf_type 8) or Q4_0 (gguf_type 2) linear
 * (scripts/convert_to_gguf.py:63-97), kept in the planes w2v_repack_q
 * writes: Bq the codes, Bs the fp16 scales [K/32][ld_s] (ld_s >= N, a
 * multiple of 8).  Converter warps expand each 64-deep k-block of W to fp16
 * straight into tensor memory (w = d*q rounded once: the values
 * w2v_dequant_f16 gives), where the MMA reads it as its A operand.  Replaces
 * ggml_mul_mat on quantised weights (GgmlScratch::linear,
 * src/ggml_backend.h:78-120).  A: fp16 [M, K] activation rows (K % 64 == 0);
 * C, bias, resid and the epilogues as w2v_gemm_f16 (not
 * W2V_EPI_F32_RESID_LN: w2v_gemm_q_ln_resid).  block_n: 0 = automatic,
 * 64/128/192/224 = one CTA per 128 weight rows x block_n activation rows,
 * -128/-192/-224 = a CTA pair per 256 weight rows x -block_n activation rows. */
int w2v_gemm_q(const void* A, long long K, long long M, const void* Bq, const void* Bs, long long ld_s,
               int gguf_type, int N, void* C, long long ldc, const float* bias, const float* resid,
               long long ldr, int epilogue, int block_n, int* err, void* stream);

/* w2v_gemm_q with the W2V_EPI_F32_RESID_LN epilogue (see w2v_gemm_f16_ln_resid). */
int w2v_gemm_q_ln_resid(const void* A, long long K, long long M, const void* Bq, const void* Bs,
                        long long ld_s, int gguf_type, int N, void* C, long long ldc, const float* bias,
                        const float* resid, long long ldr, const float* ln_stats, const float* ln_w,
                        const float* ln_b, int block_n, int* err, void* stream);

/* GGUF Q8_0 / Q4_0 blocks of weight rows [n_rows, K] (K % 64 == 0; raw
 * bytes as stored in the file, the way src/ggml_backend.h:43-50 keeps them)
 * -> the planes of w2v_gemm_q: codes = [n_rows][K] int8 (Q8_0) or
 * [n_rows][K/2] bytes of 4-bit codes (Q4_0), 16-byte aligned; scales[j*ld_s
 * + n] = fp16 scale of row n's j-th block of 32.  Rows may be written into a
 * larger plane (stacked Q/K/V): pass codes and scales offset to the first row
 * / column. */
int w2v_repack_q(const void* raw, int gguf_type, long long n_rows, long long K, void* codes, void* scales,
                 long long ld_s, void* stream);

/* Failure-detection self-test: launches a kernel whose bounded mbarrier wait
 * (the same wait the GEMM pipeline uses) is never satisfied; after limit_ms
 * (1..2000) it writes the timeout code (1) to *err and returns without
 * trapping, so the context stays usable.  No counterpart in the reference. */
int w2v_selftest_wait_timeout(int* err, int limit_ms, void* stream);

/* Expand GGUF linear weight rows ([N, K], GGUF type F32=0, F16=1, Q4_0=2,
 * Q8_0=8, raw bytes as stored in the file) to fp16 [N, K].  Block formats as
 * written by scripts/convert_to_gguf.py:63-97. */
int w2v_dequant_f16(const void* raw, int gguf_type, long long n_rows, long long K, void* out,
                    void* stream);

/* Per-utterance waveform statistics (src/wav2vec2.cpp:262-271): stats[2u] =
 * mean, stats[2u+1] = 1/sqrt(var + 1e-7), population variance. audio is
 * packed; utterance u is audio[off[u] .. off[u]+len[u]). */
int w2v_wave_stats(const float* audio, const long long* off, const int* len, int n_utt,
                   float* stats, void* stream);

/* Conv layer 0 (Cin = 1, kernel k0, stride s0, C channels) on the normalised
 * waveform, then the layer's norm and GELU (src/wav2vec2.cpp:273-287,
 * src/ops.h:24-50,76-99).
 *   norm: 0 = none, 1 = GroupNorm over time per channel (needs gn_sums,
 *   a device double buffer [n_utt][C][2] used as scratch for the
 *   statistics), 2 = LayerNorm over channels per frame.
 *   w0: fp32 [C][k0]; b0: fp32 [C] or NULL; gw/gb: fp32 [C] norm affine.
 *   out: fp16 [n_utt][rows_max][C]; frames per utterance (len-k0)/s0+1.
 *   err: device word for bounded-wait failures of the tensor-core path
 *   (k0 = 10, s0 = 5, C = 256 or 512, norm 0 or 1). */
int w2v_conv0(const float* audio, const long long* off, const int* len, const int* frames, int n_utt,
              const float* stats, const float* w0, const float* b0, int C, int k0, int s0, int norm,
              const float* gw, const float* gb, double* gn_sums, void* out, long long rows_max,
              int max_frames, int* err, void* stream);

/* w2v_conv0 for callers that cannot allocate device memory.  No counterpart
 * in the reference (which has no GPU code): same arguments and result as
 * w2v_conv0 without gn_sums; the GroupNorm statistics live in a 512 KiB
 * buffer inside the library, per device, held until process exit.
 *   Limit: with norm == 1, n_utt <= 64 and C <= 512, else W2V_ERR_CAPACITY
 *   (and nothing is launched).
 *   It calls no cudaMalloc/cudaFree.  The first call on a device looks the
 *   buffer's device address up once (make that first call before any stream
 *   capture).  Under CUDA's default lazy module loading that first lookup may
 *   also load the library's device code, which allocates device memory and
 *   can block: make one warm-up call per device from a thread that is
 *   allowed to block (not the real-time thread) and outside stream capture.
 *   All calls on a device share the buffer: calls that overlap on the GPU
 *   (different streams, no ordering) race on it. */
int w2v_conv0_noalloc(const float* audio, const long long* off, const int* len, const int* frames,
                      int n_utt, const float* stats, const float* w0, const float* b0, int C, int k0,
                      int s0, int norm, const float* gw, const float* gb, void* out, long long rows_max,
                      int max_frames, int* err, void* stream);

/* Row LayerNorm (eps 1e-5, src/ops.h:24-36) over D columns of fp16 or fp32
 * rows, optional GELU after the affine, fp32 and/or fp16 outputs.
 * Input row r of utterance u: in + (u*in_batch_rows + r)*ld_in, r < rows[u]
 * (rows == NULL: r < n_rows with one batch).  Output rows are packed
 * (out_off[u] + r) when out_off != NULL, else laid out like the input. */
int w2v_layer_norm(const void* in, int in_f16, long long ld_in, long long in_batch_rows,
                   const int* rows, const long long* out_off, int n_batch, int n_rows, int D,
                   const float* w, const float* b, int gelu, float* out32, void* out16,
                   long long ld_out, void* stream);

/* Row LayerNorm (eps 1e-5) of fp32 rows [M, D] -> fp16 rows [M, D], also
 * writing each row's (mean, 1/sqrt(var + eps)) to stats[2r], stats[2r+1] so
 * a consumer can re-derive the fp32 normalised row (w2v_gemm_f16_ln_resid)
 * without it being stored.  D a multiple of 128 (<= 2048); pointers 16-byte
 * aligned. */
int w2v_layer_norm_stats(const float* in, long long M, int D, const float* w, const float* b, void* out16,
                         float* stats, void* stream);

/* Positional conv embedding (src/wav2vec2.cpp:349-356): grouped conv1d over
 * time (kernel Kp, padding Kp/2, G groups, first T of T+1 outputs), GELU,
 * added to the input.  x: fp32 packed rows [M, H]; utterance u occupies rows
 * off[u] .. off[u]+T[u]; x = xin + gelu(conv(xin) + bias), x != xin.
 * wt: fp16 weights re-laid out by the engine as
 * [G][Kp/2][Cg/8][2 Cg][8 (ci within the chunk)], Cg = H/G: per pair of taps
 * (2p, 2p+1) one contiguous block of 8-row x 16-byte core matrices whose 2 Cg
 * rows are tap 2p's output channels, then tap 2p+1's; bias fp32 [H].
 * Cg must be 32, 48, 64 or 80; Kp even, at most 128; x, xin, wt
 * and bias 16-byte aligned.  err: device word for bounded-wait failures. */
int w2v_pos_conv(float* x, const float* xin, const long long* off, const int* T, int n_utt, int H,
                 int Kp, int G, const void* wt, const float* bias, int max_T, int* err, void* stream);

/* Bidirectional multi-head attention (src/wav2vec2.cpp:293-334), flash-style
 * online softmax in fp32, fp16 tensor-core products.  qkv: fp16 [M, 3H]
 * (q | k | v, head h at columns h*d..), out: fp16 [M, H].  Keys are limited
 * to the query's own utterance (rows off[u] .. off[u]+T[u]).  M = total rows
 * of qkv.  Head dims 64 and 128 run on tcgen05 (TMEM accumulators, bounded
 * waits reporting through err); head dim 80 on warp-level mma.sync. */
int w2v_attention(const void* qkv, void* out, const long long* off, const int* T, int n_utt, int H,
                  int n_heads, int max_T, long long M, int* err, void* stream);

/* Greedy CTC (src/ops.h:132-149): per frame argmax (first max wins), run
 * collapse into spans (id, t_start, t_end), blank runs kept.  logits fp32
 * packed [M, V]; spans written at spans + 3*off[u]; n_spans[u] = count. */
int w2v_ctc_greedy(const float* logits, const long long* off, const int* T, int n_utt, int V,
                   int* ids, int* spans, int* n_spans, int max_T, void* stream);

#ifdef __cplusplus
}
#endif
#endif
