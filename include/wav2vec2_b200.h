/* wav2vec2-b200 extensions to the reference C API (wav2vec2.h).
 *
 * The reference transcribes one utterance per call
 * (include/wav2vec2.h:40-44 in py-ai-dev/wav2vec2.cpp) and has no batch,
 * device or multi-GPU entry points (batching is a roadmap item there,
 * README.md:166).  These are the new entry points of the B200 engine.
 * All functions return 0 (W2V_STATUS_OK) on success; on failure a non-zero
 * status, with a message from wav2vec2_b200_last_error().
 */
#pragma once
#include "wav2vec2.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    W2V_STATUS_OK = 0,
    W2V_STATUS_INVALID = 1,   /* bad arguments (NULL pointers, sizes) */
    W2V_STATUS_CUDA = 2,      /* CUDA runtime or kernel launch error */
    W2V_STATUS_DEVICE = 3,    /* a kernel reported a device-side error */
    W2V_STATUS_MODEL = 4,     /* model file missing, corrupt or unsupported */
    W2V_STATUS_AUDIO = 5,     /* audio file missing, malformed or unsupported */
};

/* Message of the most recent failure on this thread ("" if none). */
const char * wav2vec2_b200_last_error(void);

/* Load a model on n_devices CUDA devices (one full weight replica each).
 * devices == NULL selects devices 0 .. n_devices-1; n_devices <= 0 selects 1.
 * max_batch bounds utterances per device batch (<= 0: 64).  Batched calls
 * length-bucket utterances and shard the batches over the devices, one host
 * thread and stream per device, with no inter-device traffic. */
struct wav2vec2_context * wav2vec2_b200_init(const char * path_model, const int * devices,
                                             int n_devices, int max_batch);

/* Number of devices the context runs on. */
int wav2vec2_b200_n_devices(const struct wav2vec2_context * ctx);

/* Model dimensions: out[0..7] = conv_dim, hidden, n_layers, n_heads, ffn,
 * vocab, pad_id, stable_layer_norm. */
int wav2vec2_b200_model_info(const struct wav2vec2_context * ctx, int * out);

/* Transcribe n_utt utterances (host memory).  results[i] receives a result to
 * release with wav2vec2_result_free (same layout as wav2vec2_transcribe). */
int wav2vec2_transcribe_batch(struct wav2vec2_context * ctx, struct wav2vec2_params params,
                              const float * const * samples, const int * n_samples, int n_utt,
                              struct wav2vec2_result ** results);

/* Frames produced for an utterance of n_samples samples (0 if too short). */
int wav2vec2_b200_n_frames(const struct wav2vec2_context * ctx, int n_samples);

/* CTC logits for n_utt utterances (host memory in and out): logits receives
 * the utterances' [T_i, vocab] fp32 blocks back to back (sum T_i rows);
 * n_frames[i] = T_i.  Used for parity checks and host-side decoders. */
int wav2vec2_b200_logits(struct wav2vec2_context * ctx, const float * const * samples,
                         const int * n_samples, int n_utt, float * logits, int * n_frames);

/* Device-resident batch on the context's first device: d_audio holds the
 * utterances back to back in device memory (n_samples on the host); runs the
 * whole path through greedy CTC on `stream` (a cudaStream_t, NULL = the
 * context's own stream) and returns without synchronising.  Results stay in
 * engine-owned device memory until the next call: see
 * wav2vec2_b200_device_outputs. */
int wav2vec2_b200_forward_device(struct wav2vec2_context * ctx, const float * d_audio,
                                 const int * n_samples, int n_utt, void * stream);

/* Device pointers of the last forward_device batch: logits [M, vocab] fp32,
 * spans int32 triples (id, t_start, t_end) for utterance i at row offset
 * off_i (sum of earlier T), n_spans int32 [n_utt]; M = total frames. */
int wav2vec2_b200_device_outputs(struct wav2vec2_context * ctx, const float ** logits,
                                 const int ** spans, const int ** n_spans, long long * M);

/* Stage-wise activations of one utterance for parity checks (fp32, host):
 * feat [T, conv_dim] (extractor output), stages [(n_layers + 2), T, hidden]:
 * block 0 = feature projection, 1 = after positional conv (+ encoder LN for
 * post-LN models), 2 + l = after encoder layer l; logits [T, vocab]. */
int wav2vec2_b200_debug_stages(struct wav2vec2_context * ctx, const float * samples, int n_samples,
                               float * feat, float * stages, float * logits);

/* Kernel timing: enable (1) / disable (0) CUDA-event timing of every kernel
 * launch on the context's devices; enabling resets the totals. */
int wav2vec2_b200_profile(struct wav2vec2_context * ctx, int enable);

/* Per-category totals on the first device since profiling was enabled:
 * names[i] (static strings), ms[i] (sum of event-timed kernel durations),
 * launches[i], flops[i] (algorithmic FLOPs of those launches).  Synchronises
 * the device stream.  Returns the number of categories (<= cap). */
int wav2vec2_b200_profile_read(struct wav2vec2_context * ctx, const char ** names, double * ms,
                               long long * launches, double * flops, int cap);

/* CTC prefix beam search on host logits [T, V] fp32, the decoder the
 * reference runs for beam_size > 1 (wv2_ctc_beam_search, src/ops.h:151-251):
 * writes the decoded token ids (runs collapsed, blank removed) to ids and
 * returns their count; -1 on bad arguments (blank outside 0..V-1,
 * beam_width < 1) or when more than cap ids result.  For host decoders that
 * consume wav2vec2_b200_logits output; runs on the calling thread, no GPU. */
int wav2vec2_b200_ctc_beam_search(const float * logits, int T, int V, int blank, int beam_width, int * ids,
                                  int cap);

/* Per-device load of the host batch path (wav2vec2_transcribe_batch,
 * wav2vec2_b200_logits) since the last reset: busy_ms[i] = device time of
 * device i's batches, each measured with CUDA events from before its first
 * upload to after its last download; batches[i], samples[i] = batches and
 * audio samples it processed.  Any output may be NULL; reset != 0 clears the
 * totals after reading.  Returns the number of devices written (<= cap), -1
 * on bad arguments.  No counterpart in the reference (single CPU). */
int wav2vec2_b200_device_stats(struct wav2vec2_context * ctx, int reset, double * busy_ms,
                               long long * batches, long long * samples, int cap);

/* Device bytes that the first device holds for the linear layers (feature
 * projection, encoder Q/K/V/out/FFN, CTC head): Q8_0 / Q4_0 linears stay
 * quantised (code plane + fp16 scale plane, expanded inside the GEMM), F16 /
 * F32 ones are fp16 rows.  The environment variable W2V_B200_EXPAND_WEIGHTS=1,
 * read when a context is created, expands every linear to fp16 rows instead.
 * -1 on a NULL context. */
long long wav2vec2_b200_linear_weight_bytes(const struct wav2vec2_context * ctx);

/* Kernel launches of the most recent forward on the first device. */
long long wav2vec2_b200_launches_per_forward(const struct wav2vec2_context * ctx);

/* Read a WAV file as mono float samples at target_sr Hz (<= 0: 16000): PCM
 * 16-bit, PCM 32-bit or float 32-bit, any channel count (averaged) and rate
 * (linear interpolation).  Same decoding, messages and results as the
 * reference CLI's reader (examples/main/main.cpp:20-82), which has no library
 * counterpart.  *samples is malloc'd (free with wav2vec2_b200_free_samples;
 * NULL when *n_samples is 0).  Returns W2V_STATUS_AUDIO on a bad file. */
int wav2vec2_b200_load_wav(const char * path, int target_sr, float ** samples, int * n_samples);
void wav2vec2_b200_free_samples(float * samples);

#ifdef __cplusplus
}
#endif
