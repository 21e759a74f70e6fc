/* wav2vec2 CTC speech recognition -- public C API.
 *
 * Drop-in for py-ai-dev/wav2vec2.cpp: the declarations, structs and semantics
 * below are those of the reference's include/wav2vec2.h:1-51 (kept identical
 * so existing callers recompile unchanged); the implementation is the
 * B200-native engine (libwav2vec2_b200.so).  Extensions (batched and
 * device-resident entry points, multi-GPU) live in wav2vec2_b200.h.
 *
 * Differences in behaviour: wav2vec2_init returns NULL on failure instead of
 * throwing a C++ exception (the reference CLI already treats NULL as failure,
 * examples/main/main.cpp:218); the message is available from
 * wav2vec2_b200_last_error().  n_threads sizes host-side decoding threads.
 */
#pragma once
#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

struct wav2vec2_context;

/* Word-level timing (populated when params.word_timestamps == true) */
struct wav2vec2_word {
    char  * text;       /* heap-allocated; freed by wav2vec2_result_free */
    float   t_start;    /* seconds */
    float   t_end;      /* seconds */
};

/* Inference result -- use wav2vec2_result_free() to release */
struct wav2vec2_result {
    char                  * transcript;  /* full text, heap-allocated */
    int                     n_frames;    /* CTC feature frames (each = 20 ms) */
    struct wav2vec2_word  * words;       /* NULL unless params.word_timestamps */
    int                     n_words;     /* 0 unless params.word_timestamps */
};

struct wav2vec2_params {
    int  n_threads;          /* default: 4 */
    int  beam_size;          /* 1 = greedy CTC, >1 = beam search (default: 1) */
    bool verbose;            /* print timing to stderr */
    bool word_timestamps;    /* populate result->words with per-word timing */
};

struct wav2vec2_params wav2vec2_default_params(void);

/* Load model from a GGUF file (reference format: scripts/convert_to_gguf.py) */
struct wav2vec2_context * wav2vec2_init(const char * path_model);
void                      wav2vec2_free(struct wav2vec2_context * ctx);

/* Transcribe raw PCM: 16 kHz mono float32 in [-1, 1] */
struct wav2vec2_result * wav2vec2_transcribe(
    struct wav2vec2_context * ctx,
    struct wav2vec2_params    params,
    const float             * samples,
    int                       n_samples);

/* Free a result returned by wav2vec2_transcribe */
void wav2vec2_result_free(struct wav2vec2_result * result);

#ifdef __cplusplus
}
#endif
