// wav2vec2-b200 engine: one model replica on one CUDA device.
//
// Owns the device weights (repacked once at load) and the per-batch device
// workspace, and runs the batched forward pass -- waveform normalisation,
// conv extractor, feature projection, positional conv, post-LN or pre-LN
// encoder, CTC head, greedy CTC -- as a fixed sequence of kernel launches on
// one stream (reference: src/wav2vec2.cpp:257-394, 477-506).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <mutex>
#include <vector>

#include "gguf.hpp"

namespace w2v {

struct ModelConfig {
    int n_conv = 0, conv_dim = 0, n_layers = 0, n_heads = 0, hidden = 0, ffn = 0, vocab = 0, pad_id = 0;
    int pos_k = 0, pos_g = 0;
    bool group_norm = true;       // feat_extract_norm == "group"
    bool stable = false;          // pre-LN encoder (stable_layer_norm)
    std::vector<int> conv_k, conv_s;
    std::vector<bool> conv_norm, conv_bias;
    std::vector<std::string> tokens;
    std::string word_delim = "|";

    static ModelConfig from_gguf(const GgufFile& gf);
    // Frames after the conv stack for n samples (reference wav2vec2.cpp:278); 0 if too short.
    int frames(long long n_samples) const;
};

// Device buffer that only grows.
struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    bool ensure(size_t bytes);   // true if the buffer was (re)allocated
    void release();
    template <typename T> T* as() const { return static_cast<T*>(p); }
};

// One linear's weights on the device: fp16 rows [N, K] (gguf_type 1), or the
// GGUF Q8_0 (8) / Q4_0 (2) blocks repacked into a code plane and a scale
// plane [K/32][N] that the dequant-fused GEMM reads (w2v_gemm_q).
struct LinearW {
    DevBuf w;             // fp16 rows, or the codes
    DevBuf s;             // quantised: fp16 scales
    int gguf_type = 1;
    int N = 0, K = 0;
    size_t bytes() const { return w.n + s.n; }
};

struct LayerWeights {
    LinearW qkv, o, fc1, fc2;
    DevBuf bqkv, bo, b1, b2, ln1w, ln1b, ln2w, ln2b;
};

// Everything one forward pass needs per batch.
struct BatchGeom {
    int n_utt = 0;
    std::vector<int> n_samples;            // per utterance
    std::vector<long long> audio_off;      // packed audio offsets
    std::vector<std::vector<int>> L;       // [layer][utt] frames after conv layer
    std::vector<int> Lmax;                 // per layer
    std::vector<long long> R;              // per layer: rows per utterance in the padded buffer
    std::vector<int> T;                    // encoder frames per utterance (= L.back())
    std::vector<long long> T_off;          // packed row offsets
    long long M = 0;                       // total frames
    int T_max = 0;
};

class Engine {
public:
    Engine(const GgufFile& gf, const ModelConfig& cfg, int device);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    const ModelConfig& cfg() const { return cfg_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    BatchGeom geometry(const std::vector<int>& n_samples) const;

    // Forward for a batch whose packed audio is in device memory.  Enqueues on
    // `st` (nullptr: the engine's stream) and returns without synchronising.
    // If dbg_feat/dbg_stages are non-null (single-utterance debug), copies the
    // extractor output and per-stage encoder activations to the host
    // (synchronous).
    void forward(const float* d_audio, const BatchGeom& g, cudaStream_t st, float* dbg_feat = nullptr,
                 float* dbg_stages = nullptr);

    // Host-memory convenience used by the C API: packs the utterances into
    // pinned memory, uploads, runs forward, downloads logits and/or spans.
    // Host threads that pack one batch's pageable audio (0: up to 8, half the
    // host's hardware threads); a context over several devices divides them.
    void set_pack_threads(int n) { pack_threads_ = n; }
    void run_host(const std::vector<const float*>& audio, const std::vector<int>& n_samples,
                  std::vector<float>* logits, std::vector<int>* spans, std::vector<int>* n_spans,
                  BatchGeom* geom_out);

    // Outputs of the last forward (device).
    const float* d_logits() const { return logits_.as<float>(); }
    const int* d_spans() const { return spans_.as<int>(); }
    const int* d_n_spans() const { return nspans_.as<int>(); }
    long long last_M() const { return last_M_; }

    // Device error word set by kernels whose bounded waits expired.
    int check_device_error();

    // Per-category kernel timing with CUDA events on the forward stream.
    // Categories: see kProfNames in engine.cpp.  set_profiling resets totals.
    void set_profiling(bool on);
    // Synchronises the stream, folds recorded events into the totals and
    // returns the number of categories written (<= cap).
    int profile_read(const char** names, double* ms, long long* launches, double* flops, int cap);
    long long launches_last_forward() const { return launches_last_; }
    // Device bytes of the linear weights (codes + scales, or fp16 rows).
    size_t linear_weight_bytes() const;
    // Host batches run since the last reset: device time from the first
    // upload to the last download of each batch (CUDA events), batch and
    // sample counts.
    void busy_stats(double* ms, long long* batches, long long* samples, bool reset);

private:
    void load(const GgufFile& gf);
    // Weight rows of GGUF linears `names` (each [N_i, K]) stacked into one
    // linear: kept quantised when they share a Q8_0 / Q4_0 type (unless the
    // engine expands every weight to fp16), else expanded to fp16.
    void upload_linears(const GgufFile& gf, const std::vector<std::string>& names, const std::vector<int>& Ns, int K,
                        LinearW& L);
    // One GEMM over packed encoder rows [M, K] with linear L's weights.
    int gemm_linear(const void* A, long long M, const LinearW& L, void* C, long long ldc, const float* bias,
                    const float* resid, int epilogue, int block_n, const float* ln_stats, const float* ln_w,
                    const float* ln_b, cudaStream_t st);
    void ensure_workspace(const BatchGeom& g);
    void upload_meta(const BatchGeom& g, cudaStream_t st);
    // The forward in three parts: begin (workspace, metadata; false if there
    // is nothing to compute), the feature extractor for utterances [u0, u1)
    // (waveform statistics, conv layers; utterances are independent there),
    // and everything after it over the whole batch.
    bool fwd_begin(const BatchGeom& g, cudaStream_t st);
    void fwd_extract(const float* d_audio, const BatchGeom& g, int u0, int u1, cudaStream_t st);
    void fwd_encode(const BatchGeom& g, cudaStream_t st, float* dbg_feat, float* dbg_stages);
    // fwd_extract over the whole batch + fwd_encode, from a captured graph when
    // this (input, lengths) pair has been seen before (after fwd_begin).
    void extract_encode(const float* d_audio, const BatchGeom& g, cudaStream_t st, float* dbg_feat,
                        float* dbg_stages);
    // Launch bookkeeping: counts the launch and, when profiling, brackets it
    // with events attributed to category `cat` with `flops` algorithmic FLOPs.
    template <typename Fn> void launch(int cat, double flops, cudaStream_t st, const char* what, Fn fn);
    void prof_fold();

    ModelConfig cfg_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;

    // weights
    DevBuf conv0_w_, conv0_b_;
    std::vector<DevBuf> conv_w_, conv_b_, conv_gw_, conv_gb_;
    DevBuf proj_lnw_, proj_lnb_, proj_b_;
    LinearW proj_w_;
    DevBuf pos_w_, pos_b_, enc_lnw_, enc_lnb_;
    std::vector<LayerWeights> layers_;
    LinearW lm_w_;
    DevBuf lm_b_;
    bool expand_weights_ = false;   // W2V_B200_EXPAND_WEIGHTS=1: every linear as fp16 rows

    // workspace
    DevBuf audio_stage_;                       // device copy of packed audio (run_host)
    DevBuf meta_;                              // packed per-batch metadata
    DevBuf stats_, gn_;
    DevBuf actA_, actB_;                       // fp16 conv ping-pong
    DevBuf feat_, pbuf_, x_, xh_, qkv_, attn_, hbuf_, ybuf_;
    DevBuf lnstats_;                           // per encoder row (mean, rstd) of the latest LayerNorm
    DevBuf logits_, ids_, spans_, nspans_;
    DevBuf err_;
    long long last_M_ = 0;
    long long launches_cur_ = 0, launches_last_ = 0;

    // Captured forwards (CUDA graphs) of Engine::forward, keyed by the input
    // pointer and the utterance lengths; valid while no workspace buffer is
    // reallocated (ws_gen_).  A geometry is captured the second time it is
    // seen, so one-off batches and the first call's lazy set-up run eagerly;
    // at most kMaxGraphs are kept (further pairs run kernel by kernel).
    struct GraphEntry {
        const float* audio;
        std::vector<int> n_samples;
        uint64_t ws_gen;
        cudaGraphExec_t exec;
        long long launches;
    };
    static constexpr size_t kMaxGraphs = 16;
    std::vector<GraphEntry> graphs_;
    std::vector<std::pair<const float*, std::vector<int>>> graph_seen_;
    uint64_t ws_gen_ = 0;
    bool graphs_enabled_ = true;   // W2V_B200_GRAPHS=0: always launch kernel by kernel
    int pack_threads_ = 0;
    void drop_graphs();

    struct ProfRec { int cat; cudaEvent_t a, b; double flops; };
    bool profiling_ = false;
    std::vector<cudaEvent_t> ev_pool_;
    std::vector<ProfRec> prof_pending_;
    std::vector<double> prof_ms_, prof_flops_;
    std::vector<long long> prof_n_;

    // pinned host staging
    float* h_audio_ = nullptr;
    size_t h_audio_n_ = 0;
    uint8_t* h_out_ = nullptr;                 // pinned: error word, spans and span counts of a host batch
    size_t h_out_n_ = 0;
    std::vector<uint8_t> meta_host_;
    cudaEvent_t meta_done_ = nullptr;
    // host-batch uploads: a copy stream and one event per utterance chunk
    static constexpr int kMaxChunks = 4;
    cudaStream_t copy_stream_ = nullptr;
    cudaEvent_t chunk_ev_[kMaxChunks] = {};
    cudaEvent_t busy0_ = nullptr, busy1_ = nullptr;
    std::mutex busy_mu_;
    double busy_ms_ = 0.0;
    long long busy_batches_ = 0, busy_samples_ = 0;

    // device pointers into meta_
    long long* d_audio_off_ = nullptr;
    int* d_len_ = nullptr;
    std::vector<int*> d_L_;
    int* d_T_ = nullptr;
    long long* d_T_off_ = nullptr;
};

}  // namespace w2v
