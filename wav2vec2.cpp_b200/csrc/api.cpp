// C API of the wav2vec2-b200 engine (include/wav2vec2.h, include/wav2vec2_b200.h).
//
// Mirrors the reference's public API (src/wav2vec2.cpp:458-533): same result
// layout and ownership (everything malloc'd, released by
// wav2vec2_result_free), same text post-processing (ids_to_text /
// spans_to_words, src/wav2vec2.cpp:396-452) and beam search
// (src/ops.h:151-251) on the host, with the forward pass on the GPU.
// C++ exceptions never cross this boundary: failures return NULL / a status
// and leave a message for wav2vec2_b200_last_error().
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <exception>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "engine.hpp"
#include "shard.hpp"
#include "audio.hpp"
#include "beam.hpp"
#include "wav2vec2_b200.h"

using namespace w2v;

struct wav2vec2_context {
    ModelConfig cfg;
    std::vector<std::unique_ptr<Engine>> engines;   // one per device
    // Batch workers for wav2vec2_transcribe_batch: the engines above, plus, on
    // contexts over several devices, a second engine per device (its own
    // stream and workspace), so that one engine packs and uploads its next
    // batch while the other's kernels run.
    std::vector<Engine*> workers;
    std::vector<std::unique_ptr<Engine>> extra;
    int max_batch = 64;
};

namespace {

thread_local std::string g_last_error;

void set_error(const std::string& e) { g_last_error = e; }

// ── detokenisation (src/wav2vec2.cpp:396-452) ───────────────────────────────

bool is_special(const std::string& s) { return s.size() >= 2 && s.front() == '<' && s.back() == '>'; }

std::string trim_spaces(const std::string& s) {
    const auto a = s.find_first_not_of(' ');
    if (a == std::string::npos) return "";
    const auto b = s.find_last_not_of(' ');
    return s.substr(a, b - a + 1);
}

std::string ids_to_text(const std::vector<int>& ids, const ModelConfig& c) {
    std::string out;
    for (int id : ids) {
        if (id == c.pad_id || id < 0 || id >= (int)c.tokens.size()) continue;
        const auto& tok = c.tokens[id];
        if (tok == c.word_delim) { out += ' '; continue; }
        if (is_special(tok)) continue;
        out += tok;
    }
    return trim_spaces(out);
}

struct Span { int id, t0, t1; };
struct Word { std::string text; int t0, t1; };

std::vector<Word> spans_to_words(const std::vector<Span>& spans, const ModelConfig& c) {
    std::vector<Word> words;
    std::string cur;
    int s0 = -1, s1 = -1;
    auto flush = [&]() {
        if (cur.empty()) return;
        std::string t = trim_spaces(cur);
        if (!t.empty()) words.push_back({t, s0, s1});
        cur.clear();
        s0 = s1 = -1;
    };
    for (const auto& sp : spans) {
        if (sp.id == c.pad_id || sp.id < 0 || sp.id >= (int)c.tokens.size()) continue;
        const auto& tok = c.tokens[sp.id];
        if (is_special(tok)) continue;
        if (tok == c.word_delim) { flush(); continue; }
        if (s0 < 0) s0 = sp.t0;
        s1 = sp.t1;
        cur += tok;
    }
    flush();
    return words;
}

// ── result assembly (src/wav2vec2.cpp:491-532) ──────────────────────────────

char* dup_str(const std::string& s) {
    char* p = (char*)malloc(s.size() + 1);
    memcpy(p, s.c_str(), s.size() + 1);
    return p;
}

wav2vec2_result* make_result(const ModelConfig& c, int T, const std::string& text, const std::vector<Word>* words) {
    auto* r = (wav2vec2_result*)calloc(1, sizeof(wav2vec2_result));
    r->n_frames = T;
    r->transcript = dup_str(text);
    if (words && !words->empty()) {
        r->n_words = (int)words->size();
        r->words = (wav2vec2_word*)malloc(r->n_words * sizeof(wav2vec2_word));
        for (int i = 0; i < r->n_words; i++) {
            const auto& w = (*words)[i];
            r->words[i].t_start = w.t0 * (320.f / 16000.f);
            r->words[i].t_end = w.t1 * (320.f / 16000.f);
            r->words[i].text = dup_str(w.text);
        }
    }
    (void)c;
    return r;
}

// Host decoding pool: device workers hand each finished batch's utterances
// to it and go straight on to their next batch, so prefix beam search (the
// reference's host decoder, src/ops.h:151-251) overlaps the GPU forward of
// the following batches.  finish() drains the queue, joins and rethrows the
// first task failure; the destructor (an error path) drains and joins only.
class DecodePool {
public:
    explicit DecodePool(int n) {
        for (int i = 0; i < n; i++) th_.emplace_back([this] { loop(); });
    }
    ~DecodePool() { join(); }
    void push(std::function<void()> f) {
        {
            std::lock_guard<std::mutex> l(m_);
            q_.push_back(std::move(f));
        }
        cv_.notify_one();
    }
    // Wait for every queued task; rethrows the first task exception.
    void finish() {
        join();
        if (err_) {
            auto e = err_;
            err_ = nullptr;
            std::rethrow_exception(e);
        }
    }

private:
    void join() {
        {
            std::lock_guard<std::mutex> l(m_);
            done_ = true;
        }
        cv_.notify_all();
        for (auto& t : th_)
            if (t.joinable()) t.join();
        th_.clear();
    }
    void loop() {
        for (;;) {
            std::function<void()> f;
            {
                std::unique_lock<std::mutex> l(m_);
                cv_.wait(l, [this] { return done_ || !q_.empty(); });
                if (q_.empty()) return;
                f = std::move(q_.front());
                q_.pop_front();
            }
            try {
                f();
            } catch (...) {
                std::lock_guard<std::mutex> l(m_);
                if (!err_) err_ = std::current_exception();
            }
        }
    }
    std::vector<std::thread> th_;
    std::deque<std::function<void()>> q_;
    std::mutex m_;
    std::condition_variable cv_;
    bool done_ = false;
    std::exception_ptr err_;
};

// Run every batch, sharded over the context's devices (shard.hpp: one host
// thread per device pulling from a shared queue; a failing device retires and
// its batch is re-queued); fn(engine, batch index list, logits, spans,
// n_spans, geometry) consumes each result on the worker thread (it may move
// the logits out).
template <typename Fn>
void run_sharded(wav2vec2_context* ctx, const float* const* samples, const int* n_samples, int n_utt,
                 bool want_logits, bool want_spans, Fn fn) {
    const auto batches = make_batches(n_samples, n_utt, ctx->max_batch, (long long)ctx->max_batch * 16000LL * 32);
    const int nw = (int)std::min(ctx->workers.size(), std::max<size_t>(batches.size(), 1));
    // the workers' packing threads share the host: half its hardware threads
    // in all, at most 8 per worker
    const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
    for (int w = 0; w < nw; w++) ctx->workers[w]->set_pack_threads(std::max(1, std::min(8, hw / (2 * nw))));
    run_batches(batches.size(), nw, [&](int w, size_t bi, std::string& err) {
        Engine* e = ctx->workers[w];
        std::vector<float> logits;
        std::vector<int> spans, nsp;
        const auto& b = batches[bi];
        std::vector<const float*> a;
        std::vector<int> ns;
        for (int i : b) { a.push_back(samples[i]); ns.push_back(n_samples[i]); }
        BatchGeom g;
        try {
            e->run_host(a, ns, want_logits ? &logits : nullptr, want_spans ? &spans : nullptr,
                        want_spans ? &nsp : nullptr, &g);
        } catch (const std::exception& ex) {
            err = std::string("device ") + std::to_string(e->device()) + ": " + ex.what();
            return false;
        }
        fn(e, b, logits, spans, nsp, g);
        return true;
    });
}

}  // namespace

// ── public API ──────────────────────────────────────────────────────────────

extern "C" {

const char* wav2vec2_b200_last_error(void) { return g_last_error.c_str(); }

wav2vec2_params wav2vec2_default_params(void) {
    wav2vec2_params p{};
    p.n_threads = 4;
    p.beam_size = 1;
    p.verbose = false;
    p.word_timestamps = false;
    return p;
}

void wav2vec2_result_free(wav2vec2_result* r) {
    if (!r) return;
    free(r->transcript);
    if (r->words) {
        for (int i = 0; i < r->n_words; i++) free(r->words[i].text);
        free(r->words);
    }
    free(r);
}

wav2vec2_context* wav2vec2_b200_init(const char* path, const int* devices, int n_devices, int max_batch) {
    try {
        if (!path) throw std::runtime_error("NULL model path");
        GgufFile gf(path);
        auto ctx = std::make_unique<wav2vec2_context>();
        ctx->cfg = ModelConfig::from_gguf(gf);
        ctx->max_batch = max_batch > 0 ? max_batch : 64;
        if (n_devices <= 0) n_devices = 1;
        int avail = 0;
        if (cudaGetDeviceCount(&avail) != cudaSuccess || avail == 0) throw std::runtime_error("no CUDA device");
        for (int i = 0; i < n_devices; i++) {
            const int d = devices ? devices[i] : i;
            if (d < 0 || d >= avail) throw std::runtime_error("invalid device index " + std::to_string(d));
            ctx->engines.push_back(std::make_unique<Engine>(gf, ctx->cfg, d));
        }
        int per_device = n_devices > 1 ? 2 : 1;
        if (const char* s = getenv("W2V_B200_ENGINES_PER_DEVICE")) per_device = std::max(1, std::min(4, atoi(s)));
        for (auto& e : ctx->engines) ctx->workers.push_back(e.get());
        for (int k = 1; k < per_device; k++)
            for (int i = 0; i < n_devices; i++) {
                ctx->extra.push_back(std::make_unique<Engine>(gf, ctx->cfg, ctx->engines[i]->device()));
                ctx->workers.push_back(ctx->extra.back().get());
            }
        return ctx.release();
    } catch (const std::exception& e) {
        set_error(e.what());
        fprintf(stderr, "wav2vec2_init: %s\n", e.what());
        return nullptr;
    }
}

wav2vec2_context* wav2vec2_init(const char* path) {
    int n = 1;
    if (const char* s = getenv("W2V_N_DEVICES")) n = std::max(1, atoi(s));
    return wav2vec2_b200_init(path, nullptr, n, 0);
}

void wav2vec2_free(wav2vec2_context* ctx) { delete ctx; }

int wav2vec2_b200_n_devices(const wav2vec2_context* ctx) { return ctx ? (int)ctx->engines.size() : 0; }

int wav2vec2_b200_model_info(const wav2vec2_context* ctx, int* out) {
    if (!ctx || !out) return W2V_STATUS_INVALID;
    const auto& c = ctx->cfg;
    out[0] = c.conv_dim; out[1] = c.hidden; out[2] = c.n_layers; out[3] = c.n_heads;
    out[4] = c.ffn; out[5] = c.vocab; out[6] = c.pad_id; out[7] = c.stable ? 1 : 0;
    return W2V_STATUS_OK;
}

int wav2vec2_b200_n_frames(const wav2vec2_context* ctx, int n_samples) {
    return ctx ? ctx->cfg.frames(n_samples) : 0;
}

int wav2vec2_transcribe_batch(wav2vec2_context* ctx, wav2vec2_params params, const float* const* samples,
                              const int* n_samples, int n_utt, wav2vec2_result** results) {
    if (!ctx || (!samples && n_utt > 0) || (!n_samples && n_utt > 0) || !results || n_utt < 0) {
        set_error("invalid arguments");
        return W2V_STATUS_INVALID;
    }
    for (int i = 0; i < n_utt; i++) {
        results[i] = nullptr;
        if (n_samples[i] < 0 || (n_samples[i] > 0 && !samples[i])) {
            set_error("invalid utterance " + std::to_string(i));
            return W2V_STATUS_INVALID;
        }
    }
    const auto t_start = std::chrono::steady_clock::now();
    const ModelConfig& c = ctx->cfg;
    const bool beam = params.beam_size > 1;
    try {
        // beam: decoded by a host pool overlapping later batches' GPU work;
        // greedy: spans come from the GPU, detokenised inline
        std::unique_ptr<DecodePool> pool;
        if (beam) pool.reset(new DecodePool(std::max(1, params.n_threads)));
        run_sharded(ctx, samples, n_samples, n_utt, beam, !beam,
                    [&](Engine*, const std::vector<int>& b, std::vector<float>& logits,
                        const std::vector<int>& spans, const std::vector<int>& nsp, const BatchGeom& g) {
                        const int nb = (int)b.size();
                        if (beam) {
                            auto lg = std::make_shared<std::vector<float>>(std::move(logits));
                            auto geo = std::make_shared<BatchGeom>(g);
                            for (int j = 0; j < nb; j++) {
                                const int u = b[j];
                                pool->push([&, lg, geo, j, u] {
                                    const int T = geo->T[j];
                                    const float* l = lg->data() + (size_t)geo->T_off[j] * c.vocab;
                                    const std::string text =
                                        ids_to_text(ctc_prefix_beam_search(l, T, c.vocab, c.pad_id, params.beam_size), c);
                                    results[u] = make_result(c, T, text, nullptr);
                                });
                            }
                            return;
                        }
                        // The batch's results are assembled locally and published
                        // only once all of them exist: if one throws, the batch is
                        // re-queued and nothing already built is left behind.
                        struct Local {
                            std::vector<wav2vec2_result*> r;
                            ~Local() {
                                for (auto* p : r) wav2vec2_result_free(p);
                            }
                        } local;
                        local.r.assign(nb, nullptr);
                        for (int j = 0; j < nb; j++) {
                            const int T = g.T[j];
                            std::vector<Span> sp;
                            std::vector<int> ids;
                            for (int k = 0; k < (T > 0 ? nsp[j] : 0); k++) {
                                const int* s = spans.data() + 3 * ((size_t)g.T_off[j] + k);
                                sp.push_back({s[0], s[1], s[2]});
                                if (s[0] != c.pad_id) ids.push_back(s[0]);
                            }
                            std::vector<Word> words;
                            if (params.word_timestamps) words = spans_to_words(sp, c);
                            local.r[j] = make_result(c, T, ids_to_text(ids, c),
                                                     params.word_timestamps ? &words : nullptr);
                        }
                        for (int j = 0; j < nb; j++) {
                            results[b[j]] = local.r[j];
                            local.r[j] = nullptr;
                        }
                    });
        if (pool) pool->finish();
    } catch (const std::exception& e) {
        for (int i = 0; i < n_utt; i++) { wav2vec2_result_free(results[i]); results[i] = nullptr; }
        set_error(e.what());
        return strstr(e.what(), "device error") ? W2V_STATUS_DEVICE : W2V_STATUS_CUDA;
    }
    if (params.verbose) {
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() -
                                                                              t_start).count();
        fprintf(stderr, "wav2vec2: %d utterances, %s(b=%d), %lld ms\n", n_utt, beam ? "beam" : "greedy",
                params.beam_size, (long long)ms);
    }
    return W2V_STATUS_OK;
}

wav2vec2_result* wav2vec2_transcribe(wav2vec2_context* ctx, wav2vec2_params params, const float* samples,
                                     int n_samples) {
    wav2vec2_result* r = nullptr;
    const float* s[1] = {samples};
    int n[1] = {n_samples};
    if (wav2vec2_transcribe_batch(ctx, params, s, n, 1, &r) != W2V_STATUS_OK) {
        fprintf(stderr, "wav2vec2_transcribe: %s\n", g_last_error.c_str());
        return nullptr;
    }
    return r;
}

int wav2vec2_b200_logits(wav2vec2_context* ctx, const float* const* samples, const int* n_samples, int n_utt,
                         float* logits, int* n_frames) {
    if (!ctx || n_utt < 0 || (n_utt > 0 && (!samples || !n_samples || !logits || !n_frames))) {
        set_error("invalid arguments");
        return W2V_STATUS_INVALID;
    }
    // output row offset of each utterance in input order
    std::vector<long long> out_off(n_utt + 1, 0);
    for (int i = 0; i < n_utt; i++) {
        if (n_samples[i] < 0 || (n_samples[i] > 0 && !samples[i])) { set_error("invalid utterance"); return W2V_STATUS_INVALID; }
        n_frames[i] = ctx->cfg.frames(n_samples[i]);
        out_off[i + 1] = out_off[i] + n_frames[i];
    }
    const int V = ctx->cfg.vocab;
    try {
        run_sharded(ctx, samples, n_samples, n_utt, true, false,
                    [&](Engine*, const std::vector<int>& b, const std::vector<float>& lg, const std::vector<int>&,
                        const std::vector<int>&, const BatchGeom& g) {
                        for (size_t j = 0; j < b.size(); j++)
                            if (g.T[j] > 0)
                                memcpy(logits + out_off[b[j]] * V, lg.data() + (size_t)g.T_off[j] * V,
                                       (size_t)g.T[j] * V * sizeof(float));
                    });
    } catch (const std::exception& e) {
        set_error(e.what());
        return strstr(e.what(), "device error") ? W2V_STATUS_DEVICE : W2V_STATUS_CUDA;
    }
    return W2V_STATUS_OK;
}

int wav2vec2_b200_forward_device(wav2vec2_context* ctx, const float* d_audio, const int* n_samples, int n_utt,
                                 void* stream) {
    if (!ctx || n_utt < 0 || (n_utt > 0 && (!d_audio || !n_samples))) {
        set_error("invalid arguments");
        return W2V_STATUS_INVALID;
    }
    try {
        Engine* e = ctx->engines[0].get();
        std::vector<int> ns(n_samples, n_samples + n_utt);
        BatchGeom g = e->geometry(ns);
        e->forward(d_audio, g, reinterpret_cast<cudaStream_t>(stream));
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return W2V_STATUS_CUDA;
    }
    return W2V_STATUS_OK;
}

int wav2vec2_b200_device_outputs(wav2vec2_context* ctx, const float** logits, const int** spans,
                                 const int** n_spans, long long* M) {
    if (!ctx) return W2V_STATUS_INVALID;
    Engine* e = ctx->engines[0].get();
    if (logits) *logits = e->d_logits();
    if (spans) *spans = e->d_spans();
    if (n_spans) *n_spans = e->d_n_spans();
    if (M) *M = e->last_M();
    return W2V_STATUS_OK;
}

int wav2vec2_b200_debug_stages(wav2vec2_context* ctx, const float* samples, int n_samples, float* feat,
                               float* stages, float* logits) {
    if (!ctx || !samples || n_samples <= 0) {
        set_error("invalid arguments");
        return W2V_STATUS_INVALID;
    }
    try {
        Engine* e = ctx->engines[0].get();
        cudaSetDevice(e->device());
        BatchGeom g = e->geometry({n_samples});
        if (g.M == 0) throw std::runtime_error("utterance too short");
        void* d = nullptr;
        if (cudaMalloc(&d, (size_t)n_samples * 4) != cudaSuccess) throw std::runtime_error("cudaMalloc");
        // same stream as the forward: a pageable cudaMemcpy may return before its DMA lands
        if (cudaMemcpyAsync(d, samples, (size_t)n_samples * 4, cudaMemcpyHostToDevice, e->stream()) != cudaSuccess) {
            cudaFree(d);
            throw std::runtime_error("audio upload");
        }
        e->forward(static_cast<float*>(d), g, e->stream(), feat, stages);
        if (logits)
            cudaMemcpyAsync(logits, e->d_logits(), (size_t)g.M * ctx->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                            e->stream());
        const cudaError_t err = cudaStreamSynchronize(e->stream());
        cudaFree(d);
        if (err != cudaSuccess) throw std::runtime_error(cudaGetErrorString(err));
        if (e->check_device_error()) throw std::runtime_error("device error (bounded wait expired)");
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return W2V_STATUS_CUDA;
    }
    return W2V_STATUS_OK;
}

int wav2vec2_b200_profile(wav2vec2_context* ctx, int enable) {
    if (!ctx) return W2V_STATUS_INVALID;
    for (auto& e : ctx->engines) e->set_profiling(enable != 0);
    return W2V_STATUS_OK;
}

int wav2vec2_b200_profile_read(wav2vec2_context* ctx, const char** names, double* ms, long long* launches,
                               double* flops, int cap) {
    if (!ctx) return -1;
    return ctx->engines[0]->profile_read(names, ms, launches, flops, cap);
}

int wav2vec2_b200_ctc_beam_search(const float* logits, int T, int V, int blank, int beam_width, int* ids,
                                  int cap) {
    if (T < 0 || V <= 0 || blank < 0 || blank >= V || beam_width < 1 || cap < 0 || (T > 0 && !logits) ||
        (cap > 0 && !ids)) {
        set_error("invalid arguments");
        return -1;
    }
    try {
        const auto r = ctc_prefix_beam_search(logits, T, V, blank, beam_width);
        if ((int)r.size() > cap) {
            set_error("output capacity too small");
            return -1;
        }
        std::copy(r.begin(), r.end(), ids);
        return (int)r.size();
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

int wav2vec2_b200_device_stats(wav2vec2_context* ctx, int reset, double* busy_ms, long long* batches,
                               long long* samples, int cap) {
    if (!ctx || cap < 0) return -1;
    // per device: the sums over its engines (a second engine's batches overlap
    // the first's, so busy_ms may exceed the wall time)
    const int nd = (int)ctx->engines.size();
    const int n = std::min<int>(cap, nd);
    for (int i = 0; i < n; i++) {
        if (busy_ms) busy_ms[i] = 0;
        if (batches) batches[i] = 0;
        if (samples) samples[i] = 0;
    }
    for (size_t k = 0; k < ctx->workers.size(); k++) {
        double ms = 0;
        long long nb = 0, ns = 0;
        ctx->workers[k]->busy_stats(&ms, &nb, &ns, reset != 0);
        const int i = (int)(k % (size_t)nd);
        if (i < n) {
            if (busy_ms) busy_ms[i] += ms;
            if (batches) batches[i] += nb;
            if (samples) samples[i] += ns;
        }
    }
    return n;
}

long long wav2vec2_b200_linear_weight_bytes(const wav2vec2_context* ctx) {
    return ctx && !ctx->engines.empty() ? (long long)ctx->engines[0]->linear_weight_bytes() : -1;
}

long long wav2vec2_b200_launches_per_forward(const wav2vec2_context* ctx) {
    return ctx ? ctx->engines[0]->launches_last_forward() : 0;
}

int wav2vec2_b200_load_wav(const char* path, int target_sr, float** samples, int* n_samples) {
    if (!samples || !n_samples) {
        set_error("invalid arguments");
        return W2V_STATUS_INVALID;
    }
    *samples = nullptr;
    *n_samples = 0;
    try {
        const std::vector<float> a = load_wav(path, target_sr > 0 ? target_sr : 16000);
        if (a.size() > (size_t)0x7fffffff) throw std::runtime_error("WAV too long");
        if (!a.empty()) {
            float* out = static_cast<float*>(std::malloc(a.size() * sizeof(float)));
            if (!out) throw std::runtime_error("out of host memory");
            std::memcpy(out, a.data(), a.size() * sizeof(float));
            *samples = out;
        }
        *n_samples = (int)a.size();
        return W2V_STATUS_OK;
    } catch (const std::exception& e) {
        set_error(e.what());
        return W2V_STATUS_AUDIO;
    }
}

void wav2vec2_b200_free_samples(float* samples) { std::free(samples); }

}  // extern "C"
