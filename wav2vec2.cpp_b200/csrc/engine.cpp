#include "engine.hpp"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <thread>

#include "w2v_kernels.h"

namespace w2v {

namespace {

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void w2v_check(int rc, const char* what) {
    if (rc != W2V_OK) {
        const cudaError_t e = cudaGetLastError();
        throw std::runtime_error(std::string(what) + " failed (status " + std::to_string(rc) + ")" +
                                 (e != cudaSuccess ? std::string(": ") + cudaGetErrorString(e) : std::string()));
    }
}
long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }

}  // namespace

enum ProfCat { P_WAVE, P_CONV0, P_GEMM_CONV, P_LN, P_GEMM_PROJ, P_POSCONV, P_GEMM_ENC, P_ATTN, P_GEMM_LM, P_CTC, P_N };
static const char* kProfNames[P_N] = {"wave_stats", "conv0", "gemm_conv", "layer_norm", "gemm_proj",
                                      "pos_conv", "gemm_encoder", "attention", "gemm_lm_head", "ctc_greedy"};

template <typename Fn>
void Engine::launch(int cat, double flops, cudaStream_t st, const char* what, Fn fn) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (profiling_) {
        if (ev_pool_.size() < 2) {
            for (int i = 0; i < 64; i++) {
                cudaEvent_t e;
                cuda_check(cudaEventCreate(&e), "cudaEventCreate");
                ev_pool_.push_back(e);
            }
        }
        a = ev_pool_.back(); ev_pool_.pop_back();
        b = ev_pool_.back(); ev_pool_.pop_back();
        cuda_check(cudaEventRecord(a, st), "cudaEventRecord");
    }
    w2v_check(fn(), what);
    launches_cur_++;
    if (profiling_) {
        cuda_check(cudaEventRecord(b, st), "cudaEventRecord");
        prof_pending_.push_back({cat, a, b, flops});
    }
}

void Engine::prof_fold() {
    if (prof_ms_.empty()) { prof_ms_.assign(P_N, 0.0); prof_flops_.assign(P_N, 0.0); prof_n_.assign(P_N, 0); }
    for (auto& r : prof_pending_) {
        float ms = 0.f;
        cudaEventSynchronize(r.b);
        if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
            prof_ms_[r.cat] += ms;
            prof_flops_[r.cat] += r.flops;
            prof_n_[r.cat] += 1;
        }
        ev_pool_.push_back(r.a);
        ev_pool_.push_back(r.b);
    }
    prof_pending_.clear();
}

void Engine::set_profiling(bool on) {
    cudaSetDevice(device_);
    prof_fold();
    profiling_ = on;
    prof_ms_.assign(P_N, 0.0);
    prof_flops_.assign(P_N, 0.0);
    prof_n_.assign(P_N, 0);
}

int Engine::profile_read(const char** names, double* ms, long long* launches, double* flops, int cap) {
    cudaSetDevice(device_);
    prof_fold();
    int n = std::min<int>(cap, P_N);
    for (int i = 0; i < n; i++) {
        if (names) names[i] = kProfNames[i];
        if (ms) ms[i] = prof_ms_.empty() ? 0.0 : prof_ms_[i];
        if (launches) launches[i] = prof_n_.empty() ? 0 : prof_n_[i];
        if (flops) flops[i] = prof_flops_.empty() ? 0.0 : prof_flops_[i];
    }
    return n;
}

void Engine::busy_stats(double* ms, long long* batches, long long* samples, bool reset) {
    std::lock_guard<std::mutex> lk(busy_mu_);
    if (ms) *ms = busy_ms_;
    if (batches) *batches = busy_batches_;
    if (samples) *samples = busy_samples_;
    if (reset) {
        busy_ms_ = 0.0;
        busy_batches_ = busy_samples_ = 0;
    }
}

// ── model configuration (src/wav2vec2.cpp:133-202) ──────────────────────────

ModelConfig ModelConfig::from_gguf(const GgufFile& gf) {
    ModelConfig c;
    c.n_conv = (int)gf.u32("wav2vec2.n_conv_layers");
    c.conv_dim = (int)gf.u32("wav2vec2.conv_dim");
    c.n_layers = (int)gf.u32("wav2vec2.n_encoder_layers");
    c.n_heads = (int)gf.u32("wav2vec2.n_heads");
    c.hidden = (int)gf.u32("wav2vec2.hidden_size");
    c.ffn = (int)gf.u32("wav2vec2.intermediate_size");
    c.vocab = (int)gf.u32("wav2vec2.vocab_size");
    c.pad_id = (int)gf.u32("wav2vec2.pad_token_id");
    c.group_norm = gf.str("wav2vec2.feat_extract_norm") == "group";
    c.pos_k = (int)gf.u32("wav2vec2.pos_conv_kernel");
    c.pos_g = (int)gf.u32("wav2vec2.pos_conv_groups");
    for (auto v : gf.arr_u32("wav2vec2.conv_kernel")) c.conv_k.push_back((int)v);
    for (auto v : gf.arr_u32("wav2vec2.conv_stride")) c.conv_s.push_back((int)v);
    c.tokens = gf.arr_str("tokenizer.ggml.tokens");
    c.vocab = (int)c.tokens.size();                       // as the reference (wav2vec2.cpp:150-151)
    if (gf.has_kv("wav2vec2.word_delimiter_token")) c.word_delim = gf.str("wav2vec2.word_delimiter_token");
    c.stable = gf.has_kv("wav2vec2.stable_layer_norm") && gf.u32("wav2vec2.stable_layer_norm") != 0;
    if ((int)c.conv_k.size() < c.n_conv || (int)c.conv_s.size() < c.n_conv || c.n_conv < 1)
        throw std::runtime_error("conv_kernel/conv_stride shorter than n_conv_layers");
    for (int i = 0; i < c.n_conv; i++) {
        const std::string p = "feature_extractor.conv_layers." + std::to_string(i);
        c.conv_norm.push_back(gf.has(p + ".layer_norm.weight"));
        c.conv_bias.push_back(gf.has(p + ".conv.bias"));
    }
    // Shapes the kernels support (all published wav2vec2 / XLS-R models fit).
    auto need = [](bool ok, const std::string& what) {
        if (!ok) throw std::runtime_error("unsupported model: " + what);
    };
    need(c.conv_dim % 64 == 0 && c.conv_dim <= 512, "conv_dim must be a multiple of 64, <= 512");
    need(c.hidden % 64 == 0 && c.ffn % 64 == 0, "hidden and intermediate sizes must be multiples of 64");
    need(c.n_heads > 0 && c.hidden % c.n_heads == 0, "hidden not divisible by n_heads");
    const int d = c.n_heads ? c.hidden / c.n_heads : 0;
    need(d == 64 || d == 80 || d == 128, "head dim must be 64, 80 or 128");
    need(c.pos_g > 0 && c.hidden % c.pos_g == 0, "hidden not divisible by pos_conv_groups");
    const int cg = c.pos_g ? c.hidden / c.pos_g : 0;
    need(cg == 32 || cg == 48 || cg == 64 || cg == 80, "hidden/pos_conv_groups must be 32, 48, 64 or 80");
    need(c.pos_k > 0 && c.pos_k % 2 == 0 && c.pos_k <= 128, "pos_conv_kernel must be even, at most 128");
    need(c.conv_k[0] <= 16, "first conv kernel must be <= 16");
    for (int i = 1; i < c.n_conv; i++)
        need(!(c.conv_norm[i] && c.group_norm), "GroupNorm is supported on conv layer 0 only");
    need(c.vocab > 0, "empty vocabulary");
    return c;
}

int ModelConfig::frames(long long n) const {
    long long L = n;
    for (int i = 0; i < n_conv; i++) {
        if (L < conv_k[i]) return 0;
        L = (L - conv_k[i]) / conv_s[i] + 1;
    }
    return (int)L;
}

// ── device buffers ──────────────────────────────────────────────────────────

bool DevBuf::ensure(size_t bytes) {
    if (bytes <= n) return false;
    release();
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
    n = bytes;
    return true;
}
void DevBuf::release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
}

// ── load ────────────────────────────────────────────────────────────────────

Engine::Engine(const GgufFile& gf, const ModelConfig& cfg, int device) : cfg_(cfg), device_(device) {
    cuda_check(cudaSetDevice(device_), "cudaSetDevice");
    cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaEventCreateWithFlags(&meta_done_, cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    for (auto& e : chunk_ev_) cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaEventCreate(&busy0_), "cudaEventCreate");
    cuda_check(cudaEventCreate(&busy1_), "cudaEventCreate");
    if (const char* e = getenv("W2V_B200_EXPAND_WEIGHTS")) expand_weights_ = atoi(e) != 0;
    if (const char* e = getenv("W2V_B200_GRAPHS")) graphs_enabled_ = atoi(e) != 0;
    err_.ensure(sizeof(int));
    // Every transfer of the engine is ordered on its own (non-blocking) stream:
    // a legacy-stream cudaMemcpy from pageable memory may return before its DMA
    // lands and is not ordered against this stream.
    cuda_check(cudaMemsetAsync(err_.p, 0, sizeof(int), stream_), "cudaMemsetAsync");
    load(gf);
    cuda_check(cudaStreamSynchronize(stream_), "weight upload");
}

Engine::~Engine() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (copy_stream_) cudaStreamSynchronize(copy_stream_);
    cudaDeviceSynchronize();   // replays of captured forwards may run on caller streams
    drop_graphs();
    auto rel = [](DevBuf& b) { b.release(); };
    for (DevBuf* b : {&conv0_w_, &conv0_b_, &proj_lnw_, &proj_lnb_, &proj_w_.w, &proj_w_.s, &proj_b_, &pos_w_, &pos_b_,
                      &enc_lnw_, &enc_lnb_, &lm_w_.w, &lm_w_.s, &lm_b_, &audio_stage_, &meta_, &stats_, &gn_, &actA_,
                      &actB_, &feat_,
                      &pbuf_, &x_, &xh_, &qkv_, &attn_, &hbuf_, &ybuf_, &lnstats_, &logits_, &ids_, &spans_, &nspans_, &err_})
        rel(*b);
    for (auto* v : {&conv_w_, &conv_b_, &conv_gw_, &conv_gb_})
        for (auto& b : *v) rel(b);
    for (auto& L : layers_)
        for (DevBuf* b : {&L.qkv.w, &L.qkv.s, &L.bqkv, &L.o.w, &L.o.s, &L.bo, &L.fc1.w, &L.fc1.s, &L.b1, &L.fc2.w,
                          &L.fc2.s, &L.b2, &L.ln1w, &L.ln1b, &L.ln2w,
                          &L.ln2b})
            rel(*b);
    if (h_audio_) cudaFreeHost(h_audio_);
    if (h_out_) cudaFreeHost(h_out_);
    prof_fold();
    for (auto e : ev_pool_) cudaEventDestroy(e);
    if (meta_done_) cudaEventDestroy(meta_done_);
    if (busy0_) cudaEventDestroy(busy0_);
    if (busy1_) cudaEventDestroy(busy1_);
    for (auto e : chunk_ev_)
        if (e) cudaEventDestroy(e);
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    if (stream_) cudaStreamDestroy(stream_);
}

// Pageable source: cudaMemcpyAsync stages the data before returning, so v may
// be released right after; the copy itself is ordered on `st`.
static void upload_floats(DevBuf& d, const std::vector<float>& v, cudaStream_t st) {
    d.ensure(v.size() * sizeof(float));
    cuda_check(cudaMemcpyAsync(d.p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice, st), "upload");
}

static std::vector<float> floats_sized(const GgufFile& gf, const std::string& name, size_t n) {
    auto v = gf.floats(name);
    if (v.size() != n) throw std::runtime_error("tensor size mismatch: " + name);
    return v;
}

// fp32 host data -> fp16 device buffer (via a temporary fp32 upload).
static void upload_f16(DevBuf& d, const std::vector<float>& v, cudaStream_t st) {
    DevBuf tmp;
    upload_floats(tmp, v, st);
    d.ensure(v.size() * 2);
    w2v_check(w2v_dequant_f16(tmp.p, 0, 1, (long long)v.size(), d.p, st), "fp16 weight conversion");
    cuda_check(cudaStreamSynchronize(st), "fp16 weight conversion");
    tmp.release();
}

void Engine::upload_linears(const GgufFile& gf, const std::vector<std::string>& names, const std::vector<int>& Ns,
                            int K, LinearW& L) {
    int N = 0, type = -1;
    bool same = true;
    for (size_t i = 0; i < names.size(); i++) {
        const auto& t = gf.tensor(names[i] + ".weight");
        // GGUF dims are innermost first: [K, N] (src/wav2vec2.cpp:116-125)
        if (t.shape.size() < 2 || (int)t.shape[0] != K || (int)t.shape[1] != Ns[i])
            throw std::runtime_error("tensor shape mismatch: " + names[i] + ".weight");
        if (t.type != GT_F32 && t.type != GT_F16 && t.type != GT_Q8_0 && t.type != GT_Q4_0)
            throw std::runtime_error("unsupported weight type " + std::to_string(t.type) + " for " + names[i]);
        if (t.nbytes != gguf_nbytes(t.type, (uint64_t)Ns[i] * K))
            throw std::runtime_error("tensor size mismatch: " + names[i] + ".weight");
        same = same && (type < 0 || (int)t.type == type);
        type = (int)t.type;
        N += Ns[i];
    }
    const bool quant = same && (type == GT_Q8_0 || type == GT_Q4_0) && K % 64 == 0 && !expand_weights_;
    L.N = N;
    L.K = K;
    L.gguf_type = quant ? type : (int)GT_F16;
    // codes [N][K] int8 or [N][K/2] 4-bit; scales [K/32][N'] fp16 with N' = N rounded up to 8 (16-byte rows)
    const size_t row_bytes = type == GT_Q8_0 ? (size_t)K : (size_t)K / 2;
    const size_t ld_s = ((size_t)N + 7) / 8 * 8;
    if (quant) {
        L.w.ensure((size_t)N * row_bytes);
        L.s.ensure((size_t)(K / 32) * ld_s * 2);
    } else {
        L.w.ensure((size_t)N * K * 2);
    }
    size_t row0 = 0;
    for (size_t i = 0; i < names.size(); i++) {
        const auto& t = gf.tensor(names[i] + ".weight");
        DevBuf raw;
        raw.ensure(t.nbytes);
        cuda_check(cudaMemcpyAsync(raw.p, t.data, t.nbytes, cudaMemcpyHostToDevice, stream_), "weight upload");
        if (quant)
            w2v_check(w2v_repack_q(raw.p, (int)t.type, Ns[i], K, L.w.as<uint8_t>() + row0 * row_bytes,
                                   L.s.as<uint16_t>() + row0, (long long)ld_s, stream_),
                      "weight repack");
        else
            w2v_check(w2v_dequant_f16(raw.p, (int)t.type, Ns[i], K, L.w.as<uint16_t>() + row0 * K, stream_),
                      "weight expansion");
        cuda_check(cudaStreamSynchronize(stream_), "weight upload");
        raw.release();
        row0 += (size_t)Ns[i];
    }
}

int Engine::gemm_linear(const void* A, long long M, const LinearW& L, void* C, long long ldc, const float* bias,
                        const float* resid, int epilogue, int block_n, const float* ln_stats, const float* ln_w,
                        const float* ln_b, cudaStream_t st) {
    int* err = err_.as<int>();
    if (L.gguf_type == GT_F16) {
        if (epilogue == W2V_EPI_F32_RESID_LN)
            return w2v_gemm_f16_ln_resid(A, L.K, 1, 1, L.K, M, 1, M * L.K, L.w.p, L.N, C, ldc, M, (int)M, bias, resid,
                                         ldc, ln_stats, ln_w, ln_b, block_n, err, st);
        return w2v_gemm_f16(A, L.K, 1, 1, L.K, M, 1, M * L.K, L.w.p, L.N, C, ldc, M, (int)M, bias, resid, ldc,
                            epilogue, block_n, err, st);
    }
    const long long ld_s = (L.N + 7) / 8 * 8;
    if (epilogue == W2V_EPI_F32_RESID_LN)
        return w2v_gemm_q_ln_resid(A, L.K, M, L.w.p, L.s.p, ld_s, L.gguf_type, L.N, C, ldc, bias, resid, ldc, ln_stats,
                                   ln_w, ln_b, 0, err, st);
    return w2v_gemm_q(A, L.K, M, L.w.p, L.s.p, ld_s, L.gguf_type, L.N, C, ldc, bias, resid, ldc, epilogue, 0, err, st);
}

size_t Engine::linear_weight_bytes() const {
    size_t n = proj_w_.bytes() + lm_w_.bytes();
    for (const auto& L : layers_) n += L.qkv.bytes() + L.o.bytes() + L.fc1.bytes() + L.fc2.bytes();
    return n;
}

void Engine::load(const GgufFile& gf) {
    const ModelConfig& c = cfg_;
    const int C = c.conv_dim, H = c.hidden, F = c.ffn, V = c.vocab;
    // conv layer 0: [C][1][k0] fp32 (src/wav2vec2.cpp:182-202)
    upload_floats(conv0_w_, floats_sized(gf, "feature_extractor.conv_layers.0.conv.weight", (size_t)C * c.conv_k[0]), stream_);
    conv_w_.resize(c.n_conv);
    conv_b_.resize(c.n_conv);
    conv_gw_.resize(c.n_conv);
    conv_gb_.resize(c.n_conv);
    for (int i = 0; i < c.n_conv; i++) {
        const std::string p = "feature_extractor.conv_layers." + std::to_string(i);
        if (c.conv_bias[i]) upload_floats(conv_b_[i], floats_sized(gf, p + ".conv.bias", C), stream_);
        if (c.conv_norm[i]) {
            upload_floats(conv_gw_[i], floats_sized(gf, p + ".layer_norm.weight", C), stream_);
            upload_floats(conv_gb_[i], floats_sized(gf, p + ".layer_norm.bias", C), stream_);
        }
        if (i == 0) continue;
        // [co][ci][k] -> implicit-GEMM B operand [co][k*C + ci]
        const int K = c.conv_k[i];
        auto w = floats_sized(gf, p + ".conv.weight", (size_t)C * C * K);
        std::vector<float> r((size_t)C * C * K);
        for (int co = 0; co < C; co++)
            for (int ci = 0; ci < C; ci++)
                for (int k = 0; k < K; k++) r[((size_t)co * K + k) * C + ci] = w[((size_t)co * C + ci) * K + k];
        upload_f16(conv_w_[i], r, stream_);
    }
    // feature projection (src/wav2vec2.cpp:205-208)
    upload_floats(proj_lnw_, floats_sized(gf, "feature_projection.layer_norm.weight", C), stream_);
    upload_floats(proj_lnb_, floats_sized(gf, "feature_projection.layer_norm.bias", C), stream_);
    upload_linears(gf, {"feature_projection.projection"}, {H}, C, proj_w_);
    upload_floats(proj_b_, floats_sized(gf, "feature_projection.projection.bias", H), stream_);
    // positional conv [H][Cg][Kp] (src/wav2vec2.cpp:211-212) -> per pair of taps
    // (2p, 2p+1), 8-channel core-matrix blocks with the two taps stacked along
    // the output channels: [G][Kp/2][Cg/8 (ci chunk)][2 Cg (tap, co)][8 (ci)]
    {
        const int G = c.pos_g, Cg = H / G, Kp = c.pos_k;
        auto w = floats_sized(gf, "encoder.pos_conv_embed.conv.weight", (size_t)H * Cg * Kp);
        std::vector<float> r(w.size());
        for (int g = 0; g < G; g++)
            for (int oc = 0; oc < Cg; oc++)
                for (int ic = 0; ic < Cg; ic++)
                    for (int k = 0; k < Kp; k++)
                        r[((((size_t)g * (Kp / 2) + k / 2) * (Cg / 8) + ic / 8) * (2 * Cg) + (k % 2) * Cg + oc) * 8 +
                          ic % 8] =
                            w[((size_t)(g * Cg + oc) * Cg + ic) * Kp + k];
        upload_f16(pos_w_, r, stream_);
        upload_floats(pos_b_, floats_sized(gf, "encoder.pos_conv_embed.conv.bias", H), stream_);
    }
    upload_floats(enc_lnw_, floats_sized(gf, "encoder.layer_norm.weight", H), stream_);
    upload_floats(enc_lnb_, floats_sized(gf, "encoder.layer_norm.bias", H), stream_);
    // encoder layers (src/wav2vec2.cpp:219-242); Q, K, V stacked into one [3H, H]
    layers_.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; l++) {
        auto& L = layers_[l];
        const std::string p = "encoder.layers." + std::to_string(l);
        upload_linears(gf, {p + ".attention.q_proj", p + ".attention.k_proj", p + ".attention.v_proj"}, {H, H, H}, H,
                       L.qkv);
        std::vector<float> bq = floats_sized(gf, p + ".attention.q_proj.bias", H);
        auto bk = floats_sized(gf, p + ".attention.k_proj.bias", H);
        auto bv = floats_sized(gf, p + ".attention.v_proj.bias", H);
        bq.insert(bq.end(), bk.begin(), bk.end());
        bq.insert(bq.end(), bv.begin(), bv.end());
        upload_floats(L.bqkv, bq, stream_);
        upload_linears(gf, {p + ".attention.out_proj"}, {H}, H, L.o);
        upload_floats(L.bo, floats_sized(gf, p + ".attention.out_proj.bias", H), stream_);
        upload_linears(gf, {p + ".feed_forward.intermediate_dense"}, {F}, H, L.fc1);
        upload_floats(L.b1, floats_sized(gf, p + ".feed_forward.intermediate_dense.bias", F), stream_);
        upload_linears(gf, {p + ".feed_forward.output_dense"}, {H}, F, L.fc2);
        upload_floats(L.b2, floats_sized(gf, p + ".feed_forward.output_dense.bias", H), stream_);
        upload_floats(L.ln1w, floats_sized(gf, p + ".layer_norm.weight", H), stream_);
        upload_floats(L.ln1b, floats_sized(gf, p + ".layer_norm.bias", H), stream_);
        upload_floats(L.ln2w, floats_sized(gf, p + ".final_layer_norm.weight", H), stream_);
        upload_floats(L.ln2b, floats_sized(gf, p + ".final_layer_norm.bias", H), stream_);
    }
    // CTC head (src/wav2vec2.cpp:245-246)
    upload_linears(gf, {"lm_head"}, {V}, H, lm_w_);
    upload_floats(lm_b_, floats_sized(gf, "lm_head.bias", V), stream_);
}

// ── per-batch geometry and workspace ────────────────────────────────────────

BatchGeom Engine::geometry(const std::vector<int>& n_samples) const {
    const ModelConfig& c = cfg_;
    BatchGeom g;
    g.n_utt = (int)n_samples.size();
    g.n_samples = n_samples;
    g.L.assign(c.n_conv, std::vector<int>(g.n_utt, 0));
    g.Lmax.assign(c.n_conv, 0);
    long long off = 0;
    for (int u = 0; u < g.n_utt; u++) {
        if (n_samples[u] < 0) throw std::runtime_error("negative sample count");
        g.audio_off.push_back(off);
        off += n_samples[u];
        long long L = n_samples[u];
        for (int i = 0; i < c.n_conv; i++) {
            L = (L < c.conv_k[i]) ? 0 : (L - c.conv_k[i]) / c.conv_s[i] + 1;
            g.L[i][u] = (int)L;
            g.Lmax[i] = std::max(g.Lmax[i], (int)L);
        }
    }
    // rows per utterance of each layer's padded buffer: a multiple of the next
    // layer's stride (the implicit GEMM reads rows in stride-phase groups)
    g.R.resize(c.n_conv);
    for (int i = 0; i < c.n_conv; i++) {
        const long long s_next = i + 1 < c.n_conv ? c.conv_s[i + 1] : 1;
        g.R[i] = std::max<long long>(round_up(std::max(g.Lmax[i], 1), s_next), s_next);
    }
    g.T = g.L.back();
    g.T_off.resize(g.n_utt);
    long long m = 0;
    for (int u = 0; u < g.n_utt; u++) {
        g.T_off[u] = m;
        m += g.T[u];
        g.T_max = std::max(g.T_max, g.T[u]);
    }
    g.M = m;
    return g;
}

void Engine::ensure_workspace(const BatchGeom& g) {
    const ModelConfig& c = cfg_;
    const size_t B = (size_t)std::max(g.n_utt, 1), C = c.conv_dim, H = c.hidden, F = c.ffn, V = c.vocab;
    const size_t M = (size_t)std::max<long long>(g.M, 1);
    size_t a0 = 0, a1 = 0;
    for (int i = 0; i < c.n_conv; i++) {
        size_t& a = (i % 2) ? a1 : a0;
        a = std::max<size_t>(a, B * (size_t)g.R[i] * C * 2);
    }
    bool re = false;
    re |= actA_.ensure(std::max<size_t>(a0, 16));
    re |= actB_.ensure(std::max<size_t>(a1, 16));
    re |= stats_.ensure(B * 2 * sizeof(float));
    re |= gn_.ensure(B * C * 2 * sizeof(double));
    re |= feat_.ensure(M * C * 2);
    re |= pbuf_.ensure(M * H * 4);
    re |= x_.ensure(M * H * 4);
    re |= ybuf_.ensure(M * H * 4);
    re |= lnstats_.ensure(M * 2 * sizeof(float));
    re |= xh_.ensure(M * H * 2);
    re |= attn_.ensure(M * H * 2);
    re |= qkv_.ensure(M * 3 * H * 2);
    re |= hbuf_.ensure(M * F * 2);
    re |= logits_.ensure(M * V * 4);
    re |= ids_.ensure(M * 4);
    re |= spans_.ensure(M * 3 * 4);
    re |= nspans_.ensure(B * 4);
    re |= meta_.ensure(B * (8 + 8 + 4 + 4 + 4 * (size_t)c.n_conv) + 64);
    if (re) {
        // captured forwards hold the old buffers' addresses
        ws_gen_++;
        drop_graphs();
    }
}

void Engine::drop_graphs() {
    // the pairs already seen stay known: their next call captures afresh
    for (auto& e : graphs_) cudaGraphExecDestroy(e.exec);
    graphs_.clear();
}

void Engine::upload_meta(const BatchGeom& g, cudaStream_t st) {
    const int B = g.n_utt, nc = cfg_.n_conv;
    const size_t bytes = (size_t)B * (8 + 8 + 4 + 4 + 4 * (size_t)nc);
    cuda_check(cudaEventSynchronize(meta_done_), "meta staging");
    if (meta_host_.size() < bytes) meta_host_.resize(bytes);
    uint8_t* h = meta_host_.data();
    size_t o = 0;
    auto put = [&](const void* src, size_t n) { memcpy(h + o, src, n); o += n; };
    put(g.audio_off.data(), 8 * (size_t)B);
    put(g.T_off.data(), 8 * (size_t)B);
    put(g.n_samples.data(), 4 * (size_t)B);
    for (int i = 0; i < nc; i++) put(g.L[i].data(), 4 * (size_t)B);
    uint8_t* d = meta_.as<uint8_t>();
    d_audio_off_ = reinterpret_cast<long long*>(d);
    d_T_off_ = reinterpret_cast<long long*>(d + 8 * (size_t)B);
    d_len_ = reinterpret_cast<int*>(d + 16 * (size_t)B);
    d_L_.resize(nc);
    for (int i = 0; i < nc; i++) d_L_[i] = reinterpret_cast<int*>(d + (20 + 4 * (size_t)i) * B);
    d_T_ = d_L_[nc - 1];
    // pageable source: the copy is staged before cudaMemcpyAsync returns
    cuda_check(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st), "meta upload");
    cuda_check(cudaEventRecord(meta_done_, st), "meta event");
}

int Engine::check_device_error() {
    int e = 0;
    cudaSetDevice(device_);
    if (cudaMemcpyAsync(&e, err_.p, sizeof(int), cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess)
        return -1;
    if (e) {
        cudaMemsetAsync(err_.p, 0, sizeof(int), stream_);
        cudaStreamSynchronize(stream_);
    }
    return e;
}

// ── forward ─────────────────────────────────────────────────────────────────

bool Engine::fwd_begin(const BatchGeom& g, cudaStream_t st) {
    cuda_check(cudaSetDevice(device_), "cudaSetDevice");
    last_M_ = g.M;
    launches_cur_ = 0;
    if (g.n_utt == 0) { launches_last_ = 0; return false; }
    ensure_workspace(g);
    upload_meta(g, st);
    if (g.M == 0) {
        cuda_check(cudaMemsetAsync(nspans_.p, 0, sizeof(int) * g.n_utt, st), "memset");
        launches_last_ = 0;
        return false;
    }
    return true;
}

void Engine::fwd_extract(const float* d_audio, const BatchGeom& g, int u0, int u1, cudaStream_t st) {
    const ModelConfig& c = cfg_;
    const int n = u1 - u0, C = c.conv_dim;
    if (n <= 0) return;
    int* err = err_.as<int>();
    // 1. waveform normalisation statistics + conv layer 0 with its norm and GELU
    launch(P_WAVE, 0.0, st, "wave_stats", [&] {
        return w2v_wave_stats(d_audio, d_audio_off_ + u0, d_len_ + u0, n, stats_.as<float>() + 2 * u0, st);
    });
    const int norm0 = c.conv_norm[0] ? (c.group_norm ? 1 : 2) : 0;
    long long f0 = 0;
    for (int u = u0; u < u1; u++) f0 += g.L[0][u];
    uint16_t* actA = actA_.as<uint16_t>();
    uint16_t* actB = actB_.as<uint16_t>();
    launch(P_CONV0, 2.0 * f0 * C * c.conv_k[0] * (norm0 == 1 ? 2 : 1), st, "conv0", [&] {
        return w2v_conv0(d_audio, d_audio_off_ + u0, d_len_ + u0, d_L_[0] + u0, n, stats_.as<float>() + 2 * u0,
                         conv0_w_.as<float>(), c.conv_bias[0] ? conv_b_[0].as<float>() : nullptr, C, c.conv_k[0],
                         c.conv_s[0], norm0, c.conv_norm[0] ? conv_gw_[0].as<float>() : nullptr,
                         c.conv_norm[0] ? conv_gb_[0].as<float>() : nullptr, gn_.as<double>(),
                         actA + (size_t)u0 * g.R[0] * C, g.R[0], g.Lmax[0], err, st);
    });
    if (norm0 == 1) launches_cur_ += 2;   // window moments and their reduction are two more kernels
    // 2. conv layers 1..n-1 as implicit GEMMs over the strided windows
    uint16_t* cur = actA;
    uint16_t* nxt = actB;
    for (int i = 1; i < c.n_conv; i++) {
        const bool ln = c.conv_norm[i];
        long long rows = 0;
        for (int u = u0; u < u1; u++) rows += g.L[i][u];
        uint16_t* in = cur + (size_t)u0 * g.R[i - 1] * C;
        uint16_t* out = nxt + (size_t)u0 * g.R[i] * C;
        if (g.Lmax[i] > 0)
            launch(P_GEMM_CONV, 2.0 * rows * C * C * c.conv_k[i], st, "gemm", [&] {
                return w2v_gemm_f16(in, C, c.conv_k[i], c.conv_s[i], C, g.R[i - 1], n, g.R[i - 1] * C,
                                    conv_w_[i].p, C, out, C, g.R[i], g.Lmax[i],
                                    c.conv_bias[i] ? conv_b_[i].as<float>() : nullptr, nullptr, C,
                                    ln ? W2V_EPI_F16 : W2V_EPI_F16_GELU, 0, err, st);
            });
        if (ln)
            launch(P_LN, 0.0, st, "conv layer_norm", [&] {
                return w2v_layer_norm(out, 1, C, g.R[i], d_L_[i] + u0, nullptr, n, 0, C, conv_gw_[i].as<float>(),
                                      conv_gb_[i].as<float>(), 1, nullptr, out, C, st);
            });
        std::swap(cur, nxt);
    }
}

void Engine::fwd_encode(const BatchGeom& g, cudaStream_t st, float* dbg_feat, float* dbg_stages) {
    const ModelConfig& c = cfg_;
    const int B = g.n_utt, C = c.conv_dim, H = c.hidden, V = c.vocab;
    int* err = err_.as<int>();
    const long long M = g.M;
    (void)err;
    // one linear over the packed rows: fp16 or dequant-fused GEMM by the weights' format
    auto plain_gemm = [&](int cat, const void* A, const LinearW& W, void* out, const DevBuf& bias,
                          const float* resid, int epi, int bn = 0) {
        launch(cat, 2.0 * M * W.N * W.K, st, "gemm", [&] {
            return gemm_linear(A, M, W, out, W.N, bias.as<float>(), resid, epi, bn, nullptr, nullptr, nullptr, st);
        });
    };
    auto dbg_copy = [&](int block, const float* src) {
        if (!dbg_stages) return;
        cuda_check(cudaMemcpyAsync(dbg_stages + (size_t)block * M * H, src, (size_t)M * H * 4, cudaMemcpyDeviceToHost,
                                   st),
                   "debug copy");
        cuda_check(cudaStreamSynchronize(st), "debug copy");
    };
    // output of the last conv layer: the ping-pong buffers alternate once per layer
    const void* cur = (c.n_conv - 1) % 2 ? actB_.p : actA_.p;
    if (dbg_feat) {
        std::vector<uint16_t> tmp((size_t)g.T[0] * C);
        cuda_check(cudaMemcpyAsync(tmp.data(), cur, tmp.size() * 2, cudaMemcpyDeviceToHost, st), "debug copy");
        cuda_check(cudaStreamSynchronize(st), "debug copy");
        for (size_t i = 0; i < tmp.size(); i++) dbg_feat[i] = f16_to_f32(tmp[i]);
    }
    // 3. feature projection: LN(conv_dim) -> packed fp16 rows -> linear
    //    (src/wav2vec2.cpp:345-347)
    launch(P_LN, 0.0, st, "projection layer_norm", [&] {
        return w2v_layer_norm(cur, 1, C, g.R[c.n_conv - 1], d_T_, d_T_off_, B, 0, C, proj_lnw_.as<float>(),
                              proj_lnb_.as<float>(), 0, nullptr, feat_.p, C, st);
    });
    plain_gemm(P_GEMM_PROJ, feat_.p, proj_w_, pbuf_.p, proj_b_, nullptr, W2V_EPI_F32);
    dbg_copy(0, pbuf_.as<float>());
    // 4. positional conv embedding + residual (src/wav2vec2.cpp:349-356)
    float* x = x_.as<float>();
    launch(P_POSCONV, 2.0 * M * c.pos_k * (H / c.pos_g) * H, st, "pos_conv", [&] {
        return w2v_pos_conv(x, pbuf_.as<float>(), d_T_off_, d_T_, B, H, c.pos_k, c.pos_g, pos_w_.p,
                            pos_b_.as<float>(), g.T_max, err, st);
    });
    const int n_heads = c.n_heads;
    double attn_flops = 0;
    for (int u = 0; u < B; u++) attn_flops += 4.0 * g.T[u] * g.T[u] * H;
    auto ln_rows = [&](const float* in, float* out32, void* out16, const DevBuf& w, const DevBuf& b) {
        launch(P_LN, 0.0, st, "layer_norm", [&] {
            return w2v_layer_norm(in, 0, H, M, nullptr, nullptr, 1, (int)M, H, w.as<float>(), b.as<float>(), 0,
                                  out32, out16, H, st);
        });
    };
    auto attention = [&] {
        launch(P_ATTN, attn_flops, st, "attention",
               [&] { return w2v_attention(qkv_.p, attn_.p, d_T_off_, d_T_, B, H, n_heads, g.T_max, M, err, st); });
    };
    if (!c.stable) {
        // post-LN encoder (src/wav2vec2.cpp:360-373).  x holds the raw
        // (pre-LayerNorm) residual stream and is updated in place: each
        // LayerNorm writes only its fp16 rows (the next GEMM's input) and the
        // rows' (mean, rstd); the next residual GEMM re-derives the fp32
        // normalised rows from x and those statistics in its epilogue, so the
        // normalised stream is never stored.
        float* lst = lnstats_.as<float>();
        auto ln_stats = [&](const DevBuf& w, const DevBuf& b) {
            launch(P_LN, 0.0, st, "layer_norm", [&] {
                return w2v_layer_norm_stats(x, M, H, w.as<float>(), b.as<float>(), xh_.p, lst, st);
            });
        };
        auto resid_ln_gemm = [&](const void* A, const LinearW& W, const DevBuf& bias, const DevBuf& lw,
                                 const DevBuf& lb) {
            launch(P_GEMM_ENC, 2.0 * M * W.N * W.K, st, "gemm", [&] {
                return gemm_linear(A, M, W, x, H, bias.as<float>(), x, W2V_EPI_F32_RESID_LN, 0, lst, lw.as<float>(),
                                   lb.as<float>(), st);
            });
        };
        auto dbg_norm = [&](int block, const DevBuf& lw, const DevBuf& lb) {   // debug: materialise LN(x)
            if (!dbg_stages) return;
            ln_rows(x, ybuf_.as<float>(), nullptr, lw, lb);
            dbg_copy(block, ybuf_.as<float>());
        };
        ln_stats(enc_lnw_, enc_lnb_);
        dbg_norm(1, enc_lnw_, enc_lnb_);
        const DevBuf* pw = &enc_lnw_;   // the LayerNorm that x currently stands for
        const DevBuf* pb = &enc_lnb_;
        for (int l = 0; l < c.n_layers; l++) {
            const auto& L = layers_[l];
            plain_gemm(P_GEMM_ENC, xh_.p, L.qkv, qkv_.p, L.bqkv, nullptr, W2V_EPI_F16);
            attention();
            resid_ln_gemm(attn_.p, L.o, L.bo, *pw, *pb);
            ln_stats(L.ln1w, L.ln1b);
            plain_gemm(P_GEMM_ENC, xh_.p, L.fc1, hbuf_.p, L.b1, nullptr, W2V_EPI_F16_GELU);
            resid_ln_gemm(hbuf_.p, L.fc2, L.b2, L.ln1w, L.ln1b);
            ln_stats(L.ln2w, L.ln2b);
            pw = &L.ln2w;
            pb = &L.ln2b;
            dbg_norm(2 + l, L.ln2w, L.ln2b);
        }
    } else {
        // pre-LN ("stable layer norm") encoder (src/wav2vec2.cpp:374-392)
        // LayerNorm of x into the next GEMM's fp16 rows (the statistics pass:
        // its (mean, rstd) output is not needed here)
        auto ln_half = [&](const DevBuf& w, const DevBuf& b) {
            if (H % 128) {   // the statistics pass takes rows of whole 128-column groups
                ln_rows(x, nullptr, xh_.p, w, b);
                return;
            }
            launch(P_LN, 0.0, st, "layer_norm", [&] {
                return w2v_layer_norm_stats(x, M, H, w.as<float>(), b.as<float>(), xh_.p, lnstats_.as<float>(), st);
            });
        };
        dbg_copy(1, x);
        for (int l = 0; l < c.n_layers; l++) {
            const auto& L = layers_[l];
            ln_half(L.ln1w, L.ln1b);
            plain_gemm(P_GEMM_ENC, xh_.p, L.qkv, qkv_.p, L.bqkv, nullptr, W2V_EPI_F16);
            attention();
            plain_gemm(P_GEMM_ENC, attn_.p, L.o, x, L.bo, x, W2V_EPI_F32_RESID);
            ln_half(L.ln2w, L.ln2b);
            plain_gemm(P_GEMM_ENC, xh_.p, L.fc1, hbuf_.p, L.b1, nullptr, W2V_EPI_F16_GELU);
            plain_gemm(P_GEMM_ENC, hbuf_.p, L.fc2, x, L.b2, x, W2V_EPI_F32_RESID);
            if (l == c.n_layers - 1) ln_rows(x, x, xh_.p, enc_lnw_, enc_lnb_);
            dbg_copy(2 + l, x);
        }
        if (c.n_layers == 0) ln_rows(x, x, xh_.p, enc_lnw_, enc_lnb_);
    }
    // 5. CTC head + greedy decode (src/wav2vec2.cpp:489, 498-503)
    plain_gemm(P_GEMM_LM, xh_.p, lm_w_, logits_.p, lm_b_, nullptr, W2V_EPI_F32, lm_w_.gguf_type == GT_F16 ? 64 : 0);
    launch(P_CTC, 0.0, st, "ctc_greedy", [&] {
        return w2v_ctc_greedy(logits_.as<float>(), d_T_off_, d_T_, B, V, ids_.as<int>(), spans_.as<int>(),
                              nspans_.as<int>(), g.T_max, st);
    });
    launches_last_ = launches_cur_;
}

void Engine::forward(const float* d_audio, const BatchGeom& g, cudaStream_t st, float* dbg_feat, float* dbg_stages) {
    if (!st) st = stream_;
    if (!fwd_begin(g, st)) return;   // workspace and metadata upload: never part of a captured graph
    extract_encode(d_audio, g, st, dbg_feat, dbg_stages);
}

void Engine::extract_encode(const float* d_audio, const BatchGeom& g, cudaStream_t st, float* dbg_feat,
                            float* dbg_stages) {
    if (graphs_enabled_ && !profiling_ && !dbg_feat && !dbg_stages) {
        // Replay a captured forward of this (input, lengths): one launch instead
        // of about a hundred, which is what a single short utterance waits on.
        for (auto& e : graphs_)
            if (e.audio == d_audio && e.ws_gen == ws_gen_ && e.n_samples == g.n_samples) {
                cuda_check(cudaGraphLaunch(e.exec, st), "cudaGraphLaunch");
                launches_last_ = e.launches;
                return;
            }
        bool seen = false;
        for (auto& k : graph_seen_)
            if (k.first == d_audio && k.second == g.n_samples) seen = true;
        // A full cache captures nothing more (the calls run kernel by kernel):
        // evicting would let a rotation over more inputs than it holds capture
        // on every call.
        if (seen && graphs_.size() < kMaxGraphs) {
            // Nothing captured is launched until the graph is instantiated: if the
            // capture or the instantiation fails, this engine stops capturing and
            // runs the forward kernel by kernel (a real error then surfaces there).
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            bool captured = false;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                try {
                    fwd_extract(d_audio, g, 0, g.n_utt, st);
                    fwd_encode(g, st, nullptr, nullptr);
                    captured = true;
                } catch (...) {
                }
                if (cudaStreamEndCapture(st, &graph) != cudaSuccess) captured = false;
                if (captured && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) captured = false;
                if (graph) cudaGraphDestroy(graph);
            }
            if (captured) {
                graphs_.push_back({d_audio, g.n_samples, ws_gen_, exec, launches_last_});
                cuda_check(cudaGraphLaunch(exec, st), "cudaGraphLaunch");
                return;
            }
            if (exec) cudaGraphExecDestroy(exec);
            cudaGetLastError();
            graphs_enabled_ = false;
            launches_cur_ = 0;   // the abandoned capture counted its launches
        }
        if (!seen) {
            if (graph_seen_.size() >= 4 * kMaxGraphs) graph_seen_.erase(graph_seen_.begin());
            graph_seen_.push_back({d_audio, g.n_samples});
        }
    }
    fwd_extract(d_audio, g, 0, g.n_utt, st);
    fwd_encode(g, st, dbg_feat, dbg_stages);
}


void Engine::run_host(const std::vector<const float*>& audio, const std::vector<int>& n_samples,
                      std::vector<float>* logits, std::vector<int>* spans, std::vector<int>* n_spans,
                      BatchGeom* geom_out) {
    cuda_check(cudaSetDevice(device_), "cudaSetDevice");
    BatchGeom g = geometry(n_samples);
    const size_t total = g.n_utt ? (size_t)(g.audio_off.back() + n_samples.back()) : 0;
    if (total > h_audio_n_) {
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        if (h_audio_) cudaFreeHost(h_audio_);
        h_audio_ = nullptr;
        cuda_check(cudaMallocHost(&h_audio_, std::max<size_t>(total, 1) * sizeof(float)), "cudaMallocHost");
        h_audio_n_ = total;
    }
    audio_stage_.ensure(std::max<size_t>(total, 1) * sizeof(float));
    // Pipelined upload: the batch is cut into up to kMaxChunks utterance
    // chunks.  Host threads pack the caller's (pageable) utterances into
    // pinned staging chunk by chunk; as soon as a chunk is packed it is copied
    // on the copy stream and the feature extractor for its utterances is
    // queued behind that copy, so the DMA and packing of later chunks overlap
    // the convolutions of earlier ones.  The encoder then runs on the batch.
    const int B = g.n_utt;
    // The first chunk is small (an eighth of the batch) so that the only
    // upload nothing overlaps is short; the rest is split evenly.
    const int nch = B >= 32 ? kMaxChunks : B >= 8 ? 2 : 1;
    std::vector<int> cu(nch + 1);
    cu[0] = 0;
    if (nch == 1) {
        cu[1] = B;
    } else {
        cu[1] = std::max(1, B / 8);
        for (int k = 2; k <= nch; k++) cu[k] = cu[1] + (int)((long long)(B - cu[1]) * (k - 1) / (nch - 1));
    }
    const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
    const int nt = std::max(1, std::min({pack_threads_ > 0 ? pack_threads_ : 8, hw / 2, std::max(1, B / nch)}));
    std::unique_ptr<std::atomic<int>[]> packed(new std::atomic<int>[nch]);
    for (int k = 0; k < nch; k++) packed[k].store(0);
    auto pack = [&](int t) {
        for (int k = 0; k < nch; k++) {
            const int n = cu[k + 1] - cu[k];
            const int u0 = cu[k] + (int)((long long)n * t / nt), u1 = cu[k] + (int)((long long)n * (t + 1) / nt);
            for (int u = u0; u < u1; u++)
                if (n_samples[u]) memcpy(h_audio_ + g.audio_off[u], audio[u], (size_t)n_samples[u] * sizeof(float));
            packed[k].fetch_add(1, std::memory_order_release);
        }
    };
    // Page-locked caller buffers need no staging: each chunk's utterances are
    // copied straight from them.
    bool pinned = B > 0;
    for (int u = 0; u < B && pinned; u++) {
        if (!n_samples[u]) continue;
        cudaPointerAttributes at{};
        pinned = cudaPointerGetAttributes(&at, audio[u]) == cudaSuccess && at.type == cudaMemoryTypeHost;
    }
    cudaGetLastError();   // a pageable pointer may leave an error from the query
    // device span of this batch: from before its first upload (copy stream)
    // to after its last download (compute stream)
    cuda_check(cudaEventRecord(busy0_, copy_stream_), "busy event");
    if (nch == 1 && fwd_begin(g, stream_)) {
        // one chunk (short batches): upload, then the whole forward, which
        // repeated batches of the same lengths replay as one captured graph
        if (pinned) {
            for (int u = 0; u < B; u++)
                if (n_samples[u])
                    cuda_check(cudaMemcpyAsync(audio_stage_.as<float>() + g.audio_off[u], audio[u],
                                               (size_t)n_samples[u] * sizeof(float), cudaMemcpyHostToDevice,
                                               copy_stream_),
                               "audio upload");
        } else {
            std::vector<std::thread> packers;
            struct Joiner {
                std::vector<std::thread>& v;
                ~Joiner() {
                    for (auto& t : v)
                        if (t.joinable()) t.join();
                }
            } joiner{packers};
            for (int t = 0; t < nt; t++) packers.emplace_back(pack, t);
            for (auto& t : packers) t.join();
            if (total)
                cuda_check(cudaMemcpyAsync(audio_stage_.as<float>(), h_audio_, total * sizeof(float),
                                           cudaMemcpyHostToDevice, copy_stream_),
                           "audio upload");
        }
        cuda_check(cudaEventRecord(chunk_ev_[0], copy_stream_), "chunk event");
        cuda_check(cudaStreamWaitEvent(stream_, chunk_ev_[0], 0), "chunk wait");
        extract_encode(audio_stage_.as<float>(), g, stream_, nullptr, nullptr);
    } else if (pinned && fwd_begin(g, stream_)) {
        for (int k = 0; k < nch; k++) {
            for (int u = cu[k]; u < cu[k + 1]; u++)
                if (n_samples[u])
                    cuda_check(cudaMemcpyAsync(audio_stage_.as<float>() + g.audio_off[u], audio[u],
                                               (size_t)n_samples[u] * sizeof(float), cudaMemcpyHostToDevice,
                                               copy_stream_),
                               "audio upload");
            cuda_check(cudaEventRecord(chunk_ev_[k], copy_stream_), "chunk event");
            cuda_check(cudaStreamWaitEvent(stream_, chunk_ev_[k], 0), "chunk wait");
            fwd_extract(audio_stage_.as<float>(), g, cu[k], cu[k + 1], stream_);
        }
        fwd_encode(g, stream_, nullptr, nullptr);
    } else if (!pinned && fwd_begin(g, stream_)) {
        std::vector<std::thread> packers;
        struct Joiner {
            std::vector<std::thread>& v;
            ~Joiner() {
                for (auto& t : v)
                    if (t.joinable()) t.join();
            }
        } joiner{packers};
        for (int t = 0; t < nt; t++) packers.emplace_back(pack, t);
        for (int k = 0; k < nch; k++) {
            while (packed[k].load(std::memory_order_acquire) < nt) std::this_thread::yield();
            const long long b0 = g.audio_off[cu[k]];
            const long long b1 = g.audio_off[cu[k + 1] - 1] + n_samples[cu[k + 1] - 1];
            if (b1 > b0)
                cuda_check(cudaMemcpyAsync(audio_stage_.as<float>() + b0, h_audio_ + b0,
                                           (size_t)(b1 - b0) * sizeof(float), cudaMemcpyHostToDevice, copy_stream_),
                           "audio upload");
            cuda_check(cudaEventRecord(chunk_ev_[k], copy_stream_), "chunk event");
            cuda_check(cudaStreamWaitEvent(stream_, chunk_ev_[k], 0), "chunk wait");
            fwd_extract(audio_stage_.as<float>(), g, cu[k], cu[k + 1], stream_);
        }
        for (auto& t : packers) t.join();
        fwd_encode(g, stream_, nullptr, nullptr);
    }
    if (g.M > 0 && logits) {
        logits->resize((size_t)g.M * cfg_.vocab);
        cuda_check(cudaMemcpyAsync(logits->data(), logits_.p, logits->size() * 4, cudaMemcpyDeviceToHost, stream_),
                   "logits download");
    }
    // The device error word, the spans and the span counts come back through
    // one pinned staging buffer and one synchronisation.
    const size_t sp_bytes = spans && g.M > 0 ? (size_t)g.M * 3 * sizeof(int) : 0;
    const size_t ns_bytes = n_spans && g.M > 0 ? (size_t)g.n_utt * sizeof(int) : 0;
    const size_t out_bytes = 16 + sp_bytes + ns_bytes;
    if (out_bytes > h_out_n_) {
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        if (h_out_) cudaFreeHost(h_out_);
        h_out_ = nullptr;
        cuda_check(cudaMallocHost(&h_out_, out_bytes), "cudaMallocHost");
        h_out_n_ = out_bytes;
    }
    cuda_check(cudaMemcpyAsync(h_out_, err_.p, sizeof(int), cudaMemcpyDeviceToHost, stream_), "error word download");
    if (sp_bytes)
        cuda_check(cudaMemcpyAsync(h_out_ + 16, spans_.p, sp_bytes, cudaMemcpyDeviceToHost, stream_), "spans download");
    if (ns_bytes)
        cuda_check(cudaMemcpyAsync(h_out_ + 16 + sp_bytes, nspans_.p, ns_bytes, cudaMemcpyDeviceToHost, stream_),
                   "spans download");
    cuda_check(cudaEventRecord(busy1_, stream_), "busy event");
    cuda_check(cudaStreamSynchronize(stream_), "forward");
    {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, busy0_, busy1_) == cudaSuccess) {
            std::lock_guard<std::mutex> lk(busy_mu_);
            busy_ms_ += ms;
            busy_batches_ += 1;
            busy_samples_ += (long long)total;
        }
        cudaGetLastError();
    }
    int e = 0;
    memcpy(&e, h_out_, sizeof(int));
    if (e) {
        cudaMemsetAsync(err_.p, 0, sizeof(int), stream_);
        cudaStreamSynchronize(stream_);
        throw std::runtime_error("device error " + std::to_string(e) + " (bounded wait expired)");
    }
    if (spans && g.M > 0) {
        spans->resize((size_t)g.M * 3);
        memcpy(spans->data(), h_out_ + 16, sp_bytes);
    }
    if (n_spans) {
        n_spans->assign(g.n_utt, 0);
        if (ns_bytes) memcpy(n_spans->data(), h_out_ + 16 + sp_bytes, ns_bytes);
    }
    if (geom_out) *geom_out = std::move(g);
}

}  // namespace w2v
