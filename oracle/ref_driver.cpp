// Oracle driver around the reference's own, unmodified sources.
//
// Test infrastructure only: built by oracle/Makefile into oracle/_ref/ from
// the reference checkout, linked with the oracle's ggml-API shim.  It pulls
// src/wav2vec2.cpp into this translation unit so that the reference's
// file-static forward-pass stages (feature_extract, encode, self_attention)
// can be called directly and their fp32 outputs returned as golden data; the
// reference's public C API does not expose logits.
//
// All entry points catch the reference's C++ exceptions and return -1/NULL.
#include "wav2vec2.cpp"   // reference src/wav2vec2.cpp (found via -I<ref>/src)

extern "C" {

wav2vec2_context * w2vref_init(const char * path) {
    try { return wav2vec2_init(path); }
    catch (const std::exception & e) { fprintf(stderr, "w2vref_init: %s\n", e.what()); return nullptr; }
}

void w2vref_free(wav2vec2_context * ctx) { wav2vec2_free(ctx); }

// Model hyper-parameters as the reference parsed them (wav2vec2.cpp:133-156).
// out[0..9] = conv_dim, hidden, n_layers, n_heads, intermediate, vocab, pad_id,
//             stable_layer_norm, n_conv_layers, feat_norm_is_group
int w2vref_info(const wav2vec2_context * ctx, int * out) {
    const auto & m = ctx->model;
    out[0] = m.conv_dim; out[1] = m.hidden; out[2] = m.n_enc_layers; out[3] = m.n_heads;
    out[4] = m.intermediate; out[5] = m.vocab_size; out[6] = m.pad_id;
    out[7] = m.stable_layer_norm ? 1 : 0; out[8] = m.n_conv_layers;
    out[9] = m.feat_norm == "group" ? 1 : 0;
    return 0;
}

// CNN feature extractor output [T, conv_dim] (wav2vec2.cpp:257-289). Returns T.
int w2vref_features(wav2vec2_context * ctx, const float * samples, int n, float * out, long cap) {
    try {
        auto f = feature_extract(ctx->model, samples, n);
        if ((long)f.size() > cap) return -1;
        memcpy(out, f.data(), f.size() * sizeof(float));
        return (int)(f.size() / ctx->model.conv_dim);
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_features: %s\n", e.what()); return -1; }
}

// Encoder output [T, hidden] from features (wav2vec2.cpp:340-394).
int w2vref_encode(wav2vec2_context * ctx, const float * feat, int T, int n_threads, float * out) {
    try {
        auto x = encode(ctx->model, ctx->scratch, feat, T, n_threads);
        memcpy(out, x.data(), x.size() * sizeof(float));
        return T;
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_encode: %s\n", e.what()); return -1; }
}

// Encoder activations after each stage, for stage-wise parity: out holds
// (n_layers + 2) blocks of [T, hidden]: block 0 = feature projection output,
// block 1 = after the positional conv (+ encoder LN for post-LN models),
// block 2 + l = after encoder layer l.  The stage sequence is the reference's
// encode() (wav2vec2.cpp:340-394) driven step by step with its own primitives.
int w2vref_encode_stages(wav2vec2_context * ctx, const float * feat, int T, int n_threads, float * out) {
    try {
        const auto & m = ctx->model;
        auto & scratch = ctx->scratch;
        const int H = m.hidden;
        const size_t blk = (size_t)T * H;
        std::vector<float> feat_norm(feat, feat + (size_t)T * m.conv_dim);
        wv2_layer_norm(feat_norm.data(), m.proj_ln_w.data(), m.proj_ln_b.data(), T, m.conv_dim);
        auto x = scratch.linear(m.proj_w, feat_norm.data(), T, m.conv_dim, H, m.proj_b, n_threads);
        memcpy(out, x.data(), blk * sizeof(float));
        int pk = m.pos_conv_kernel, pg = m.pos_conv_groups;
        auto pos = wv2_conv1d(x.data(), m.pos_w.data(), m.pos_b.data(), T, H, H, pk, 1, pk / 2, pg);
        int use_T = std::min(T, (int)pos.size() / H);
        for (auto & v : pos) v = wv2_gelu(v);
        for (int t = 0; t < use_T; t++)
            for (int i = 0; i < H; i++) x[t * H + i] += pos[t * H + i];
        std::vector<float> attn_buf((size_t)T * H), ln_buf((size_t)T * H);
        if (!m.stable_layer_norm) {
            wv2_layer_norm(x.data(), m.enc_ln_w.data(), m.enc_ln_b.data(), T, H);
            memcpy(out + blk, x.data(), blk * sizeof(float));
            int l = 0;
            for (const auto & el : m.enc_layers) {
                self_attention(el, scratch, attn_buf.data(), x.data(), T, H, m.n_heads, n_threads);
                for (size_t i = 0; i < blk; i++) x[i] += attn_buf[i];
                wv2_layer_norm(x.data(), el.ln1_w.data(), el.ln1_b.data(), T, H);
                auto ff1 = scratch.linear(el.ff.fc1_w, x.data(), T, H, m.intermediate, el.ff.fc1_b, n_threads);
                for (auto & v : ff1) v = wv2_gelu(v);
                auto ff2 = scratch.linear(el.ff.fc2_w, ff1.data(), T, m.intermediate, H, el.ff.fc2_b, n_threads);
                for (size_t i = 0; i < blk; i++) x[i] += ff2[i];
                wv2_layer_norm(x.data(), el.ln2_w.data(), el.ln2_b.data(), T, H);
                memcpy(out + (2 + l++) * blk, x.data(), blk * sizeof(float));
            }
        } else {
            memcpy(out + blk, x.data(), blk * sizeof(float));
            int l = 0;
            for (const auto & el : m.enc_layers) {
                std::copy(x.begin(), x.end(), ln_buf.begin());
                wv2_layer_norm(ln_buf.data(), el.ln1_w.data(), el.ln1_b.data(), T, H);
                self_attention(el, scratch, attn_buf.data(), ln_buf.data(), T, H, m.n_heads, n_threads);
                for (size_t i = 0; i < blk; i++) x[i] += attn_buf[i];
                std::copy(x.begin(), x.end(), ln_buf.begin());
                wv2_layer_norm(ln_buf.data(), el.ln2_w.data(), el.ln2_b.data(), T, H);
                auto ff1 = scratch.linear(el.ff.fc1_w, ln_buf.data(), T, H, m.intermediate, el.ff.fc1_b, n_threads);
                for (auto & v : ff1) v = wv2_gelu(v);
                auto ff2 = scratch.linear(el.ff.fc2_w, ff1.data(), T, m.intermediate, H, el.ff.fc2_b, n_threads);
                for (size_t i = 0; i < blk; i++) x[i] += ff2[i];
                memcpy(out + (2 + l++) * blk, x.data(), blk * sizeof(float));
            }
            // the final encoder LN belongs to the last stage block
            wv2_layer_norm(x.data(), m.enc_ln_w.data(), m.enc_ln_b.data(), T, H);
            memcpy(out + (size_t)(1 + (l > 0 ? l : 0)) * blk, x.data(), blk * sizeof(float));
        }
        return T;
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_encode_stages: %s\n", e.what()); return -1; }
}

// CTC logits [T, vocab] for one utterance: the reference's transcribe path up
// to the lm_head linear (wav2vec2.cpp:485-489). Returns T.
int w2vref_logits(wav2vec2_context * ctx, const float * samples, int n, int n_threads,
                  float * out, long cap) {
    try {
        const auto & m = ctx->model;
        auto feat = feature_extract(m, samples, n);
        int T = (int)feat.size() / m.conv_dim;
        auto enc = encode(m, ctx->scratch, feat.data(), T, n_threads);
        auto logits = ctx->scratch.linear(m.lm_w, enc.data(), T, m.hidden, m.vocab_size, m.lm_b, n_threads);
        if ((long)logits.size() > cap) return -1;
        memcpy(out, logits.data(), logits.size() * sizeof(float));
        return T;
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_logits: %s\n", e.what()); return -1; }
}

// Logits from given encoder features: lm_head(encode(feat)).
int w2vref_logits_from_features(wav2vec2_context * ctx, const float * feat, int T, int n_threads,
                                float * out) {
    try {
        const auto & m = ctx->model;
        auto enc = encode(m, ctx->scratch, feat, T, n_threads);
        auto logits = ctx->scratch.linear(m.lm_w, enc.data(), T, m.hidden, m.vocab_size, m.lm_b, n_threads);
        memcpy(out, logits.data(), logits.size() * sizeof(float));
        return T;
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_logits_from_features: %s\n", e.what()); return -1; }
}

// Reference public-API transcription (wav2vec2.cpp:477-533); returns the
// transcript length copied into buf (NUL-terminated), or -1.
int w2vref_transcribe(wav2vec2_context * ctx, const float * samples, int n, int n_threads,
                      int beam, char * buf, int cap) {
    try {
        auto p = wav2vec2_default_params();
        p.n_threads = n_threads; p.beam_size = beam;
        auto * r = wav2vec2_transcribe(ctx, p, samples, n);
        int len = (int)strlen(r->transcript);
        if (len + 1 > cap) { wav2vec2_result_free(r); return -1; }
        memcpy(buf, r->transcript, len + 1);
        wav2vec2_result_free(r);
        return len;
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_transcribe: %s\n", e.what()); return -1; }
}

// Greedy CTC spans from logits (ops.h:132-149): out = [id, t0, t1] triples.
int w2vref_greedy_spans(const float * logits, int T, int V, int * out, int cap_spans) {
    auto s = wv2_ctc_greedy_spans(logits, T, V);
    if ((int)s.size() > cap_spans) return -1;
    for (size_t i = 0; i < s.size(); i++) { out[3*i] = s[i].token_id; out[3*i+1] = s[i].t_start; out[3*i+2] = s[i].t_end; }
    return (int)s.size();
}

// The reference's greedy post-processing on given logits, exactly as its
// public transcribe call runs it (wav2vec2.cpp:497-503, 515-530): greedy
// spans, pad filter, ids_to_text and spans_to_words, with the word times
// converted to seconds by the same float expression.  text receives the
// transcript; words receives the words separated by '\n'; times[2i],
// times[2i+1] = start, end of word i.  Returns the number of words, or -1.
int w2vref_words_from_logits(wav2vec2_context * ctx, const float * logits, int T, char * text, int text_cap,
                             char * words, int words_cap, float * times, int max_words) {
    try {
        const auto & m = ctx->model;
        auto spans = wv2_ctc_greedy_spans(logits, T, m.vocab_size);
        std::vector<int> ids;
        for (const auto & sp : spans)
            if (sp.token_id != m.pad_id) ids.push_back(sp.token_id);
        std::string t = ids_to_text(ids, m.pad_id, m.vocab, m.word_delimiter);
        auto ws = spans_to_words(spans, m.pad_id, m.vocab, m.word_delimiter);
        if ((int)t.size() + 1 > text_cap || (int)ws.size() > max_words) return -1;
        memcpy(text, t.c_str(), t.size() + 1);
        std::string joined;
        for (size_t i = 0; i < ws.size(); i++) {
            if (i) joined += '\n';
            joined += ws[i].word;
            times[2 * i] = ws[i].t_start * (320.f / 16000.f);
            times[2 * i + 1] = ws[i].t_end * (320.f / 16000.f);
        }
        if ((int)joined.size() + 1 > words_cap) return -1;
        memcpy(words, joined.c_str(), joined.size() + 1);
        return (int)ws.size();
    } catch (const std::exception & e) { fprintf(stderr, "w2vref_words_from_logits: %s\n", e.what()); return -1; }
}

// Prefix beam search from logits (ops.h:162-251).
int w2vref_beam_search(const float * logits, int T, int V, int blank, int beam, int * out, int cap) {
    auto ids = wv2_ctc_beam_search(logits, T, V, blank, beam);
    if ((int)ids.size() > cap) return -1;
    for (size_t i = 0; i < ids.size(); i++) out[i] = ids[i];
    return (int)ids.size();
}

// Single reference primitives for known-answer comparisons (ops.h:18-106).
float w2vref_gelu(float x) { return wv2_gelu(x); }
void w2vref_layer_norm(float * x, const float * w, const float * b, int T, int D) { wv2_layer_norm(x, w, b, T, D); }
void w2vref_group_norm(float * x, const float * w, const float * b, int T, int C) { wv2_group_norm(x, w, b, T, C); }
void w2vref_softmax(float * x, int n) { wv2_softmax(x, n); }
int w2vref_conv1d(const float * x, const float * w, const float * b, int L, int Cin, int Cout,
                  int K, int stride, int pad, int groups, float * out) {
    auto y = wv2_conv1d(x, w, b, L, Cin, Cout, K, stride, pad, groups);
    memcpy(out, y.data(), y.size() * sizeof(float));
    return (int)(y.size() / Cout);
}

}  // extern "C"
