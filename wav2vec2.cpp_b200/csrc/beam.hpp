// CTC prefix beam search on host logits (the reference's host decoder,
// src/ops.h:151-251: Graves 2006 prefix search in the log domain, beam of
// `width` prefixes, blank id `blank`).
//
// Same search and the same float arithmetic per state as the reference, in a
// different data structure:
//   * prefixes are nodes of a trie (parent, last token) that lives for the
//     whole utterance; a child is found by hashing (parent, token), so a step
//     never copies or compares token vectors (the reference keys an ordered
//     map by whole token vectors, O(length) per comparison);
//   * the candidates of a frame sit in a flat array indexed through a
//     per-node stamp, so each lookup is O(1).
// Each candidate's two log-probabilities receive at most two contributions
// per frame (its own continuation and its parent's extension), and
// log_sum_exp is symmetric, so the order in which beams are expanded does not
// change any value.  Ties are broken by an explicit rule: higher score first,
// then the lexicographically smaller token sequence (the reference iterates
// its map in that order when it picks the final prefix; while pruning, exact
// score ties among finite scores do not occur in practice and ties at the
// -1e30 floor never displace a finite-score prefix).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <unordered_map>
#include <vector>

namespace w2v {

inline float lse2(float a, float b) {
    if (a <= -1e29f) return b;
    if (b <= -1e29f) return a;
    const float hi = a > b ? a : b, lo = a > b ? b : a;
    return hi + log1pf(expf(lo - hi));
}

class PrefixTrie {
public:
    PrefixTrie() { add(-1, -1); }
    int child(int p, int tok) {
        const uint64_t key = ((uint64_t)(uint32_t)p << 32) | (uint32_t)tok;
        auto it = kids_.find(key);
        if (it != kids_.end()) return it->second;
        const int n = add(p, tok);
        kids_.emplace(key, n);
        return n;
    }
    int last(int n) const { return tok_[n]; }
    int size() const { return (int)tok_.size(); }
    std::vector<int> tokens(int n) const {
        std::vector<int> t((size_t)depth_[n]);
        for (int i = depth_[n] - 1; i >= 0; i--, n = parent_[n]) t[(size_t)i] = tok_[n];
        return t;
    }
    // token sequence of a before that of b (lexicographic, a proper prefix first)
    bool lex_less(int a, int b) const {
        if (a == b) return false;
        const auto x = tokens(a), y = tokens(b);
        return std::lexicographical_compare(x.begin(), x.end(), y.begin(), y.end());
    }

private:
    int add(int p, int tok) {
        parent_.push_back(p);
        tok_.push_back(tok);
        depth_.push_back(p < 0 ? 0 : depth_[p] + 1);
        return (int)tok_.size() - 1;
    }
    std::vector<int> parent_, tok_, depth_;
    std::unordered_map<uint64_t, int> kids_;
};

inline std::vector<int> ctc_prefix_beam_search(const float* logits, int T, int V, int blank, int width) {
    constexpr float kFloor = -1e30f;
    struct Beam {
        int node;
        float pb, pnb;       // log P(prefix, path ends in blank / in its last token)
    };
    if (width < 1) width = 1;
    PrefixTrie trie;
    std::vector<Beam> cur{{0, 0.f, kFloor}}, next;
    std::vector<int> stamp, slot;      // candidate slot of a node in this frame
    std::vector<float> lp((size_t)V);
    std::vector<std::pair<float, int>> order;
    for (int t = 0; t < T; t++) {
        const float* row = logits + (size_t)t * V;
        float mx = row[0];
        for (int v = 1; v < V; v++) mx = row[v] > mx ? row[v] : mx;
        float z = 0.f;
        for (int v = 0; v < V; v++) z += expf(row[v] - mx);
        const float lz = mx + logf(z);
        for (int v = 0; v < V; v++) lp[(size_t)v] = row[v] - lz;
        next.clear();
        auto cand = [&](int node) -> Beam& {
            if (node >= (int)stamp.size()) {
                stamp.resize((size_t)trie.size() * 2 + 64, -1);
                slot.resize(stamp.size());
            }
            if (stamp[(size_t)node] != t) {
                stamp[(size_t)node] = t;
                slot[(size_t)node] = (int)next.size();
                next.push_back({node, kFloor, kFloor});
            }
            return next[(size_t)slot[(size_t)node]];
        };
        for (size_t bi = 0; bi < cur.size(); bi++) {
            const Beam b = cur[bi];
            const float total = lse2(b.pb, b.pnb);
            const int last = trie.last(b.node);
            {
                Beam& s = cand(b.node);
                s.pb = lse2(s.pb, total + lp[(size_t)blank]);
            }
            for (int ch = 0; ch < V; ch++) {
                if (ch == blank) continue;
                const float l = lp[(size_t)ch];
                const int q = trie.child(b.node, ch);
                if (ch == last) {
                    // the same token again without a blank continues the prefix;
                    // after a blank it starts a new copy of the token
                    Beam& s = cand(b.node);
                    s.pnb = lse2(s.pnb, b.pnb + l);
                    Beam& e = cand(q);
                    e.pnb = lse2(e.pnb, b.pb + l);
                } else {
                    Beam& e = cand(q);
                    e.pnb = lse2(e.pnb, total + l);
                }
            }
        }
        // keep the `width` best: higher score, then the smaller token sequence
        order.clear();
        for (size_t i = 0; i < next.size(); i++) order.push_back({lse2(next[i].pb, next[i].pnb), (int)i});
        auto better = [&](const std::pair<float, int>& a, const std::pair<float, int>& b) {
            if (a.first != b.first) return a.first > b.first;
            return trie.lex_less(next[(size_t)a.second].node, next[(size_t)b.second].node);
        };
        const size_t keep = std::min(order.size(), (size_t)width);
        std::partial_sort(order.begin(), order.begin() + (long)keep, order.end(), better);
        cur.clear();
        for (size_t i = 0; i < keep; i++) cur.push_back(next[(size_t)order[i].second]);
    }
    int best = -1;
    float bs = kFloor;
    for (const Beam& b : cur) {
        const float s = lse2(b.pb, b.pnb);
        if (best < 0 || s > bs || (s == bs && trie.lex_less(b.node, best))) {
            bs = s;
            best = b.node;
        }
    }
    // the reference returns the empty sequence unless some prefix beats its floor
    if (best < 0 || !(bs > kFloor)) return {};
    return trie.tokens(best);
}

}  // namespace w2v
