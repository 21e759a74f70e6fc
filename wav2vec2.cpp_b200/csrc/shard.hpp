// Utterance batching and the multi-device batch scheduler.
//
// The reference transcribes one utterance per call on one host
// (include/wav2vec2.h:40-44); utterances share no state, so the engine
// shards them: length-bucketed batches are pulled from a shared queue by one
// worker (host thread + CUDA stream) per device.  No data crosses devices.
//
// A worker whose batch fails (a device error, a failed launch) retires and
// its batch goes back on the queue for the remaining workers; the call fails
// only when no worker is left.  Header-only so the scheduler can be tested on
// the CPU with fake workers.
#pragma once
#include <algorithm>
#include <condition_variable>
#include <deque>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace w2v {

// Batches of utterance indices, longest first: at most max_batch utterances
// and at most max_padded padded samples (batch size x longest utterance) per
// batch, so conv-extractor padding stays small and memory bounded.
inline std::vector<std::vector<int>> make_batches(const int* n_samples, int n_utt, int max_batch,
                                                  long long max_padded) {
    std::vector<int> order(n_utt);
    for (int i = 0; i < n_utt; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return n_samples[a] > n_samples[b]; });
    std::vector<std::vector<int>> batches;
    std::vector<int> cur;
    long long cur_max = 0;
    for (int i : order) {
        const long long n = std::max(n_samples[i], 1);
        const long long new_max = std::max(cur_max, n);
        if (!cur.empty() && ((int)cur.size() >= max_batch || new_max * (long long)(cur.size() + 1) > max_padded)) {
            batches.push_back(cur);
            cur.clear();
            cur_max = 0;
        }
        cur.push_back(i);
        cur_max = std::max(cur_max, n);
    }
    if (!cur.empty()) batches.push_back(cur);
    return batches;
}

// Run batches 0..n_batches-1 on n_workers workers.  fn(worker, batch) returns
// true on success; on false (or an exception) the worker retires and the
// batch is re-queued.  Throws std::runtime_error if every worker retired
// before all batches completed; `first_error` holds the first failure text.
inline void run_batches(size_t n_batches, int n_workers,
                        const std::function<bool(int, size_t, std::string&)>& fn) {
    std::mutex mu;
    std::condition_variable cv;
    std::deque<size_t> pending;
    for (size_t b = 0; b < n_batches; b++) pending.push_back(b);
    size_t in_flight = 0, done = 0;
    int alive = n_workers;
    std::string first_error;
    auto worker = [&](int w) {
        for (;;) {
            size_t b;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return !pending.empty() || in_flight == 0; });
                if (pending.empty()) return;         // nothing queued, nothing that could come back
                b = pending.front();
                pending.pop_front();
                in_flight++;
            }
            std::string err;
            bool ok = false;
            try {
                ok = fn(w, b, err);
            } catch (const std::exception& e) {
                err = e.what();
            }
            std::lock_guard<std::mutex> lk(mu);
            in_flight--;
            if (ok) {
                done++;
                cv.notify_all();
                continue;
            }
            if (first_error.empty()) first_error = "worker " + std::to_string(w) + ": " + err;
            pending.push_front(b);                   // re-queue for the surviving workers
            alive--;
            cv.notify_all();
            return;
        }
    };
    if (n_workers <= 1) {
        worker(0);
    } else {
        std::vector<std::thread> th;
        for (int w = 0; w < n_workers; w++) th.emplace_back(worker, w);
        for (auto& t : th) t.join();
    }
    if (done != n_batches) {
        (void)alive;
        throw std::runtime_error(first_error.empty() ? "batch scheduler: batches left unprocessed" : first_error);
    }
}

}  // namespace w2v
