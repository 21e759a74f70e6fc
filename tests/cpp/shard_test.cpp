// CPU test driver for the batch planner and the fault-tolerant scheduler
// (wav2vec2.cpp_b200/csrc/shard.hpp).  Prints one JSON object per scenario.
#include <atomic>
#include <chrono>
#include <cstdio>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "shard.hpp"

using namespace w2v;

static void plan(int n_utt, int max_batch, long long max_padded, unsigned seed) {
    std::vector<int> n(n_utt);
    unsigned x = seed;
    for (auto& v : n) { x = x * 1103515245u + 12345u; v = 32000 + (int)((x >> 8) % 448000); }
    auto b = make_batches(n.data(), n_utt, max_batch, max_padded);
    printf("{\"scenario\":\"plan\",\"n\":[");
    for (int i = 0; i < n_utt; i++) printf("%s%d", i ? "," : "", n[i]);
    printf("],\"batches\":[");
    for (size_t i = 0; i < b.size(); i++) {
        printf("%s[", i ? "," : "");
        for (size_t j = 0; j < b[i].size(); j++) printf("%s%d", j ? "," : "", b[i][j]);
        printf("]");
    }
    printf("]}\n");
}

static void sched(int n_batches, int n_workers, int fail_worker, int fail_after) {
    std::mutex mu;
    std::vector<int> owner(n_batches, -1), runs(n_batches, 0);
    std::vector<int> calls(n_workers, 0);
    bool threw = false;
    std::string msg;
    try {
        run_batches(n_batches, n_workers, [&](int w, size_t b, std::string& err) {
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
            std::lock_guard<std::mutex> lk(mu);
            runs[b]++;
            if ((w == fail_worker || fail_worker == -2) && calls[w]++ >= fail_after) {
                err = "injected failure";
                return false;
            }
            owner[b] = w;
            return true;
        });
    } catch (const std::exception& e) {
        threw = true;
        msg = e.what();
    }
    printf("{\"scenario\":\"sched\",\"threw\":%s,\"msg\":\"%s\",\"owner\":[", threw ? "true" : "false", msg.c_str());
    for (int i = 0; i < n_batches; i++) printf("%s%d", i ? "," : "", owner[i]);
    printf("],\"runs\":[");
    for (int i = 0; i < n_batches; i++) printf("%s%d", i ? "," : "", runs[i]);
    printf("]}\n");
}

int main() {
    plan(300, 64, 64LL * 16000 * 32, 1);
    plan(10, 4, 4LL * 16000 * 32, 2);
    plan(0, 64, 64LL * 16000 * 32, 3);
    sched(40, 4, -1, 0);      // no failure
    sched(40, 4, 2, 1);       // worker 2 fails on its second batch -> re-queued
    sched(40, 3, -2, 0);      // every worker fails -> error
    sched(7, 1, -1, 0);       // single worker
    return 0;
}
