// Launch counter and event-pair profiler (host side only).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "prof.cuh"

namespace altxs {
namespace {

std::atomic<int64_t> g_launches{0};
std::atomic<uint32_t> g_mask{0xffffffffu};  // kernel classes recorded while profiling

struct Profiler {
    std::mutex mu;
    bool on = false;
    std::vector<cudaEvent_t> ev;  // pairs
    std::vector<int> cls;
    size_t used = 0;
    int pending_cls = -1;
};
Profiler g_prof;
constexpr size_t kMaxPairs = 16384;

}  // namespace

void prof_begin(cudaStream_t s, int c) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!g_prof.on || c < 0 || c > 31 || !((g_mask.load(std::memory_order_relaxed) >> c) & 1u)) return;
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (g_prof.used >= g_prof.cls.size()) {
        g_prof.pending_cls = -1;
        return;
    }
    cudaEventRecord(g_prof.ev[2 * g_prof.used], s);
    g_prof.pending_cls = c;
}

void prof_end(cudaStream_t s) {
    if (!g_prof.on) return;
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (g_prof.pending_cls < 0) return;
    cudaEventRecord(g_prof.ev[2 * g_prof.used + 1], s);
    g_prof.cls[g_prof.used] = g_prof.pending_cls;
    g_prof.used++;
    g_prof.pending_cls = -1;
}

}  // namespace altxs

using namespace altxs;

namespace altxs {
namespace {
thread_local int g_last_cuda_error = 0;
}
void note_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
}  // namespace altxs

extern "C" {

int altxs_last_cuda_error(void) { return altxs::g_last_cuda_error; }

int64_t altxs_launch_count(void) { return g_launches.load(); }

int altxs_profile(int enable) {
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (enable) {
        if (g_prof.ev.empty()) {
            g_prof.ev.resize(2 * kMaxPairs);
            g_prof.cls.resize(kMaxPairs);
            for (auto &e : g_prof.ev)
                if (cudaEventCreate(&e) != cudaSuccess) return ALTXS_ECUDA;
        }
        g_prof.used = 0;
        g_prof.pending_cls = -1;
        g_prof.on = true;
    } else {
        g_prof.on = false;
    }
    return ALTXS_OK;
}

int altxs_profile_mask(uint32_t mask) {
    g_mask.store(mask);
    return ALTXS_OK;
}

int altxs_profile_read(int n_classes, double *ms, int64_t *counts) {
    if (n_classes < 0 || (n_classes > 0 && (!ms || !counts))) return ALTXS_EINVAL;
    std::lock_guard<std::mutex> lk(g_prof.mu);
    for (int c = 0; c < n_classes; ++c) {
        ms[c] = 0.0;
        counts[c] = 0;
    }
    for (size_t i = 0; i < g_prof.used; ++i) {
        if (cudaEventSynchronize(g_prof.ev[2 * i + 1]) != cudaSuccess) return ALTXS_ECUDA;
        float t = 0.f;
        if (cudaEventElapsedTime(&t, g_prof.ev[2 * i], g_prof.ev[2 * i + 1]) != cudaSuccess) return ALTXS_ECUDA;
        const int c = g_prof.cls[i];
        if (c >= 0 && c < n_classes) {
            ms[c] += t;
            counts[c] += 1;
        }
    }
    return (int)g_prof.used;
}

}  // extern "C"
