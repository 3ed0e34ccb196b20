// api.cu -- status plumbing shared by every k3c_* entry point.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace k3c {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_err[0] = 0; }

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Event pairs per stage, recorded only while timing is enabled.
struct StageTimer {
    std::mutex mu;
    bool on = false;
    std::vector<cudaEvent_t> pending[STAGE_N];  // begin,end,begin,end...
    double ms[STAGE_N] = {};
    long long n[STAGE_N] = {};
};
static StageTimer g_timer;

static void record(int stage, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_timer.mu);
    if (!g_timer.on || stage < 0 || stage >= STAGE_N) return;
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    cudaEventRecord(e, s);
    g_timer.pending[stage].push_back(e);
}
void stage_begin(int stage, cudaStream_t s) { record(stage, s); }
void stage_end(int stage, cudaStream_t s) { record(stage, s); }

}  // namespace k3c

extern "C" const char *k3c_last_error(void) { return k3c::g_err; }

extern "C" const char *k3c_version(void) { return "k3c 0.1 sm_100a"; }

extern "C" long long k3c_launch_count(void) { return k3c::g_launches.load(); }

extern "C" void k3c_timing_enable(int on) {
    std::lock_guard<std::mutex> lk(k3c::g_timer.mu);
    k3c::g_timer.on = on != 0;
}

extern "C" int k3c_timing_read(double *ms, long long *count, int nstage) {
    using namespace k3c;
    std::lock_guard<std::mutex> lk(g_timer.mu);
    for (int st = 0; st < STAGE_N; st++) {
        auto &v = g_timer.pending[st];
        for (size_t i = 0; i + 1 < v.size(); i += 2) {
            float t = 0.f;
            if (cudaEventSynchronize(v[i + 1]) != cudaSuccess ||
                cudaEventElapsedTime(&t, v[i], v[i + 1]) != cudaSuccess)
                return set_error(K3C_ECUDA, "timing: event query failed");
            g_timer.ms[st] += t;
            g_timer.n[st] += 1;
        }
        for (auto e : v) cudaEventDestroy(e);
        v.clear();
    }
    for (int st = 0; st < nstage && st < STAGE_N; st++) {
        if (ms) ms[st] = g_timer.ms[st];
        if (count) count[st] = g_timer.n[st];
        g_timer.ms[st] = 0;
        g_timer.n[st] = 0;
    }
    return K3C_OK;
}
