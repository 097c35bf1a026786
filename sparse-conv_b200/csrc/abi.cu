// C-ABI plumbing shared by every entry point: version, per-thread error message, and
// the launch check that turns a failed CUDA launch into SPCONV_ERR_CUDA.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace spconv {

static thread_local char g_last_error[512] = "";
static std::atomic<uint64_t> g_wait_limit_ns{kWaitLimitNs};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
        return SPCONV_ERR_CUDA;
    }
    return SPCONV_OK;
}

// Stage timer: per stage, a pool of (start, end) event pairs recorded on the launch stream.
struct StageTimer {
    std::mutex mu;
    int cap = 0;
    std::vector<cudaEvent_t> ev[SPCONV_NUM_STAGES][2];
    int used[SPCONV_NUM_STAGES] = {0};

    void release() {
        for (int s = 0; s < SPCONV_NUM_STAGES; ++s) {
            for (int k = 0; k < 2; ++k) {
                for (cudaEvent_t e : ev[s][k]) cudaEventDestroy(e);
                ev[s][k].clear();
            }
            used[s] = 0;
        }
        cap = 0;
    }
};
static StageTimer g_timer;

void stage_mark(int stage, int which, cudaStream_t stream) {
    if (g_timer.cap == 0) return;
    std::lock_guard<std::mutex> lk(g_timer.mu);
    if (g_timer.cap == 0 || g_timer.used[stage] >= g_timer.cap) return;
    cudaEventRecord(g_timer.ev[stage][which][g_timer.used[stage]], stream);
    if (which == 1) g_timer.used[stage]++;
}

}  // namespace spconv

extern "C" int spconv_stage_timing(int max_calls) {
    using namespace spconv;
    std::lock_guard<std::mutex> lk(g_timer.mu);
    g_timer.release();
    if (max_calls <= 0) return SPCONV_OK;
    for (int s = 0; s < SPCONV_NUM_STAGES; ++s)
        for (int k = 0; k < 2; ++k) {
            g_timer.ev[s][k].resize(max_calls);
            for (int i = 0; i < max_calls; ++i) {
                if (cudaEventCreate(&g_timer.ev[s][k][i]) != cudaSuccess) {
                    g_timer.ev[s][k].resize(i);
                    g_timer.release();
                    return check_launch("cudaEventCreate");
                }
            }
        }
    g_timer.cap = max_calls;
    return SPCONV_OK;
}

extern "C" int spconv_stage_times_ms(double *total_ms, int64_t *launches, int n) {
    using namespace spconv;
    std::lock_guard<std::mutex> lk(g_timer.mu);
    if (n > SPCONV_NUM_STAGES) n = SPCONV_NUM_STAGES;
    for (int s = 0; s < n; ++s) {
        double sum = 0.0;
        for (int i = 0; i < g_timer.used[s]; ++i) {
            float ms = 0.0f;
            if (cudaEventSynchronize(g_timer.ev[s][1][i]) != cudaSuccess ||
                cudaEventElapsedTime(&ms, g_timer.ev[s][0][i], g_timer.ev[s][1][i]) != cudaSuccess) {
                check_launch("stage timing");
                return -1;
            }
            sum += ms;
        }
        if (total_ms) total_ms[s] = sum;
        if (launches) launches[s] = g_timer.used[s];
    }
    return n;
}

extern "C" int spconv_abi_version(void) { return SPCONV_ABI_VERSION; }

extern "C" uint64_t spconv_set_wait_limit_ns(uint64_t limit_ns) {
    const uint64_t v = limit_ns == 0 ? spconv::kWaitLimitNs : limit_ns;
    return spconv::g_wait_limit_ns.exchange(v);
}

extern "C" const char *spconv_last_error(void) { return spconv::g_last_error; }
