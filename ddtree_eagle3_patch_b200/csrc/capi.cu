// Error reporting and device queries shared by the C-ABI entry points.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace ddt {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

// Kernels launched by this library since load (every launch goes through
// check_launch); read by ddt_launch_count().
static std::atomic<unsigned long long> g_launches{0};

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(DDT_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return DDT_OK;
}

// Programmatic dependent launch of the decode-layer kernels (ddt_set_pdl).
static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

unsigned pdl_attr(cudaLaunchAttribute* a) {
    if (!g_pdl.load(std::memory_order_relaxed)) return 0;
    a->id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a->val.programmaticStreamSerializationAllowed = 1;
    return 1;
}

}  // namespace ddt

extern "C" int ddt_set_pdl(int enabled) { return ddt::g_pdl.exchange(enabled ? 1 : 0); }

extern "C" const char* ddt_last_error(void) { return ddt::g_last_error; }

extern "C" int ddt_abi_version(void) { return 1; }

extern "C" uint64_t ddt_launch_count(void) { return ddt::g_launches.load(std::memory_order_relaxed); }

extern "C" int ddt_sm_count(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    if (device < 0 || device >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cache[device] = n;
    }
    return cache[device];
}
