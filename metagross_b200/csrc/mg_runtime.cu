// Host-side runtime pieces of the C ABI: error text, version, device queries.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "mg_common.cuh"

namespace mg {

static thread_local char g_last_error[512] = "";

mg_status set_error(mg_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return s;
}

mg_status check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return MG_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace mg

extern "C" const char* mg_version(void) { return "metagross_b200 0.1.0 (sm_100a)"; }

extern "C" const char* mg_last_error(void) { return mg::g_last_error; }
