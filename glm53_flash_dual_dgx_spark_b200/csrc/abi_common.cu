// Library-wide C-ABI entry points (version, last error) and host helpers.
#include "abi_common.h"

#include <mutex>
#include <string>

namespace nvfp4kv {

namespace {
thread_local std::string g_last_error;
thread_local cudaEvent_t g_ev_start = nullptr, g_ev_stop = nullptr;
std::mutex g_sm_mutex;
int g_sm_count[64] = {0};
}  // namespace

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(NVFP4KV_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return NVFP4KV_OK;
}

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lk(g_sm_mutex);
    if (g_sm_count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

void take_kernel_events(cudaEvent_t* start, cudaEvent_t* stop) {
    *start = g_ev_start;
    *stop = g_ev_stop;
    g_ev_start = g_ev_stop = nullptr;
}

}  // namespace nvfp4kv

extern "C" int nvfp4kv_version(void) { return 100; }

extern "C" int nvfp4kv_set_kernel_events(void* start, void* stop) {
    if ((start == nullptr) != (stop == nullptr))
        return nvfp4kv::fail(NVFP4KV_EINVAL, "set_kernel_events: give both events or neither");
    nvfp4kv::g_ev_start = static_cast<cudaEvent_t>(start);
    nvfp4kv::g_ev_stop = static_cast<cudaEvent_t>(stop);
    return NVFP4KV_OK;
}

extern "C" const char* nvfp4kv_last_error(void) { return nvfp4kv::g_last_error.c_str(); }
