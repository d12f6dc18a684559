// Error state, version and device queries of the openquant_b200 C ABI.
#include "oq_common.cuh"

#include <mutex>

namespace oq {

namespace {
thread_local std::string g_last_error;

void vset(const char *fmt, va_list ap) {
    char buf[1024];
    vsnprintf(buf, sizeof(buf), fmt, ap);
    g_last_error = buf;
}
}  // namespace

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
}

void clear_error() { g_last_error.clear(); }

int invalid(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
    return OQ_ERR_INVALID;
}

int check_launch(const char *what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

int sm_count() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace oq

extern "C" const char *oq_version(void) { return "openquant_b200 0.1.0 sm_100a"; }

extern "C" const char *oq_last_error(void) { return oq::g_last_error.c_str(); }

extern "C" int oq_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    int count = 0;
    for (int d = 0; d < n; ++d) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) == cudaSuccess && major == 10)
            ++count;
    }
    return count;
}
