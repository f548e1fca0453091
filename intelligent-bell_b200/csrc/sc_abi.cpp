// sc_abi.cpp — error reporting, version and small host utilities of the C ABI.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "sc_internal.h"

namespace sc {

namespace {
thread_local char g_last_error[512] = {0};

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
std::mutex g_attr_mutex;
}  // namespace

int32_t set_error(int32_t code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int32_t ok() {
    g_last_error[0] = '\0';
    return SC_OK;
}

int32_t cuda_error(cudaError_t e, const char* what) {
    return set_error(SC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < kMaxDevices) {
        std::lock_guard<std::mutex> lock(g_attr_mutex);
        if (g_sm_count[dev] == 0) {
            int n = 0;
            if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                n <= 0)
                n = 148;
            g_sm_count[dev] = n;
        }
        return g_sm_count[dev];
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    return n;
}

void default_inv_freq(int32_t head_dim, double theta, float* out) {
    for (int i = 0; i < head_dim / 2; ++i) {
        const float expo = (2.0f * static_cast<float>(i)) / static_cast<float>(head_dim);
        const float p = static_cast<float>(pow(theta, static_cast<double>(expo)));
        out[i] = 1.0f / p;
    }
}

}  // namespace sc

extern "C" {

const char* sc_last_error(void) { return sc::g_last_error; }

int32_t sc_abi_version(void) { return SC_ABI_VERSION; }

int32_t sc_preload_kernels(void) {
    cudaError_t e = sc::preload_dense_kernels();
    if (e == cudaSuccess) e = sc::preload_paged_kernels();
    if (e == cudaSuccess) e = sc::preload_quantize_kernels(true);
    if (e == cudaSuccess) e = sc::preload_shift_kernels();
    if (e != cudaSuccess) return sc::cuda_error(e, "loading the kernels");
    return sc::ok();
}

}  // extern "C"
