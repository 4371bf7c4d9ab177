// status.cu — status codes, per-thread error messages and small device
// queries behind the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <string>

#include "qc_common.cuh"

namespace qc {

namespace {
thread_local std::string g_last_error;

std::mutex g_sm_mutex;
int g_sm_cache[64] = {0};
}  // namespace

int set_error(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int check_cuda(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return 0;
    return set_error(static_cast<int>(err), "CUDA error in %s: %s (%s)", what,
                     cudaGetErrorName(err), cudaGetErrorString(err));
}

int device_sm_count(int *sms) {
    int dev = 0;
    QC_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 0 && dev < 64) {
        std::lock_guard<std::mutex> lock(g_sm_mutex);
        if (g_sm_cache[dev] > 0) {
            *sms = g_sm_cache[dev];
            return 0;
        }
    }
    int n = 0;
    QC_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev),
                "cudaDeviceGetAttribute(MultiProcessorCount)");
    if (dev >= 0 && dev < 64) {
        std::lock_guard<std::mutex> lock(g_sm_mutex);
        g_sm_cache[dev] = n;
    }
    *sms = n;
    return 0;
}

}  // namespace qc

extern "C" {

const char *quantem_cuda_last_error(void) { return qc::g_last_error.c_str(); }

const char *quantem_cuda_status_string(int status) {
    switch (status) {
        case QC_OK: return "QC_OK";
        case QC_ERR_INVALID_ARGUMENT: return "QC_ERR_INVALID_ARGUMENT";
        case QC_ERR_WORKSPACE_TOO_SMALL: return "QC_ERR_WORKSPACE_TOO_SMALL";
        case QC_ERR_NO_DEVICE: return "QC_ERR_NO_DEVICE";
        case QC_ERR_TENSOR_MAP: return "QC_ERR_TENSOR_MAP";
        default:
            if (status > 0 && status < 10000)
                return cudaGetErrorName(static_cast<cudaError_t>(status));
            return "QC_ERR_UNKNOWN";
    }
}

int quantem_cuda_cudart_version(void) { return CUDART_VERSION; }

}  // extern "C"
