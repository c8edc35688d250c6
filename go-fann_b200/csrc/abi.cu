// abi.cu — host-side plumbing shared by every C-ABI entry point: the
// per-thread last-error string and CUDA status mapping.
#include <cstdarg>
#include <cstring>

#include "common.cuh"

namespace gofann {

namespace {
thread_local char g_last_error[512] = "";
}

void set_error(const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int fail(int status, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int cuda_status(cudaError_t err, const char* what)
{
    set_error("%s: %s", what, cudaGetErrorString(err));
    return GOFANN_ERR_CUDA;
}

int sm_count()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return n;
}

size_t l2_bytes()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrL2CacheSize, dev) != cudaSuccess) return 0;
    return static_cast<size_t>(n);
}

}  // namespace gofann

extern "C" {

int gofann_abi_version(void) { return GOFANN_ABI_VERSION; }

const char* gofann_last_error(void) { return gofann::g_last_error; }

int gofann_device_sm_count(void) { return gofann::sm_count(); }

}  // extern "C"
