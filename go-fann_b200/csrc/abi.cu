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

int gofann_string_peq(const uint8_t* pattern, uint32_t length, uint32_t* peq_out)
{
    if ((!pattern && length) || !peq_out) return gofann::fail(GOFANN_ERR_INVALID, "string_peq: null argument");
    if (length > GOFANN_FUZZY_MAX_LENGTH)
        return gofann::fail(GOFANN_ERR_UNSUPPORTED, "string_peq: fuzzy pattern of %u bytes (at most %d)", length,
                            GOFANN_FUZZY_MAX_LENGTH);
    for (int c = 0; c < 128; ++c) peq_out[c] = 0u;
    for (uint32_t i = 0; i < length; ++i) {
        if (pattern[i] >= 128)
            return gofann::fail(GOFANN_ERR_UNSUPPORTED, "string_peq: fuzzy pattern byte %u at %u is not ASCII",
                                pattern[i], i);
        peq_out[pattern[i]] |= 1u << i;
    }
    return GOFANN_OK;
}

}  // extern "C"
