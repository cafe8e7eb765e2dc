// Error state of the C ABI: a per-thread message and the status strings.
#include "common.cuh"

#include <cstdarg>
#include <cstdio>

namespace l2k
{
namespace
{
thread_local char g_message[512] = "";
}

int set_error(int status, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_message, sizeof(g_message), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char *what)
{
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    return L2K_OK;
}

int num_sms()
{
    static int n = [] {
        int dev = 0, v = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
        {
            cudaGetLastError();
            return kNumSMs;
        }
        return v;
    }();
    return n;
}
} // namespace l2k

extern "C" const char *l2k_status_string(int status)
{
    switch (status)
    {
    case L2K_OK:
        return "ok";
    case L2K_ERR_INVALID_ARGUMENT:
        return "invalid argument";
    case L2K_ERR_UNSUPPORTED_DTYPE:
        return "unsupported dtype";
    case L2K_ERR_UNSUPPORTED_SHAPE:
        return "unsupported shape";
    case L2K_ERR_CUDA:
        return "CUDA error";
    default:
        return "unknown status";
    }
}

extern "C" const char *l2k_last_error_message(void) { return l2k::g_message; }

extern "C" int l2k_abi_version(void) { return 1; }
