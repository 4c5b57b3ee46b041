// Error reporting and device queries of the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "mb_common.cuh"

static thread_local char g_last_error[512] = "";

int mb_fail(int code, const char* fmt, ...)
{
    // a failed CUDA call also leaves its error as the thread's last error: it is
    // reported here, so clear it (the next call's launch check must not see it)
    if (code == MB_ECUDA) (void)cudaGetLastError();
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int mb_check_launch(const char* what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return MB_OK;
}

int mb_num_sms()
{
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

extern "C" const char* mb_last_error(void) { return g_last_error; }

extern "C" int mb_version(void) { return 1; }

extern "C" int mb_device_check(void)
{
    int dev = 0, major = 0, minor = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
        return mb_fail(MB_EUNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                       minor);
    return MB_OK;
}
