// Library runtime: per-thread error message, device selection, SM count, version.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace muyo {

static thread_local char t_error[512] = "";

void set_error(const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(t_error, sizeof(t_error), fmt, ap);
    va_end(ap);
}

void clear_error() { t_error[0] = '\0'; }

int sm_count()
{
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace muyo

extern "C" const char* muyo_cuda_last_error(void) { return muyo::t_error; }

extern "C" const char* muyo_cuda_version(void) { return "muyo_cuda 0.1.0 sm_100a"; }

extern "C" int muyo_cuda_init(int device)
{
    muyo::clear_error();
    MUYO_REQUIRE(device >= 0, "init: device %d is negative", device);
    int n = 0;
    MUYO_CUDA_TRY(cudaGetDeviceCount(&n));
    MUYO_REQUIRE(device < n, "init: device %d of %d", device, n);
    MUYO_CUDA_TRY(cudaSetDevice(device));
    MUYO_CUDA_TRY(cudaFree(nullptr));  // create the primary context now, not inside a timed region
    int major = 0, minor = 0;
    MUYO_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    MUYO_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0) {
        muyo::set_error("init: device %d is sm_%d%d; this library is built for sm_100a only", device, major, minor);
        return MUYO_EUNSUPPORTED;
    }
    return MUYO_OK;
}

extern "C" int muyo_cuda_shutdown(void)
{
    muyo::clear_error();
    MUYO_CUDA_TRY(cudaDeviceSynchronize());
    return MUYO_OK;
}
