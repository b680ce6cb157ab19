// Shared helpers of the sm_100a decode-step kernels: error reporting at the C-ABI, streaming loads,
// warp reductions and F16 conversion.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "muyo_cuda.h"

namespace muyo {

// ---- errors at the ABI ---------------------------------------------------------------------------

void set_error(const char* fmt, ...);
void clear_error();

#define MUYO_REQUIRE(cond, ...)        \
    do {                               \
        if (!(cond)) {                 \
            ::muyo::set_error(__VA_ARGS__); \
            return MUYO_EINVAL;        \
        }                              \
    } while (0)

#define MUYO_CUDA_TRY(expr)                                                                     \
    do {                                                                                        \
        cudaError_t muyo_err_ = (expr);                                                         \
        if (muyo_err_ != cudaSuccess) {                                                         \
            ::muyo::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(muyo_err_), __FILE__, \
                              __LINE__);                                                        \
            return MUYO_ECUDA;                                                                  \
        }                                                                                       \
    } while (0)

// Checks the launch that was just issued (configuration errors are synchronous).
#define MUYO_LAUNCH_CHECK() MUYO_CUDA_TRY(cudaGetLastError())

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches kernel k; with pdl the launch carries the programmatic-stream-serialization attribute,
// so that (inside a captured graph) it may start while the kernel before it drains.
template <typename... Params, typename... Args>
inline cudaError_t launch_kernel(void (*k)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                                 Args... args)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// Number of SMs of the current device (cached per device).
int sm_count();

// ---- device helpers ------------------------------------------------------------------------------

constexpr int WARP = 32;

// 16-byte load of data read once per decode step (weights): no L1 allocation.
// Programmatic dependent launch. pdl_wait() returns once the grids this one depends on have
// completed and their writes are visible (at once when the kernel was launched without the
// programmatic-serialization attribute); pdl_trigger() lets the next kernel on the stream start
// launching. Kernels here call pdl_trigger() only after their own pdl_wait(), so a kernel's code
// before its wait may read anything written two or more kernels back, but nothing of the kernel
// right before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_stream16(const void* p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ld_stream16f(const void* p)
{
    uint4 r = ld_stream16(p);
    return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z), __uint_as_float(r.w));
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t bits)
{
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = bits;
    return __half22float2(h);
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// (value, index) pair with the greedy tie rule of src/Sampler.cpp:32-43: a larger value wins, an
// equal value with a lower index wins (the first index of the maximum). NaN never wins.
__device__ __forceinline__ bool pair_better(float v, int i, float bv, int bi)
{
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (pair_better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// Block-wide sum; `red` is shared scratch of at least 32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0)
        red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0)
        red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    return t;
}

// SiLU(g) * u as src/Swiglu.cpp:56 (g / (1 + exp(-g)) * u), IEEE division and CUDA's accurate expf.
__device__ __forceinline__ float silu_mul(float g, float u)
{
    return __fdiv_rn(g, 1.0f + expf(-g)) * u;
}

}  // namespace muyo
