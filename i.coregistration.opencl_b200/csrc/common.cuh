// SPDX-License-Identifier: Unlicense
//
// Shared helpers of the CUDA sources: error reporting (fatal or recorded,
// see ocl_backend.h), activation functions with the reference's
// definitions (ops.cl:23-37), element load/store for float and bfloat16
// storage, and the per-launch profiler behind ops_report.

#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "ocl_backend.h"
#include "ops.h"

struct _cl_mem {
    void *ptr;
    size_t bytes;
    int owned;
};

namespace coreg {

// Report an error: fatal (exit 1) or recorded for coreg_last_error.
void fail(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
// True while an error is recorded on this thread (entry points return).
bool pending();
// Fail on a CUDA error, naming what.
bool cuda_ok(cudaError_t e, const char *what);
// Fail with the launch error of the last kernel, if any.
bool launch_ok(const char *what);

// The current backend of the thread's last ops_init / model call, for the
// profiler.
struct Prof {
    const char *what;
    cudaStream_t st;
    cudaEvent_t e0, e1;
    bool on;
    Prof(const struct ocl_backend *ocl, const char *what);
    ~Prof();
};

inline cudaStream_t stream_of(const struct ocl_backend *ocl)
{
    return (cudaStream_t)ocl->queue;
}

inline float *fptr(cl_mem m, long off = 0)
{
    return m ? (float *)m->ptr + off : nullptr;
}

inline unsigned cdiv(long a, long b) { return (unsigned)((a + b - 1) / b); }

// Element counts passed as int to kernels (the reference's count(),
// ops.c:79-84).
bool count_ok(long n, const char *what);

}  // namespace coreg

// ---------------------------------------------------------------- device

#define ACTF_NONE 0
#define ACTF_GELU 1
#define ACTF_RELU 2
#define ACTF_LEAKY 3
#define ACTF_GELU_TANH 4

__device__ __forceinline__ float apply_act(float v, int act, float slope)
{
    switch (act) {
    case ACTF_GELU:
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    case ACTF_RELU:
        return fmaxf(v, 0.0f);
    case ACTF_LEAKY:
        return v >= 0.0f ? v : slope * v;
    case ACTF_GELU_TANH:
        return 0.5f * v *
               (1.0f + tanhf(0.79788456080286536f * (v + 0.044715f * v * v * v)));
    }
    return v;
}

__device__ __forceinline__ float ldf(const float *p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16 *p)
{
    return __bfloat162float(*p);
}
__device__ __forceinline__ void stf(float *p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16 *p, float v)
{
    *p = __float2bfloat16_rn(v);
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

// Sum over a block of blockDim.x threads (a multiple of 32, <= 1024);
// every thread gets the result. red: 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float *red)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0)
        red[wid] = v;
    __syncthreads();
    v = lane < nw ? red[lane] : 0.0f;
    return warp_sum(v);
}

__device__ __forceinline__ float block_max(float v, float *red)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0)
        red[wid] = v;
    __syncthreads();
    v = lane < nw ? red[lane] : -INFINITY;
    return warp_max(v);
}
