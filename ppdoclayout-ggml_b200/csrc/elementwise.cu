// elementwise.cu — bias + activation (op 5) and contiguous copy (op 6).
//
// Reference: ppdl_bias_act_kernel (patches/ggml-ppdl.patch:417-432) and
// ppdl_copy_kernel (:434-438).  Grid-stride loops sized to the SM count, with
// 16-byte accesses when the pointers and the plane size allow it.
#include "common.cuh"
#include "kernels.h"

namespace ppdl {

namespace {

__global__ void bias_act_kernel(const float *__restrict__ x, const float *__restrict__ bias,
                                float *__restrict__ y, long long n, long long plane, int C,
                                int act) {
    pdl_begin();
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float v = x[i];
        if (bias) v = __fadd_rn(v, bias[(i / plane) % C]);
        y[i] = act_apply(v, act);
    }
}

__global__ void bias_act_kernel_v4(const float4 *__restrict__ x, const float *__restrict__ bias,
                                   float4 *__restrict__ y, long long n4, long long plane4, int C,
                                   int act) {
    pdl_begin();
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 v = x[i];
        if (bias) {
            const float b = bias[(i / plane4) % C];
            v.x = __fadd_rn(v.x, b); v.y = __fadd_rn(v.y, b);
            v.z = __fadd_rn(v.z, b); v.w = __fadd_rn(v.w, b);
        }
        v.x = act_apply(v.x, act); v.y = act_apply(v.y, act);
        v.z = act_apply(v.z, act); v.w = act_apply(v.w, act);
        y[i] = v;
    }
}

__global__ void copy_kernel(const float4 *__restrict__ x, float4 *__restrict__ y, long long n4) {
    pdl_begin();
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
        y[i] = x[i];
}

__global__ void copy_kernel_tail(const float *__restrict__ x, float *__restrict__ y,
                                 long long from, long long n) {
    pdl_begin();
    const long long i = from + (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = x[i];
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace

Status launch_bias_act(const float *x, const float *bias, float *y, long long n, long long plane,
                       int C, int act, cudaStream_t stream) {
    if (n < 0 || plane <= 0 || C <= 0) return ERR_SHAPE;
    if (n == 0) return OK;
    const int grid_cap = sm_count() * 8;
    if (((uintptr_t)x | (uintptr_t)y) % 16 == 0 && plane % 4 == 0) {
        const long long n4 = n / 4;
        const int grid = (int)(cdiv(n4, 256) < grid_cap ? cdiv(n4, 256) : grid_cap);
        pdl_launch(bias_act_kernel_v4, grid, 256, 0, stream, (const float4 *)x, bias, (float4 *)y,
                   n4, plane / 4, C, act);
    } else {
        const int grid = (int)(cdiv(n, 256) < grid_cap ? cdiv(n, 256) : grid_cap);
        pdl_launch(bias_act_kernel, grid, 256, 0, stream, x, bias, y, n, plane, C, act);
    }
    return cuda_status();
}

Status launch_copy(const float *x, float *y, long long n, cudaStream_t stream) {
    if (n < 0) return ERR_SHAPE;
    if (n == 0) return OK;
    long long done = 0;
    if (((uintptr_t)x | (uintptr_t)y) % 16 == 0) {
        const long long n4 = n / 4;
        if (n4) {
            const int grid_cap = sm_count() * 8;
            const int grid = (int)(cdiv(n4, 256) < grid_cap ? cdiv(n4, 256) : grid_cap);
            pdl_launch(copy_kernel, grid, 256, 0, stream, (const float4 *)x, (float4 *)y, n4);
        }
        done = n4 * 4;
    }
    if (done < n) pdl_launch(copy_kernel_tail, cdiv(n - done, 256), 256, 0, stream, x, y, done, n);
    return cuda_status();
}

}  // namespace ppdl
