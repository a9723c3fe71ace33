// norm.cuh - RMS norm of f32 rows, the contract of the HIP executor's rvh_rms_norm
// (runtime/hip/rvhip.h:43, rvhip.hip:75-90) and the arithmetic of the CPU op (ops.rs:131-139):
//
//     mean  = (f32)(sum_i (f64)x_i^2 / width)
//     scale = 1 / sqrt(mean + eps)                     (f32, correctly rounded)
//     out_i = x_i * scale [* post when post != 1] [* w_i]   (each product rounded)
//
// One warp per row: each lane sums its elements' squares in f64 (the squares of f32 values are
// exact in f64), the lanes' partial sums meet in a shuffle tree; the row is then read again
// (from L1/L2) to write the output. HBM-bound: 4 B read and 4 B written per element.
#pragma once
#include "common.cuh"

namespace rvc {

constexpr int NORM_WARPS = 8;  // rows per CTA

template <bool VEC>
__global__ void __launch_bounds__(NORM_WARPS * 32) k_rms_norm(const float *__restrict__ x, float *out,
                                                             const float *__restrict__ w, int rows, int width,
                                                             float eps, float post) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * NORM_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *xr = x + (size_t)row * width;
    float *o = out + (size_t)row * width;
    double s = 0.0;
    if (VEC) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        for (int i = lane; i < width / 4; i += 32) {
            const float4 v = x4[i];
            s += (double)v.x * (double)v.x;
            s += (double)v.y * (double)v.y;
            s += (double)v.z * (double)v.z;
            s += (double)v.w * (double)v.w;
        }
    } else {
        for (int i = lane; i < width; i += 32) s += (double)xr[i] * (double)xr[i];
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    const float mean = (float)(s / (double)width);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    const bool has_post = post != 1.0f;
    if (VEC) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        float4 *o4 = reinterpret_cast<float4 *>(o);
        for (int i = lane; i < width / 4; i += 32) {
            float4 v = x4[i];
            v.x = __fmul_rn(v.x, scale), v.y = __fmul_rn(v.y, scale);
            v.z = __fmul_rn(v.z, scale), v.w = __fmul_rn(v.w, scale);
            if (has_post) {
                v.x = __fmul_rn(v.x, post), v.y = __fmul_rn(v.y, post);
                v.z = __fmul_rn(v.z, post), v.w = __fmul_rn(v.w, post);
            }
            if (w) {
                const float4 g = w4[i];
                v.x = __fmul_rn(v.x, g.x), v.y = __fmul_rn(v.y, g.y);
                v.z = __fmul_rn(v.z, g.z), v.w = __fmul_rn(v.w, g.w);
            }
            o4[i] = v;
        }
    } else {
        for (int i = lane; i < width; i += 32) {
            float v = __fmul_rn(xr[i], scale);
            if (has_post) v = __fmul_rn(v, post);
            if (w) v = __fmul_rn(v, w[i]);
            o[i] = v;
        }
    }
}

}  // namespace rvc
