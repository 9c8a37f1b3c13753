// norm.cuh -- RMSNorm and the fused residual-add + RMSNorm.
//
// Reference kernel: engine/kernels/rmsnorm.cu:3-17 (one CTA per row, two passes
// over global x with 2-byte loads).  Here one warp owns a row: the row is read
// once with 16-byte loads into registers, the sum of squares is reduced with
// warp shuffles, and out = x * rsqrt(mean + eps) * w is formed in f32 and
// rounded once -- the same arithmetic order as the reference ((x*inv)*w).
#pragma once

#include "kvb_common.cuh"

namespace kvb {

// NV = 16-byte chunks held per lane; the row has hidden/8 <= 32*NV chunks.
template <typename T, int NV, bool kAdd>
__global__ void __launch_bounds__(128) rmsnorm_warp_kernel(uint4* __restrict__ x,
                                                           const uint4* __restrict__ y,
                                                           const uint4* __restrict__ w,
                                                           uint4* __restrict__ out, int rows,
                                                           int chunks, float inv_hidden,
                                                           float eps) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    uint4* xr = x + (size_t)row * chunks;
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int c = lane + 32 * k;
        if (c < chunks) {
            unpack8<T>(xr[c], v[k]);
            if (kAdd) {
                float d[8];
                unpack8<T>(y[(size_t)row * chunks + c], d);
#pragma unroll
                for (int e = 0; e < 8; ++e) d[e] += v[k][e];
                const uint4 s = pack8<T>(d);  // residual rounded to the activation type
                xr[c] = s;
                unpack8<T>(s, v[k]);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
        }
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss * inv_hidden + eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int c = lane + 32 * k;
        if (c < chunks) {
            float wf[8];
            unpack8<T>(w[c], wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[k][e] = v[k][e] * inv * wf[e];
            out[(size_t)row * chunks + c] = pack8<T>(v[k]);
        }
    }
}

// Few rows (decode batches): one CTA per row, one 16-byte chunk per thread
// (blockDim = hidden / 8), so a row's loads are all in flight at once.
template <typename T, bool kAdd>
__global__ void __launch_bounds__(1024) rmsnorm_row_kernel(uint4* __restrict__ x,
                                                          const uint4* __restrict__ y,
                                                          const uint4* __restrict__ w,
                                                          uint4* __restrict__ out, int chunks,
                                                          float inv_hidden, float eps) {
    __shared__ float red[32];
    const size_t row = blockIdx.x;
    const int c = threadIdx.x;
    const int lane = c & 31, warp = c >> 5;
    float v[8], wf[8];
    unpack8<T>(x[row * chunks + c], v);
    unpack8<T>(w[c], wf);
    if (kAdd) {
        float d[8];
        unpack8<T>(y[row * chunks + c], d);
#pragma unroll
        for (int e = 0; e < 8; ++e) d[e] += v[e];
        const uint4 s = pack8<T>(d);  // residual rounded to the activation type
        x[row * chunks + c] = s;
        unpack8<T>(s, v);
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float r = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
        r = warp_sum(r);
        if (lane == 0) red[0] = r;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] * inv_hidden + eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * wf[e];
    out[row * chunks + c] = pack8<T>(v);
}

// Any width, any alignment: one CTA per row, two passes over the row.
template <typename T, bool kAdd>
__global__ void __launch_bounds__(256) rmsnorm_generic_kernel(T* __restrict__ x,
                                                              const T* __restrict__ y,
                                                              const T* __restrict__ w,
                                                              T* __restrict__ out, int hidden,
                                                              float eps) {
    __shared__ float red[8];
    T* xr = x + (size_t)blockIdx.x * hidden;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = Elem<T>::to_f(xr[i]);
        if (kAdd) {
            const T s = Elem<T>::from_f(v + Elem<T>::to_f(y[(size_t)blockIdx.x * hidden + i]));
            xr[i] = s;
            v = Elem<T>::to_f(s);
        }
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        r = warp_sum(r);
        if (threadIdx.x == 0) red[0] = r;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x)
        out[(size_t)blockIdx.x * hidden + i] =
            Elem<T>::from_f(Elem<T>::to_f(xr[i]) * inv * Elem<T>::to_f(w[i]));
}

}  // namespace kvb
