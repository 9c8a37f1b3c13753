// elementwise.cuh -- embedding gather, residual add, bf16->f16 conversion,
// SiLU*mul and greedy argmax.  All are HBM-bound copies/maps: 16-byte
// vector loads and stores on the aligned fast path, a scalar path for odd
// widths or unaligned views.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

// ---------------------------------------------------------------- embedding gather
// One warp per output row; lanes copy 16-byte chunks.  Reference kernel:
// engine/kernels/embedding.cu:3-10 (2-byte copies, one CTA per row).
__global__ void __launch_bounds__(128) embedding_gather_vec_kernel(
    const int32_t* __restrict__ ids, const uint4* __restrict__ table, uint4* __restrict__ out,
    int t, int chunks_per_row, int vocab) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= t) return;
    const int id = ids[row];
    uint4* dst = out + (size_t)row * chunks_per_row;
    if (id < 0 || id >= vocab) {
        for (int c = lane; c < chunks_per_row; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint4* src = table + (size_t)id * chunks_per_row;
#pragma unroll 4
    for (int c = lane; c < chunks_per_row; c += 32) dst[c] = src[c];
}

__global__ void embedding_gather_scalar_kernel(const int32_t* __restrict__ ids,
                                               const uint16_t* __restrict__ table,
                                               uint16_t* __restrict__ out, int hidden, int vocab) {
    const int row = blockIdx.x;
    const int id = ids[row];
    uint16_t* dst = out + (size_t)row * hidden;
    const bool ok = id >= 0 && id < vocab;
    const uint16_t* src = table + (size_t)(ok ? id : 0) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = ok ? src[i] : (uint16_t)0;
}

// ---------------------------------------------------------------- residual add
// x[i] = round(x[i] + y[i]).  Reference: engine/kernels/elementwise.cu:4-9.
template <typename T>
__global__ void add_vec_kernel(uint4* __restrict__ x, const uint4* __restrict__ y, size_t nvec) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
         i += (size_t)gridDim.x * blockDim.x) {
        float a[8], b[8];
        unpack8<T>(x[i], a);
        unpack8<T>(y[i], b);
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] += b[k];
        x[i] = pack8<T>(a);
    }
}
template <typename T>
__global__ void add_scalar_kernel(T* __restrict__ x, const T* __restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        x[i] = Elem<T>::from_f(Elem<T>::to_f(x[i]) + Elem<T>::to_f(y[i]));
}

// ---------------------------------------------------------------- bf16 -> f16
// Reference: engine/kernels/elementwise.cu:11-20 (one atomic per bad value);
// here one atomic per warp.
__global__ void bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ in, __half* __restrict__ out,
                                   size_t n, uint32_t* __restrict__ bad) {
    uint32_t cnt = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = __bfloat162float(in[i]);
        if (!(fabsf(v) <= 65504.f)) ++cnt;
        out[i] = __float2half_rn(v);
    }
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(bad, cnt);
}

// ---------------------------------------------------------------- SiLU * mul
// out[r, i] = g / (1 + exp(-g)) * u with g = gu[r, i], u = gu[r, inter + i].
// Reference: engine/kernels/silu_mul.cu:3-12 (64-bit div/mod per element);
// here a 2-D grid (column chunk, row) and 8 elements per thread.
__device__ __forceinline__ float silu_mul_f(float g, float u) { return g / (1.0f + __expf(-g)) * u; }

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(const uint4* __restrict__ gu,
                                                           uint4* __restrict__ out,
                                                           int chunks /* inter/8 */, int rows) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= chunks) return;
    for (size_t r = blockIdx.y; r < (size_t)rows; r += gridDim.y) {
        const uint4 gv = ld_stream(gu + r * 2 * chunks + c);
        const uint4 uv = ld_stream(gu + r * 2 * chunks + chunks + c);
        float g[8], u[8];
        unpack8<T>(gv, g);
        unpack8<T>(uv, u);
#pragma unroll
        for (int k = 0; k < 8; ++k) g[k] = silu_mul_f(g[k], u[k]);
        st_stream(out + r * chunks + c, pack8<T>(g));
    }
}
template <typename T>
__global__ void silu_mul_scalar_kernel(const T* __restrict__ gu, T* __restrict__ out, int inter,
                                       int rows) {
    for (size_t r = blockIdx.y; r < (size_t)rows; r += gridDim.y)
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < inter; i += gridDim.x * blockDim.x) {
            const float g = Elem<T>::to_f(gu[r * 2 * inter + i]);
            const float u = Elem<T>::to_f(gu[r * 2 * inter + inter + i]);
            out[r * inter + i] = Elem<T>::from_f(silu_mul_f(g, u));
        }
}

// ---------------------------------------------------------------- greedy argmax
// First index of the row's maximum; NaN and -inf never win, so a row with no
// value above -inf gives 0 (the CPU reference's scan: strict > from -inf, index 0).
// The merge is a maximum over (value descending, index ascending), so the order in
// which partials meet does not change the result.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i && v2 > -INFINITY)) {
        v = v2;
        i = i2;
    }
}
__device__ __forceinline__ void argmax_warp(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        argmax_merge(v, i, v2, i2);
    }
}

// One 8-CTA cluster per row: CTA r scans the row's r-th contiguous slice (`slice`
// elements, a multiple of 4) with kArgmaxUnroll independent loads in flight per
// thread, and CTA 0 merges the eight partials through distributed shared memory.
// A 128,256-token row is 64 KB per SM, one batch of loads (one CTA per row kept a
// single SM's loads waiting on L2 latency ~60 times in a row).
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxUnroll = 8;
__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const float* __restrict__ logits, int vocab, int slice,
                  int32_t* __restrict__ ids, int32_t* __restrict__ adv,
                  int32_t* __restrict__ adv2, int vec4) {
    const uint32_t rank = cluster_rank();
    const size_t row = blockIdx.x / kArgmaxCluster;
    const float* l = logits + row * (size_t)vocab;
    const int lo = (int)min((int64_t)vocab, (int64_t)rank * slice);
    const int hi = (int)min((int64_t)vocab, (int64_t)lo + slice);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if (vec4) {  // vocab and slice are multiples of 4, the row 16-byte aligned
        const float4* l4 = reinterpret_cast<const float4*>(l);
        const int hi4 = hi / 4;
        for (int c0 = lo / 4 + (int)threadIdx.x; c0 < hi4; c0 += kArgmaxThreads * kArgmaxUnroll) {
            float4 v[kArgmaxUnroll];
#pragma unroll
            for (int u = 0; u < kArgmaxUnroll; ++u) {
                const int c = c0 + u * kArgmaxThreads;
                if (c < hi4) v[u] = l4[c];
            }
#pragma unroll
            for (int u = 0; u < kArgmaxUnroll; ++u) {
                const int c = c0 + u * kArgmaxThreads;
                if (c < hi4) {
                    argmax_merge(best, bi, v[u].x, 4 * c);
                    argmax_merge(best, bi, v[u].y, 4 * c + 1);
                    argmax_merge(best, bi, v[u].z, 4 * c + 2);
                    argmax_merge(best, bi, v[u].w, 4 * c + 3);
                }
            }
        }
    } else {
        for (int c = lo + (int)threadIdx.x; c < hi; c += kArgmaxThreads) argmax_merge(best, bi, l[c], c);
    }
    argmax_warp(best, bi);
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    __shared__ float part_v;  // this CTA's partial, read by CTA 0 of the cluster
    __shared__ int part_i;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        best = lane < kArgmaxThreads / 32 ? sv[lane] : -INFINITY;
        bi = lane < kArgmaxThreads / 32 ? si[lane] : 0x7fffffff;
        argmax_warp(best, bi);
        if (lane == 0) {
            part_v = best;
            part_i = bi;
        }
    }
    cluster_sync();  // every CTA's partial is written
    if (rank == 0 && warp == 0) {
        best = lane < kArgmaxCluster ? dsmem_ld(&part_v, lane) : -INFINITY;
        bi = lane < kArgmaxCluster ? dsmem_ld(&part_i, lane) : 0x7fffffff;
        argmax_warp(best, bi);
        if (lane == 0) {
            ids[row] = bi == 0x7fffffff ? 0 : bi;  // all -inf / NaN rows give index 0
            if (adv) adv[row] += 1;
            if (adv2) adv2[row] += 1;
        }
    }
    cluster_sync();  // no CTA leaves while CTA 0 may still read its partial
}

}  // namespace kvb
