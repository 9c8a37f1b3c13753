// norm.cuh -- RMSNorm and the fused residual-add + RMSNorm.
//
// Reference kernel: engine/kernels/rmsnorm.cu:3-17 (one CTA per row, two passes
// over global x with 2-byte loads).  Here every row is read from HBM once, in
// 16-byte pieces, and held in registers while its sum of squares is reduced.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

// Many rows: persistent CTAs (kNormBulkPerSm per SM), CTA c owning the
// contiguous rows [c*rows/grid, (c+1)*rows/grid).  One lane streams them into a
// shared-memory ring with bulk copies, kNormBulkWarps rows per stage (x, and y
// when the residual add is fused); consumer warp j normalises row j of each
// stage: the row is unpacked into registers, the sum of squares reduced with
// warp shuffles, and out = x * rsqrt(mean + eps) * w formed in f32 and rounded
// once -- the reference's arithmetic order ((x*inv)*w).  The ring keeps ~96 KB
// of every CTA's reads in flight whatever the per-row work, so the kernel runs
// at the speed of a device-to-device copy of the same bytes.
// NV = 16-byte chunks per lane (the row has chunks <= 32*NV of them).
constexpr int kNormBulkWarps = 4;
constexpr int kNormBulkThreads = 32 * (kNormBulkWarps + 1);
constexpr int kNormBulkPerSm = 2;
constexpr int kNormBulkRingBytes = 96 * 1024;

__host__ __device__ constexpr int norm_bulk_stage_bytes(int chunks, bool add) {
    return kNormBulkWarps * chunks * 16 * (add ? 2 : 1);
}
// Stages of the ring for a row width: as many as fit kNormBulkRingBytes, 2..12.
__host__ __device__ constexpr int norm_bulk_stages(int chunks, bool add) {
    return kNormBulkRingBytes / norm_bulk_stage_bytes(chunks, add) < 2 ? 2
           : kNormBulkRingBytes / norm_bulk_stage_bytes(chunks, add) > 12
               ? 12
               : kNormBulkRingBytes / norm_bulk_stage_bytes(chunks, add);
}
// Dynamic shared memory: 24 mbarriers (256 B), the weights, then the ring.
__host__ __device__ constexpr int norm_bulk_smem_bytes(int chunks, bool add) {
    return 256 + ((chunks * 16 + 127) & ~127) +
           norm_bulk_stages(chunks, add) * norm_bulk_stage_bytes(chunks, add);
}
// Upper bound of norm_bulk_smem_bytes over the widths one NV serves (chunks <= 32*NV).
__host__ __device__ constexpr int norm_bulk_smem_cap(int nv, bool add) {
    return 256 + 32 * nv * 16 +
           (2 * norm_bulk_stage_bytes(32 * nv, add) > kNormBulkRingBytes
                ? 2 * norm_bulk_stage_bytes(32 * nv, add)
                : kNormBulkRingBytes);
}

// kFull: chunks == 32*NV (every lane holds NV chunks; no per-chunk guards).
// Weights sit in registers for NV <= 8, in shared memory above that.
template <typename T, int NV, bool kAdd, bool kFull>
__global__ void __launch_bounds__(kNormBulkThreads) rmsnorm_bulk_kernel(
    uint4* __restrict__ x, const uint4* __restrict__ y, const uint4* __restrict__ w,
    uint4* __restrict__ out, int rows, int chunks_arg, float inv_hidden, float eps) {
    constexpr bool kWReg = NV <= 8;
    const int chunks = kFull ? 32 * NV : chunks_arg;
    extern __shared__ __align__(128) uint8_t norm_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(norm_smem);  // [12]
    uint64_t* empty = full + 12;                                 // [12]
    uint4* ws = reinterpret_cast<uint4*>(norm_smem + 256);
    // ring after the weights, 128-byte aligned
    uint8_t* ring = norm_smem + 256 + ((chunks * 16 + 127) & ~127);
    const int stages = norm_bulk_stages(chunks, kAdd);
    const int row_bytes = chunks * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (int)((long long)blockIdx.x * rows / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * rows / gridDim.x);
    const int groups = (r1 - r0 + kNormBulkWarps - 1) / kNormBulkWarps;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNormBulkWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == kNormBulkWarps) {  // producer
        if (lane != 0) return;
        int issued = 0;
        for (int g = 0; g < groups; ++g) {
            const int s = g % stages;
            if (g >= stages && !mbar_wait(&empty[s], ((g / stages) - 1) & 1)) break;
            const int row = r0 + g * kNormBulkWarps;
            const uint32_t n = (uint32_t)min(kNormBulkWarps, r1 - row) * row_bytes;
            uint8_t* dst = ring + (size_t)s * norm_bulk_stage_bytes(chunks, kAdd);
            mbar_expect_tx(&full[s], kAdd ? 2 * n : n);
            bulk_load(dst, x + (size_t)row * chunks, n, &full[s]);
            if (kAdd) bulk_load(dst + kNormBulkWarps * row_bytes, y + (size_t)row * chunks, n, &full[s]);
            ++issued;
        }
        // no copy may still be landing in this CTA's shared memory when it exits
        for (int g = max(0, issued - stages); g < issued; ++g)
            mbar_wait(&full[g % stages], (g / stages) & 1);
        return;
    }
    uint4 wr[kWReg ? NV : 1];
    if (kWReg) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int c = lane + 32 * k;
            if (kFull || c < chunks) wr[k] = w[c];
        }
    } else {
        for (int c = threadIdx.x; c < chunks; c += 32 * kNormBulkWarps) ws[c] = w[c];
        named_bar_sync(1, 32 * kNormBulkWarps);  // the consumer warps only
    }
    for (int g = 0; g < groups; ++g) {
        const int s = g % stages;
        if (!mbar_wait(&full[s], (g / stages) & 1)) return;
        const int row = r0 + g * kNormBulkWarps + warp;
        if (row < r1) {
            const uint8_t* st = ring + (size_t)s * norm_bulk_stage_bytes(chunks, kAdd);
            const uint4* xs = reinterpret_cast<const uint4*>(st + warp * row_bytes);
            const uint4* ys = reinterpret_cast<const uint4*>(st + (kNormBulkWarps + warp) * row_bytes);
            uint4* xg = x + (size_t)row * chunks;
            uint4* og = out + (size_t)row * chunks;
            float v[NV][8];
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                const int c = lane + 32 * k;
                if (kFull || c < chunks) {
                    unpack8<T>(xs[c], v[k]);
                    if (kAdd) {
                        float d[8];
                        unpack8<T>(ys[c], d);
#pragma unroll
                        for (int e = 0; e < 8; ++e) d[e] += v[k][e];
                        const uint4 r = pack8<T>(d);  // residual rounded to the activation type
                        xg[c] = r;
                        unpack8<T>(r, v[k]);
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // the row is in registers now
            ss = warp_sum(ss);
            const float inv = rsqrtf(ss * inv_hidden + eps);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                const int c = lane + 32 * k;
                if (kFull || c < chunks) {
                    float wf[8];
                    unpack8<T>(kWReg ? wr[kWReg ? k : 0] : ws[c], wf);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[k][e] = v[k][e] * inv * wf[e];
                    og[c] = pack8<T>(v[k]);
                }
            }
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
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
    // a projection launched as this grid's programmatic dependent may start streaming
    // its weights now; it reads this kernel's output only after the grid completes.
    // This kernel is itself launched that way: nothing is read before the preceding
    // kernel has completed.
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
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

// Embedding gather fused with the RMSNorm that follows it (the first norm of a
// decode step): x row r = table[ids[r]] (a zero row for an id outside the table,
// as embedding_gather_vec_kernel), out row r = RMSNorm(x row r) * w with the
// arithmetic of rmsnorm_row_kernel<T, false>, so x and out equal the two-launch
// form bit for bit.  One CTA per row, one 16-byte chunk per thread.
template <typename T>
__global__ void __launch_bounds__(1024) embedding_rmsnorm_row_kernel(
    const int32_t* __restrict__ ids, const uint4* __restrict__ table, const uint4* __restrict__ w,
    uint4* __restrict__ x, uint4* __restrict__ out, int chunks, int vocab, float inv_hidden,
    float eps) {
    __shared__ float red[32];
    asm volatile("griddepcontrol.launch_dependents;");  // as rmsnorm_row_kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t row = blockIdx.x;
    const int c = threadIdx.x;
    const int lane = c & 31, warp = c >> 5;
    const int id = ids[row];
    uint4 e = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab) e = table[(size_t)id * chunks + c];
    x[row * chunks + c] = e;
    float v[8], wf[8];
    unpack8<T>(e, v);
    unpack8<T>(w[c], wf);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
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
    for (int k = 0; k < 8; ++k) v[k] = v[k] * inv * wf[k];
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
