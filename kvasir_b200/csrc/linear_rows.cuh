// linear_rows.cuh -- the projections of decode-sized batches on the tensor
// cores: Y[r, o] = sum_k X[r, k] W[o, k] for up to 128 rows.
//
// This is the reference's gemm_nt / linear_f16 (engine/src/gpu/gemm.rs:17-88, one
// cublasGemmEx call) at the shapes a decode step has: a few rows of X against a
// weight matrix of millions of elements.  The product is then a stream of W from
// HBM (rows * 2 flops per weight byte), and the kernel is built to keep that
// stream running from the first cycle to the last:
//   * one CTA per (128-row tile of W, slice of the K dimension), one wave over
//     the SMs.  The `splits` CTAs of a tile form a thread-block cluster.  Each
//     owns 1/splits of the output tile and reads the others' partial sums of
//     those outputs from their shared memory (distributed shared memory, all
//     loads in flight at once), adding the slices in slice order, so the result
//     does not depend on timing;
//   * warp 4 streams W in 16 KB chunks (128 rows x 64 elements, 128-byte
//     swizzle) together with the matching 64-column chunk of X through a ring of
//     stages (TMA, no multicast); warp 5 issues tcgen05.mma kind::f16 (M = 128
//     rows of W, N = the row count padded to 16/32/64/128, f32 accumulator in
//     TMEM); warps 0-3 move the accumulator to shared memory, one TMEM lane (W
//     row) per thread;
//   * the launch is a programmatic dependent of the kernel before it: the W
//     chunks of the first stages are requested before griddepcontrol.wait, since
//     W does not depend on that kernel; X is loaded, and Y written, after it.
// kGlu: the gate/up projection fused with SiLU*mul.  A tile holds 64 gate rows
// of W_gu and the 64 up rows of the same outputs (rows j and inter + j).  The
// reduced G and U are rounded to the 16-bit type and combined with the
// arithmetic of silu_mul_vec_kernel, so the output is what the projection
// followed by kvb_silu_mul gives for the same G and U; the [rows, 2 * inter]
// intermediate is never written.
//
// Every mbarrier wait is bounded and TMEM is released on every path; every CTA
// passes both cluster barriers on every path.
#pragma once

#include "elementwise.cuh"  // silu_mul_f
#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kLrTile = 128;                   // W rows per tile (MMA M)
constexpr int kLrK = 64;                       // K elements per chunk: one 128-byte row
constexpr int kLrWBytes = kLrTile * kLrK * 2;  // 16 KB of W per chunk
constexpr int kLrMaxRows = 128;
constexpr int kLrMaxSplits = 8;                // portable cluster size
constexpr int kLrThreads = 6 * 32;
constexpr int kLrTmaWarp = 4, kLrMmaWarp = 5;
constexpr int kLrRingBudget = 210 * 1024;      // bytes in flight per SM: the W stream's depth
constexpr int kLrMaxStages = 12;

__host__ __device__ constexpr int lr_stage_bytes(int n) { return kLrWBytes + n * 128; }
__host__ __device__ constexpr int lr_stages(int n) {
    return kLrRingBudget / lr_stage_bytes(n) < kLrMaxStages ? kLrRingBudget / lr_stage_bytes(n)
                                                             : kLrMaxStages;
}
__host__ __device__ constexpr int lr_smem_bytes(int n) {
    return lr_stages(n) * lr_stage_bytes(n) + 1024;  // + alignment slack
}

struct LinearRowsArgs {
    int rows;     // rows of X and Y (<= the kernel's N)
    int out;      // columns of Y: W rows, or inter for kGlu
    int glu_up;   // kGlu: first up row of W_gu (= inter)
    int kchunks;  // ceil(in / 64)
    int splits;   // CTAs per tile = cluster size
    void* y;      // [rows][out]
};

// Four floats of the partial tile of cluster CTA `rank` at this CTA's address p
// (a plain shared-memory load for this CTA itself).
__device__ __forceinline__ float4 lr_part4(const float* p, int rank, int self) {
    if (rank == self) return *reinterpret_cast<const float4*>(p);
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(dsmem_addr(p, (uint32_t)rank)));
    return v;
}

template <int N, bool kGlu, typename T>
__global__ void __launch_bounds__(kLrThreads, 1)
    linear_rows_kernel(const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap xmap, LinearRowsArgs a, uint32_t fmt) {
    constexpr int kStages = lr_stages(N);
    constexpr int kStage = lr_stage_bytes(N);
    constexpr int kCols = N < 32 ? 32 : N;  // TMEM columns (a power of two >= 32)
    constexpr int kLd = N < 32 ? N : 32;    // columns per TMEM load
    // the tile in units: (row, 4 W rows) of 16 bytes, or for kGlu (row, 4 gate/up
    // pairs) of 32 bytes, gate values first; contiguous in shared memory
    constexpr int kUnitsPerRow = kGlu ? 16 : 32;
    constexpr int kUnits = N * kUnitsPerRow;
    constexpr int kUnitFloats = kGlu ? 8 : 4;
    static_assert(kStages >= 2 && kStages * kStage >= N * kLrTile * 4,
                  "the ring holds at least two stages and the f32 tile");
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[kStages], empty[kStages], d_full;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_err;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    float* part = reinterpret_cast<float*>(smem);  // over the ring, at the end
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_split = a.splits;
    const int tile = (int)blockIdx.x / n_split, split = (int)blockIdx.x % n_split;
    const int c0 = split * a.kchunks / n_split;
    const int nc = (split + 1) * a.kchunks / n_split - c0;  // >= 1: splits <= kchunks
    // the units of the output tile this CTA sums over the slices and writes
    const int u0 = split * kUnits / n_split, u1 = (split + 1) * kUnits / n_split;

    // a kernel launched as this grid's programmatic dependent may start its prologue
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == kLrTmaWarp && lane == 0) {
        tma_prefetch_desc(&wmap);
        tma_prefetch_desc(&xmap);
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&d_full, 1);
        s_err = 0;
        fence_mbar_init();
    }
    if (warp == kLrMmaWarp) tmem_alloc(&tmem_slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == kLrTmaWarp) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            auto load_w = [&](int s, int c) {
                uint8_t* dst = smem + s * kStage;
                if constexpr (kGlu) {
                    tma_load_2d(dst, &wmap, &full[s], c * kLrK, tile * 64);
                    tma_load_2d(dst + kLrWBytes / 2, &wmap, &full[s], c * kLrK, a.glu_up + tile * 64);
                } else {
                    tma_load_2d(dst, &wmap, &full[s], c * kLrK, tile * kLrTile);
                }
            };
            auto load_x = [&](int s, int c) {
                tma_load_2d(smem + s * kStage + kLrWBytes, &xmap, &full[s], c * kLrK, 0);
            };
            const int pre = nc < kStages ? nc : kStages;
            for (int i = 0; i < pre; ++i) {
                mbar_expect_tx(&full[i], kStage);  // W and X of the stage
                load_w(i, c0 + i);
            }
            // X is written by the preceding kernel (a no-op without a programmatic launch)
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; ++i) load_x(i, c0 + i);
            int it = pre;
            for (; it < nc; ++it) {
                const int s = it % kStages;
                if (!mbar_wait(&empty[s], ((it - kStages) / kStages) & 1)) {
                    s_err = 1;
                    break;
                }
                mbar_expect_tx(&full[s], kStage);
                load_w(s, c0 + it);
                load_x(s, c0 + it);
            }
            if (s_err) {  // let every copy this CTA issued land before it goes on (bounded)
                for (int j = it - kStages < 0 ? 0 : it - kStages; j < it; ++j)
                    mbar_wait(&full[j % kStages], (j / kStages) & 1);
            }
        }
        __syncwarp();
    } else if (warp == kLrMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_f16(kLrTile, N, fmt, 0, 0);
        const uint64_t d0 = sdesc_sw128(smem_u32(smem), 16, 1024);
        constexpr uint64_t kStageDesc = kStage >> 4, kXDesc = kLrWBytes >> 4;
        bool ok = true;
        for (int i = 0; i < nc; ++i) {
            const int s = i % kStages;
            ok = __all_sync(0xffffffffu, !s_err && mbar_wait(&full[s], (i / kStages) & 1));
            if (!ok) break;
            tc_fence_after();
            const uint64_t dw = d0 + kStageDesc * (uint64_t)s, dx = dw + kXDesc;
#pragma unroll
            for (int k = 0; k < kLrK / 16; ++k)
                umma_f16(tmem, dw + 2 * k, dx + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);  // the stage is free once these finish
        }
        if (!ok && lane == 0) s_err = 1;
        umma_commit(&d_full);   // arrives when every MMA above has finished
        mbar_wait(&d_full, 0);  // TMEM is released below only after that
        __syncwarp();
    } else {
        // ------------------------------------------------------------ accumulator -> units
        // The tile in unit order over the ring: every MMA has read its stages when
        // d_full completes, and every copy into them has landed.  Thread m holds W
        // row m of the tile for all N rows of X; a row of X takes 128 floats in both
        // unit orders, at offset mo.
        const int m = warp * 32 + lane;
        const int mo = kGlu ? ((m & 63) >> 2) * 8 + (m >= 64 ? 4 : 0) + (m & 3) : m;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        if (__all_sync(0xffffffffu, mbar_wait(&d_full, 0))) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < N; c += kLd) {
                float v[kLd];
                if constexpr (kLd == 32) tmem_ld32(tmem + lane_off + (uint32_t)c, v);
                else tmem_ld16(tmem + lane_off + (uint32_t)c, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < kLd; ++j) part[(c + j) * kLrTile + mo] = v[j];
            }
        } else if (lane == 0) {
            s_err = 1;
        }
    }
    // every partial tile of the cluster is in shared memory; TMEM is read no more
    tc_fence_before();
    if (n_split > 1) cluster_sync();
    else __syncthreads();
    if (warp == kLrMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
    // the preceding grid may still read Y's buffer until it completes
    asm volatile("griddepcontrol.wait;" ::: "memory");
    T* y = static_cast<T*>(a.y);
    for (int u = u0 + (int)threadIdx.x; u < u1; u += kLrThreads) {
        const int r = u / kUnitsPerRow, m4 = (u % kUnitsPerRow) * 4;
        const int o = tile * (kGlu ? 64 : kLrTile) + m4;
        if (r >= a.rows || o >= a.out) continue;
        // all slices' loads in flight at once, then the sum in slice order (the same
        // sum on every run)
        const float* src = part + u * kUnitFloats;
        float4 v[kLrMaxSplits], hv[kGlu ? kLrMaxSplits : 1];
#pragma unroll
        for (int p = 0; p < kLrMaxSplits; ++p) {
            if (p < n_split) {
                v[p] = lr_part4(src, p, split);
                if constexpr (kGlu) hv[p] = lr_part4(src + 4, p, split);
            }
        }
        float4 g = v[0], h = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (kGlu) h = hv[0];
#pragma unroll
        for (int p = 1; p < kLrMaxSplits; ++p) {
            if (p < n_split) {
                g.x += v[p].x;
                g.y += v[p].y;
                g.z += v[p].z;
                g.w += v[p].w;
                if constexpr (kGlu) {
                    h.x += hv[p].x;
                    h.y += hv[p].y;
                    h.z += hv[p].z;
                    h.w += hv[p].w;
                }
            }
        }
        uint2 w;
        if constexpr (kGlu) {
            // the projection's 16-bit G and U, then SiLU*mul as silu_mul_vec_kernel does
            const float2 g01 = Elem<T>::unpack(Elem<T>::pack(g.x, g.y));
            const float2 g23 = Elem<T>::unpack(Elem<T>::pack(g.z, g.w));
            const float2 h01 = Elem<T>::unpack(Elem<T>::pack(h.x, h.y));
            const float2 h23 = Elem<T>::unpack(Elem<T>::pack(h.z, h.w));
            w.x = Elem<T>::pack(silu_mul_f(g01.x, h01.x), silu_mul_f(g01.y, h01.y));
            w.y = Elem<T>::pack(silu_mul_f(g23.x, h23.x), silu_mul_f(g23.y, h23.y));
        } else {
            w.x = Elem<T>::pack(g.x, g.y);
            w.y = Elem<T>::pack(g.z, g.w);
        }
        *reinterpret_cast<uint2*>(y + (size_t)r * a.out + o) = w;
    }
    if (n_split > 1) cluster_sync();  // no CTA leaves while a peer may still read its tile
}

}  // namespace kvb
