// lm_head.cuh -- the tied LM head and greedy argmax in one pass: the f32 logits
// of up to 32 rows are formed on the tensor cores and reduced to each row's
// argmax on chip, never written to memory.
//
// D[v, r] = sum_k W[v, k] x[r, k] for one 128-row vocabulary tile v0 .. v0+127
// is tcgen05.mma kind::f16 with M = 128 (vocabulary rows, A = W, K-major) and
// N = 16 or 32 (the rows r, B = x, K-major), f32 accumulate in TMEM.  One CTA
// per SM walks the vocabulary tiles blockIdx.x, + gridDim.x, ...:
//   warp 4   TMA producer: x (all of it, once: N rows x hidden, 128-byte
//            swizzled chunks of 64 elements) and then W in 16 KB chunks of
//            128 rows x 64 elements through a kLmStages ring (no multicast)
//   warp 5   MMA issuer (whole warp, elected lane): per tile, hidden / 16
//            MMAs into one of two TMEM accumulators, commits that free the W
//            stages and announce the finished tile
//   warps 0-3  epilogue, one thread per vocabulary row of the tile (= TMEM
//            lane): loads its N logits, frees the accumulator, and keeps per
//            row r the best (value, first index) seen so far in registers.
// At the end the four epilogue warps merge their bests, and the CTA writes one
// (value, index) partial per row to the workspace; lm_head_argmax_finish_kernel
// merges the CTAs' partials into ids (and advances the decode counters).  The
// rule is kvb_argmax_f32's: the first index of the maximum; NaN never wins, a
// -inf never wins a tie, and a row with nothing above -inf gives 0.
//
// HBM-bound: W (vocab x hidden x 2 B, 525 MB for Llama-3.2-1B) is read once;
// x is read once per CTA from L2.  Every mbarrier wait is bounded; TMEM is
// freed on every path.
#pragma once

#include "elementwise.cuh"  // argmax_merge / argmax_warp: the argmax rule
#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kLmMaxCtas = 256;                    // partials per row in the workspace
constexpr int kLmRows = 128;                       // vocabulary rows per tile (MMA M)
constexpr int kLmK = 64;                           // elements per chunk: one 128-byte row
constexpr int kLmStages = 5;
constexpr int kLmStageBytes = kLmRows * kLmK * 2;  // 16 KB of W
constexpr int kLmMaxRows = 32;
constexpr int kLmMaxXBytes = 128 * 1024;           // x held in shared memory
constexpr int kLmThreads = 6 * 32;
constexpr int kLmTmaWarp = 4, kLmMmaWarp = 5;

__host__ __device__ constexpr int lm_smem_bytes(int n, int hidden) {
    return n * hidden * 2 + kLmStages * kLmStageBytes + 1024;
}

struct LmArgs {
    int vocab, hidden, rows, n_tiles;
    float* part_v;    // [gridDim.x][rows] best value of each CTA
    int32_t* part_i;  // [gridDim.x][rows] its index
};

template <int N>
__global__ void __launch_bounds__(kLmThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap wmap,
                          const __grid_constant__ CUtensorMap xmap, LmArgs a, uint32_t fmt) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t x_full, full[kLmStages], empty[kLmStages], d_full[2], d_empty[2], mma_done;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_err;
    __shared__ float red_v[4][N];
    __shared__ int red_i[4][N];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* sx = smem;                           // kchunks x [N rows][128 B]
    const int kchunks = a.hidden / kLmK;
    uint8_t* sw = sx + (size_t)kchunks * N * 128;  // kLmStages x 16 KB
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Launched as a programmatic dependent of the kernel before it: W (never the output
    // of a kernel still running) is requested before griddepcontrol.wait, x after it.
    // The merge kernel after this one may launch at once; it waits for this grid.
    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        mbar_init(&x_full, 1);
        for (int s = 0; s < kLmStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int d = 0; d < 2; ++d) {
            mbar_init(&d_full[d], 1);
            mbar_init(&d_empty[d], 128);
        }
        mbar_init(&mma_done, 1);
        s_err = 0;
        fence_mbar_init();
    }
    if (warp == kLmMmaWarp) tmem_alloc(&tmem_slot, 64);  // two N-column accumulators
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == kLmTmaWarp) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            tma_prefetch_desc(&xmap);
            int it = 0;
            bool x_issued = false;
            for (int t = blockIdx.x; t < a.n_tiles && !s_err; t += gridDim.x) {
                for (int c = 0; c < kchunks; ++c, ++it) {
                    const int s = it % kLmStages;
                    if (it == kLmStages && !x_issued) {  // the ring is full: now x
                        asm volatile("griddepcontrol.wait;" ::: "memory");
                        mbar_expect_tx(&x_full, (uint32_t)(kchunks * N * 128));
                        for (int k = 0; k < kchunks; ++k)
                            tma_load_2d(sx + (size_t)k * N * 128, &xmap, &x_full, k * kLmK, 0);
                        x_issued = true;
                    }
                    if (it >= kLmStages && !mbar_wait(&empty[s], ((it - kLmStages) / kLmStages) & 1)) {
                        s_err = 1;
                        break;
                    }
                    mbar_expect_tx(&full[s], kLmStageBytes);
                    tma_load_2d(sw + s * kLmStageBytes, &wmap, &full[s], c * kLmK, t * kLmRows);
                }
            }
            if (!x_issued) {  // fewer W chunks than stages in this CTA
                asm volatile("griddepcontrol.wait;" ::: "memory");
                mbar_expect_tx(&x_full, (uint32_t)(kchunks * N * 128));
                for (int k = 0; k < kchunks; ++k)
                    tma_load_2d(sx + (size_t)k * N * 128, &xmap, &x_full, k * kLmK, 0);
            }
            if (s_err) {  // let every copy this CTA issued land before it exits (bounded)
                for (int j = it - kLmStages < 0 ? 0 : it - kLmStages; j < it; ++j)
                    mbar_wait(&full[j % kLmStages], (j / kLmStages) & 1);
                mbar_wait(&x_full, 0);
            }
        }
    } else if (warp == kLmMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_f16(kLmRows, N, fmt, 0, 0);
        const uint64_t dx0 = sdesc_sw128(smem_u32(sx), 16, 1024);
        const uint64_t dw0 = sdesc_sw128(smem_u32(sw), 16, 1024);
        constexpr uint64_t kXChunk = (N * 128) >> 4, kWStage = kLmStageBytes >> 4;
        bool ok = __all_sync(0xffffffffu, mbar_wait(&x_full, 0));
        int it = 0, lt = 0;
        for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x, ++lt) {
            const int d = lt & 1;
            if (lt >= 2) ok = __all_sync(0xffffffffu, !s_err && mbar_wait(&d_empty[d], ((lt - 2) >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            const uint32_t dt = tmem + (uint32_t)(d * 32);
            for (int c = 0; c < kchunks; ++c, ++it) {
                const int s = it % kLmStages;
                ok = __all_sync(0xffffffffu, !s_err && mbar_wait(&full[s], (it / kLmStages) & 1));
                if (!ok) break;
                tc_fence_after();
                const uint64_t dw = dw0 + kWStage * s, dx = dx0 + kXChunk * c;
#pragma unroll
                for (int k = 0; k < kLmK / 16; ++k)
                    umma_f16(dt, dw + 2 * k, dx + 2 * k, idesc, (c | k) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);  // the W stage is free once these finish
            }
            if (!ok) break;
            umma_commit(&d_full[d]);
        }
        if (!ok && lane == 0) s_err = 1;
        umma_commit(&mma_done);  // no MMA may still run when TMEM is released below
        mbar_wait(&mma_done, 0);
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue warps
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float bv[N];
        int bi[N];
#pragma unroll
        for (int r = 0; r < N; ++r) {
            bv[r] = -INFINITY;
            bi[r] = 0x7fffffff;
        }
        int lt = 0;
        for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x, ++lt) {
            const int d = lt & 1;
            if (!__all_sync(0xffffffffu, !s_err && mbar_wait(&d_full[d], (lt >> 1) & 1))) {
                s_err = 1;
                break;
            }
            tc_fence_after();
            float v[N];
            if constexpr (N == 32) tmem_ld32(tmem + (uint32_t)(d * 32) + lane_off, v);
            else tmem_ld16(tmem + (uint32_t)(d * 32) + lane_off, v);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&d_empty[d]);  // the MMA warp may refill this accumulator
            const int vi = t * kLmRows + warp * 32 + lane;
            if (vi < a.vocab) {
#pragma unroll
                for (int r = 0; r < N; ++r) argmax_merge(bv[r], bi[r], v[r], vi);
            }
        }
        // merge the warp's 32 rows, then the four warps (named barrier 1, 128 threads)
#pragma unroll
        for (int r = 0; r < N; ++r) {
            float x = bv[r];
            int i = bi[r];
            argmax_warp(x, i);
            if (lane == 0) {
                red_v[warp][r] = x;
                red_i[warp][r] = i;
            }
        }
        named_bar_sync(1, 128);
        // the partials' buffer was last read by an earlier merge kernel
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (threadIdx.x < a.rows) {
            const int r = threadIdx.x;
            float x = red_v[0][r];
            int i = red_i[0][r];
#pragma unroll
            for (int w = 1; w < 4; ++w) argmax_merge(x, i, red_v[w][r], red_i[w][r]);
            a.part_v[(size_t)blockIdx.x * a.rows + r] = x;
            a.part_i[(size_t)blockIdx.x * a.rows + r] = i;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kLmMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

// Merges the per-CTA partials: one warp per row; ids[r], then the counters.
__global__ void __launch_bounds__(32) lm_head_argmax_finish_kernel(const float* part_v,
                                                                   const int32_t* part_i,
                                                                   int n_parts, int rows,
                                                                   int32_t* ids, int32_t* adv,
                                                                   int32_t* adv2) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the partials of the pass before
    const int r = blockIdx.x, lane = threadIdx.x;
    float x = -INFINITY;
    int i = 0x7fffffff;
    for (int p = lane; p < n_parts; p += 32)
        argmax_merge(x, i, part_v[(size_t)p * rows + r], part_i[(size_t)p * rows + r]);
    argmax_warp(x, i);
    if (lane == 0) {
        ids[r] = i == 0x7fffffff ? 0 : i;  // all -inf / NaN rows give index 0
        if (adv) adv[r] += 1;
        if (adv2) adv2[r] += 1;
    }
}

}  // namespace kvb
