// attn_prefill.cuh -- causal GQA prefill attention on the 5th-generation
// tensor cores (tcgen05 / TMEM), head_dim 64.
//
// One CTA computes a 128-query tile of one head of one sequence.  Q (128x64),
// and double-buffered K/V tiles (64 keys x 64 dims) arrive by TMA with
// 128-byte swizzle (no multicast), each completing an mbarrier.  Per K/V tile:
//   S = Q K^T      tcgen05.mma kind::f16, M=128 N=64, K=64 (4 x K16), D in TMEM
//   softmax        each of the 128 threads owns one query row: tcgen05.ld the
//                  S row, causal mask on the diagonal tiles, online max/sum in
//                  the log2 domain, P rounded to 16 bits and stored to shared
//                  memory in the canonical 128B-swizzled K-major layout
//   O_t = P V      tcgen05.mma, M=128 N=64 K=64, V read MN-major from the
//                  same TMA tile; O_t lands in TMEM and is folded into the
//                  row's f32 accumulator in registers (O = O*alpha + O_t)
// Causal tile skipping: a 128-row tile at query offset q0 only visits keys
// [0, pos0 + q0 + 128).  Grid order puts the longest tiles first.
// Every mbarrier wait is bounded; TMEM is released on every exit path.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kPfRows = 128;     // query rows per CTA (MMA M)
constexpr int kPfKeys = 64;      // keys per K/V tile (MMA N of S, K of O)
constexpr int kPfQBytes = kPfRows * 64 * 2;    // 16 KB
constexpr int kPfKVBytes = kPfKeys * 64 * 2;   // 8 KB
constexpr int kPfPBytes = kPfRows * kPfKeys * 2;  // 16 KB
constexpr int kPfSmemBytes = kPfQBytes + 4 * kPfKVBytes + 2 * kPfPBytes + 1024;
constexpr uint32_t kPfTmemCols = 128;  // S: cols [0,64), O tile: cols [64,128)

struct PrefillArgs {
    int t, pos0, n_q, n_kv, group, n_qtiles;
    float scale_log2;
    uint16_t* out;
    long long out_row_stride;
};

template <typename T>
__global__ void __launch_bounds__(128, 2) attn_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_q, bar_s, bar_o;
    __shared__ uint64_t bar_kv[2];
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* sq = smem;
    uint8_t* skv = smem + kPfQBytes;  // [buf][K | V]
    uint8_t* sp = skv + 4 * kPfKVBytes;

    const int h = blockIdx.x, seq = blockIdx.y;
    const int qt = a.n_qtiles - 1 - (int)blockIdx.z;  // longest tiles first
    const int q0 = qt * kPfRows;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int kvh = h / a.group;
    const int rows_valid = min(kPfRows, a.t - q0);
    const int key_end = a.pos0 + q0 + rows_valid;  // keys [0, key_end) are visible to this tile
    const int n_tiles = (key_end + kPfKeys - 1) / kPfKeys;
    const int diag_key = a.pos0 + q0;               // tiles with keys > diag_key need the mask
    const int my_pos = a.pos0 + q0 + tid;           // absolute position of this thread's row

    if (tid == 0) {
        mbar_init(&bar_q, 1);
        mbar_init(&bar_s, 1);
        mbar_init(&bar_o, 1);
        mbar_init(&bar_kv[0], 1);
        mbar_init(&bar_kv[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tmem_slot, kPfTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t t_s = tmem, t_o = tmem + 64;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

    const uint32_t fmt = Elem<T>::kDtype == KVB_BF16 ? 1u : 0u;
    const uint32_t idesc_s = idesc_f16(kPfRows, kPfKeys, fmt, 0, 0);
    const uint32_t idesc_o = idesc_f16(kPfRows, 64, fmt, 0, 1);
    const int kv_plane = seq * a.n_kv + kvh;

    // Error state shared by the CTA so that every thread leaves the tile loop
    // at the same barrier.
    __shared__ volatile int s_err;
    if (tid == 0) s_err = 0;
    uint32_t kv_issued[2] = {0, 0}, kv_done[2] = {0, 0};  // meaningful in thread 0 only
    __syncthreads();
    if (tid == 0) {
        tma_prefetch_desc(&qmap);
        mbar_expect_tx(&bar_q, kPfQBytes);
        tma_load_3d(sq, &qmap, &bar_q, h * 64, q0, seq);
        for (int j = 0; j < 2 && j < n_tiles; ++j) {
            mbar_expect_tx(&bar_kv[j], 2 * kPfKVBytes);
            tma_load_3d(skv + (2 * j) * kPfKVBytes, &kmap, &bar_kv[j], 0, j * kPfKeys, kv_plane);
            tma_load_3d(skv + (2 * j + 1) * kPfKVBytes, &vmap, &bar_kv[j], 0, j * kPfKeys, kv_plane);
            kv_issued[j]++;
        }
        if (!mbar_wait(&bar_q, 0)) s_err = 1;
    }

    float oacc[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) oacc[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    const uint32_t sq_a = smem_u32(sq), sp_a = smem_u32(sp);

    for (int j = 0; j < n_tiles; ++j) {
        const int buf = j & 1;
        const uint32_t sk_a = smem_u32(skv + (2 * buf) * kPfKVBytes);
        const uint32_t sv_a = smem_u32(skv + (2 * buf + 1) * kPfKVBytes);
        // ---- S = Q K^T
        if (tid == 0) {
            if (!s_err) {
                if (mbar_wait(&bar_kv[buf], kv_done[buf] & 1))
                    kv_done[buf]++;
                else
                    s_err = 1;
            }
            tc_fence_after();
            if (!s_err) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma_f16(t_s, sdesc_sw128(sq_a + 32 * ks, 16, 1024),
                             sdesc_sw128(sk_a + 32 * ks, 16, 1024), idesc_s, ks > 0);
            }
            umma_commit(&bar_s);  // arrives even when nothing was issued
        }
        if (!mbar_wait(&bar_s, j & 1)) s_err = 1;
        tc_fence_after();
        // ---- softmax on this thread's row
        float s[64];
        tmem_ld32(t_s + lane_off, s);
        tmem_ld32(t_s + lane_off + 32, s + 32);
        tmem_wait_ld();
        const bool need_mask = j * kPfKeys + kPfKeys - 1 > diag_key;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            float v = s[c] * a.scale_log2;
            if (need_mask && j * kPfKeys + c > my_pos) v = -INFINITY;
            s[c] = v;
            mx = fmaxf(mx, v);
        }
        const float mn = fmaxf(m, mx);
        const float alpha = exp2f(m - mn);
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            s[c] = exp2f(s[c] - mn);
            sum += s[c];
        }
        l = l * alpha + sum;
        m = mn;
        // P row -> shared memory as two 16-bit tiles, head and remainder
        // (P = hi + lo, see split_pack), each 128B-swizzled K-major: 16-byte
        // chunk ch of row r at r*128 + ((ch ^ (r & 7)) * 16).
        {
            uint8_t* prow_h = sp + tid * 128;
            uint8_t* prow_l = sp + kPfPBytes + tid * 128;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                uint4 vh, vl;
                split_pack<T>(s[8 * ch + 0], s[8 * ch + 1], vh.x, vl.x);
                split_pack<T>(s[8 * ch + 2], s[8 * ch + 3], vh.y, vl.y);
                split_pack<T>(s[8 * ch + 4], s[8 * ch + 5], vh.z, vl.z);
                split_pack<T>(s[8 * ch + 6], s[8 * ch + 7], vh.w, vl.w);
                *reinterpret_cast<uint4*>(prow_h + ((ch ^ (tid & 7)) << 4)) = vh;
                *reinterpret_cast<uint4*>(prow_l + ((ch ^ (tid & 7)) << 4)) = vl;
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- O_t = P_hi V + P_lo V
        if (tid == 0) {
            tc_fence_after();
            if (!s_err) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma_f16(t_o, sdesc_sw128(sp_a + 32 * ks, 16, 1024),
                             sdesc_sw128(sv_a + ks * 16 * 128, 64 * 128, 1024), idesc_o, ks > 0);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma_f16(t_o, sdesc_sw128(sp_a + kPfPBytes + 32 * ks, 16, 1024),
                             sdesc_sw128(sv_a + ks * 16 * 128, 64 * 128, 1024), idesc_o, 1);
            }
            umma_commit(&bar_o);
        }
        if (!mbar_wait(&bar_o, j & 1)) s_err = 1;
        tc_fence_after();
        if (tid == 0 && !s_err && j + 2 < n_tiles) {  // both MMAs on this buffer are done
            mbar_expect_tx(&bar_kv[buf], 2 * kPfKVBytes);
            tma_load_3d(skv + (2 * buf) * kPfKVBytes, &kmap, &bar_kv[buf], 0, (j + 2) * kPfKeys,
                        kv_plane);
            tma_load_3d(skv + (2 * buf + 1) * kPfKVBytes, &vmap, &bar_kv[buf], 0,
                        (j + 2) * kPfKeys, kv_plane);
            kv_issued[buf]++;
        }
        float ot[64];
        tmem_ld32(t_o + lane_off, ot);
        tmem_ld32(t_o + lane_off + 32, ot + 32);
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < 64; ++d) oacc[d] = oacc[d] * alpha + ot[d];
        tc_fence_before();
        __syncthreads();
        if (s_err) break;  // read after the barrier: the same value in every thread
    }
    const bool ok = !s_err;
    if (!ok && tid == 0) {
        // Give every copy this CTA issued a bounded chance to land before exit.
        for (int b2 = 0; b2 < 2; ++b2)
            while (kv_done[b2] < kv_issued[b2]) {
                mbar_wait(&bar_kv[b2], kv_done[b2] & 1);
                kv_done[b2]++;
            }
        mbar_wait(&bar_q, 0);
    }

    // ---- epilogue: normalise and store this thread's row
    if (ok && tid < rows_valid) {
        const float inv = 1.f / l;
        T* orow = reinterpret_cast<T*>(a.out) + ((size_t)seq * a.t + q0 + tid) * a.out_row_stride +
                  (size_t)h * 64;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = oacc[8 * ch + e] * inv;
            *reinterpret_cast<uint4*>(orow + 8 * ch) = pack8<T>(f);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kPfTmemCols);
    }
}

}  // namespace kvb
