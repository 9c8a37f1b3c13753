// attn_prefill.cuh -- causal GQA prefill attention on the 5th-generation
// tensor cores (tcgen05 / TMEM), head_dim 64, warp-specialised.
//
// One CTA (one per SM) computes 256 query rows of one head of one sequence as
// two 128-row tiles, A and B, that share every K/V tile:
//   warp 16  TMA producer: Q_A, Q_B once, then 64-key K/V tiles into a
//            3-stage ring (cp.async.bulk.tensor, 128B swizzle, no multicast)
//   warp 17  MMA issuer (one lane): S_q = Q_q K^T (tcgen05.mma kind::f16,
//            M=128 N=64, f32 accumulators in TMEM, two S buffers per tile)
//            and O_q = P_q V (M=128 N=64, V read MN-major from the same tile)
//   warps 0-7 / 8-15  softmax for tile A / B, two threads per query row (32
//            columns each): tcgen05.ld of the S row half, causal mask on the
//            diagonal, online max/sum in the log2 domain, P to shared memory as
//            a 16-bit head plus a 16-bit remainder (two MMAs, so P keeps ~16
//            significant bits), O tile folded into f32 accumulators in registers.
// Issue order per K/V tile j: S_A(j+1), S_B(j+1), then P_A(j) V, P_B(j) V as each P
// arrives, so the next S is ready when a softmax thread finishes the current one.
// P, O and S are double-buffered; each buffer has its own ready barrier.
// Every mbarrier wait is bounded; a failed wait sets a CTA-wide flag that
// every role checks before its next wait; TMEM is freed on every path.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kPfRows = 128;                      // rows per Q tile (MMA M)
constexpr int kPfTiles = 2;                       // Q tiles per CTA
constexpr int kPfKeys = 64;                       // keys per K/V tile
constexpr int kPfStages = 6;                      // K/V ring depth
constexpr int kPfQBytes = kPfRows * 64 * 2;       // 16 KB
constexpr int kPfKVBytes = kPfKeys * 64 * 2;      // 8 KB (K or V)
// Q[2] + K/V ring (P lives in TMEM, over the S columns it was computed from)
constexpr int kPfSmemBytes = kPfTiles * kPfQBytes + kPfStages * 2 * kPfKVBytes + 1024;
constexpr int kPfSoftmaxWarps = 16;               // 8 per Q tile, two threads per row
constexpr int kTmaWarp = kPfSoftmaxWarps, kMmaWarp = kPfSoftmaxWarps + 1;
constexpr int kPfThreads = (kPfSoftmaxWarps + 2) * 32;
constexpr uint32_t kPfTmemCols = 512;             // S[tile][2] and O[tile][2], 64 columns each

// acc[0:16] = acc * alpha + (16 TMEM columns of this thread's lane at taddr)
__device__ __forceinline__ void fold_o16(uint32_t taddr, float* acc, float alpha) {
    float ot[16];
    tmem_ld16(taddr, ot);
    tmem_wait_ld();
#pragma unroll
    for (int d = 0; d < 16; ++d) acc[d] = fmaf(acc[d], alpha, ot[d]);
}

struct PrefillArgs {
    int t, pos0, n_q, n_kv, group, n_qblocks;
    float scale_log2;
    uint16_t* out;
    long long out_row_stride;
};

struct PrefillBars {
    uint64_t q_full;
    uint64_t kv_full[kPfStages], kv_empty[kPfStages];
    uint64_t s_full[kPfTiles][2];
    // One P-ready and one O-ready barrier per buffer: a warp that runs one tile
    // ahead arrives on the other buffer's barrier, never on a phase still in use.
    uint64_t p_full[kPfTiles][2], o_full[kPfTiles][2];
    uint64_t mma_done;  // every MMA of the CTA has completed (before TMEM is freed)
};

template <typename T>
// 18 warps: two SM sub-partitions host 5 warps each, which caps a thread at 96 registers.
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ PrefillBars bars;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_err;
    // Row-max exchange between the two threads of a row, per tile parity (slots 0, 1),
    // and the final row-sum exchange (slot 2, never shared with a row-max round).
    __shared__ float xmax[kPfTiles][3][2][kPfRows];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* sq = smem;                                  // [tile] Q
    uint8_t* skv = sq + kPfTiles * kPfQBytes;            // [stage][K | V]

    const int h = blockIdx.x, seq = blockIdx.y;
    const int qb = a.n_qblocks - 1 - (int)blockIdx.z;    // longest blocks first
    const int q0 = qb * kPfTiles * kPfRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = h / a.group;
    const int kv_plane = seq * a.n_kv + kvh;

    // Per tile: valid rows and the number of K/V tiles it visits (causal).
    // (Scalars, not arrays: a runtime-indexed array would live in local memory.)
    const int rows_valid0 = max(0, min(kPfRows, a.t - q0));
    const int rows_valid1 = max(0, min(kPfRows, a.t - q0 - kPfRows));
    const int n_tiles0 = rows_valid0 ? (a.pos0 + q0 + rows_valid0 + kPfKeys - 1) / kPfKeys : 0;
    const int n_tiles1 =
        rows_valid1 ? (a.pos0 + q0 + kPfRows + rows_valid1 + kPfKeys - 1) / kPfKeys : 0;
    const int n_kv_tiles = max(n_tiles0, n_tiles1);
    auto n_tiles = [&](int q) { return q ? n_tiles1 : n_tiles0; };

    if (tid == 0) {
        mbar_init(&bars.q_full, 1);
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&bars.kv_full[s], 1);
            mbar_init(&bars.kv_empty[s], 1);
        }
        for (int q = 0; q < kPfTiles; ++q) {
            for (int b = 0; b < 2; ++b) {
                mbar_init(&bars.s_full[q][b], 1);
                mbar_init(&bars.p_full[q][b], 2 * kPfRows);
                mbar_init(&bars.o_full[q][b], 1);
            }
        }
        mbar_init(&bars.mma_done, 1);
        s_err = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(&tmem_slot, kPfTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t fmt = Elem<T>::kDtype == KVB_BF16 ? 1u : 0u;

    if (warp == kTmaWarp) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&kmap);
            tma_prefetch_desc(&vmap);
            const int nq_tiles = rows_valid1 ? 2 : 1;
            mbar_expect_tx(&bars.q_full, nq_tiles * kPfQBytes);
            for (int q = 0; q < nq_tiles; ++q)
                tma_load_3d(sq + q * kPfQBytes, &qmap, &bars.q_full, h * 64, q0 + q * kPfRows, seq);
            int issued = 0;
            for (int j = 0; j < n_kv_tiles; ++j) {
                const int st = j % kPfStages;
                if (j >= kPfStages && !mbar_wait(&bars.kv_empty[st], ((j - kPfStages) / kPfStages) & 1)) {
                    s_err = 1;
                    break;
                }
                if (s_err) break;
                mbar_expect_tx(&bars.kv_full[st], 2 * kPfKVBytes);
                tma_load_3d(skv + (2 * st) * kPfKVBytes, &kmap, &bars.kv_full[st], 0, j * kPfKeys,
                            kv_plane);
                tma_load_3d(skv + (2 * st + 1) * kPfKVBytes, &vmap, &bars.kv_full[st], 0,
                            j * kPfKeys, kv_plane);
                issued = j + 1;
            }
            if (s_err) {
                // let every copy this CTA issued land before the CTA exits (bounded)
                for (int j = max(0, issued - kPfStages); j < issued; ++j)
                    mbar_wait(&bars.kv_full[j % kPfStages], (j / kPfStages) & 1);
                mbar_wait(&bars.q_full, 0);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(kPfRows, kPfKeys, fmt, 0, 0);
            const uint32_t idesc_o = idesc_f16(kPfRows, 64, fmt, 0, 1);
            // Descriptors are built once; per MMA only the 16-byte start-address field
            // (bits 0-13) moves, by adding a constant: issue cost, not the tensor core,
            // otherwise bounds a single issuing thread at these small N.
            const uint64_t dq0 = sdesc_sw128(smem_u32(sq), 16, 1024);
            const uint64_t dk0 = sdesc_sw128(smem_u32(skv), 16, 1024);
            const uint64_t dv0 = sdesc_sw128(smem_u32(skv) + kPfKVBytes, 64 * 128, 1024);
            constexpr uint64_t kQTile = kPfQBytes >> 4, kStage = (2 * kPfKVBytes) >> 4;
            // S_q[j & 1] = Q_q K_j^T.  Buffer j&1 last held P(j-2), read by P(j-2) V, which
            // this thread issued earlier: MMAs of one thread run in issue order.
            auto issue_s = [&](int q, int j) {
                const int st = j % kPfStages, b = j & 1;
                const uint32_t d = tmem + (uint32_t)((q * 2 + b) * 64);
                const uint64_t da = dq0 + kQTile * q, db = dk0 + kStage * st;
                umma_f16(d, da, db, idesc_s, 0);
                umma_f16(d, da + 2, db + 2, idesc_s, 1);  // +32 bytes: next 16 dims
                umma_f16(d, da + 4, db + 4, idesc_s, 1);
                umma_f16(d, da + 6, db + 6, idesc_s, 1);
                umma_commit(&bars.s_full[q][b]);
            };
            // O_q[j&1] = P_q,hi V_j + P_q,lo V_j with P read from TMEM (the S buffer:
            // P_hi in its columns 0-31, P_lo in 32-63, two keys per column).
            auto issue_pv = [&](int q, int j) -> bool {
                const int st = j % kPfStages, b = j & 1;
                if (!mbar_wait(&bars.p_full[q][b], (j >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(256 + (q * 2 + b) * 64);
                const uint32_t p = tmem + (uint32_t)((q * 2 + b) * 64);
                const uint64_t dv = dv0 + kStage * st;  // +2048 bytes (>> 4 = 128): next 16 keys
                umma_f16_ts(d, p + 0, dv + 0, idesc_o, 0);
                umma_f16_ts(d, p + 8, dv + 128, idesc_o, 1);
                umma_f16_ts(d, p + 16, dv + 256, idesc_o, 1);
                umma_f16_ts(d, p + 24, dv + 384, idesc_o, 1);
                umma_f16_ts(d, p + 32, dv + 0, idesc_o, 1);
                umma_f16_ts(d, p + 40, dv + 128, idesc_o, 1);
                umma_f16_ts(d, p + 48, dv + 256, idesc_o, 1);
                umma_f16_ts(d, p + 56, dv + 384, idesc_o, 1);
                umma_commit(&bars.o_full[q][b]);
                return true;
            };
            bool ok = mbar_wait(&bars.q_full, 0);
            // prologue: S for tile 0 of both Q tiles
            if (ok) ok = mbar_wait(&bars.kv_full[0], 0);
            for (int q = 0; q < kPfTiles && ok; ++q)
                if (n_tiles(q) > 0) issue_s(q, 0);
            // Per K/V tile j: first S(j+1) for both tiles (their S buffers were read by
            // softmax one tile ago), then P(j) V for both as their P arrive -- so the
            // next S is ready when a softmax warpgroup finishes with the current one.
            for (int j = 0; j < n_kv_tiles && ok; ++j) {
                if (j + 1 < n_kv_tiles)
                    ok = mbar_wait(&bars.kv_full[(j + 1) % kPfStages], ((j + 1) / kPfStages) & 1);
                for (int q = 0; q < kPfTiles && ok; ++q)
                    if (j + 1 < n_tiles(q)) issue_s(q, j + 1);
                for (int q = 0; q < kPfTiles && ok; ++q) {
                    if (j < n_tiles(q)) ok = issue_pv(q, j);
                    if (s_err) ok = false;
                }
                if (ok) umma_commit(&bars.kv_empty[j % kPfStages]);  // stage j free once all MMAs so far finish
            }
            if (!ok) s_err = 1;
            // No MMA may still be running when TMEM is released below.
            umma_commit(&bars.mma_done);
            mbar_wait(&bars.mma_done, 0);
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        // Two threads per query row: warps 8q..8q+3 take columns 0-31 and warps
        // 8q+4..8q+7 columns 32-63 of the same 128 TMEM lanes.  The row maximum is
        // exchanged once per tile through shared memory (a 64-thread named barrier
        // per warp pair); the row sum stays per thread until the end.  Error
        // decisions are exchanged through the same barrier, so both threads of a
        // row always take the same number of barrier steps.
        const int q = warp >> 3;                // Q tile
        const int half = (warp >> 2) & 1;       // column half of the S / O tiles
        const int quarter = warp & 3;           // TMEM lane quarter
        const int row = quarter * 32 + lane;    // row of the tile (= TMEM lane)
        const int col0 = half * 32;
        const uint32_t bar_id = 1 + q * 4 + quarter;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        auto t_o = [&](int b) {
            return tmem + (uint32_t)(256 + (q * 2 + b) * 64 + col0) + lane_off;
        };
        const int my_pos = a.pos0 + q0 + q * kPfRows + row;
        const int diag_key = a.pos0 + q0 + q * kPfRows;  // keys above need the causal mask
        const int nt = n_tiles(q);
        float oacc[32];
#pragma unroll
        for (int d = 0; d < 32; ++d) oacc[d] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_pending = 1.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            const bool good = ok && !s_err && mbar_wait(&bars.s_full[q][b], (j >> 1) & 1);
            float s[32];
            float mx = -INFINITY;
            const uint32_t t_sp = tmem + (uint32_t)((q * 2 + b) * 64) + lane_off;  // S, then P
            if (good) {
                tc_fence_after();
                tmem_ld32(t_sp + col0, s);
                tmem_wait_ld();
                if (j * kPfKeys + kPfKeys - 1 > diag_key) {
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        if (j * kPfKeys + col0 + c > my_pos) s[c] = -INFINITY;
                }
                float mx4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) mx4[i] = s[i];
#pragma unroll
                for (int c = 4; c < 32; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
                mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            }
            xmax[q][b][half][row] = good ? mx : __int_as_float(0x7fffffff);  // NaN = failed
            named_bar_sync(bar_id, 64);
            const float pmx = xmax[q][b][half ^ 1][row];
            if (!good || isnan(pmx)) ok = false;
            if (!ok) continue;
            // Raw scores: the max is taken before scaling (the scale is positive).
            const float mn = fmaxf(m, fmaxf(mx, pmx) * a.scale_log2);  // running max, log2
            const float alpha = ex2_approx(m - mn);
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                s[c] = ex2_approx(fmaf(s[c], a.scale_log2, -mn));  // exp2(s*scale - max)
                sum4[c & 3] += s[c];
            }
            l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            m = mn;
            // P_j -> TMEM over the S columns it came from: P_hi (two keys per 32-bit
            // column) in columns 16*half .. +15, P_lo in 32 + 16*half .. +15.  Both
            // threads of the row have their S in registers (the max exchange above
            // came after both loads), so overwriting S here is safe.
            {
                uint32_t pk[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {  // heads; s keeps the remainders
                    pk[k] = Elem<T>::pack(s[2 * k], s[2 * k + 1]);
                    const float2 hv = Elem<T>::unpack(pk[k]);
                    s[2 * k] -= hv.x;
                    s[2 * k + 1] -= hv.y;
                }
                tmem_st16(t_sp + 16 * half, pk);
#pragma unroll
                for (int k = 0; k < 16; ++k) pk[k] = Elem<T>::pack(s[2 * k], s[2 * k + 1]);
                tmem_st16(t_sp + 32 + 16 * half, pk);
                tmem_wait_st();
            }
            tc_fence_before();
            mbar_arrive(&bars.p_full[q][b]);
            if (j > 0) {  // fold the previous tile's P V (TMEM buffer (j-1)&1)
                if (s_err || !mbar_wait(&bars.o_full[q][b ^ 1], ((j - 1) >> 1) & 1)) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                fold_o16(t_o(b ^ 1), oacc, alpha_pending);
                fold_o16(t_o(b ^ 1) + 16, oacc + 16, alpha_pending);
                tc_fence_before();
            }
            alpha_pending = alpha;
        }
        if (nt > 0) {
            const bool good = ok && !s_err &&
                              mbar_wait(&bars.o_full[q][(nt - 1) & 1], ((nt - 1) >> 1) & 1);
            if (good) {
                tc_fence_after();
                fold_o16(t_o((nt - 1) & 1), oacc, alpha_pending);
                fold_o16(t_o((nt - 1) & 1) + 16, oacc + 16, alpha_pending);
            }
            xmax[q][2][half][row] = good ? l : __int_as_float(0x7fffffff);
            named_bar_sync(bar_id, 64);
            const float pl = xmax[q][2][half ^ 1][row];
            if (good && !isnan(pl)) {
                if (row < (q ? rows_valid1 : rows_valid0)) {
                    const float inv = 1.f / (l + pl);
                    T* orow = reinterpret_cast<T*>(a.out) +
                              ((size_t)seq * a.t + q0 + q * kPfRows + row) * a.out_row_stride +
                              (size_t)h * 64 + col0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = oacc[8 * k + e] * inv;
                        *reinterpret_cast<uint4*>(orow + 8 * k) = pack8<T>(f);
                    }
                }
            } else {
                s_err = 1;
            }
        }
        if (!ok) s_err = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kPfTmemCols);
    }
}

}  // namespace kvb
