// attn_prefill.cuh -- causal GQA prefill attention on the 5th-generation
// tensor cores (tcgen05 / TMEM), head_dim 64, warp-specialised.
//
// One CTA (one per SM) computes 256 query rows of one head of one sequence as
// two 128-row tiles, A and B, that share every 128-key K/V tile:
//   warp 8   TMA producer: Q_A, Q_B once, then K/V tiles (128 keys x 64 dims,
//            16 KB each) into a 4-stage ring (cp.async.bulk.tensor, 128-byte
//            swizzle, no multicast)
//   warp 9   MMA issuer (whole warp, one elected lane issues):
//              S_q  = Q_q K_j^T       tcgen05.mma kind::f16, M=128 N=128 K=64,
//                                     f32 accumulator in TMEM
//              O_q += P_q,j V_j       M=128 N=64 K=128, f16 P read from TMEM (TS
//                                     form), f16 V; O accumulated in TMEM across
//                                     all key tiles
//   warps 10-11  (bf16 inputs) convert each V tile in shared memory to f16,
//            in place, scaled by 2^-E (below)
//   warps 0-3 / 4-7  softmax for tile A / B, one thread per query row (= TMEM
//            lane): the whole 128-key S row in registers, causal mask on the
//            diagonal tile, row max and sum in the log2 domain without any
//            exchange between threads; P goes back to TMEM over the S columns
//            it came from as f16.
// Why f16 for P V: P in [0, 256] as bf16 (8 significant bits) puts the output
// ~3e-3 off for unit-scale inputs; f16 (11 bits) keeps it within ~5e-4, inside
// the 2e-3 bar.  The tensor core takes one type for both operands, so bf16 V
// becomes f16 as V * 2^-E.  E starts at 0 and is raised (never lowered) when a
// tile holds an |entry| >= 2^(15+E), so no scaled entry overflows f16; O is
// kept in units of 2^E, rescaled with the running max when E moves, and the
// final O is multiplied back by 2^E.  Entries below 2^-14 * 2^E lose relative
// precision in f16 (absolute error <= 2^-25 * 2^E each).
// Lazy rescaling: the running max m is raised only when a tile's max exceeds it
// by more than 2^8; P = 2^(s - m) then stays below 256, and O (in TMEM) and the
// row sum are rescaled only on those rare raises.  When the softmax thread holds
// S_q(j), every MMA issued before S_q(j) -- P_q(j-1) V_(j-1) included -- has
// completed (a commit tracks all earlier MMAs of the issuing thread), so the
// thread may rescale its O row in place before it hands P_q(j) back.
// Issue order per key tile j: P_A(j) V_j, S_A(j+1), P_B(j) V_j, S_B(j+1): while
// one tile's softmax runs, the tensor core works on the other tile.  S_q(j+1)
// overwrites the TMEM columns that P_q(j) V_j reads; MMAs issued by one thread
// execute in issue order, so the read precedes the overwrite.
// Every mbarrier wait is bounded; a failed wait sets a CTA-wide flag that
// every role checks before its next wait; TMEM is freed on every path.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kPfRows = 128;                      // rows per Q tile (MMA M)
constexpr int kPfTiles = 2;                       // Q tiles per CTA
constexpr int kPfKeys = 128;                      // keys per K/V tile (S MMA N)
constexpr int kPfStages = 4;                      // K/V ring depth
constexpr int kPfQBytes = kPfRows * 64 * 2;       // 16 KB
constexpr int kPfKVBytes = kPfKeys * 64 * 2;      // 16 KB (K or V)
constexpr int kPfSmemBytes = kPfTiles * kPfQBytes + kPfStages * 2 * kPfKVBytes + 1024;
constexpr int kPfSoftmaxWarps = 8;                // 4 per Q tile, one thread per row
constexpr int kTmaWarp = kPfSoftmaxWarps, kMmaWarp = kPfSoftmaxWarps + 1;
constexpr int kConvWarp = kPfSoftmaxWarps + 2;    // two V-conversion warps
constexpr int kPfThreads = (kPfSoftmaxWarps + 4) * 32;
constexpr int kMaxVShift = 112;                   // E cap (2^-E stays a normal f32)
// S_A, S_B (128 columns each, P over them), O_A, O_B (64 each): 384 of 512.
constexpr uint32_t kPfTmemCols = 512;
constexpr uint32_t kPfTmemO = 2 * kPfKeys;
constexpr float kPfRescaleLog2 = 8.0f;            // raise m only past 2^8

struct PrefillArgs {
    int t, pos0, n_q, n_kv, group, n_qblocks;
    float scale_log2;
    uint16_t* out;
    long long out_row_stride;
};

struct PrefillBars {
    uint64_t q_full;
    uint64_t kv_full[kPfStages], kv_empty[kPfStages];
    uint64_t s_full[kPfTiles];   // S_q(j) in TMEM (phase j)
    uint64_t p_full[kPfTiles];   // P_q(j) in TMEM, O_q row rescaled (128 arrivals, phase j)
    uint64_t o_done[kPfTiles];   // last P_q V completed: O_q final
    uint64_t v_ready[kPfStages]; // V tile of the stage converted to f16 (64 arrivals)
    uint64_t mma_done;           // every MMA of the CTA has completed (before TMEM is freed)
};

__device__ __forceinline__ bool warp_all(bool p) { return __all_sync(0xffffffffu, p); }

// f32 pair -> packed f16x2 (round to nearest even), a in the low half.
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}
// Nonzero if either bf16 half of w has |x| >= the bf16 magnitude `thr` (thr <=
// 0x7f80): 15-bit magnitudes plus (0x8000 - thr) carry into bit 15 exactly then.
__device__ __forceinline__ uint32_t bf16x2_at_least(uint32_t w, uint32_t add2) {
    return ((w & 0x7fff7fffu) + add2) & 0x80008000u;
}

// ---- packed f32x2 arithmetic (one instruction for two lanes of f32 work)
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// 2^x for a pair on the FMA pipe, to take load off the MUFU unit that ex2.approx
// uses.  x = n + f with n = round(x) (added to the exponent field) and f in
// [-1/2, 1/2], where a degree-3 polynomial fitted here to 2^f (weighted least
// squares on Chebyshev nodes, max relative error 7.5e-5, below the 2^-11
// rounding of the f16 P it feeds) supplies the mantissa.  x is clamped to
// [-126, 2^22]: below 2^-126 the result is not a number of any consequence to
// a softmax weight.  round(x) comes from adding 1.5 * 2^23, which leaves it in
// the low mantissa bits of the sum.
__device__ __forceinline__ void exp2_poly_pair(float& x0, float& x1) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const uint64_t x = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
    const uint64_t magic = f2_pack(kMagic, kMagic);
    const uint64_t t = f2_add(x, magic);
    const uint64_t f = f2_sub(x, f2_sub(t, magic));
    uint64_t p = f2_fma(f2_pack(0.055171654f, 0.055171654f), f, f2_pack(0.24261113f, 0.24261113f));
    p = f2_fma(p, f, f2_pack(0.69326097f, 0.69326097f));
    p = f2_fma(p, f, f2_pack(0.99992806f, 0.99992806f));
    float p0, p1, t0, t1;
    f2_unpack(p, p0, p1);
    f2_unpack(t, t0, t1);
    x0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
    x1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

template <typename T>
// 12 warps, three per SM sub-partition (16K registers each): at most 168 registers.
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ PrefillBars bars;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_err;
    __shared__ int v_shift[kPfStages];      // E in force for the stage's converted V tile
    __shared__ uint32_t conv_xchg[2][2];    // per conversion warp: overflow flag, max magnitude
    constexpr bool kConvertV = Elem<T>::kDtype == KVB_BF16;
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
            mbar_init(&bars.v_ready[s], 64);
            v_shift[s] = 0;
        }
        for (int q = 0; q < kPfTiles; ++q) {
            mbar_init(&bars.s_full[q], 1);
            mbar_init(&bars.p_full[q], kPfRows);
            mbar_init(&bars.o_done[q], 1);
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
        // The whole warp runs this loop converged; umma_* / umma_commit issue from
        // one elected lane.  Wait results are made warp-uniform.
        const uint32_t idesc_s = idesc_f16(kPfRows, kPfKeys, fmt, 0, 0);
        const uint32_t idesc_o = idesc_f16(kPfRows, 64, 0, 0, 1);  // f16 P, f16 V
        // Descriptors are built once; per MMA only the 16-byte start-address field
        // (bits 0-13) moves, by adding a constant.
        const uint64_t dq0 = sdesc_sw128(smem_u32(sq), 16, 1024);
        const uint64_t dk0 = sdesc_sw128(smem_u32(skv), 16, 1024);
        const uint64_t dv0 = sdesc_sw128(smem_u32(skv) + kPfKVBytes, 64 * 128, 1024);
        constexpr uint64_t kQTile = kPfQBytes >> 4, kStage = (2 * kPfKVBytes) >> 4;
        // S_q = Q_q K_j^T: four K=16 steps of 32 bytes along the 128-byte rows.
        auto issue_s = [&](int q, int j) {
            const uint32_t d = tmem + (uint32_t)(q * kPfKeys);
            const uint64_t da = dq0 + kQTile * q, db = dk0 + kStage * (j % kPfStages);
            umma_f16(d, da, db, idesc_s, 0);
            umma_f16(d, da + 2, db + 2, idesc_s, 1);
            umma_f16(d, da + 4, db + 4, idesc_s, 1);
            umma_f16(d, da + 6, db + 6, idesc_s, 1);
            umma_commit(&bars.s_full[q]);
        };
        // O_q += P_q V_j: f16 P in the S columns 0-63 (keys 2c, 2c+1 in column c);
        // V_j read MN-major, 16 keys (2048 bytes) per step.
        auto issue_pv = [&](int q, int j) {
            const uint32_t d = tmem + kPfTmemO + (uint32_t)(q * 64);
            const uint32_t p = tmem + (uint32_t)(q * kPfKeys);
            const uint64_t dv = dv0 + kStage * (j % kPfStages);
            umma_f16_ts(d, p, dv, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
            for (int k = 1; k < 8; ++k) umma_f16_ts(d, p + 8 * k, dv + 128 * k, idesc_o, 1);
        };
        bool ok = warp_all(mbar_wait(&bars.q_full, 0) && mbar_wait(&bars.kv_full[0], 0));
        for (int q = 0; q < kPfTiles && ok; ++q)
            if (n_tiles(q) > 0) issue_s(q, 0);
        int kv_ready = 0;  // highest key tile known to be in shared memory
        for (int j = 0; j < n_kv_tiles && ok; ++j) {
            for (int q = 0; q < kPfTiles && ok; ++q) {
                if (j >= n_tiles(q)) continue;
                ok = warp_all(!s_err && mbar_wait(&bars.p_full[q], j & 1) &&
                              (!kConvertV || mbar_wait(&bars.v_ready[j % kPfStages],
                                                       (j / kPfStages) & 1)));
                if (!ok) break;
                tc_fence_after();
                issue_pv(q, j);
                if (j + 1 < n_tiles(q)) {
                    if (kv_ready < j + 1) {
                        ok = warp_all(mbar_wait(&bars.kv_full[(j + 1) % kPfStages],
                                                ((j + 1) / kPfStages) & 1));
                        if (!ok) break;
                        kv_ready = j + 1;
                    }
                    issue_s(q, j + 1);
                } else {
                    umma_commit(&bars.o_done[q]);
                }
            }
            if (ok) umma_commit(&bars.kv_empty[j % kPfStages]);  // stage free once these finish
        }
        if (!ok && lane == 0) s_err = 1;
        // No MMA may still be running when TMEM is released below.
        umma_commit(&bars.mma_done);
        mbar_wait(&bars.mma_done, 0);
        __syncwarp();
    } else if (warp >= kConvWarp) {
        // ------------------------------------------------------------ V conversion
        // Warp kConvWarp + c converts 16-byte chunks c*32 + lane + 64 i of the V
        // tile (all 1024 chunks between the two warps) from bf16 to f16 * 2^-E.
        if constexpr (kConvertV) {
            const int cw = warp - kConvWarp;
            const int ct = cw * 32 + lane;
            int e = 0;  // E: V is stored as V * 2^-E
            bool ok = true;
            for (int j = 0; j < n_kv_tiles; ++j) {
                const int st = j % kPfStages;
                const bool here = warp_all(!s_err && mbar_wait(&bars.kv_full[st], (j / kPfStages) & 1));
                uint4* vt = reinterpret_cast<uint4*>(skv + (2 * st + 1) * kPfKVBytes);
                uint4 w[16];
                // |v| >= 2^(15 + E): bf16 magnitude (127 + 15 + E) << 7
                const uint32_t thr = (uint32_t)min(127 + 15 + e, 255) << 7;
                const uint32_t add = 0x8000u - min(thr, 0x7f80u);
                const uint32_t add2 = add | (add << 16);
                uint32_t big = 0;
                if (here) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        w[i] = vt[ct + 64 * i];
                        big |= bf16x2_at_least(w[i].x, add2) | bf16x2_at_least(w[i].y, add2) |
                               bf16x2_at_least(w[i].z, add2) | bf16x2_at_least(w[i].w, add2);
                    }
                }
                // Both warps must agree on failure and on E for the tile: exchange the
                // flags (and, on the rare overflow path, the largest magnitude) through
                // shared memory; both warps pass every named barrier of an iteration.
                const bool any_big = __any_sync(0xffffffffu, big != 0);
                if (lane == 0) conv_xchg[cw][0] = (any_big ? 1u : 0u) | (here ? 0u : 2u);
                named_bar_sync(1, 64);
                const uint32_t flags = conv_xchg[0][0] | conv_xchg[1][0];
                if (flags & 2u) {
                    ok = false;
                    break;
                }
                if (flags & 1u) {
                    uint32_t mag = 0;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mag = max(mag, max(u[k] & 0x7fffu, (u[k] >> 16) & 0x7fffu));
                    }
                    mag = __reduce_max_sync(0xffffffffu, mag);
                    if (lane == 0) conv_xchg[cw][1] = mag;
                    named_bar_sync(1, 64);
                    mag = max(conv_xchg[0][1], conv_xchg[1][1]);
                    // largest |v| < 2^(x - 126) with x = its biased exponent: E >= x - 141
                    e = min(max(e, (int)(mag >> 7) - 141), kMaxVShift);
                }
                const float sc = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-E
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float lo = __uint_as_float(u[k] << 16) * sc;
                        const float hi = __uint_as_float(u[k] & 0xffff0000u) * sc;
                        u[k] = pack_f16x2(lo, hi);
                    }
                    vt[ct + 64 * i] = make_uint4(u[0], u[1], u[2], u[3]);
                }
                if (ct == 0) v_shift[st] = e;
                fence_async_smem();  // generic-proxy writes -> visible to the tensor core
                mbar_arrive(&bars.v_ready[st]);
                named_bar_sync(1, 64);  // conv_xchg is reused by the next tile
            }
            if (!ok && lane == 0) s_err = 1;
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        // Warp w serves tile w >> 2 and TMEM lanes 32 (w & 3) .. +31: thread = row.
        // Wait results are made warp-uniform (tcgen05.ld / st are warp-collective).
        const int q = warp >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t t_s = tmem + (uint32_t)(q * kPfKeys) + lane_off;       // S, then P
        const uint32_t t_o = tmem + kPfTmemO + (uint32_t)(q * 64) + lane_off;  // O
        const int my_pos = a.pos0 + q0 + q * kPfRows + row;
        const int diag_key = a.pos0 + q0 + q * kPfRows;  // keys above need the causal mask
        const int nt = n_tiles(q);
        float m = -INFINITY, l = 0.f;  // running max (log2 units) and row sum
        int e_cur = 0;                 // E of the V tiles accumulated into O so far
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            ok = warp_all(!s_err && mbar_wait(&bars.s_full[q], j & 1));
            if (!ok) break;
            tc_fence_after();
            float s[kPfKeys];
            tmem_ld32(t_s, s);
            tmem_ld32(t_s + 32, s + 32);
            tmem_ld32(t_s + 64, s + 64);
            tmem_ld32(t_s + 96, s + 96);
            tmem_wait_ld();
            if (j * kPfKeys + kPfKeys - 1 > diag_key) {
#pragma unroll
                for (int c = 0; c < kPfKeys; ++c)
                    if (j * kPfKeys + c > my_pos) s[c] = -INFINITY;
            }
            float mx8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
            for (int c = 8; c < kPfKeys; c += 16)
#pragma unroll
                for (int i = 0; i < 8; ++i) mx8[i] = max3f(mx8[i], s[c + i], s[c + 8 + i]);
            // Raw scores: the max is taken before scaling (the scale is positive).
            const float mt = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]),
                                   fmaxf(mx8[6], mx8[7])) *
                             a.scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m + kPfRescaleLog2) {  // always at j = 0 (m = -inf; row 0 of a tile sees key 0)
                alpha = ex2_approx(m - mt);  // 0 at j = 0
                rescale = j > 0;
                m = mt;
            }
            // V_j's scale: O (in units of 2^E) follows E before P_j V_j is added.
            int de = 0;
            if (kConvertV) {
                ok = warp_all(!s_err && mbar_wait(&bars.v_ready[j % kPfStages], (j / kPfStages) & 1));
                if (!ok) break;
                const int e_j = v_shift[j % kPfStages];
                if (j > 0) de = e_j - e_cur;
                e_cur = e_j;
            }
            // P_j = 2^(s*scale - m) <= 2^8 -> TMEM as f16 over the S columns 0-63 (keys
            // 2c, 2c+1 in column c), 32 keys at a time so that each store is in flight
            // while the next keys are computed.  One key pair in four takes 2^x from
            // the FMA pipe, the others from MUFU.  This thread's S loads completed above.
            uint64_t sum2[4] = {0, 0, 0, 0};  // four f32 pairs of partial row sums (+0.0f bits)
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                uint32_t pk[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    float p0 = fmaf(s[32 * ch + 2 * k], a.scale_log2, -m);
                    float p1 = fmaf(s[32 * ch + 2 * k + 1], a.scale_log2, -m);
                    if ((k & 3) == 0) {
                        exp2_poly_pair(p0, p1);
                    } else {
                        p0 = ex2_approx(p0);
                        p1 = ex2_approx(p1);
                    }
                    sum2[k & 3] = f2_add(sum2[k & 3], f2_pack(p0, p1));
                    pk[k] = pack_f16x2(p0, p1);
                }
                tmem_st16(t_s + 16 * ch, pk);
            }
            float r0, r1, r2, r3, r4, r5, r6, r7;
            f2_unpack(f2_add(sum2[0], sum2[1]), r0, r1);
            f2_unpack(f2_add(sum2[2], sum2[3]), r2, r3);
            (void)r4; (void)r5; (void)r6; (void)r7;
            l = l * alpha + ((r0 + r1) + (r2 + r3));
            if (__any_sync(0xffffffffu, rescale) || de != 0) {  // O row *= f (O is idle, see above; S is dead)
                const float f = (rescale ? alpha : 1.f) * __uint_as_float((uint32_t)(127 - de) << 23);
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float o[32];
                    tmem_ld32(t_o + 32 * hf, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int d = 0; d < 32; ++d) o[d] *= f;
                    tmem_st32(t_o + 32 * hf, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars.p_full[q]);
        }
        if (ok && nt > 0) {
            ok = warp_all(!s_err && mbar_wait(&bars.o_done[q], 0));
            if (ok) {
                tc_fence_after();
                const float inv = __uint_as_float((uint32_t)(127 + e_cur) << 23) / l;  // 2^E / l
                const bool valid = row < (q ? rows_valid1 : rows_valid0);
                T* orow = reinterpret_cast<T*>(a.out) +
                          ((size_t)seq * a.t + q0 + q * kPfRows + row) * a.out_row_stride +
                          (size_t)h * 64;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float o[32];
                    tmem_ld32(t_o + 32 * hf, o);
                    tmem_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            float f[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) f[e] = o[8 * k + e] * inv;
                            *reinterpret_cast<uint4*>(orow + 32 * hf + 8 * k) = pack8<T>(f);
                        }
                    }
                }
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
