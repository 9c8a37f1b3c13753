// attn_prefill.cuh -- causal GQA prefill attention on the 5th-generation
// tensor cores (tcgen05 / TMEM), head_dim 64, warp-specialised.
//
// One CTA computes one 128-row query tile of one head of one sequence; two
// CTAs share an SM (256 TMEM columns and ~89 KB of shared memory each), so
// that while one CTA's softmax waits for its tensor-core work the other one's
// runs -- two independent pipelines, nothing shared between them:
//   warp 4   TMA producer: Q once, then 96-key K/V tiles (12 KB each) into a
//            3-stage ring (cp.async.bulk.tensor, 128-byte swizzle, no multicast)
//   warp 5   MMA issuer (whole warp, one elected lane issues):
//              S  = Q K_j^T       tcgen05.mma kind::f16, M=128 N=96 K=64, f32 in
//                                 TMEM, two S buffers (tile j in buffer j & 1)
//              O += P_j V_j       M=128 N=64, P read from TMEM (TS form); O
//                                 accumulated in TMEM across all key tiles
//   warps 0-3  softmax, one thread per query row (= TMEM lane): the 96-key S
//            row in registers, causal mask on the diagonal tiles, row max and
//            sum in the log2 domain without any exchange between threads.
// TMEM: S0 columns 0-95, S1 96-191, O 192-255.  96-key tiles are what lets two
// S buffers and O fit the 256 columns of a CTA: S(j+1) is computed while the
// softmax threads work on S(j).  Issue order P(j) V(j), S(j+2): S(j+2) reuses
// the buffer of P(j), which P(j) V(j) has read -- MMAs issued by one thread
// execute in issue order.
// P goes back to TMEM over the S columns it came from.  bf16 inputs: P as a
// bf16 head (columns 0-47 of the buffer, the truncated upper half of each f32)
// plus a bf16 remainder (48-95), two
// MMAs per key step, so P keeps ~16 significant bits (bf16 P alone, 8 bits,
// puts the output ~3e-3 off for unit-scale inputs, outside the 2e-3 bar).
// f16 inputs: P as one f16 (columns 0-47), within ~5e-4.
// Lazy rescaling: the running max m is raised only when a tile's max exceeds it
// by more than 2^8; P = 2^(s - m) then stays below 256, and O (in TMEM) and the
// row sum are rescaled only on those rare raises, after the previous P V has
// finished writing O.
// Every mbarrier wait is bounded; a failed wait sets a CTA-wide flag that
// every role checks before its next wait; TMEM is freed on every path.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

constexpr int kPfRows = 128;                      // query rows per CTA (MMA M)
constexpr int kPfKeys = 96;                       // keys per K/V tile (S MMA N)
constexpr int kPfStages = 3;                      // K/V ring depth
constexpr int kPfQBytes = kPfRows * 64 * 2;       // 16 KB
constexpr int kPfKVBytes = kPfKeys * 64 * 2;      // 12 KB (K or V)
constexpr int kPfSmemBytes = kPfQBytes + kPfStages * 2 * kPfKVBytes + 1024;
constexpr int kPfSoftmaxWarps = 4;                // one thread per row
constexpr int kTmaWarp = kPfSoftmaxWarps, kMmaWarp = kPfSoftmaxWarps + 1;
constexpr int kPfThreads = (kPfSoftmaxWarps + 2) * 32;
constexpr int kPfCtasPerSm = 2;
// S[2] (96 columns each, P over them), then O (64): all 256.
constexpr uint32_t kPfTmemCols = 256;
constexpr uint32_t kPfTmemO = 2 * kPfKeys;
constexpr int kPfPCols = kPfKeys / 2;             // 16-bit P: two keys per column
constexpr float kPfRescaleLog2 = 8.0f;            // raise m only past 2^8

struct PrefillArgs {
    int t, pos0, n_q, n_kv, group, n_qblocks;
    float scale_log2;
    uint16_t* out;
    long long out_row_stride;
    // Paged cache (block_table != nullptr): kmap / vmap are 2-D maps over the pools'
    // rows of 64 elements ([n_blocks][n_kv][block_size] rows, box 32 rows); key k of
    // sequence s is row (block_table[s * max_blocks + k / block_size] * n_kv + kvh)
    // * block_size + k % block_size, block_size a multiple of 32.
    const int32_t* block_table;
    int max_blocks, block_size, n_blocks;
};
constexpr int kPfPagedPiece = 32;                 // rows per paged tensor copy (4 KB)
constexpr int kPfTableSmem = 1024;                // block-table entries cached in smem
constexpr int kPfPagedPieces = kPfKeys / kPfPagedPiece;

struct PrefillBars {
    uint64_t q_full;
    uint64_t kv_full[kPfStages], kv_empty[kPfStages];
    // One S-ready and one P-ready barrier per S buffer (tile j uses buffer j & 1):
    // a thread that runs a tile ahead arrives on the other buffer's barrier.
    uint64_t s_full[2];
    uint64_t p_full[2];  // 128 arrivals
    // P(j) V(j) has completed (phase j).  A softmax thread holding S(j) knows
    // P(j-2) V completed (S(j) was issued after it), so only P(j-1) V can be
    // pending when it waits here: a parity wait is unambiguous there.
    uint64_t pv_done;
    uint64_t o_done;     // last P V completed: O final (one phase)
    uint64_t mma_done;   // every MMA of the CTA has completed (before TMEM is freed)
};

__device__ __forceinline__ bool warp_all(bool p) { return __all_sync(0xffffffffu, p); }

// f32 pair -> packed f16x2 (round to nearest even), a in the low half.
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
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
// Two f32 as a packed bf16 head (the upper halves of their bit patterns, i.e.
// truncated) and the packed bf16 remainder (p - head, rounded): the pair keeps
// ~16 significant bits.  prmt picks bytes 2-3 of each operand.
__device__ __forceinline__ void split_bf16_pair(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(hi) : "r"(__float_as_uint(p0)), "r"(__float_as_uint(p1)));
    float r0, r1;
    f2_unpack(f2_sub(f2_pack(p0, p1), f2_pack(__uint_as_float(__float_as_uint(p0) & 0xffff0000u),
                                              __uint_as_float(__float_as_uint(p1) & 0xffff0000u))),
              r0, r1);
    lo = Elem<__nv_bfloat16>::pack(r0, r1);
}

// kOutF32: the rows are written as f32 (a.out holds floats), the values that the
// 16-bit form rounds once.
template <typename T, bool kOutF32 = false>
// 2 CTAs x 6 warps: three warps on each SM sub-partition (16K registers each),
// at most 168 registers a thread.
__global__ void __launch_bounds__(kPfThreads, kPfCtasPerSm)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ PrefillBars bars;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_err;
    __shared__ int s_table[kPfTableSmem];  // paged: this sequence's block-table row
    // bf16: P as head + remainder (two MMAs per key step); f16: P as one f16.
    constexpr bool kSplitP = Elem<T>::kDtype == KVB_BF16;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* sq = smem;                  // Q
    uint8_t* skv = sq + kPfQBytes;       // [stage][K | V]

    const int h = blockIdx.x, seq = blockIdx.y;
    const int qb = a.n_qblocks - 1 - (int)blockIdx.z;    // longest blocks first
    const int q0 = qb * kPfRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = h / a.group;
    const int kv_plane = seq * a.n_kv + kvh;
    const int rows_valid = max(0, min(kPfRows, a.t - q0));
    // key tiles this query tile visits (causal)
    const int nt = rows_valid ? (a.pos0 + q0 + rows_valid + kPfKeys - 1) / kPfKeys : 0;

    if (tid == 0) {
        mbar_init(&bars.q_full, 1);
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&bars.kv_full[s], 1);
            mbar_init(&bars.kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars.s_full[b], 1);
            mbar_init(&bars.p_full[b], kPfRows);
        }
        mbar_init(&bars.pv_done, 1);
        mbar_init(&bars.o_done, 1);
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
        // Paged: the whole warp first copies the blocks this CTA visits into shared
        // memory (one global read per block, not per tile piece on the issuing lane).
        const int seq_len = a.pos0 + a.t;
        const int kv_end = min(seq_len, nt * kPfKeys);
        const bool pow2 = a.block_table && (a.block_size & (a.block_size - 1)) == 0;
        const int bs_shift = pow2 ? __ffs(a.block_size) - 1 : 0;
        const int n_lb = a.block_table ? (kv_end + a.block_size - 1) / a.block_size : 0;
        const bool cached = n_lb <= kPfTableSmem;
        if (a.block_table && cached) {
            for (int i = lane; i < n_lb; i += 32)
                s_table[i] = i < a.max_blocks ? a.block_table[(size_t)seq * a.max_blocks + i]
                                              : a.n_blocks;  // reported below
            __syncwarp();
        }
        if (lane == 0 && nt > 0) {
            tma_prefetch_desc(&kmap);
            tma_prefetch_desc(&vmap);
            mbar_expect_tx(&bars.q_full, kPfQBytes);
            tma_load_3d(sq, &qmap, &bars.q_full, h * 64, q0, seq);
            int issued = 0;
            // Paged: block of each 32-key piece of a tile (kPastEnd: past the sequence end);
            // the next tile's entries are read while this one's copies are in flight.
            constexpr int kPastEnd = -2147483647 - 1;
            auto piece_block = [&](int k) -> int {
                if (k >= seq_len) return kPastEnd;
                const int lb = pow2 ? k >> bs_shift : k / a.block_size;
                if (cached) return s_table[lb];
                return lb < a.max_blocks ? a.block_table[(size_t)seq * a.max_blocks + lb]
                                         : a.n_blocks;  // reported below
            };
            int nblk[kPfPagedPieces];
            if (a.block_table) {
#pragma unroll
                for (int i = 0; i < kPfPagedPieces; ++i) nblk[i] = piece_block(i * kPfPagedPiece);
            }
            for (int j = 0; j < nt; ++j) {
                const int st = j % kPfStages;
                if (j >= kPfStages && !mbar_wait(&bars.kv_empty[st], ((j - kPfStages) / kPfStages) & 1)) {
                    s_err = 1;
                    break;
                }
                if (s_err) break;
                uint8_t* kdst = skv + (2 * st) * kPfKVBytes;
                uint8_t* vdst = kdst + kPfKVBytes;
                if (!a.block_table) {
                    mbar_expect_tx(&bars.kv_full[st], 2 * kPfKVBytes);
                    tma_load_3d(kdst, &kmap, &bars.kv_full[st], 0, j * kPfKeys, kv_plane);
                    tma_load_3d(vdst, &vmap, &bars.kv_full[st], 0, j * kPfKeys, kv_plane);
                } else {
                    // 32-key pieces, each inside one block; pieces past the sequence end
                    // are not loaded (the MMA warp zeroes those V rows).  A table entry
                    // outside the pool is reported and read as zeros (rows past the map).
                    int rows[kPfPagedPieces];
                    uint32_t bytes = 0;
#pragma unroll
                    for (int i = 0; i < kPfPagedPieces; ++i) {
                        const int k = j * kPfKeys + i * kPfPagedPiece;
                        const int blk = nblk[i];
                        rows[i] = -1;
                        if (blk == kPastEnd) continue;
                        if (blk < 0 || blk >= a.n_blocks) {
                            raise_dev_error(kDevErrBadPosition);
                            rows[i] = a.n_blocks * a.n_kv * a.block_size;
                        } else {
                            rows[i] = (blk * a.n_kv + kvh) * a.block_size +
                                      (pow2 ? k & (a.block_size - 1) : k % a.block_size);
                        }
                        bytes += 2 * kPfPagedPiece * 128;
                    }
                    mbar_expect_tx(&bars.kv_full[st], bytes);
#pragma unroll
                    for (int i = 0; i < kPfPagedPieces; ++i) {
                        if (rows[i] < 0) continue;
                        tma_load_2d(kdst + i * kPfPagedPiece * 128, &kmap, &bars.kv_full[st], 0,
                                    rows[i]);
                        tma_load_2d(vdst + i * kPfPagedPiece * 128, &vmap, &bars.kv_full[st], 0,
                                    rows[i]);
                    }
                    if (j + 1 < nt) {
#pragma unroll
                        for (int i = 0; i < kPfPagedPieces; ++i)
                            nblk[i] = piece_block((j + 1) * kPfKeys + i * kPfPagedPiece);
                    }
                }
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
        const uint32_t idesc_o = idesc_f16(kPfRows, 64, fmt, 0, 1);
        // Descriptors are built once; per MMA only the 16-byte start-address field
        // (bits 0-13) moves, by adding a constant.
        const uint64_t dq = sdesc_sw128(smem_u32(sq), 16, 1024);
        const uint64_t dk0 = sdesc_sw128(smem_u32(skv), 16, 1024);
        const uint64_t dv0 = sdesc_sw128(smem_u32(skv) + kPfKVBytes, 64 * 128, 1024);
        constexpr uint64_t kStage = (2 * kPfKVBytes) >> 4;
        // S = Q K_j^T: four K=16 steps of 32 bytes along the 128-byte rows.
        auto issue_s = [&](int j) {
            const uint32_t d = tmem + (uint32_t)((j & 1) * kPfKeys);
            const uint64_t db = dk0 + kStage * (j % kPfStages);
            umma_f16(d, dq, db, idesc_s, 0);
            umma_f16(d, dq + 2, db + 2, idesc_s, 1);
            umma_f16(d, dq + 4, db + 4, idesc_s, 1);
            umma_f16(d, dq + 6, db + 6, idesc_s, 1);
            umma_commit(&bars.s_full[j & 1]);
        };
        // O += P_j V_j: P (head, then remainder for bf16) in the S columns, two keys
        // per column; V_j read MN-major, 16 keys (2048 bytes) per step.
        auto issue_pv = [&](int j) {
            const uint32_t d = tmem + kPfTmemO;
            const uint32_t p = tmem + (uint32_t)((j & 1) * kPfKeys);
            const uint64_t dv = dv0 + kStage * (j % kPfStages);
            umma_f16_ts(d, p, dv, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
            for (int k = 1; k < kPfKeys / 16; ++k) umma_f16_ts(d, p + 8 * k, dv + 128 * k, idesc_o, 1);
            if (kSplitP) {
#pragma unroll
                for (int k = 0; k < kPfKeys / 16; ++k)
                    umma_f16_ts(d, p + kPfPCols + 8 * k, dv + 128 * k, idesc_o, 1);
            }
            umma_commit(&bars.pv_done);
        };
        bool ok = nt > 0 && warp_all(mbar_wait(&bars.q_full, 0));
        for (int j = 0; j < 2 && j < nt && ok; ++j) {  // S for key tiles 0 and 1
            ok = warp_all(mbar_wait(&bars.kv_full[j % kPfStages], (j / kPfStages) & 1));
            if (ok) issue_s(j);
        }
        for (int j = 0; j < nt && ok; ++j) {
            ok = warp_all(!s_err && mbar_wait(&bars.p_full[j & 1], (j >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            if (a.block_table && (j + 1) * kPfKeys > a.pos0 + a.t) {
                // Paged: V rows past the sequence end hold whatever the pool holds there
                // (a contiguous map reads zeros); P is 0 on them, but 0 * NaN is not 0.
                uint4* vt = reinterpret_cast<uint4*>(skv + (2 * (j % kPfStages) + 1) * kPfKVBytes);
                for (int i = (a.pos0 + a.t - j * kPfKeys) * 8 + lane; i < kPfKeys * 8; i += 32)
                    vt[i] = make_uint4(0u, 0u, 0u, 0u);
                fence_async_smem();
                __syncwarp();
            }
            issue_pv(j);  // then S(j + 2) reuses buffer j & 1 (read by this P V first)
            if (j + 1 == nt) umma_commit(&bars.o_done);
            if (j + 2 < nt) {
                ok = warp_all(mbar_wait(&bars.kv_full[(j + 2) % kPfStages], ((j + 2) / kPfStages) & 1));
                if (!ok) break;
                issue_s(j + 2);
            }
            umma_commit(&bars.kv_empty[j % kPfStages]);  // stage free once these finish
        }
        if (!ok && nt > 0 && lane == 0) s_err = 1;
        // No MMA may still be running when TMEM is released below.
        umma_commit(&bars.mma_done);
        mbar_wait(&bars.mma_done, 0);
        __syncwarp();
    } else {
        // ------------------------------------------------------------ softmax warps
        // Warp w serves TMEM lanes 32 w .. +31: thread = row.  Wait results are made
        // warp-uniform (tcgen05.ld / st are warp-collective).
        const int row = warp * 32 + lane;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const uint32_t t_o = tmem + kPfTmemO + lane_off;  // O
        const int my_pos = a.pos0 + q0 + row;
        const int diag_key = a.pos0 + q0;  // keys above need the causal mask
        float m = -INFINITY, l = 0.f;      // running max (log2 units) and row sum
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            const uint32_t t_s = tmem + (uint32_t)(b * kPfKeys) + lane_off;  // S, then P
            ok = warp_all(!s_err && mbar_wait(&bars.s_full[b], (j >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            float s[kPfKeys];
#pragma unroll
            for (int c = 0; c < kPfKeys; c += 32) tmem_ld32(t_s + c, s + c);
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
            for (int c = 8; c + 16 <= kPfKeys; c += 16)
#pragma unroll
                for (int i = 0; i < 8; ++i) mx8[i] = max3f(mx8[i], s[c + i], s[c + 8 + i]);
            if ((kPfKeys - 8) % 16 != 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(mx8[i], s[kPfKeys - 8 + i]);
            }
            // Raw scores: the max is taken before scaling (the scale is positive).
            const float mt = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]),
                                   fmaxf(mx8[6], mx8[7])) *
                             a.scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m + kPfRescaleLog2) {  // always at j = 0 (m = -inf; every row sees key 0)
                alpha = ex2_approx(m - mt);  // 0 at j = 0
                rescale = j > 0;
                m = mt;
            }
            // P_j = 2^(s*scale - m) <= 2^8 -> TMEM over the S columns (keys 2c, 2c+1 in
            // column c; bf16 remainders in columns 48 + c), 32 keys at a time.  This
            // thread's S loads completed above.
            uint64_t sum2[4] = {0, 0, 0, 0};  // four f32 pairs of partial row sums (+0.0f bits)
#pragma unroll
            for (int ch = 0; ch < kPfKeys / 32; ++ch) {
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float p0 = ex2_approx(fmaf(s[32 * ch + 2 * k], a.scale_log2, -m));
                    const float p1 = ex2_approx(fmaf(s[32 * ch + 2 * k + 1], a.scale_log2, -m));
                    sum2[k & 3] = f2_add(sum2[k & 3], f2_pack(p0, p1));
                    if (kSplitP) split_bf16_pair(p0, p1, ph[k], pl[k]);
                    else ph[k] = pack_f16x2(p0, p1);
                }
                tmem_st16(t_s + 16 * ch, ph);
                if (kSplitP) tmem_st16(t_s + kPfPCols + 16 * ch, pl);
            }
            float r0, r1, r2, r3;
            f2_unpack(f2_add(sum2[0], sum2[1]), r0, r1);
            f2_unpack(f2_add(sum2[2], sum2[3]), r2, r3);
            l = l * alpha + ((r0 + r1) + (r2 + r3));
            if (__any_sync(0xffffffffu, rescale)) {
                // O row *= alpha, once P(j-1) V(j-1) has finished writing O
                ok = warp_all(!s_err && mbar_wait(&bars.pv_done, (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const float f = rescale ? alpha : 1.f;
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
            mbar_arrive(&bars.p_full[b]);
        }
        if (ok && nt > 0) {
            ok = warp_all(!s_err && mbar_wait(&bars.o_done, 0));
            if (ok) {
                tc_fence_after();
                const float inv = 1.f / l;
                const bool valid = row < rows_valid;
                const size_t orow_off =
                    ((size_t)seq * a.t + q0 + row) * a.out_row_stride + (size_t)h * 64;
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
                            if constexpr (kOutF32) {
                                float4* orow = reinterpret_cast<float4*>(
                                    reinterpret_cast<float*>(a.out) + orow_off + 32 * hf + 8 * k);
                                orow[0] = make_float4(f[0], f[1], f[2], f[3]);
                                orow[1] = make_float4(f[4], f[5], f[6], f[7]);
                            } else {
                                T* orow = reinterpret_cast<T*>(a.out) + orow_off;
                                *reinterpret_cast<uint4*>(orow + 32 * hf + 8 * k) = pack8<T>(f);
                            }
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
