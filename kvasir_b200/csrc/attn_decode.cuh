// attn_decode.cuh -- split-KV GQA decode attention for head_dim 64.
//
// Work unit: one CTA per (key chunk, kv head, sequence).  The group of
// n_q/n_kv query heads that share a kv head is handled by the same CTA, so
// every K/V byte crosses HBM once (the reference kernel,
// engine/kernels/attention.cu:5-57, re-reads K/V once per query head and reads
// keys with a head_dim stride across threads).
//
// Data path per warp, per 64-key tile:
//   TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast) brings the K
//   and V tiles (8 KB each) into shared memory, each completing its own
//   mbarrier, so that the next K tile loads while this tile's softmax and
//   P V run, and the next V tile once P V has read this one;
//   S = Q K^T runs on the tensor cores as m16n8k16 MMAs with the group's
//   query heads as the 16 rows (padded), K fragments via ldmatrix;
//   an online softmax in f32 (exp2, running max / sum) turns S into P;
//   O += P V with P re-used from registers and V fragments via ldmatrix.trans.
// The four warps of a CTA take interleaved tiles of the chunk, merge their
// (max, sum, O) states through shared memory, and either write the final
// rows (single-chunk sequences) or an unnormalised partial that
// attn_combine_kernel folds across chunks.  The kernel is HBM-bound: per key
// it reads 256 bytes (K+V) and does 4*64*2*2 = 1024 useful flops.
#pragma once

#include "kvb_ptx.cuh"
#include "rope.cuh"

namespace kvb {

constexpr int kDecTileKeys = 64;
constexpr int kDecWarps = 4;
constexpr int kDecTileBytes = kDecTileKeys * 64 * 2;  // one K (or V) tile
// the tiles, a chunk's folded state (G <= 16 heads x 66 floats), alignment slack
constexpr int kDecSmemBytes = kDecWarps * 2 * kDecTileBytes + 16 * 66 * 4 + 1024;

struct DecodeArgs {
    const uint16_t* q;
    long long q_row_stride;
    const int32_t* lens;     // per-sequence key count (device) or nullptr
    int len_const;           // key count when lens == nullptr
    int max_len;
    int n_kv, group, max_seq;
    long long seq_rows;      // rows (of 64 elements) between sequences in the cache
    float scale_log2;        // softmax scale * log2(e)
    uint16_t* out;
    long long out_row_stride;
    float* ws;               // split-KV partials, or nullptr when chunks == 1
    int chunk_keys;          // keys per CTA (multiple of 256)
    int max_chunks;
    // Paged cache (block_table != nullptr): K/V pools [n_blocks][n_kv][block_size][64];
    // key k of sequence b lives in block block_table[b * max_blocks + k / block_size].
    const int32_t* block_table;
    int max_blocks, block_size, n_blocks;
    // Fused RoPE + KV append (rope_cos != nullptr; kvb_rope_attention_decode): the new
    // token of sequence b is key lens[b] - 1; q (a.q) and the new k, v are read
    // unrotated from the sequence's qkv row, q is rotated in registers, and the CTA of
    // the last chunk writes the rotated k and the v to that cache row before its tensor
    // copies read it.
    const float* rope_cos;
    const float* rope_sin;
    int rope_max_pos;
    uint16_t* kc_w;
    uint16_t* vc_w;
    long long cache_seq_stride;  // elements between sequences' caches
    int fold;                    // chunks folded in-kernel through a cluster (see the kernel)
    // The cache rows before each sequence's new key are final (no kernel that can still
    // be running writes them: the decode-step driver's launches).  The first K/V tiles
    // are then requested before griddepcontrol.wait; otherwise nothing is read before it.
    int kv_ready;
};

// First row (of 64 elements) of the 64-key tile starting at key kt0 (a multiple of
// 64) of kv head kvh of sequence b.  Paged: block_size is a multiple of 64, so the
// tile lies inside one block; an entry outside [0, n_blocks) is reported and mapped
// past the end of the pool, where the tensor copy reads zeros.
__device__ __forceinline__ int decode_tile_row(const DecodeArgs& a, int b, int kvh, int row_base,
                                               int kt0, int blk) {
    if (!a.block_table) return row_base + kt0;
    if (blk < 0 || blk >= a.n_blocks) {
        raise_dev_error(kDevErrBadPosition);
        return a.n_blocks * a.n_kv * a.block_size;
    }
    return (blk * a.n_kv + kvh) * a.block_size + kt0 % a.block_size;
}
__device__ __forceinline__ int decode_block_of(const DecodeArgs& a, int b, int kt0) {
    if (!a.block_table) return 0;
    const int lb = kt0 / a.block_size;
    return lb < a.max_blocks ? a.block_table[(size_t)b * a.max_blocks + lb] : -1;
}

__device__ __forceinline__ int decode_len(const DecodeArgs& a, int b) {
    int len = a.lens ? a.lens[b] : a.len_const;
    if (len < 0 || len > a.max_len) {
        if (threadIdx.x == 0) raise_dev_error(kDevErrBadLength);
        len = len < 0 ? 0 : a.max_len;
    }
    return len;
}

// One chunk of attn_decode_kernel: chunk slot `from_end` (counted from the end of
// the sequence) of kv head kvh of sequence b.  Called by every thread of the CTA.
// Its result goes to the output row (a one-chunk sequence), to `fold` (this CTA's
// shared memory, for the cluster fold) or to the workspace.
template <typename T, bool kRope>
__device__ __forceinline__ void decode_chunk(const CUtensorMap& kmap, const CUtensorMap& vmap,
                                             const DecodeArgs& a, uint8_t* smem, uint64_t* bars,
                                             int kvh, int b, int from_end, float* fold) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int G = a.group;

    const int len = decode_len(a, b);
    const int n_chunks = (len + a.chunk_keys - 1) / a.chunk_keys;
    T* outb = reinterpret_cast<T*>(a.out) + (size_t)b * a.out_row_stride + (size_t)kvh * G * 64;
    if (len == 0) {  // no keys: defined as a zero output row
        if (a.kv_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (from_end == 0)
            for (int i = threadIdx.x; i < G * 64; i += blockDim.x) outb[i] = Elem<T>::from_f(0.f);
        return;
    }
    if (from_end >= n_chunks) return;
    const int chunk = n_chunks - 1 - from_end;
    const int key_begin = chunk * a.chunk_keys;
    const int key_end = min(len, key_begin + a.chunk_keys);

    int rope_p = -1;  // fused RoPE: the new token's position (-1: none, or out of range)
    if (kRope) {
        rope_p = len - 1;
        if (rope_p >= a.rope_max_pos) {
            if (threadIdx.x == 0) raise_dev_error(kDevErrBadPosition);
            rope_p = -1;
        }
    }
    // this CTA appends the new key (fused RoPE, last chunk): CTA-uniform
    const bool appends = kRope && rope_p >= 0 && chunk == n_chunks - 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * kDecWarps; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    uint8_t* ktile = smem + warp * 2 * kDecTileBytes;
    uint8_t* vtile = ktile + kDecTileBytes;
    uint64_t* bar_k = &bars[warp];              // this warp's K tile
    uint64_t* bar_v = &bars[kDecWarps + warp];  // and its V tile, completed separately
    const int row_base = (int)((long long)b * a.seq_rows + (long long)kvh * a.max_seq);
    // paged: lane 0 reads the block of its next tile while the current one loads
    int blk_next = lane == 0 ? decode_block_of(a, b, key_begin + warp * kDecTileKeys) : 0;
    auto tile_row = [&](int kt0) {  // lane 0: cache row of keys kt0 .. kt0 + 63
        const int row = decode_tile_row(a, b, kvh, row_base, kt0, blk_next);
        const int kn = kt0 + kDecWarps * kDecTileKeys;
        if (kn < key_end) blk_next = decode_block_of(a, b, kn);
        return row;
    };
    auto issue_k = [&](int row) {
        mbar_expect_tx(bar_k, kDecTileBytes);
        tma_load_2d(ktile, &kmap, bar_k, 0, row);
    };
    auto issue_v = [&](int row) {
        mbar_expect_tx(bar_v, kDecTileBytes);
        tma_load_2d(vtile, &vmap, bar_v, 0, row);
    };
    // The first tile's copy is in flight while q is loaded (and the new row written):
    // only the tile that holds the new key waits for that write.
    const int kt_first = key_begin + warp * kDecTileKeys;
    const bool early = kt_first < key_end && !(appends && rope_p < kt_first + kDecTileKeys);
    if (early && lane == 0) {
        const int row = tile_row(kt_first);
        issue_k(row);
        issue_v(row);
    }
    if (a.kv_ready) asm volatile("griddepcontrol.wait;" ::: "memory");  // q, the new row

    if (appends) {
        const T* kin = reinterpret_cast<const T*>(a.q) + (size_t)b * a.q_row_stride +
                       (size_t)(a.n_kv * G + kvh) * 64;
        const T* vin = kin + (size_t)a.n_kv * 64;
        size_t row = (size_t)b * a.cache_seq_stride + ((size_t)kvh * a.max_seq + rope_p) * 64;
        bool write = true;
        if (a.block_table) {  // paged: the block holding position rope_p
            const int lb = rope_p / a.block_size;
            const int blk = a.block_table[(size_t)b * a.max_blocks + lb];
            if (blk < 0 || blk >= a.n_blocks) {  // reported; the tile read sees zeros there
                if (threadIdx.x == 0) raise_dev_error(kDevErrBadPosition);
                write = false;
            }
            row = (((size_t)blk * a.n_kv + kvh) * a.block_size + (rope_p - lb * a.block_size)) * 64;
        }
        T* kout = reinterpret_cast<T*>(a.kc_w) + row;
        T* vout = reinterpret_cast<T*>(a.vc_w) + row;
        const int t = threadIdx.x;
        if (write && t < 32) {
            const float x0 = Elem<T>::to_f(kin[t]), x1 = Elem<T>::to_f(kin[t + 32]);
            const float cs = a.rope_cos[(size_t)rope_p * 32 + t];
            const float sn = a.rope_sin[(size_t)rope_p * 32 + t];
            kout[t] = Elem<T>::from_f(rot_a(x0, x1, cs, sn));
            kout[t + 32] = Elem<T>::from_f(rot_b(x0, x1, cs, sn));
        } else if (write && t >= 64) {
            vout[t - 64] = vin[t - 64];
        }
        // the tensor copies below read this row through the async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __syncthreads();  // written before the copy of its tile is issued
    }

    const uint32_t kb = smem_u32(ktile), vb = smem_u32(vtile);

    // Q fragments (A operand, rows = the group's heads, padded to 16).
    uint32_t qa[4][4];
    {
        const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.q_row_stride +
                      (size_t)kvh * G * 64;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int d0 = 16 * s + 2 * c;
            qa[s][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * 64 + d0) : 0u;
            qa[s][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * 64 + d0) : 0u;
            qa[s][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * 64 + d0 + 8) : 0u;
            qa[s][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * 64 + d0 + 8) : 0u;
        }
        if (kRope && rope_p >= 0) {
            // rotate_half in registers: dims j (s = 0, 1) pair with j + 32 (s = 2, 3);
            // the same f32 operations and one rounding as the RoPE kernels
            const float* cr = a.rope_cos + (size_t)rope_p * 32;
            const float* sr = a.rope_sin + (size_t)rope_p * 32;
#pragma unroll
            for (int s = 0; s < 2; ++s)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int j = 16 * s + 2 * c + (r >= 2 ? 8 : 0);
                    const float2 lo = Elem<T>::unpack(qa[s][r]), hi = Elem<T>::unpack(qa[s + 2][r]);
                    const float c0 = cr[j], c1 = cr[j + 1], s0 = sr[j], s1 = sr[j + 1];
                    qa[s][r] = Elem<T>::pack(rot_a(lo.x, hi.x, c0, s0), rot_a(lo.y, hi.y, c1, s1));
                    qa[s + 2][r] = Elem<T>::pack(rot_b(lo.x, hi.x, c0, s0), rot_b(lo.y, hi.y, c1, s1));
                }
        }
    }

    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    // One K and one V copy per warp at a time, each on its own barrier: the next
    // tile's K is requested as soon as S = Q K^T has read this one (its load runs
    // under the softmax and P V), its V once P V has read this V.  k_out / v_out:
    // a copy is outstanding (warp-uniform; lane 0 issues).
    uint32_t phase_k = 0, phase_v = 0;
    bool k_out = early, v_out = early;
    int row_next = 0;  // lane 0: row of the tile whose V is requested after P V
    bool ok = true;

    for (int kt0 = kt_first; kt0 < key_end; kt0 += kDecWarps * kDecTileKeys) {
        const int nk = min(kDecTileKeys, key_end - kt0);
        const int kt_next = kt0 + kDecWarps * kDecTileKeys;
        if (!k_out) {  // the first tile, when it waited for the new key's row
            if (lane == 0) {
                const int row = tile_row(kt0);
                issue_k(row);
                issue_v(row);
            }
            k_out = v_out = true;
        }
        ok = mbar_wait(bar_k, phase_k);
        if (!ok) break;
        phase_k ^= 1;
        k_out = false;

        // ---- S = Q K^T : 16 x 64 per warp
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
            const int r = 8 * j + (lane & 7);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int ch = 4 * hf + (lane >> 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + r * 128 + ((ch ^ (lane & 7)) << 4), b0, b1, b2, b3);
                mma_16816<T>(s[j], qa[2 * hf], b0, b1);
                mma_16816<T>(s[j], qa[2 * hf + 1], b2, b3);
            }
        }
        __syncwarp();
        fence_async_smem();  // generic-proxy reads of the K tile precede the next TMA write
        if (kt_next < key_end) {
            if (lane == 0) {
                row_next = tile_row(kt_next);
                issue_k(row_next);
            }
            k_out = true;
        }
        // ---- online softmax (log2 domain); rows g (e = 0,1) and g + 8 (e = 2,3)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = 8 * j + 2 * c + (e & 1);
                s[j][e] = key < nk ? s[j][e] * a.scale_log2 : -INFINITY;
            }
            mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
            mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s[j][0] = exp2f(s[j][0] - mn0);
            s[j][1] = exp2f(s[j][1] - mn0);
            s[j][2] = exp2f(s[j][2] - mn1);
            s[j][3] = exp2f(s[j][3] - mn1);
            sum0 += s[j][0] + s[j][1];
            sum1 += s[j][2] + s[j][3];
        }
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
        l0 = l0 * al0 + sum0;
        l1 = l1 * al1 + sum1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= al0;
            o[j][1] *= al0;
            o[j][2] *= al1;
            o[j][3] *= al1;
        }
        ok = mbar_wait(bar_v, phase_v);
        if (!ok) break;
        phase_v ^= 1;
        v_out = false;
        if (nk < kDecTileKeys) {  // rows past the sequence end: zero V so that 0 * garbage stays 0
            uint4* vz = reinterpret_cast<uint4*>(vtile);
            for (int i = nk * 8 + lane; i < kDecTileKeys * 8; i += 32) vz[i] = make_uint4(0, 0, 0, 0);
            __syncwarp();
        }
        // ---- O += P V : P from registers, V^T fragments via ldmatrix.trans.
        // P is split into a 16-bit head and a 16-bit remainder (P = hi + lo)
        // and both are multiplied: a single 16-bit P would carry a 2^-9
        // relative error into every weight, above the 2e-3 attention bar.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t ph[4], pl[4];
            split_pack<T>(s[2 * kk][0], s[2 * kk][1], ph[0], pl[0]);
            split_pack<T>(s[2 * kk][2], s[2 * kk][3], ph[1], pl[1]);
            split_pack<T>(s[2 * kk + 1][0], s[2 * kk + 1][1], ph[2], pl[2]);
            split_pack<T>(s[2 * kk + 1][2], s[2 * kk + 1][3], ph[3], pl[3]);
            const int key = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                const int ch = 2 * jp + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + key * 128 + ((ch ^ (lane & 7)) << 4), b0, b1, b2, b3);
                mma_16816<T>(o[2 * jp], ph, b0, b1);
                mma_16816<T>(o[2 * jp + 1], ph, b2, b3);
                mma_16816<T>(o[2 * jp], pl, b0, b1);
                mma_16816<T>(o[2 * jp + 1], pl, b2, b3);
            }
        }
        __syncwarp();
        fence_async_smem();  // generic-proxy reads of the V tile precede the next TMA write
        if (kt_next < key_end) {
            if (lane == 0) issue_v(row_next);
            v_out = true;
        }
    }
    if (!ok) {
        // A copy did not complete in time (the error word is set): wait once
        // more, bounded, for each copy still outstanding, so that none lands in
        // shared memory after the CTA exits, and contribute an empty state.
        if (k_out) mbar_wait(bar_k, phase_k);
        if (v_out) mbar_wait(bar_v, phase_v);
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    }

    // ---- merge the four warps' states through shared memory (own K tile area)
    float* wo = reinterpret_cast<float*>(ktile);  // [16 rows][64] O, then m[16], l[16]
    float* wm = wo + 16 * 64;
    float* wl = wm + 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = 8 * j + 2 * c;
        wo[g * 64 + d] = o[j][0];
        wo[g * 64 + d + 1] = o[j][1];
        wo[(g + 8) * 64 + d] = o[j][2];
        wo[(g + 8) * 64 + d + 1] = o[j][3];
    }
    if (c == 0) {
        wm[g] = m0;
        wl[g] = l0;
        wm[g + 8] = m1;
        wl[g + 8] = l1;
    }
    __syncthreads();
    float* wsb = nullptr;
    if (n_chunks > 1)
        wsb = fold ? fold : a.ws + (((size_t)b * a.n_kv + kvh) * a.max_chunks + chunk) * (size_t)G * 66;
    for (int i = threadIdx.x; i < G * 64; i += blockDim.x) {
        const int r = i >> 6, d = i & 63;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w)
            M = fmaxf(M, reinterpret_cast<const float*>(smem + w * 2 * kDecTileBytes)[16 * 64 + r]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) {
            const float* base = reinterpret_cast<const float*>(smem + w * 2 * kDecTileBytes);
            const float mw = base[16 * 64 + r];
            const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
            L += base[16 * 64 + 16 + r] * f;
            O += base[r * 64 + d] * f;
        }
        if (n_chunks == 1) {
            outb[i] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
        } else {
            wsb[i] = O;
            if (d == 0) {
                wsb[G * 64 + r] = M;
                wsb[G * 65 + r] = L;
            }
        }
    }
}

// Grid (kv head, sequence, chunk slot), or with a.fold (chunk slot, kv head,
// sequence) in clusters of max_chunks CTAs.  The slot counts chunks from the END
// of the sequence, and the last slot holds every sequence's last, partial chunk.
// CTAs are dispatched slot by slot, so full chunks go first and the final wave
// holds the shortest pieces of work (longest first: a shorter tail).
// The combine pass (a programmatic dependent) may launch once every CTA got here;
// it still waits for this grid's completion before it reads any partial.  This
// kernel is launched the same way after the qkv projection: it reads memory that
// the preceding kernels write only after griddepcontrol.wait -- at once, or with
// a.kv_ready after requesting its first K/V tiles (those rows are final, and the
// lengths were written by an earlier step).
// a.fold: the chunks of one (sequence, kv head) form a cluster, and the CTA of the
// last chunk folds the others' partial states through distributed shared memory
// with the arithmetic of attn_combine_kernel (so the rows are the same bits), in
// place of the workspace and the combine pass.  For small grids, where every
// cluster is resident at once.  Every CTA of a cluster with keys passes both
// cluster barriers; a cluster of an empty sequence passes none.
template <typename T, bool kRope>
__global__ void __launch_bounds__(128, 3) attn_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                             const __grid_constant__ CUtensorMap vmap,
                                                             DecodeArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[2 * kDecWarps];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    asm volatile("griddepcontrol.launch_dependents;");
    if (!a.kv_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
    const int slot = a.fold ? (int)blockIdx.x : (int)blockIdx.z;
    const int kvh = a.fold ? (int)blockIdx.y : (int)blockIdx.x;
    const int b = a.fold ? (int)blockIdx.z : (int)blockIdx.y;
    const int from_end = a.max_chunks - 1 - slot;
    float* st = reinterpret_cast<float*>(smem + kDecWarps * 2 * kDecTileBytes);  // [G][66]
    decode_chunk<T, kRope>(kmap, vmap, a, smem, bars, kvh, b, from_end, a.fold ? st : nullptr);
    if (!a.fold) return;
    const int G = a.group;
    const int len = decode_len(a, b);
    if (len == 0) return;  // the whole cluster: its row was written as zeros
    const int n_chunks = (len + a.chunk_keys - 1) / a.chunk_keys;
    cluster_sync();  // every chunk's state is in its CTA's shared memory
    if (n_chunks > 1 && slot == a.max_chunks - 1) {
        // chunk c of the sequence is cluster rank max_chunks - n_chunks + c
        const uint32_t r0 = (uint32_t)(a.max_chunks - n_chunks);
        T* outb = reinterpret_cast<T*>(a.out) + (size_t)b * a.out_row_stride + (size_t)kvh * G * 64;
        for (int i = threadIdx.x; i < G * 64; i += blockDim.x) {
            const int r = i >> 6;
            float Mn = -INFINITY;
            for (int c = 0; c < n_chunks; ++c) Mn = fmaxf(Mn, dsmem_ld(st + G * 64 + r, r0 + c));
            float Lu = 0.f, Ou = 0.f;
            for (int c = 0; c < n_chunks; ++c) {
                const float mc = dsmem_ld(st + G * 64 + r, r0 + c);
                const float f = mc == -INFINITY ? 0.f : exp2f(mc - Mn);
                Lu += dsmem_ld(st + G * 65 + r, r0 + c) * f;
                Ou += dsmem_ld(st + i, r0 + c) * f;
            }
            outb[i] = Elem<T>::from_f(Ou / Lu);
        }
    }
    cluster_sync();  // no CTA leaves while the fold may still read its state
}

// Folds the per-chunk partials of every (sequence, kv head) with more than one chunk.
// The CTA first stages the partials of up to kCombineSmemBytes worth of chunks in
// shared memory with coalesced loads (one round of memory latency for all of them),
// then each thread folds its output elements from there: the row max M over the
// chunks, then L = sum l_c 2^(m_c - M) and O = sum o_c 2^(m_c - M).  Launched as a
// programmatic dependent of the decode kernel: griddepcontrol.wait holds it until
// every decode CTA has finished and its partials are visible, while its launch and
// CTA set-up overlap the decode kernel's last wave.
constexpr int kCombineSmemBytes = 48 * 1024;
constexpr int kCombineThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(DecodeArgs a) {
    extern __shared__ float sp[];
    // the projection after this pass (a programmatic dependent) may start streaming its
    // weights; it reads the attention output only after this grid completes
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int kvh = blockIdx.x, b = blockIdx.y;
    const int G = a.group;
    const int len = decode_len(a, b);
    const int n_chunks = (len + a.chunk_keys - 1) / a.chunk_keys;
    if (n_chunks <= 1) return;
    const int per = G * 66;                          // floats per chunk: O[G][64], m[G], l[G]
    const int cap = kCombineSmemBytes / (per * 4);   // chunks per round (>= 11: G <= 16)
    const float* base = a.ws + ((size_t)b * a.n_kv + kvh) * a.max_chunks * (size_t)per;
    T* outb = reinterpret_cast<T*>(a.out) + (size_t)b * a.out_row_stride + (size_t)kvh * G * 64;
    constexpr int kPer = 4;  // outputs per thread: G * 64 <= 1024
    float M[kPer], L[kPer], O[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        M[u] = -INFINITY;
        L[u] = O[u] = 0.f;
    }
    for (int c0 = 0; c0 < n_chunks; c0 += cap) {
        const int nc = min(cap, n_chunks - c0);
        const float* src = base + (size_t)c0 * per;
        __syncthreads();  // the previous round's reads are done
#pragma unroll 8
        for (int k = threadIdx.x; k < nc * per; k += kCombineThreads) sp[k] = src[k];
        __syncthreads();
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * kCombineThreads;
            if (i >= G * 64) break;
            const int r = i >> 6;
            float Mn = M[u];
            for (int c = 0; c < nc; ++c) Mn = fmaxf(Mn, sp[c * per + G * 64 + r]);
            const float f0 = M[u] == -INFINITY ? 0.f : exp2f(M[u] - Mn);  // earlier rounds
            float Lu = L[u] * f0, Ou = O[u] * f0;
            for (int c = 0; c < nc; ++c) {
                const float mc = sp[c * per + G * 64 + r];
                const float f = mc == -INFINITY ? 0.f : exp2f(mc - Mn);
                Lu += sp[c * per + G * 65 + r] * f;
                Ou += sp[c * per + i] * f;
            }
            M[u] = Mn;
            L[u] = Lu;
            O[u] = Ou;
        }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int i = threadIdx.x + u * kCombineThreads;
        if (i < G * 64) outb[i] = Elem<T>::from_f(O[u] / L[u]);
    }
}

}  // namespace kvb
