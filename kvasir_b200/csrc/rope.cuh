// rope.cuh -- RoPE (rotate_half), KV-cache append, and the fused pass that
// does both in one read of the qkv row.
//
// Reference kernels: engine/kernels/rope.cu:3-19 (one thread per (head, pair),
// 2-byte loads) and engine/kernels/elementwise.cu:22-34 (kv_append, div/mod per
// element).  Here one CTA owns one qkv row: each thread rotates 8 pairs of a
// head with two 16-byte loads, the f32 cos/sin come in as float4s, and with
// do_append the rotated k and the raw v chunks are also stored to the cache.
// The rotation is x0*c - x1*s, x1*c + x0*s evaluated with explicitly
// unfused f32 multiplies and adds, the exact f32 sequence of the reference
// test (engine/tests/kernels.rs:121-132), then rounded once.
#pragma once

#include "kvb_ptx.cuh"

namespace kvb {

struct RopeArgs {
    uint16_t* qkv;
    int n_q, n_kv, hd, row_stride;
    int rows_per_seq;        // rows of one sequence (T for a prefill call, 1 for batched decode)
    const int32_t* pos_arr;  // per-sequence start position (device) or nullptr
    int pos0;                // start position when pos_arr == nullptr
    const float* cos_t;
    const float* sin_t;
    int max_pos;             // rows of the cos/sin table
    uint16_t* kc;
    uint16_t* vc;
    long long seq_stride;    // elements between consecutive sequences' caches
    int max_seq;             // positions per sequence (paged: max_blocks * block_size)
    int do_rope, do_append;
    // Paged cache (block_table != nullptr): kc/vc are pools [n_blocks][n_kv][block_size][hd];
    // position p of sequence s lives in block block_table[s * max_blocks + p / block_size].
    const int32_t* block_table;
    int max_blocks, block_size, n_blocks;
};

// Cache element offset of (kv head 0, position p) of sequence seq, and the stride
// between kv heads.  Returns false (and reports) when a paged block entry lies
// outside the pool; the caller then writes nothing for the row.
__device__ __forceinline__ bool rope_cache_base(const RopeArgs& a, int seq, int p, size_t& kv0,
                                                size_t& head_stride, bool report) {
    if (!a.block_table) {
        kv0 = (size_t)seq * a.seq_stride + (size_t)p * a.hd;
        head_stride = (size_t)a.max_seq * a.hd;
        return true;
    }
    const int lb = p / a.block_size;
    const int blk = a.block_table[(size_t)seq * a.max_blocks + lb];  // lb < max_blocks: p < max_seq
    if (blk < 0 || blk >= a.n_blocks) {
        if (report) raise_dev_error(kDevErrBadPosition);
        return false;
    }
    kv0 = ((size_t)blk * a.n_kv * a.block_size + (size_t)(p - lb * a.block_size)) * a.hd;
    head_stride = (size_t)a.block_size * a.hd;
    return true;
}

__device__ __forceinline__ float rot_a(float x0, float x1, float c, float s) {
    return __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
}
__device__ __forceinline__ float rot_b(float x0, float x1, float c, float s) {
    return __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

__device__ __forceinline__ bool rope_row_position(const RopeArgs& a, int row, int& seq, int& p) {
    seq = row / a.rows_per_seq;
    p = (a.pos_arr ? a.pos_arr[seq] : a.pos0) + row % a.rows_per_seq;
    const bool bad = p < 0 || (a.do_rope && p >= a.max_pos) || (a.do_append && p >= a.max_seq);
    if (bad && threadIdx.x == 0) raise_dev_error(kDevErrBadPosition);
    return !bad;
}

// head_dim % 16 == 0 and 16-byte aligned rows.
template <typename T>
__global__ void __launch_bounds__(256) rope_append_vec_kernel(RopeArgs a) {
    const int row = blockIdx.x;
    int seq, p;
    if (!rope_row_position(a, row, seq, p)) return;
    const int half = a.hd >> 1;
    const int cpr = a.hd >> 4;  // 8-pair chunks per head
    const int n_rope = (a.n_q + a.n_kv) * cpr;
    const int n_items = n_rope + a.n_kv * (a.hd >> 3);
    uint16_t* rowp = a.qkv + (size_t)row * a.row_stride;
    size_t kv0 = 0, hs = 0;
    if (a.do_append && !rope_cache_base(a, seq, p, kv0, hs, threadIdx.x == 0)) return;
    for (int it = threadIdx.x; it < n_items; it += blockDim.x) {
        if (it < n_rope) {
            const int h = it / cpr, j = it - h * cpr;
            if (h < a.n_q && !a.do_rope) continue;
            uint4* pa = reinterpret_cast<uint4*>(rowp + h * a.hd + 8 * j);
            uint4* pb = reinterpret_cast<uint4*>(rowp + h * a.hd + 8 * j + half);
            uint4 va = *pa, vb = *pb;
            if (a.do_rope) {
                float x0[8], x1[8];
                unpack8<T>(va, x0);
                unpack8<T>(vb, x1);
                const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)p * half + 8 * j);
                const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)p * half + 8 * j);
                const float4 c0 = c4[0], c1 = c4[1], s0 = s4[0], s1 = s4[1];
                const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                float ra[8], rb[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ra[e] = rot_a(x0[e], x1[e], c[e], s[e]);
                    rb[e] = rot_b(x0[e], x1[e], c[e], s[e]);
                }
                va = pack8<T>(ra);
                vb = pack8<T>(rb);
                *pa = va;
                *pb = vb;
            }
            if (a.do_append && h >= a.n_q) {
                const size_t dst = kv0 + (size_t)(h - a.n_q) * hs;
                *reinterpret_cast<uint4*>(a.kc + dst + 8 * j) = va;
                *reinterpret_cast<uint4*>(a.kc + dst + 8 * j + half) = vb;
            }
        } else if (a.do_append) {
            const int vi = it - n_rope;
            const int per = a.hd >> 3;
            const int kvh = vi / per, c = vi - kvh * per;
            const uint4 v =
                *reinterpret_cast<const uint4*>(rowp + (a.n_q + a.n_kv) * a.hd + kvh * a.hd + 8 * c);
            const size_t dst = kv0 + (size_t)kvh * hs;
            *reinterpret_cast<uint4*>(a.vc + dst + 8 * c) = v;
        }
    }
}

// One warp per qkv row, four rows per CTA (rotate with or without append;
// head_dim = 16 * CPR with CPR dividing 32, 16-byte aligned rows).  Lane l
// always handles 8-pair chunk j = l mod CPR, so its cos/sin are loaded once per
// row; it visits heads l / CPR, + 32 / CPR, ... and issues every load of a batch
// of up to 6 heads before the first rotation.  Same arithmetic as the kernels
// above, bit for bit.
template <typename T, int CPR>
__global__ void __launch_bounds__(128) rope_append_warp_kernel(RopeArgs a, int rows) {
    constexpr int kHeadStep = 32 / CPR;
    constexpr int kBatch = 6;
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int seq = row / a.rows_per_seq;
    const int p = (a.pos_arr ? a.pos_arr[seq] : a.pos0) + row % a.rows_per_seq;
    if (p < 0 || p >= a.max_pos || (a.do_append && p >= a.max_seq)) {
        if (lane == 0) raise_dev_error(kDevErrBadPosition);
        return;
    }
    constexpr int half = CPR * 8;
    const int j = lane % CPR;
    const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)p * half + 8 * j);
    const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)p * half + 8 * j);
    const float4 c0 = c4[0], c1 = c4[1], s0 = s4[0], s1 = s4[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    uint16_t* rowp = a.qkv + (size_t)row * a.row_stride;
    size_t kv0 = 0, hs = 0;
    if (a.do_append && !rope_cache_base(a, seq, p, kv0, hs, lane == 0)) return;
    const int n_heads = a.n_q + a.n_kv;
    for (int h0 = lane / CPR; h0 < n_heads; h0 += kBatch * kHeadStep) {
        uint4 va[kBatch], vb[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            const int h = h0 + k * kHeadStep;
            if (h < n_heads) {
                va[k] = *reinterpret_cast<const uint4*>(rowp + h * 2 * half + 8 * j);
                vb[k] = *reinterpret_cast<const uint4*>(rowp + h * 2 * half + 8 * j + half);
            }
        }
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            const int h = h0 + k * kHeadStep;
            if (h < n_heads) {
                float x0[8], x1[8], ra[8], rb[8];
                unpack8<T>(va[k], x0);
                unpack8<T>(vb[k], x1);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ra[e] = rot_a(x0[e], x1[e], c[e], sn[e]);
                    rb[e] = rot_b(x0[e], x1[e], c[e], sn[e]);
                }
                const uint4 oa = pack8<T>(ra), ob = pack8<T>(rb);
                *reinterpret_cast<uint4*>(rowp + h * 2 * half + 8 * j) = oa;
                *reinterpret_cast<uint4*>(rowp + h * 2 * half + 8 * j + half) = ob;
                if (a.do_append && h >= a.n_q) {
                    const size_t dst = kv0 + (size_t)(h - a.n_q) * hs;
                    *reinterpret_cast<uint4*>(a.kc + dst + 8 * j) = oa;
                    *reinterpret_cast<uint4*>(a.kc + dst + 8 * j + half) = ob;
                }
            }
        }
    }
    if (a.do_append) {  // raw v heads into the cache, 16 bytes per lane per step
        const int per = (2 * half) >> 3;
        const uint16_t* vrow = rowp + (size_t)n_heads * 2 * half;
        for (int vi = lane; vi < a.n_kv * per; vi += 32) {
            const int kvh = vi / per, cc = vi - kvh * per;
            const uint4 v = *reinterpret_cast<const uint4*>(vrow + kvh * 2 * half + 8 * cc);
            const size_t dst = kv0 + (size_t)kvh * hs;
            *reinterpret_cast<uint4*>(a.vc + dst + 8 * cc) = v;
        }
    }
}

// Many rows (prefill), rotate with or without append, head_dim = 16 * CPR:
// persistent CTAs each own the contiguous rows [c*rows/grid, (c+1)*rows/grid).
// One lane streams the rows' q, k (and v) heads into a shared-memory ring with
// bulk copies, kWarps rows per stage; warp j rotates row j of a stage from
// shared memory and stores q and k back in place, k and v to the cache.  A warp
// fetches its next row's cos/sin (and block-table entry) before it waits for
// the row's copy.  Lane l handles 8-pair chunk l mod CPR of heads l / CPR,
// + 32 / CPR, ...: the same arithmetic as the kernels above, bit for bit.
// The launcher takes 16 warps (one CTA per SM) when two 16-row stages fit in
// shared memory, else 8 or 4: with fewer rows in flight per SM the per-row
// latency of the consumer warps, not HBM, sets the pace.
constexpr int kRopeBulkRingBytes = 96 * 1024;

// Bytes of one row that the kernel copies: q and k heads, and v when appending.
__host__ __device__ inline int rope_bulk_row_bytes(const RopeArgs& a) {
    return (a.n_q + a.n_kv + (a.do_append ? a.n_kv : 0)) * a.hd * 2;
}
__host__ __device__ inline int rope_bulk_stages(const RopeArgs& a, int warps) {
    const int st = kRopeBulkRingBytes / (warps * rope_bulk_row_bytes(a));
    return st < 2 ? 2 : st > 12 ? 12 : st;
}
__host__ __device__ inline int rope_bulk_smem_bytes(const RopeArgs& a, int warps) {
    return 256 + rope_bulk_stages(a, warps) * warps * rope_bulk_row_bytes(a);
}

template <typename T, int CPR, int kWarps, int kBatch = 1>
__global__ void __launch_bounds__(32 * (kWarps + 1)) rope_append_bulk_kernel(RopeArgs a, int rows) {
    constexpr int kHeadStep = 32 / CPR;
    constexpr int half = CPR * 8;
    extern __shared__ __align__(128) uint8_t rope_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(rope_smem);  // [12]
    uint64_t* empty = full + 12;                                 // [12]
    uint8_t* ring = rope_smem + 256;
    const int row_bytes = rope_bulk_row_bytes(a);
    const int stage_bytes = kWarps * row_bytes;
    const int stages = rope_bulk_stages(a, kWarps);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (int)((long long)blockIdx.x * rows / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * rows / gridDim.x);
    const int groups = (r1 - r0 + kWarps - 1) / kWarps;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == kWarps) {  // producer
        if (lane != 0) return;
        int issued = 0;
        for (int g = 0; g < groups; ++g) {
            const int s = g % stages;
            if (g >= stages && !mbar_wait(&empty[s], ((g / stages) - 1) & 1)) break;
            const int row = r0 + g * kWarps;
            const int n = min(kWarps, r1 - row);
            mbar_expect_tx(&full[s], (uint32_t)(n * row_bytes));
            for (int i = 0; i < n; ++i)
                bulk_load(ring + (size_t)s * stage_bytes + i * row_bytes,
                          a.qkv + (size_t)(row + i) * a.row_stride, (uint32_t)row_bytes, &full[s]);
            ++issued;
        }
        for (int g = max(0, issued - stages); g < issued; ++g)
            mbar_wait(&full[g % stages], (g / stages) & 1);
        return;
    }
    const int j = lane % CPR;
    const int n_heads = a.n_q + a.n_kv;
    for (int g = 0; g < groups; ++g) {
        const int s = g % stages;
        const int row = r0 + g * kWarps + warp;
        // row metadata and cos/sin first: their loads overlap the wait for the copy
        bool ok = row < r1;
        int seq = 0, p = 0;
        float c[8], sn[8];
        size_t kv0 = 0, hs = 0;
        if (ok) {
            seq = row / a.rows_per_seq;
            p = (a.pos_arr ? a.pos_arr[seq] : a.pos0) + row % a.rows_per_seq;
            if (p < 0 || p >= a.max_pos || (a.do_append && p >= a.max_seq)) {
                if (lane == 0) raise_dev_error(kDevErrBadPosition);
                ok = false;
            }
        }
        if (ok) {
            const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)p * half + 8 * j);
            const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)p * half + 8 * j);
            const float4 c0 = c4[0], c1 = c4[1], s0 = s4[0], s1 = s4[1];
            c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w;
            c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
            sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
            sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
            if (a.do_append && !rope_cache_base(a, seq, p, kv0, hs, lane == 0)) ok = false;
        }
        if (!mbar_wait(&full[s], (g / stages) & 1)) return;
        if (ok) {
            const uint16_t* src =
                reinterpret_cast<const uint16_t*>(ring + (size_t)s * stage_bytes + warp * row_bytes);
            uint16_t* rowp = a.qkv + (size_t)row * a.row_stride;
            for (int h0 = lane / CPR; h0 < n_heads; h0 += kBatch * kHeadStep) {
                uint4 va[kBatch], vb[kBatch];
#pragma unroll
                for (int k = 0; k < kBatch; ++k) {
                    const int h = h0 + k * kHeadStep;
                    if (h < n_heads) {
                        va[k] = *reinterpret_cast<const uint4*>(src + h * 2 * half + 8 * j);
                        vb[k] = *reinterpret_cast<const uint4*>(src + h * 2 * half + 8 * j + half);
                    }
                }
#pragma unroll
                for (int k = 0; k < kBatch; ++k) {
                    const int h = h0 + k * kHeadStep;
                    if (h < n_heads) {
                        float x0[8], x1[8], ra[8], rb[8];
                        unpack8<T>(va[k], x0);
                        unpack8<T>(vb[k], x1);
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            ra[e] = rot_a(x0[e], x1[e], c[e], sn[e]);
                            rb[e] = rot_b(x0[e], x1[e], c[e], sn[e]);
                        }
                        const uint4 oa = pack8<T>(ra), ob = pack8<T>(rb);
                        *reinterpret_cast<uint4*>(rowp + h * 2 * half + 8 * j) = oa;
                        *reinterpret_cast<uint4*>(rowp + h * 2 * half + 8 * j + half) = ob;
                        if (a.do_append && h >= a.n_q) {
                            const size_t dst = kv0 + (size_t)(h - a.n_q) * hs;
                            *reinterpret_cast<uint4*>(a.kc + dst + 8 * j) = oa;
                            *reinterpret_cast<uint4*>(a.kc + dst + 8 * j + half) = ob;
                        }
                    }
                }
            }
            if (a.do_append) {  // raw v heads into the cache, 16 bytes per lane per step
                constexpr int per = (2 * half) >> 3;
                const uint16_t* vrow = src + (size_t)n_heads * 2 * half;
                for (int vi = lane; vi < a.n_kv * per; vi += 32) {
                    const int kvh = vi / per, cc = vi - kvh * per;
                    const uint4 v = *reinterpret_cast<const uint4*>(vrow + kvh * 2 * half + 8 * cc);
                    *reinterpret_cast<uint4*>(a.vc + kv0 + (size_t)kvh * hs + 8 * cc) = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// Any even head_dim, any alignment.
template <typename T>
__global__ void __launch_bounds__(256) rope_append_scalar_kernel(RopeArgs a) {
    const int row = blockIdx.x;
    int seq, p;
    if (!rope_row_position(a, row, seq, p)) return;
    const int half = a.hd >> 1;
    T* rowp = reinterpret_cast<T*>(a.qkv) + (size_t)row * a.row_stride;
    T* kc = reinterpret_cast<T*>(a.kc);
    T* vc = reinterpret_cast<T*>(a.vc);
    size_t kv0 = 0, hs = 0;
    if (a.do_append && !rope_cache_base(a, seq, p, kv0, hs, threadIdx.x == 0)) return;
    if (!a.do_rope) {  // plain kv_append: any head_dim, element copies
        for (int it = threadIdx.x; it < 2 * a.n_kv * a.hd; it += blockDim.x) {
            const int is_v = it >= a.n_kv * a.hd;
            const int i = it - is_v * a.n_kv * a.hd;
            const int kvh = i / a.hd, d = i - kvh * a.hd;
            const size_t dst = kv0 + (size_t)kvh * hs + d;
            (is_v ? vc : kc)[dst] = rowp[(a.n_q + is_v * a.n_kv) * a.hd + i];
        }
        return;
    }
    const int n_rope = (a.n_q + a.n_kv) * half;
    const int n_items = n_rope + a.n_kv * a.hd;
    for (int it = threadIdx.x; it < n_items; it += blockDim.x) {
        if (it < n_rope) {
            const int h = it / half, j = it - h * half;
            if (h < a.n_q && !a.do_rope) continue;
            T* v = rowp + h * a.hd;
            T ta = v[j], tb = v[j + half];
            if (a.do_rope) {
                const float x0 = Elem<T>::to_f(ta), x1 = Elem<T>::to_f(tb);
                const float c = a.cos_t[(size_t)p * half + j], s = a.sin_t[(size_t)p * half + j];
                ta = Elem<T>::from_f(rot_a(x0, x1, c, s));
                tb = Elem<T>::from_f(rot_b(x0, x1, c, s));
                v[j] = ta;
                v[j + half] = tb;
            }
            if (a.do_append && h >= a.n_q) {
                const size_t dst = kv0 + (size_t)(h - a.n_q) * hs;
                kc[dst + j] = ta;
                kc[dst + j + half] = tb;
            }
        } else if (a.do_append) {
            const int vi = it - n_rope;
            const int kvh = vi / a.hd, d = vi - kvh * a.hd;
            const size_t dst = kv0 + (size_t)kvh * hs;
            vc[dst + d] = rowp[(a.n_q + a.n_kv) * a.hd + kvh * a.hd + d];
        }
    }
}

}  // namespace kvb
