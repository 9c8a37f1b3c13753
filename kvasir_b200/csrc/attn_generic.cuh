// attn_generic.cuh -- causal GQA attention for any head_dim <= 256 and any
// group size: the general path behind kvb_attention when the specialised
// kernels do not apply (e.g. the reference's head_dim 128 test case).
//
// One warp per (query row, head).  Keys are scored 32 at a time (one key per
// lane), the block's scores fold into an online softmax (running max / sum in
// f32), and each lane accumulates head_dim/32 output dims with coalesced reads
// of the value rows.  Same math as engine/kernels/attention.cu:5-57 without its
// shared-memory score buffer, so there is no kv-length cap.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

struct GenericAttnArgs {
    const uint16_t* q;
    long long q_row_stride;   // elements between query rows
    const uint16_t* kc;
    const uint16_t* vc;
    long long seq_stride;     // elements between sequences' caches
    int rows_per_seq;         // query rows per sequence (T), 1 for batched decode
    const int32_t* lens;      // per-sequence key count (device) or nullptr
    int pos0;                 // when lens == nullptr: row r attends keys [0, pos0 + r%T]
    int max_len;              // upper bound on lens[] (larger values are clamped + flagged)
    int n_q, n_kv, hd, max_seq;
    float scale;
    uint16_t* out;
    long long out_row_stride;
};

template <typename T>
__global__ void __launch_bounds__(128) attn_generic_kernel(GenericAttnArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * 4 + warp;
    const int row = blockIdx.x;
    if (h >= a.n_q) return;
    const int seq = row / a.rows_per_seq;
    int len;
    if (a.lens) {
        len = a.lens[seq];
        if (len < 0 || len > a.max_len) {
            if (lane == 0) raise_dev_error(kDevErrBadLength);
            len = len < 0 ? 0 : a.max_len;
        }
    } else {
        len = a.pos0 + row % a.rows_per_seq + 1;
    }
    const int kvh = h / (a.n_q / a.n_kv);
    const T* q = reinterpret_cast<const T*>(a.q) + (size_t)row * a.q_row_stride + (size_t)h * a.hd;
    const T* kb = reinterpret_cast<const T*>(a.kc) + (size_t)seq * a.seq_stride +
                  (size_t)kvh * a.max_seq * a.hd;
    const T* vb = reinterpret_cast<const T*>(a.vc) + (size_t)seq * a.seq_stride +
                  (size_t)kvh * a.max_seq * a.hd;
    T* o = reinterpret_cast<T*>(a.out) + (size_t)row * a.out_row_stride + (size_t)h * a.hd;

    __shared__ float qs[4][256];
    for (int d = lane; d < a.hd; d += 32) qs[warp][d] = Elem<T>::to_f(q[d]) * a.scale;
    __syncwarp();

    constexpr int kMaxDims = 8;  // head_dim <= 256
    float acc[kMaxDims];
#pragma unroll
    for (int i = 0; i < kMaxDims; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int j0 = 0; j0 < len; j0 += 32) {
        const int j = j0 + lane;
        float s = -INFINITY;
        if (j < len) {
            const T* kr = kb + (size_t)j * a.hd;
            float dot = 0.f;
            for (int d = 0; d < a.hd; ++d) dot += qs[warp][d] * Elem<T>::to_f(kr[d]);
            s = dot;
        }
        const float mb = warp_max(s);
        const float mn = fmaxf(m, mb);
        const float alpha = __expf(m - mn);
        const float p = (j < len) ? __expf(s - mn) : 0.f;
        l = l * alpha + warp_sum(p);
#pragma unroll
        for (int i = 0; i < kMaxDims; ++i) acc[i] *= alpha;
        const int nb = min(32, len - j0);
        for (int jj = 0; jj < nb; ++jj) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
            const T* vr = vb + (size_t)(j0 + jj) * a.hd;
#pragma unroll
            for (int i = 0; i < kMaxDims; ++i) {
                const int d = lane + 32 * i;
                if (d < a.hd) acc[i] += pj * Elem<T>::to_f(vr[d]);
            }
        }
        m = mn;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < kMaxDims; ++i) {
        const int d = lane + 32 * i;
        if (d < a.hd) o[d] = Elem<T>::from_f(acc[i] * inv);
    }
}

}  // namespace kvb
