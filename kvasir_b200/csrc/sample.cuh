// sample.cuh -- temperature / top-p (nucleus) sampling over f32 logits, one
// thread-block cluster of 8 (or 16) CTAs per row, entirely on the device.
//
// The reference plans this on the host over the copied logits
// (DESIGN.md:24,109 of kvasir: "greedy / temperature / top-p", seeded so that
// the same seed and logits give the same token).  Here only the sampled id
// leaves the GPU.  Definitions (restated by the CPU oracle):
//   w_i   = floor(2^32 * expf((l_i - max l) * inv_temp)), an integer; 0 for NaN /
//           -inf logits (a row holding +inf samples its first +inf, as the argmax);
//   key_i = the logit's bits mapped to an unsigned order (monotone in l_i);
//   K*    = the largest key with  sum_{key_j >= K*} w_j >= ceil(top_p * sum_j w_j)
//           (every token tied at K* is kept: the nucleus without sorting);
//   u24   = the top 24 bits of SplitMix64(seed + SplitMix64(counter << 32 | row));
//   id    = the first index i, in vocabulary order, whose running sum of kept
//           weights exceeds floor(u24 * sum_kept w / 2^24).
// All sums are exact integers, so the id depends only on the weights.
// K* is found by a mass-weighted select over the keys with no sort: a first
// histogram of w by the log-scaled key distance below the row's maximum (exact
// below 128, then 128 buckets per power of two, so logits that differ in their
// low bits still spread over many buckets), then radix passes of up to 12 bits
// over the chosen bucket's exact distance range, fed only by its tokens.
// temperature <= 0 is greedy (the argmax kernel).
//
// Layout on the GPU: the row's vocabulary is cut into 8 contiguous slices, one
// per CTA of a cluster, so a row streams through 8 SMs (16 slices and SMs when
// the rows are too few to give every SM a CTA); each CTA reads its slice from
// HBM / L2 once into shared memory and runs every pass from there.  Every cluster-wide
// quantity (max, normaliser, digit histograms, kept mass per slice) is a
// per-CTA partial in shared memory that each CTA reads from all of them through
// distributed shared memory and sums in rank order: every CTA derives the same
// K* and draw, and the CTA whose slice holds the drawn token writes it.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int kSampleThreads = 512;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kSampleCluster = 8;              // CTAs per row's cluster; 16 (a non-portable
constexpr int kSampleClusterWide = 16;         // cluster size) when few rows leave SMs idle
constexpr int kSampleMaxSlice = 40960;          // tokens per CTA: vocabularies up to 327680
constexpr int kSampleStageMax = kSampleMaxSlice * 4;

// SplitMix64 (G. Steele, D. Lea, C. Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014): the finaliser of a Weyl sequence.
__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ inline float sample_uniform(uint64_t seed, uint32_t row, uint32_t counter) {
    const uint64_t z = splitmix64(seed + splitmix64(((uint64_t)counter << 32) | row));
    return (float)(z >> 40) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ uint32_t order_key(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float sample_weight(float x, float m, float inv_temp) {
    return (x > -INFINITY) ? expf((x - m) * inv_temp) : 0.f;  // NaN and -inf weigh nothing
}

__device__ __forceinline__ float block_max_f(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = lane < kSampleWarps ? red[lane] : -INFINITY;
    return warp_max(v);
}
__device__ __forceinline__ float block_sum_f(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = lane < kSampleWarps ? red[lane] : 0.f;
    return warp_sum(v);
}

// Weights in 32-bit fixed point (w <= 1): every histogram, mass and running
// sum below is an exact integer, independent of the order the GPU adds in.
// Histograms hold the high and low 16 bits of the weights in two u32 arrays
// (native shared-memory atomics; a slice of <= 40960 tokens cannot overflow).
constexpr float kFixScale = 4294967296.0f;  // 2^32
__device__ __forceinline__ uint64_t fixed_weight(float x, float m, float inv_temp) {
    return (uint64_t)(sample_weight(x, m, inv_temp) * kFixScale);
}
__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ uint64_t block_sum_u64(uint64_t v, uint64_t* red64) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_u64(v);
    __syncthreads();
    if (lane == 0) red64[warp] = v;
    __syncthreads();
    v = lane < kSampleWarps ? red64[lane] : 0ull;
    return warp_sum_u64(v);
}
__device__ __forceinline__ uint64_t dsmem_ld64(const uint64_t* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(remote)
                 : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
    uint64_t v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(remote));
    return v;
}

// Log-linear bucket of a key distance below the row's maximum: exact below 128,
// then 128 buckets per power of two (buckets 0 .. kLogBuckets - 1, increasing
// with d).  A bucket spans at most 2^24 distances: two 12-bit refinement passes.
constexpr int kLogSubBits = 7;
constexpr int kLogSub = 1 << kLogSubBits;
constexpr int kLogBuckets = kLogSub + (32 - kLogSubBits) * kLogSub;  // 3328
constexpr int kRadixBits = 12;                                        // refinement digits
constexpr int kHistBuckets = 1 << kRadixBits;                         // >= kLogBuckets
static_assert(kLogBuckets <= kHistBuckets, "first-pass buckets exceed the histogram");
__device__ __forceinline__ int log_bucket(uint32_t d) {
    if (d < (uint32_t)kLogSub) return (int)d;
    const int e = 31 - __clz(d);  // kLogSubBits .. 31
    return kLogSub + (e - kLogSubBits) * kLogSub +
           (int)((d >> (e - kLogSubBits)) & (uint32_t)(kLogSub - 1));
}
// The distances [lo, lo + 2^width_log2) of a bucket.
__device__ __forceinline__ void log_bucket_range(int b, uint32_t& lo, int& width_log2) {
    if (b < kLogSub) {
        lo = (uint32_t)b;
        width_log2 = 0;
        return;
    }
    const int e = kLogSubBits + (b - kLogSub) / kLogSub, f = (b - kLogSub) % kLogSub;
    lo = ((uint32_t)kLogSub + (uint32_t)f) << (e - kLogSubBits);
    width_log2 = e - kLogSubBits;
}

__device__ __forceinline__ void hist_add(uint32_t* hist_hi, uint32_t* hist_lo, int bucket,
                                         uint64_t w) {
    atomicAdd(&hist_hi[bucket], (uint32_t)(w >> 16));
    atomicAdd(&hist_lo[bucket], (uint32_t)(w & 0xFFFFu));
}

template <int kCluster>
__global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(const float* __restrict__ logits, int vocab, float inv_temp, float top_p,
                  uint64_t seed, const int32_t* __restrict__ counters, int32_t* __restrict__ ids,
                  int32_t* __restrict__ adv, int32_t* __restrict__ adv2, int vec4) {
    static_assert(kHistBuckets / kCluster <= kSampleThreads, "a share is one bucket per thread");
    extern __shared__ float4 slice_smem[];  // this CTA's slice of the row
    __shared__ float red[kSampleWarps];
    __shared__ uint64_t red64[kSampleWarps];
    __shared__ uint32_t hist_hi[kHistBuckets], hist_lo[kHistBuckets];  // this CTA's histogram (read by
                                                      // the cluster): high / low 16 bits
    __shared__ uint64_t hist_sum[kHistBuckets / kCluster];  // the cluster's sums of this CTA's share
    __shared__ uint64_t part_share;                    // and their mass (read by the cluster)
    __shared__ float part_m;                   // this CTA's max (read by the cluster)
    __shared__ uint64_t part_z, part_kept;     // its normaliser and kept mass (read by the cluster)
    __shared__ int part_i;                     // its first +inf index
    __shared__ uint64_t wmass[kSampleWarps];
    __shared__ float s_m;
    __shared__ uint64_t s_total, s_above, s_t, s_base;
    __shared__ uint32_t s_digit;
    __shared__ uint64_t s_share_above, s_kept[kCluster];
    __shared__ int s_owner, s_warp, s_cross, s_low, s_share;
    const uint32_t rank = cluster_rank();
    const int row = blockIdx.x / kCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* l = logits + (size_t)row * vocab;
    const uint32_t counter = counters ? (uint32_t)counters[row] : 0u;
    // this CTA's slice, a multiple of 4 elements long
    const int slice = ((vocab + kCluster - 1) / kCluster + 3) & ~3;
    const int v0 = min(vocab, (int)rank * slice), v1 = min(vocab, v0 + slice);
    const float4* l4 = reinterpret_cast<const float4*>(l);
    const float* sl = reinterpret_cast<const float*>(slice_smem);
    // element i / float4 q of the row, from this CTA's staged slice
    auto at = [&](int i) -> float { return sl[i - v0]; };
    auto at4 = [&](int q) -> float4 { return slice_smem[q - v0 / 4]; };
    // visits every element of the slice
    auto for_slice = [&](auto&& f) {
        if (vec4) {
            for (int q = v0 / 4 + tid; q < v1 / 4; q += kSampleThreads) {
                const float4 x = at4(q);
                f(4 * q, x.x);
                f(4 * q + 1, x.y);
                f(4 * q + 2, x.z);
                f(4 * q + 3, x.w);
            }
        } else {
            for (int i = v0 + tid; i < v1; i += kSampleThreads) f(i, at(i));
        }
    };

    // ---- the slice into shared memory (4 independent loads in flight per thread)
    // and the max over the row
    float m = -INFINITY;
    {
        float* dst = reinterpret_cast<float*>(slice_smem);
        if (vec4) {
            const int q0 = v0 / 4, q1 = v1 / 4;
            for (int q = q0 + tid; q < q1; q += 4 * kSampleThreads) {
                float4 x[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (q + k * kSampleThreads < q1) x[k] = l4[q + k * kSampleThreads];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (q + k * kSampleThreads < q1) {
                        slice_smem[q + k * kSampleThreads - q0] = x[k];
                        m = fmaxf(fmaxf(m, fmaxf(x[k].x, x[k].y)), fmaxf(x[k].z, x[k].w));
                    }
            }
        } else {
            for (int i = v0 + tid; i < v1; i += kSampleThreads) {
                const float x = l[i];
                dst[i - v0] = x;
                m = fmaxf(m, x);
            }
        }
    }
    __syncthreads();  // the slice is in shared memory
    m = block_max_f(m, red);
    if (tid == 0) part_m = m;
    cluster_sync();
    if (warp == 0) {  // one lane per CTA of the cluster
        const float mm = warp_max(lane < kCluster ? dsmem_ld(&part_m, (uint32_t)lane) : -INFINITY);
        if (lane == 0) {
            s_m = mm;
            part_i = 0x7fffffff;
        }
    }
    __syncthreads();
    m = s_m;
    int chosen = -1;  // set by the one thread that writes the id
    if (m == INFINITY) {  // all the mass sits on +inf: the first such index, as the argmax
        for_slice([&](int i, float x) {
            if (x == INFINITY) atomicMin(&part_i, i);
        });
        cluster_sync();
        if (rank == 0 && tid == 0) {
            int first = 0x7fffffff;
            for (uint32_t r = 0; r < kCluster; ++r) first = min(first, dsmem_ld(&part_i, r));
            chosen = first;
        }
    } else if (m == -INFINITY) {  // nothing but NaN / -inf: index 0, as the argmax
        if (rank == 0 && tid == 0) chosen = 0;
    } else {
        // ---- normaliser and the first digit histogram in one pass
        const bool nucleus = top_p < 1.f;
        for (int b = tid; b < kLogBuckets; b += kSampleThreads) hist_hi[b] = hist_lo[b] = 0u;
        __syncthreads();
        // first histogram: by log-scaled key distance below the maximum, which spreads
        // tokens of nearly equal logits over many buckets; index kLogBuckets - 1 - bucket, so that
        // higher indices hold higher keys
        const uint32_t kmax = order_key(m);
        uint64_t z = 0;
        for_slice([&](int, float x) {
            const uint64_t w = fixed_weight(x, m, inv_temp);
            z += w;
            if (nucleus && w)
                hist_add(hist_hi, hist_lo, kLogBuckets - 1 - log_bucket(kmax - order_key(x)), w);
        });
        z = block_sum_u64(z, red64);
        if (tid == 0) part_z = z;
        cluster_sync();  // partials and histograms of pass 0 complete everywhere
        if (warp == 0) {  // one lane per CTA of the cluster
            const uint64_t zz =
                warp_sum_u64(lane < kCluster ? dsmem_ld64(&part_z, (uint32_t)lane) : 0ull);
            if (lane == 0) s_total = zz;
        }
        __syncthreads();
        const uint64_t total = s_total;
        uint32_t kstar = 0;
        if (nucleus) {
            // the nucleus needs at least this much fixed-point mass
            const uint64_t target = (uint64_t)ceil((double)top_p * (double)total);
            // Finds, in the cluster's histogram of nb buckets (higher index = higher keys),
            // the bucket where the mass counted from the top first reaches the target
            // (above = mass of the keys above all of them); returns it and the mass above it.
            // If every bucket falls short (weights truncated to 0) the lowest nonempty one.
            auto select = [&](int nb, uint64_t above, uint32_t& digit, uint64_t& above_out) {
                // 1. CTA `rank` owns the buckets [b0, b1): it sums them over the cluster
                //    (consecutive threads read consecutive buckets of every CTA: whole
                //    128-byte lines) into hist_sum, and publishes their mass
                const int share = (nb + kCluster - 1) / kCluster;  // <= kSampleThreads
                const int b0 = min(nb, (int)rank * share), b1 = min(nb, b0 + share);
                uint64_t part = 0;
                if (b0 + tid < b1) {
                    const int b = b0 + tid;
                    uint32_t vh[kCluster], vl[kCluster];
#pragma unroll
                    for (uint32_t r = 0; r < kCluster; ++r) {
                        vh[r] = dsmem_ld_at(dsmem_addr(&hist_hi[b], r));
                        vl[r] = dsmem_ld_at(dsmem_addr(&hist_lo[b], r));
                    }
#pragma unroll
                    for (uint32_t r = 0; r < kCluster; ++r)
                        part += ((uint64_t)vh[r] << 16) + vl[r];
                    hist_sum[tid] = part;
                }
                part = block_sum_u64(part, red64);
                if (tid == 0) part_share = part;
                cluster_sync();  // every share is summed; no CTA reads hist_hi / hist_lo again
                // 2. the share where the mass counted from the top first reaches the target,
                //    else the lowest nonempty share (all CTAs decide alike from the 8 masses)
                if (warp == 0) {  // one lane per CTA's share
                    const uint64_t mr =
                        lane < kCluster ? dsmem_ld64(&part_share, (uint32_t)lane) : 0ull;
                    uint64_t suf = mr;  // mass of the shares from this one up
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint64_t y = __shfl_down_sync(0xffffffffu, suf, o);
                        if (lane + o < 32) suf += y;
                    }
                    const uint32_t crosses =
                        __ballot_sync(0xffffffffu, mr > 0 && above + suf >= target);
                    const uint32_t nonempty = __ballot_sync(0xffffffffu, mr > 0);
                    const int cr = crosses ? 31 - __clz((int)crosses)
                                           : (nonempty ? __ffs((int)nonempty) - 1 : -1);
                    const uint64_t cr_above =
                        __shfl_sync(0xffffffffu, above + suf - mr, cr < 0 ? 0 : cr);
                    if (lane == 0) {
                        s_share = cr;
                        s_share_above = cr_above;
                        s_cross = -1;
                        s_low = 0x7fffffff;
                    }
                }
                __syncthreads();
                const int cr = s_share;
                if (cr < 0) {  // no mass at all: nothing to refine
                    digit = 0;
                    above_out = above;
                    return;
                }
                // 3. that share's buckets, one per thread, from the CTA that summed them
                const int c0 = min(nb, cr * share), n = min(nb, c0 + share) - c0;
                const uint64_t own = tid < n ? dsmem_ld64(&hist_sum[tid], (uint32_t)cr) : 0ull;
                // mass of the buckets above this thread's: a suffix scan over the block
                uint64_t inc = own;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint64_t y = __shfl_down_sync(0xffffffffu, inc, o);
                    if (lane + o < 32) inc += y;
                }
                if (lane == 0) red64[warp] = inc;
                __syncthreads();
                uint64_t above_warps = 0;
                for (int w = warp + 1; w < kSampleWarps; ++w) above_warps += red64[w];
                const uint64_t ex = s_share_above + above_warps + (inc - own);  // above mine
                if (own > 0 && ex + own >= target) atomicMax(&s_cross, tid);
                if (own > 0) atomicMin(&s_low, tid);
                __syncthreads();
                // the crossing bucket, else (every bucket short) the lowest nonempty one
                const int pick = s_cross >= 0 ? s_cross : s_low;
                if (tid == pick) {
                    s_digit = (uint32_t)(c0 + tid);
                    s_above = ex;
                }
                __syncthreads();
                digit = s_digit;
                above_out = s_above;
            };
            uint32_t d0;
            uint64_t above;
            select(kLogBuckets, 0, d0, above);
            // the chosen bucket is the key distances [lo, lo + 2^nbits): refine over
            // r = (lo + 2^nbits - 1) - distance, whose higher values are higher keys
            uint32_t lo;
            int nbits;
            log_bucket_range(kLogBuckets - 1 - (int)d0, lo, nbits);
            const uint64_t hi = (uint64_t)lo + (1ull << nbits);
            uint32_t prefix = 0;
            // as few passes of at most kRadixBits as the range needs, their digits balanced
            // (13 bits: 7 + 6), so that each histogram and select is as small as it can be
            const int passes = (nbits + kRadixBits - 1) / kRadixBits;
            for (int done = 0, pass = 0; done < nbits; ++pass) {
                const int bits = (nbits - done + passes - pass - 1) / (passes - pass);
                const int shift = nbits - done - bits;
                for (int b = tid; b < (1 << bits); b += kSampleThreads) hist_hi[b] = hist_lo[b] = 0u;
                __syncthreads();
                for_slice([&](int, float x) {
                    const uint32_t dist = kmax - order_key(x);
                    if (dist < lo || (uint64_t)dist >= hi) return;
                    const uint32_t r = (uint32_t)(hi - 1 - dist);
                    if ((r >> (shift + bits)) != prefix) return;
                    const uint64_t w = fixed_weight(x, m, inv_temp);
                    if (w) hist_add(hist_hi, hist_lo, (int)((r >> shift) & ((1u << bits) - 1)), w);
                });
                cluster_sync();  // every CTA's histogram of this pass is complete
                uint32_t digit;
                select(1 << bits, above, digit, above);
                prefix = (prefix << bits) | digit;
                done += bits;
            }
            kstar = kmax - (uint32_t)(hi - 1 - prefix);
        }
        // ---- the draw: kept mass per warp segment of this slice, then per CTA
        const int seg = (v1 - v0 + kSampleWarps - 1) / kSampleWarps;
        const int s0 = min(v1, v0 + warp * seg), s1 = min(v1, s0 + seg);
        uint64_t ws = 0;
        for (int i = s0 + lane; i < s1; i += 32) {
            const float x = at(i);
            if (order_key(x) >= kstar) ws += fixed_weight(x, m, inv_temp);
        }
        ws = warp_sum_u64(ws);
        if (lane == 0) wmass[warp] = ws;
        __syncthreads();
        if (tid == 0) {
            uint64_t cm = 0;
            for (int w = 0; w < kSampleWarps; ++w) cm += wmass[w];
            part_kept = cm;
        }
        cluster_sync();
        if (warp == 0) {  // one lane per CTA of the cluster
            const uint64_t v = lane < kCluster ? dsmem_ld64(&part_kept, (uint32_t)lane) : 0ull;
            if (lane < kCluster) s_kept[lane] = v;
        }
        __syncthreads();
        if (tid == 0) {
            uint64_t pm[kCluster], sum = 0;
            for (int r = 0; r < kCluster; ++r) {
                pm[r] = s_kept[r];
                sum += pm[r];
            }
            // t = floor(u24 * kept / 2^24), in 128-bit integer arithmetic
            const uint64_t u24 =
                (uint64_t)(sample_uniform(seed, (uint32_t)row, counter) * 16777216.0f);
            const uint64_t t = (__umul64hi(sum, u24) << 40) | ((sum * u24) >> 24);
            int owner = -1, last = -1;
            uint64_t base = 0, base_last = 0, acc = 0;
            for (int r = 0; r < kCluster; ++r) {
                if (pm[r] > 0) {
                    last = r;
                    base_last = acc;
                    if (owner < 0 && acc + pm[r] > t) {
                        owner = r;
                        base = acc;
                    }
                }
                acc += pm[r];
            }
            if (owner < 0) {  // cannot happen with exact sums; kept for safety
                owner = last;
                base = base_last;
            }
            s_owner = owner;
            s_t = t;
            if (owner == (int)rank) {  // the warp of this slice that holds the draw
                int wsel = -1, wlast = -1;
                uint64_t wb = base, wb_last = base, a2 = base;
                for (int w = 0; w < kSampleWarps; ++w) {
                    if (wmass[w] > 0) {
                        wlast = w;
                        wb_last = a2;
                        if (wsel < 0 && a2 + wmass[w] > t) {
                            wsel = w;
                            wb = a2;
                        }
                    }
                    a2 += wmass[w];
                }
                if (wsel < 0) {
                    wsel = wlast;
                    wb = wb_last;
                }
                s_warp = wsel;
                s_base = wb;
            }
        }
        __syncthreads();
        if (s_owner == (int)rank && warp == s_warp) {
            const uint64_t t = s_t;
            uint64_t base = s_base;
            int last = -1, found = -1;
            for (int c = s0; c < s1; c += 32) {
                const int i = c + lane;
                uint64_t w = 0;
                if (i < s1) {
                    const float x = at(i);
                    if (order_key(x) >= kstar) w = fixed_weight(x, m, inv_temp);
                }
                uint64_t inc = w;  // inclusive scan over the 32 lanes, in index order
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint64_t y = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += y;
                }
                const uint32_t hit = __ballot_sync(0xffffffffu, w > 0 && base + inc > t);
                const uint32_t pos = __ballot_sync(0xffffffffu, w > 0);
                if (pos) last = c + 31 - __clz(pos);
                if (hit) {
                    found = c + __ffs(hit) - 1;
                    break;
                }
                base += __shfl_sync(0xffffffffu, inc, 31);
            }
            if (lane == 0) chosen = found >= 0 ? found : last;
        }
    }
    if (chosen >= 0) ids[row] = chosen;
    cluster_sync();  // no CTA leaves while another may still read its shared memory,
                     // and every CTA has read the row's counter
    if (rank == 0 && tid == 0) {
        if (adv) adv[row] += 1;
        if (adv2) adv2[row] += 1;
    }
}

}  // namespace kvb
