/*
 * kvb_oracle.c -- CPU oracle for the kvasir per-layer Llama kernel chain.
 *
 * TEST INFRASTRUCTURE ONLY (see kvb_oracle.h): the checker for the CUDA path,
 * never part of it.  Every function cites the reference file:line whose CPU
 * computation it restates.  Built with -ffp-contract=off so f32 expressions
 * round exactly as the Rust reference tests evaluate them (Rust never fuses
 * a*b-c into an FMA).
 */
#include "kvb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* 16-bit float conversion.  Restates the IEEE binary16 / bfloat16 round-to-
 * nearest-even conversions that the reference gets from the `half` crate
 * 2.7.1 (reference Cargo.lock:407-408; used as f16::from_f32 / to_f32 in
 * engine/tests/kernels.rs:9-15) and from __float2half in its kernels. */

static inline uint32_t f32_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}
static inline float bits_f32(uint32_t u) {
    float x;
    memcpy(&x, &u, 4);
    return x;
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0x1f) return bits_f32(sign | 0x7f800000u | (m << 13)); /* inf / nan */
    if (e == 0) {
        /* zero or subnormal: m * 2^-24 is exact in f32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

static uint16_t f32_to_f16(float x) {
    uint32_t u = f32_bits(x);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;   /* nan -> quiet nan */
    if (a >= 0x477ff000u) return sign | 0x7c00u;  /* >= 65520 rounds to inf */
    uint32_t e = a >> 23;
    if (e >= 113) { /* normal f16 */
        uint32_t mant = a & 0x7fffffu;
        uint32_t r = ((e - 112u) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
        return sign | (uint16_t)r;
    }
    /* subnormal f16 or zero: value in units of 2^-24 (f32 denormals are far
     * below half a unit and round to zero) */
    if (e == 0) return sign;
    uint32_t full = (a & 0x7fffffu) | 0x800000u;
    uint32_t s = 126u - e;
    if (s > 31) return sign;
    uint32_t q = full >> s;
    uint32_t rem = full & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return sign | (uint16_t)q;
}

static inline float bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

static uint16_t f32_to_bf16(float x) {
    uint32_t u = f32_bits(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float kvo_to_f32(uint16_t bits, int dtype) {
    return dtype == KVO_F16 ? f16_to_f32(bits) : bf16_to_f32(bits);
}
uint16_t kvo_from_f32(float x, int dtype) {
    return dtype == KVO_F16 ? f32_to_f16(x) : f32_to_bf16(x);
}
void kvo_to_f32_array(const uint16_t* in, float* out, size_t n, int dtype) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_to_f32(in[i], dtype);
}
void kvo_from_f32_array(const float* in, uint16_t* out, size_t n, int dtype) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_from_f32(in[i], dtype);
}

/* ------------------------------------------------------------------------ */
static int g_threads = 1;

void kvo_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int kvo_get_threads(void) { return g_threads; }

/* ------------------------------------------------------------------------ */
/* Seeded normal generator: counter-based splitmix64 hash + Box-Muller.  The
 * value at index i depends only on (seed, i), so fills are reproducible for
 * any thread count. */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

void kvo_fill_normal(uint16_t* out, size_t n, double mean, double std, uint64_t seed, int dtype) {
    const uint64_t s = mix64(seed);
    const long long pairs = (long long)((n + 1) / 2);
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (long long p = 0; p < pairs; ++p) {
        uint64_t h1 = mix64(s ^ (uint64_t)(2 * p));
        uint64_t h2 = mix64(s ^ (uint64_t)(2 * p + 1));
        double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740993.0); /* (0,1] */
        double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);         /* [0,1) */
        double r = sqrt(-2.0 * log(u1));
        double th = 6.283185307179586 * u2;
        size_t i = (size_t)(2 * p);
        out[i] = kvo_from_f32((float)(mean + std * r * cos(th)), dtype);
        if (i + 1 < n) out[i + 1] = kvo_from_f32((float)(mean + std * r * sin(th)), dtype);
    }
}

/* ------------------------------------------------------------------------ */
/* engine/tests/kernels.rs:44-47 -- out row t is table row ids[t].  Ids outside
 * [0, vocab) give a zero row (the reference range-checks ids on the host,
 * reference DESIGN.md:80; the CUDA path defines the same zero-row result). */
void kvo_embedding_gather(const int32_t* ids, size_t t, const uint16_t* table, size_t vocab,
                          uint16_t* out, size_t hidden) {
    for (size_t r = 0; r < t; ++r) {
        int32_t id = ids[r];
        if (id < 0 || (size_t)id >= vocab)
            memset(out + r * hidden, 0, hidden * 2);
        else
            memcpy(out + r * hidden, table + (size_t)id * hidden, hidden * 2);
    }
}

/* engine/tests/kernels.rs:62-70 -- f64 mean of squares, inv = 1/sqrt(ms+eps),
 * want = (x * inv * w) as f32. */
void kvo_rmsnorm(const uint16_t* x, const uint16_t* w, float* out, size_t rows, size_t hidden,
                 float eps, int dtype) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (long long r = 0; r < (long long)rows; ++r) {
        const uint16_t* row = x + (size_t)r * hidden;
        double ss = 0.0;
        for (size_t i = 0; i < hidden; ++i) {
            double v = (double)kvo_to_f32(row[i], dtype);
            ss += v * v;
        }
        double ms = ss / (double)hidden;
        double inv = 1.0 / sqrt(ms + (double)eps);
        for (size_t i = 0; i < hidden; ++i)
            out[(size_t)r * hidden + i] = (float)((double)kvo_to_f32(row[i], dtype) * inv *
                                                  (double)kvo_to_f32(w[i], dtype));
    }
}

/* engine/tests/kernels.rs:121-132 -- rotate_half on every q and k head of each
 * qkv row, pairs (j, j+hd/2), in f32: x0*c - x1*s and x1*c + x0*s, with c/s
 * from the f32 table row pos0+t.  The v slice is copied unchanged
 * (kernels.rs:134-137). */
void kvo_rope(const uint16_t* qkv, const float* cos_t, const float* sin_t, float* out, size_t t,
              size_t pos0, size_t n_q, size_t n_kv, size_t head_dim, int dtype) {
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    const size_t half = head_dim / 2;
    for (size_t i = 0; i < t * stride; ++i) out[i] = kvo_to_f32(qkv[i], dtype);
    for (size_t tok = 0; tok < t; ++tok) {
        for (size_t h = 0; h < n_q + n_kv; ++h) {
            float* v = out + tok * stride + h * head_dim;
            for (size_t j = 0; j < half; ++j) {
                float c = cos_t[(pos0 + tok) * half + j];
                float s = sin_t[(pos0 + tok) * half + j];
                float x0 = v[j], x1 = v[j + half];
                v[j] = x0 * c - x1 * s;
                v[j + half] = x1 * c + x0 * s;
            }
        }
    }
}

/* engine/tests/kernels.rs:220-232 -- k and v slices of qkv row t land at
 * kc/vc[(h*max_seq + pos0+t)*hd + d]; every other slot is untouched. */
void kvo_kv_append(const uint16_t* qkv, uint16_t* kc, uint16_t* vc, size_t t, size_t pos0,
                   size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq) {
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    for (size_t tok = 0; tok < t; ++tok) {
        const uint16_t* row = qkv + tok * stride;
        for (size_t h = 0; h < n_kv; ++h) {
            size_t dst = (h * max_seq + pos0 + tok) * head_dim;
            memcpy(kc + dst, row + n_q * head_dim + h * head_dim, head_dim * 2);
            memcpy(vc + dst, row + (n_q + n_kv) * head_dim + h * head_dim, head_dim * 2);
        }
    }
}

/* One query head against keys [0, kv_len) of one kv head, in f64
 * (engine/tests/kernels.rs:273-287): scores = q.k * scale, softmax with max
 * subtraction, out[d] = sum_j p_j v_j[d] / sum_j p_j. */
static void attend_one(const float* q, const uint16_t* kbase, const uint16_t* vbase,
                       size_t kv_len, size_t head_dim, double scale, float* out, int dtype,
                       double* scores) {
    double m = -INFINITY;
    for (size_t j = 0; j < kv_len; ++j) {
        const uint16_t* k = kbase + j * head_dim;
        double acc = 0.0;
        for (size_t d = 0; d < head_dim; ++d) acc += (double)q[d] * (double)kvo_to_f32(k[d], dtype);
        acc *= scale;
        scores[j] = acc;
        if (acc > m) m = acc;
    }
    double denom = 0.0;
    for (size_t j = 0; j < kv_len; ++j) {
        scores[j] = exp(scores[j] - m);
        denom += scores[j];
    }
    for (size_t d = 0; d < head_dim; ++d) {
        double acc = 0.0;
        for (size_t j = 0; j < kv_len; ++j)
            acc += scores[j] * (double)kvo_to_f32(vbase[j * head_dim + d], dtype);
        out[d] = (float)(acc / denom);
    }
}

/* engine/tests/kernels.rs:264-289 -- causal GQA attention over the
 * contiguous cache: query t (position pos0+t) of head h attends keys
 * [0, pos0+t] of kv head h/(n_q/n_kv), scale 1/sqrt(hd) (kernels.rs:350). */
void kvo_attention(const uint16_t* qkv, const uint16_t* kc, const uint16_t* vc, float* out,
                   size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim,
                   size_t max_seq, int dtype) {
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    const size_t group = n_q / n_kv;
    const double scale = 1.0 / sqrt((double)head_dim);
#pragma omp parallel num_threads(g_threads)
    {
        double* scores = (double*)malloc(sizeof(double) * (pos0 + t + 1));
        float* q = (float*)malloc(sizeof(float) * head_dim);
#pragma omp for schedule(dynamic) collapse(2)
        for (long long tok = 0; tok < (long long)t; ++tok) {
            for (long long h = 0; h < (long long)n_q; ++h) {
                size_t kvh = (size_t)h / group;
                for (size_t d = 0; d < head_dim; ++d)
                    q[d] = kvo_to_f32(qkv[(size_t)tok * stride + (size_t)h * head_dim + d], dtype);
                attend_one(q, kc + kvh * max_seq * head_dim, vc + kvh * max_seq * head_dim,
                           pos0 + (size_t)tok + 1, head_dim, scale,
                           out + ((size_t)tok * n_q + (size_t)h) * head_dim, dtype, scores);
            }
        }
        free(scores);
        free(q);
    }
}

/* Batched single-query decode over per-sequence caches laid out
 * [n_seq][n_kv][max_seq][hd]: the same f64 formula as kvo_attention
 * (engine/tests/kernels.rs:264-289) for one query per sequence that attends
 * keys [0, lens[b]). */
void kvo_attention_decode(const uint16_t* q, size_t q_row_stride, const uint16_t* kc,
                          const uint16_t* vc, const int32_t* lens, size_t n_seq, size_t n_q,
                          size_t n_kv, size_t head_dim, size_t max_seq, double scale,
                          float* out, int dtype) {
    const size_t group = n_q / n_kv;
    size_t max_len = 1;
    for (size_t b = 0; b < n_seq; ++b)
        if ((size_t)lens[b] > max_len) max_len = (size_t)lens[b];
#pragma omp parallel num_threads(g_threads)
    {
        double* scores = (double*)malloc(sizeof(double) * max_len);
        float* qf = (float*)malloc(sizeof(float) * head_dim);
#pragma omp for schedule(dynamic) collapse(2)
        for (long long b = 0; b < (long long)n_seq; ++b) {
            for (long long h = 0; h < (long long)n_q; ++h) {
                size_t kvh = (size_t)h / group;
                size_t base = (((size_t)b * n_kv + kvh) * max_seq) * head_dim;
                for (size_t d = 0; d < head_dim; ++d)
                    qf[d] = kvo_to_f32(q[(size_t)b * q_row_stride + (size_t)h * head_dim + d], dtype);
                attend_one(qf, kc + base, vc + base, (size_t)lens[b], head_dim, scale,
                           out + ((size_t)b * n_q + (size_t)h) * head_dim, dtype, scores);
            }
        }
        free(scores);
        free(qf);
    }
}

/* engine/tests/kernels.rs:151-158 -- out[r][i] = g/(1+exp(-g))*u in f64,
 * g = gu[r][i], u = gu[r][inter+i]. */
void kvo_silu_mul(const uint16_t* gu, float* out, size_t t, size_t inter, int dtype) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (long long r = 0; r < (long long)t; ++r) {
        for (size_t i = 0; i < inter; ++i) {
            double g = (double)kvo_to_f32(gu[(size_t)r * 2 * inter + i], dtype);
            double u = (double)kvo_to_f32(gu[(size_t)r * 2 * inter + inter + i], dtype);
            out[(size_t)r * inter + i] = (float)(g / (1.0 + exp(-g)) * u);
        }
    }
}

/* engine/tests/kernels.rs:172-174 -- exact: out = round16(f32(x) + f32(y)). */
void kvo_add(const uint16_t* x, const uint16_t* y, uint16_t* out, size_t n, int dtype) {
    for (size_t i = 0; i < n; ++i)
        out[i] = kvo_from_f32(kvo_to_f32(x[i], dtype) + kvo_to_f32(y[i], dtype), dtype);
}

/* engine/tests/kernels.rs:181-193 and engine/kernels/elementwise.cu:11-20 --
 * dst = f16(bf16 value), and count the values with !(|v| <= 65504). */
uint32_t kvo_bf16_to_f16(const uint16_t* src, uint16_t* dst, size_t n) {
    uint32_t bad = 0;
    for (size_t i = 0; i < n; ++i) {
        float v = bf16_to_f32(src[i]);
        if (!(fabsf(v) <= 65504.0f)) bad++;
        dst[i] = f32_to_f16(v);
    }
    return bad;
}

/* engine/tests/kernels.rs:318-326 -- y[r][c] = sum_k x[r][k]*w[c][k] in f64. */
void kvo_linear(const uint16_t* x, const uint16_t* w, float* y, size_t t, size_t in_dim,
                size_t out_dim, int dtype) {
    float* xf = (float*)malloc(sizeof(float) * t * in_dim);
    kvo_to_f32_array(x, xf, t * in_dim, dtype);
#pragma omp parallel num_threads(g_threads)
    {
        float* wrow = (float*)malloc(sizeof(float) * in_dim);
#pragma omp for schedule(static)
        for (long long c = 0; c < (long long)out_dim; ++c) {
            const uint16_t* wc = w + (size_t)c * in_dim;
            for (size_t k = 0; k < in_dim; ++k) wrow[k] = kvo_to_f32(wc[k], dtype);
            for (size_t r = 0; r < t; ++r) {
                const float* xr = xf + r * in_dim;
                double acc = 0.0;
                for (size_t k = 0; k < in_dim; ++k) acc += (double)xr[k] * (double)wrow[k];
                y[r * out_dim + (size_t)c] = (float)acc;
            }
        }
        free(wrow);
    }
    free(xf);
}

/* Greedy sampling: first index of the row maximum (NaN never wins).  The
 * reference plans host greedy sampling over f32 logits (reference
 * DESIGN.md:24,109; engine/src/sampling.rs is an empty stub). */
void kvo_argmax(const float* logits, size_t rows, size_t vocab, int32_t* out) {
    for (size_t r = 0; r < rows; ++r) {
        const float* l = logits + r * vocab;
        float best = -INFINITY;
        int32_t bi = 0;
        for (size_t i = 0; i < vocab; ++i)
            if (l[i] > best) {
                best = l[i];
                bi = (int32_t)i;
            }
        out[r] = bi;
    }
}

/* ------------------------------------------------------------------------ */
/* engine/src/model/rope.rs:3-25 -- base inv_freq[j] = 1/theta^(2j/hd) in f64;
 * llama3 scaling keeps high frequencies (wavelen < orig/high), divides low
 * frequencies (wavelen > orig/low) by factor, and blends in between with
 * smooth = (orig/wavelen - low)/(high - low). */
void kvo_inv_freq(size_t head_dim, double theta, int scaled, double factor, double low_freq_factor,
                  double high_freq_factor, double orig_max_pos, double* out) {
    const double pi = 3.14159265358979323846;
    for (size_t j = 0; j < head_dim / 2; ++j) {
        double f = 1.0 / pow(theta, 2.0 * (double)j / (double)head_dim);
        if (scaled) {
            double low_wavelen = orig_max_pos / low_freq_factor;
            double high_wavelen = orig_max_pos / high_freq_factor;
            double wavelen = 2.0 * pi / f;
            if (wavelen < high_wavelen) {
                /* high frequency: unchanged */
            } else if (wavelen > low_wavelen) {
                f = f / factor;
            } else {
                double smooth =
                    (orig_max_pos / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor);
                f = (1.0 - smooth) * f / factor + smooth * f;
            }
        }
        out[j] = f;
    }
}

/* engine/src/model/rope.rs:27-39 -- cos/sin[p][j] = (f32)cos/sin(p * inv[j]) in f64. */
void kvo_cos_sin_table(size_t head_dim, double theta, int scaled, double factor,
                       double low_freq_factor, double high_freq_factor, double orig_max_pos,
                       size_t max_pos, float* cos_t, float* sin_t) {
    const size_t half = head_dim / 2;
    double* inv = (double*)malloc(sizeof(double) * half);
    kvo_inv_freq(head_dim, theta, scaled, factor, low_freq_factor, high_freq_factor, orig_max_pos,
                 inv);
    for (size_t p = 0; p < max_pos; ++p)
        for (size_t j = 0; j < half; ++j) {
            double a = (double)p * inv[j];
            cos_t[p * half + j] = (float)cos(a);
            sin_t[p * half + j] = (float)sin(a);
        }
    free(inv);
}

/* ------------------------------------------------------------------------ */
static void round_array(const float* in, uint16_t* out, size_t n, int dtype) {
    kvo_from_f32_array(in, out, n, dtype);
}

/* Rounding dither of the composed decode step (kvo_set_round_dither): each value
 * is scaled by (1 + u * rel), u uniform in [-1, 1) from a counter-based hash,
 * before it is rounded to 16 bits.  It models the freedom of another correct
 * evaluation whose sums are formed in f32 and in another order (a GPU): such a
 * sum differs from the f64 one by a small relative amount, and where that
 * straddles a rounding boundary the 16-bit results differ by one ulp.  Applied
 * only at rounding points that follow a sum (norms, projections, attention,
 * SiLU), not after RoPE or the residual add, which both sides compute exactly
 * alike. */
static double g_dither_rel = 0.0;
static uint64_t g_dither_ctr = 0;

void kvo_set_round_dither(double rel, uint64_t seed) {
    g_dither_rel = rel;
    g_dither_ctr = mix64(seed);
}

static void round_dithered(const float* in, uint16_t* out, size_t n, int dtype) {
    if (g_dither_rel <= 0.0) {
        round_array(in, out, n, dtype);
        return;
    }
    for (size_t i = 0; i < n; ++i) {
        const uint64_t h = mix64(g_dither_ctr++);
        const double u = (double)(h >> 11) * (2.0 / 9007199254740992.0) - 1.0; /* [-1, 1) */
        out[i] = kvo_from_f32((float)((double)in[i] * (1.0 + u * g_dither_rel)), dtype);
    }
}

/* One decode step, composed as the reference's planned forward pass orders
 * it (reference DESIGN.md:36-74, §3 call stack of the planned llama.rs):
 * embedding -> per layer [rmsnorm, qkv linear, rope, kv_append, attention,
 * o linear, residual add, rmsnorm, gate/up linear, silu_mul, down linear,
 * residual add] -> final rmsnorm -> tied LM head (f32 logits) -> argmax. */
void kvo_decode_step(const kvo_model_dims* d, const kvo_model_weights* w, const float* cos_t,
                     const float* sin_t, uint16_t* kc, uint16_t* vc, const int32_t* ids,
                     const int32_t* pos, size_t n_seq, float* logits, int32_t* ids_out, int dtype) {
    const size_t H = d->hidden, I = d->inter, hd = d->head_dim;
    const size_t qd = d->n_q * hd, kvd = d->n_kv * hd, qkvd = qd + 2 * kvd;
    const size_t layer_cache = d->n_kv * d->max_seq * hd;
    const size_t seq_cache = d->n_layers * layer_cache;

    uint16_t* x = (uint16_t*)malloc(2 * H);
    uint16_t* hbuf = (uint16_t*)malloc(2 * H);
    uint16_t* qkv = (uint16_t*)malloc(2 * qkvd);
    uint16_t* attn = (uint16_t*)malloc(2 * qd);
    uint16_t* o = (uint16_t*)malloc(2 * H);
    uint16_t* gu = (uint16_t*)malloc(2 * 2 * I);
    uint16_t* act = (uint16_t*)malloc(2 * I);
    float* f = (float*)malloc(sizeof(float) * (2 * I > qkvd ? 2 * I : qkvd));

    for (size_t b = 0; b < n_seq; ++b) {
        const int32_t p = pos[b];
        const int32_t len = p + 1;
        kvo_embedding_gather(&ids[b], 1, w->embed, d->vocab, x, H);
        for (size_t l = 0; l < d->n_layers; ++l) {
            uint16_t* kl = kc + b * seq_cache + l * layer_cache;
            uint16_t* vl = vc + b * seq_cache + l * layer_cache;
            kvo_rmsnorm(x, w->attn_norm[l], f, 1, H, d->eps, dtype);
            round_dithered(f, hbuf, H, dtype);
            kvo_linear(hbuf, w->w_qkv[l], f, 1, H, qkvd, dtype);
            round_dithered(f, qkv, qkvd, dtype);
            kvo_rope(qkv, cos_t, sin_t, f, 1, (size_t)p, d->n_q, d->n_kv, hd, dtype);
            round_array(f, qkv, qkvd, dtype);
            kvo_kv_append(qkv, kl, vl, 1, (size_t)p, d->n_q, d->n_kv, hd, d->max_seq);
            kvo_attention_decode(qkv, qkvd, kl, vl, &len, 1, d->n_q, d->n_kv, hd, d->max_seq,
                                 1.0 / sqrt((double)hd), f, dtype);
            round_dithered(f, attn, qd, dtype);
            kvo_linear(attn, w->w_o[l], f, 1, qd, H, dtype);
            round_dithered(f, o, H, dtype);
            kvo_add(x, o, x, H, dtype);
            kvo_rmsnorm(x, w->mlp_norm[l], f, 1, H, d->eps, dtype);
            round_dithered(f, hbuf, H, dtype);
            kvo_linear(hbuf, w->w_gu[l], f, 1, H, 2 * I, dtype);
            round_dithered(f, gu, 2 * I, dtype);
            kvo_silu_mul(gu, f, 1, I, dtype);
            round_dithered(f, act, I, dtype);
            kvo_linear(act, w->w_down[l], f, 1, I, H, dtype);
            round_dithered(f, o, H, dtype);
            kvo_add(x, o, x, H, dtype);
        }
        kvo_rmsnorm(x, w->final_norm, f, 1, H, d->eps, dtype);
        round_dithered(f, hbuf, H, dtype);
        kvo_linear(hbuf, w->embed, logits + b * d->vocab, 1, H, d->vocab, dtype);
        kvo_argmax(logits + b * d->vocab, 1, d->vocab, &ids_out[b]);
    }
    free(x);
    free(hbuf);
    free(qkv);
    free(attn);
    free(o);
    free(gu);
    free(act);
    free(f);
}
