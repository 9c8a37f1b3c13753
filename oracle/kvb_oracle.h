/*
 * kvb_oracle.h -- CPU oracle for the kvasir per-layer Llama kernel chain.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * kvasir_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load it.  Nothing in the product links
 * or calls it.
 *
 * Each function restates, in plain C, the CPU reference computation that the
 * kvasir reference tests use to check its GPU kernels (engine/tests/kernels.rs)
 * or the host setup code of the reference (engine/src/model/rope.rs).  The
 * file:line each one follows is given at its definition in kvb_oracle.c.
 *
 * Parity pinning.  The reference ships no golden vectors and cannot be built
 * here (Rust toolchain absent), so the oracle is pinned by (1) every
 * known-answer test the reference holds for this path (rope.rs:56-74,
 * config.rs:156-171, the exactness checks of tests/kernels.rs), restated in
 * tests/test_oracle.py, and (2) golden vectors produced by HuggingFace
 * transformers' Llama modules, the numerical target the reference's own
 * design names (reference DESIGN.md:124-131), committed under tests/golden/
 * with the script that made them.
 *
 * 16-bit element arrays are passed as raw uint16_t bit patterns with a dtype
 * tag: KVO_BF16 (0) or KVO_F16 (1).
 */
#ifndef KVB_ORACLE_H
#define KVB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { KVO_BF16 = 0, KVO_F16 = 1 };

/* ---- 16-bit float conversion (IEEE round-to-nearest-even) ---- */
float kvo_to_f32(uint16_t bits, int dtype);
uint16_t kvo_from_f32(float x, int dtype);
void kvo_to_f32_array(const uint16_t* in, float* out, size_t n, int dtype);
void kvo_from_f32_array(const float* in, uint16_t* out, size_t n, int dtype);

/* ---- threading for the timed CPU baseline (results do not depend on it) ---- */
void kvo_set_threads(int n);
int kvo_get_threads(void);

/* ---- seeded generator (splitmix64 + Box-Muller) ---- */
void kvo_fill_normal(uint16_t* out, size_t n, double mean, double std, uint64_t seed, int dtype);

/* ---- kernels of the chain ---- */
void kvo_embedding_gather(const int32_t* ids, size_t t, const uint16_t* table, size_t vocab,
                          uint16_t* out, size_t hidden);
void kvo_rmsnorm(const uint16_t* x, const uint16_t* w, float* out, size_t rows, size_t hidden,
                 float eps, int dtype);
void kvo_rope(const uint16_t* qkv, const float* cos_t, const float* sin_t, float* out, size_t t,
              size_t pos0, size_t n_q, size_t n_kv, size_t head_dim, int dtype);
void kvo_kv_append(const uint16_t* qkv, uint16_t* kc, uint16_t* vc, size_t t, size_t pos0,
                   size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq);
void kvo_attention(const uint16_t* qkv, const uint16_t* kc, const uint16_t* vc, float* out,
                   size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim,
                   size_t max_seq, int dtype);
void kvo_attention_decode(const uint16_t* q, size_t q_row_stride, const uint16_t* kc,
                          const uint16_t* vc, const int32_t* lens, size_t n_seq, size_t n_q,
                          size_t n_kv, size_t head_dim, size_t max_seq, double scale,
                          float* out, int dtype);
void kvo_silu_mul(const uint16_t* gu, float* out, size_t t, size_t inter, int dtype);
void kvo_add(const uint16_t* x, const uint16_t* y, uint16_t* out, size_t n, int dtype);
uint32_t kvo_bf16_to_f16(const uint16_t* src, uint16_t* dst, size_t n);
void kvo_linear(const uint16_t* x, const uint16_t* w, float* y, size_t t, size_t in_dim,
                size_t out_dim, int dtype);
void kvo_argmax(const float* logits, size_t rows, size_t vocab, int32_t* out);

/* ---- host setup: llama3-scaled RoPE tables ---- */
void kvo_inv_freq(size_t head_dim, double theta, int scaled, double factor, double low_freq_factor,
                  double high_freq_factor, double orig_max_pos, double* out);
void kvo_cos_sin_table(size_t head_dim, double theta, int scaled, double factor,
                       double low_freq_factor, double high_freq_factor, double orig_max_pos,
                       size_t max_pos, float* cos_t, float* sin_t);

/* ---- one decode step of a Llama decoder, composed from the functions above ----
 * Weights are 16-bit arrays in the reference layout (engine/src/model/weights.rs:13-27):
 * per layer attn_norm[h], w_qkv[(q+2kv), h], w_o[h, q], mlp_norm[h], w_gu[2i, h],
 * w_down[h, i]; embed[v, h] doubles as the LM head (tied).  KV caches are
 * kc/vc[seq][layer][n_kv][max_seq][hd].  Each sequence b reads token ids[b] at
 * position pos[b]; the step writes K/V at pos[b], logits[b][v] (f32) and the
 * greedy argmax ids_out[b].  Intermediate activations are rounded to the
 * 16-bit dtype at the same points the GPU chain rounds them. */
typedef struct {
    size_t hidden, inter, n_layers, n_q, n_kv, head_dim, vocab, max_seq;
    float eps;
} kvo_model_dims;

typedef struct {
    const uint16_t* embed;
    const uint16_t* final_norm;
    const uint16_t* const* attn_norm;
    const uint16_t* const* w_qkv;
    const uint16_t* const* w_o;
    const uint16_t* const* mlp_norm;
    const uint16_t* const* w_gu;
    const uint16_t* const* w_down;
} kvo_model_weights;

/* Rounding dither of kvo_decode_step (0 = off, the default): every value rounded to
 * 16 bits after a sum (norms, projections, attention, SiLU) is first scaled by
 * (1 + u*rel), u uniform in [-1, 1), seeded.  Two runs, dithered and not, show how
 * far the logits move when the 16-bit roundings of the chain land as another
 * correct evaluation in f32 may land them. */
void kvo_set_round_dither(double rel, uint64_t seed);

void kvo_decode_step(const kvo_model_dims* d, const kvo_model_weights* w, const float* cos_t,
                     const float* sin_t, uint16_t* kc, uint16_t* vc, const int32_t* ids,
                     const int32_t* pos, size_t n_seq, float* logits, int32_t* ids_out, int dtype);

#ifdef __cplusplus
}
#endif
#endif
