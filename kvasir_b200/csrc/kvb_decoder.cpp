// kvb_decoder.cpp -- decode-step driver: one token for each of n_seq
// independent sequences through an n_layers Llama decoder, composed from the
// kvb_* kernels and cuBLAS projections and replayed as one CUDA graph.
//
// Layer order follows the reference's planned forward pass (reference
// DESIGN.md:36-74, §3 of its call stack): rmsnorm -> qkv projection -> RoPE +
// KV append -> attention -> o projection -> residual add -> rmsnorm -> gate/up
// projection -> SiLU*mul -> down projection -> residual add; then the final
// norm, the tied LM head (f32 logits) and greedy argmax.  The residual add is
// fused into the following rmsnorm (kvb_add_rmsnorm); RoPE, the KV append and
// decode attention are one launch (kvb_rope_attention_decode, in the step form
// that starts its K/V reads before the preceding kernel completes) on contiguous
// caches at head_dim 64.  All device memory is caller-owned.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "kvb_host.h"

extern "C" int kvb_blas_set_workspace(kvb_blas_t b, void* ws, size_t len);
extern "C" int kvb_blas_set_autotune(kvb_blas_t b, int enable);

namespace {

constexpr size_t kAlign = 256;
constexpr size_t kBlasWorkspace = 32u << 20;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Layout {  // byte offsets into the workspace
    size_t x, h, qkv, attn, o, gu, act, logits, ids_in, ids_out, pos, lens, attn_ws, lm_ws, blas_ws,
        total;
    size_t attn_ws_len, lm_ws_len;
};

Layout make_layout(const kvb_decoder_config& c) {
    const size_t e = 2;  // 16-bit activations
    const size_t B = (size_t)c.n_seq;
    const size_t qd = (size_t)c.n_q * c.head_dim, kvd = (size_t)c.n_kv * c.head_dim;
    Layout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes);
        return at;
    };
    L.x = take(B * c.hidden * e);
    L.h = take(B * c.hidden * e);
    L.qkv = take(B * (qd + 2 * kvd) * e);
    L.attn = take(B * qd * e);
    L.o = take(B * c.hidden * e);
    L.gu = take(B * 2 * (size_t)c.inter * e);
    L.act = take(B * (size_t)c.inter * e);
    L.logits = take(B * (size_t)c.vocab * 4);
    L.ids_in = take(B * 4);
    L.ids_out = take(B * 4);
    L.pos = take(B * 4);
    L.lens = take(B * 4);
    L.attn_ws_len = kvb_attention_decode_workspace_bytes(B, (size_t)c.max_seq, (size_t)c.n_q,
                                                         (size_t)c.n_kv, (size_t)c.head_dim);
    L.attn_ws = take(L.attn_ws_len);
    L.lm_ws_len = B <= 32 ? kvb_lm_head_argmax_workspace_bytes(B) : 0;
    L.lm_ws = take(L.lm_ws_len);
    L.blas_ws = take(kBlasWorkspace);
    L.total = off;
    return L;
}

}  // namespace

struct kvb_decoder_s {
    kvb_decoder_config cfg;
    Layout lay;
    uint8_t* ws = nullptr;
    const void* embed = nullptr;
    const void* lm_head = nullptr;  // untied checkpoints; nullptr: the embedding table
    float temperature = 0.f;        // <= 0: greedy
    float top_p = 1.f;
    uint64_t seed = 0;
    bool fused_lm_head = false;     // greedy steps: kvb_lm_head_argmax where it applies
    bool row_projections = false;   // kvb_linear_rows / kvb_linear_silu_mul where they apply
    const void* final_norm = nullptr;
    std::vector<const void*> attn_norm, w_qkv, w_o, mlp_norm, w_gu, w_down;
    uint8_t* kc = nullptr;
    uint8_t* vc = nullptr;
    // paged cache (kvb_decoder_use_paged_cache): per-layer pools of pool_len
    // elements, one block table shared by all layers
    uint8_t* kpool = nullptr;
    uint8_t* vpool = nullptr;
    size_t pool_len = 0, max_blocks = 0, block_size = 0;
    const int32_t* block_table = nullptr;
    const float* cos_t = nullptr;
    const float* sin_t = nullptr;
    kvb_blas_t blas = nullptr;
    cudaStream_t capture_stream = nullptr;  // private: the legacy stream cannot be captured
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int own_launches = 0, lib_launches = 0;

    template <typename T = void>
    T* at(size_t off) const {
        return reinterpret_cast<T*>(ws + off);
    }
};

static int record_step(kvb_decoder_s* d, kvb_stream_t s) {
    const kvb_decoder_config& c = d->cfg;
    const size_t B = (size_t)c.n_seq, H = (size_t)c.hidden, I = (size_t)c.inter;
    const size_t hd = (size_t)c.head_dim, nq = (size_t)c.n_q, nkv = (size_t)c.n_kv;
    const size_t qd = nq * hd, kvd = nkv * hd, qkvd = qd + 2 * kvd;
    const size_t max_seq = (size_t)c.max_seq;
    const size_t seq_stride = nkv * max_seq * hd;          // elements per sequence per layer
    const size_t layer_elems = B * seq_stride;              // elements per layer cache
    const size_t table_len = max_seq * (hd / 2);
    const int dt = c.dtype;
    const Layout& L = d->lay;
    int own = 0, lib = 0;
    int st;
#define STEP(call, is_lib)         \
    do {                           \
        st = (call);               \
        if (st != KVB_OK) return st; \
        (is_lib) ? ++lib : ++own;  \
    } while (0)

    // embedding gather + layer 0's attention norm (one launch for decode-sized batches)
    STEP(kvb_embedding_rmsnorm(s, d->at<int32_t>(L.ids_in), B, d->embed, (size_t)c.vocab * H,
                               d->attn_norm[0], H, d->at(L.x), B * H, d->at(L.h), B * H, H, c.eps,
                               dt),
         false);
    if (!kvb::embedding_rmsnorm_fused(B, H, d->embed, d->attn_norm[0], d->at(L.x), d->at(L.h)))
        ++own;  // it ran as two launches
    // one projection y[B, out] = x[B, in] w^T: this library's kernel for decode-sized
    // batches where enabled and supported, else cuBLAS
    const bool rows_proj = d->row_projections && B <= 128;
    auto proj = [&](const void* x, size_t in, const void* w, void* y, size_t out) -> int {
        if (rows_proj) {
            const int r = kvb_linear_rows(s, x, B * in, w, out * in, y, B * out, B, in, out, 0, dt);
            if (r != KVB_ERR_UNSUPPORTED) {
                if (r == KVB_OK) ++own;
                return r;
            }
        }
        const int r = kvb_linear(d->blas, s, x, B * in, w, out * in, y, B * out, B, in, out, dt, 0);
        if (r == KVB_OK) ++lib;
        return r;
    };
    for (int l = 0; l < c.n_layers; ++l) {
        st = proj(d->at(L.h), H, d->w_qkv[l], d->at(L.qkv), qkvd);
        if (st != KVB_OK) return st;
        if (!d->block_table) {
            uint8_t* kl = d->kc + (size_t)l * layer_elems * 2;
            uint8_t* vl = d->vc + (size_t)l * layer_elems * 2;
            if (hd == 64 && nq / nkv <= 16) {  // RoPE, KV append and attention: one launch
                STEP(kvb::rope_attention_decode_in_step(
                         s, d->at(L.qkv), B * qkvd, d->cos_t, d->sin_t, table_len, kl, vl,
                         seq_stride, layer_elems, d->at<int32_t>(L.lens), B, max_seq, nq, nkv, hd,
                         max_seq, 1.0f / sqrtf((float)hd), d->at(L.attn), qd, d->at(L.attn_ws),
                         L.attn_ws_len, dt),
                     false);
            } else {
                STEP(kvb_rope_kv_append_batched(s, d->at(L.qkv), B, d->at<int32_t>(L.pos), d->cos_t,
                                                d->sin_t, table_len, kl, vl, seq_stride,
                                                layer_elems, nq, nkv, hd, max_seq, dt),
                     false);
                STEP(kvb_attention_decode(s, d->at(L.qkv), qkvd, kl, vl, seq_stride, layer_elems,
                                          d->at<int32_t>(L.lens), B, max_seq, nq, nkv, hd, max_seq,
                                          1.0f / sqrtf((float)hd), d->at(L.attn), qd,
                                          d->at(L.attn_ws), L.attn_ws_len, dt),
                     false);
            }
        } else {
            uint8_t* kl = d->kpool + (size_t)l * d->pool_len * 2;
            uint8_t* vl = d->vpool + (size_t)l * d->pool_len * 2;
            // paged mode requires head_dim 64 and 64-key blocks: always one launch
            STEP(kvb::rope_attention_decode_paged_in_step(
                     s, d->at(L.qkv), B * qkvd, d->cos_t, d->sin_t, table_len, kl, vl,
                     d->pool_len, d->block_table, d->max_blocks, d->block_size,
                     d->at<int32_t>(L.lens), B, max_seq, nq, nkv, hd, 1.0f / sqrtf((float)hd),
                     d->at(L.attn), qd, d->at(L.attn_ws), L.attn_ws_len, dt),
                 false);
        }
        own += kvb::decode_combine_launches(B, max_seq, nq, nkv, hd, d->at(L.attn_ws),
                                            L.attn_ws_len);  // the split-KV combine pass
        st = proj(d->at(L.attn), qd, d->w_o[l], d->at(L.o), H);
        if (st != KVB_OK) return st;
        STEP(kvb_add_rmsnorm(s, d->at(L.x), B * H, d->at(L.o), B * H, d->mlp_norm[l], H, d->at(L.h),
                             B * H, B, H, c.eps, dt),
             false);
        int gst = KVB_ERR_UNSUPPORTED;
        if (rows_proj) {  // gate/up projection and SiLU*mul in one pass
            gst = kvb_linear_silu_mul(s, d->at(L.h), B * H, d->w_gu[l], 2 * I * H, d->at(L.act),
                                      B * I, B, H, I, 0, dt);
            if (gst != KVB_OK && gst != KVB_ERR_UNSUPPORTED) return gst;
            if (gst == KVB_OK) ++own;
        }
        if (gst != KVB_OK) {
            STEP(kvb_linear(d->blas, s, d->at(L.h), B * H, d->w_gu[l], 2 * I * H, d->at(L.gu),
                            B * 2 * I, B, H, 2 * I, dt, 0),
                 true);
            STEP(kvb_silu_mul(s, d->at(L.gu), B * 2 * I, d->at(L.act), B * I, B, I, dt), false);
        }
        st = proj(d->at(L.act), I, d->w_down[l], d->at(L.o), H);
        if (st != KVB_OK) return st;
        const void* next_norm = (l + 1 < c.n_layers) ? d->attn_norm[l + 1] : d->final_norm;
        STEP(kvb_add_rmsnorm(s, d->at(L.x), B * H, d->at(L.o), B * H, next_norm, H, d->at(L.h), B * H,
                             B, H, c.eps, dt),
             false);
    }
    const void* head = d->lm_head ? d->lm_head : d->embed;
    int fst = KVB_ERR_UNSUPPORTED;
    if (d->fused_lm_head && d->temperature <= 0.f && L.lm_ws_len > 0) {
        // LM head + greedy argmax in one pass: the logits are never stored
        fst = kvb_lm_head_argmax(s, d->at(L.h), B * H, head, (size_t)c.vocab * H, B, H,
                                 (size_t)c.vocab, d->at(L.lm_ws), L.lm_ws_len,
                                 d->at<int32_t>(L.ids_out), d->at<int32_t>(L.pos),
                                 d->at<int32_t>(L.lens), dt);
        if (fst != KVB_OK && fst != KVB_ERR_UNSUPPORTED) return fst;
        if (fst == KVB_OK) own += 2;  // the pass and the merge of its per-CTA partials
    }
    if (fst != KVB_OK) {
        STEP(kvb_linear(d->blas, s, d->at(L.h), B * H, head, (size_t)c.vocab * H,
                        d->at<float>(L.logits), B * (size_t)c.vocab, B, H, (size_t)c.vocab, dt, 1),
             true);
        // sampling reads each sequence's position as its counter, then advances it
        STEP(kvb_sample_f32(s, d->at<float>(L.logits), B, (size_t)c.vocab, d->temperature, d->top_p,
                            d->seed, d->at<int32_t>(L.pos), d->at<int32_t>(L.ids_out),
                            d->at<int32_t>(L.pos), d->at<int32_t>(L.lens)),
             false);
    }
    cudaError_t e = cudaMemcpyAsync(d->at(L.ids_in), d->at(L.ids_out), B * 4,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder: ids copy");
#undef STEP
    d->own_launches = own;
    d->lib_launches = lib;
    return KVB_OK;
}

extern "C" {

size_t kvb_decoder_workspace_bytes(const kvb_decoder_config* cfg) {
    if (!cfg) return 0;
    return make_layout(*cfg).total;
}

int kvb_decoder_create(kvb_decoder_t* out, const kvb_decoder_config* cfg,
                       const kvb_decoder_weights* w, void* kc, void* vc, const float* cos_t,
                       const float* sin_t, void* workspace, size_t workspace_len) {
    KVB_CHECK(out && cfg && w && kc && vc && cos_t && sin_t && workspace,
              "decoder_create: null argument");
    const kvb_decoder_config& c = *cfg;
    KVB_CHECK_DTYPE(c.dtype);
    KVB_CHECK(c.hidden > 0 && c.inter > 0 && c.n_layers > 0 && c.n_q > 0 && c.n_kv > 0 &&
                  c.head_dim > 0 && c.vocab > 0 && c.max_seq > 0 && c.n_seq > 0,
              "decoder_create: every dimension must be positive");
    KVB_CHECK(c.n_q % c.n_kv == 0, "decoder_create: n_q %d not a multiple of n_kv %d", c.n_q, c.n_kv);
    KVB_CHECK(c.head_dim % 2 == 0, "decoder_create: odd head_dim %d", c.head_dim);
    const Layout L = make_layout(c);
    KVB_CHECK(workspace_len >= L.total, "decoder_create: workspace of %zu bytes, need %zu",
              workspace_len, L.total);
    kvb_decoder_s* d = new kvb_decoder_s();
    d->cfg = c;
    d->lay = L;
    d->ws = static_cast<uint8_t*>(workspace);
    d->embed = w->embed;
    d->final_norm = w->final_norm;
    for (int l = 0; l < c.n_layers; ++l) {
        d->attn_norm.push_back(w->attn_norm[l]);
        d->w_qkv.push_back(w->w_qkv[l]);
        d->w_o.push_back(w->w_o[l]);
        d->mlp_norm.push_back(w->mlp_norm[l]);
        d->w_gu.push_back(w->w_gu[l]);
        d->w_down.push_back(w->w_down[l]);
    }
    d->kc = static_cast<uint8_t*>(kc);
    d->vc = static_cast<uint8_t*>(vc);
    d->cos_t = cos_t;
    d->sin_t = sin_t;
    int st = kvb_blas_create(&d->blas);
    if (st == KVB_OK) st = kvb_blas_set_workspace(d->blas, d->at(L.blas_ws), kBlasWorkspace);
    if (st == KVB_OK) st = kvb_blas_set_autotune(d->blas, 1);
    if (st == KVB_OK) {
        cudaError_t e = cudaStreamCreateWithFlags(&d->capture_stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) st = kvb::cuda_fail(e, "decoder_create: capture stream");
    }
    if (st == KVB_OK) {
        cudaError_t e = cudaMemset(d->ws, 0, L.blas_ws);  // activations, counters, ids
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) st = kvb::cuda_fail(e, "decoder_create: workspace clear");
    }
    if (st != KVB_OK) {
        if (d->capture_stream) cudaStreamDestroy(d->capture_stream);
        kvb_blas_destroy(d->blas);
        delete d;
        return st;
    }
    *out = d;
    return KVB_OK;
}

int kvb_decoder_destroy(kvb_decoder_t d) {
    if (!d) return KVB_OK;
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    if (d->capture_stream) cudaStreamDestroy(d->capture_stream);
    kvb_blas_destroy(d->blas);
    delete d;
    return KVB_OK;
}

// The captured step holds the old pointers: the next step records a new graph.
static void drop_graph(kvb_decoder_t d) {
    if (d->exec) {
        cudaGraphExecDestroy(d->exec);
        d->exec = nullptr;
    }
    if (d->graph) {
        cudaGraphDestroy(d->graph);
        d->graph = nullptr;
    }
}

int kvb_decoder_use_paged_cache(kvb_decoder_t d, void* k_pools, void* v_pools, size_t pool_len,
                                const int32_t* block_table, size_t max_blocks, size_t block_size) {
    KVB_CHECK(d && k_pools && v_pools && block_table, "decoder_use_paged_cache: null argument");
    const kvb_decoder_config& c = d->cfg;
    const size_t per_block = (size_t)c.n_kv * block_size * (size_t)c.head_dim;
    KVB_CHECK(block_size > 0 && pool_len > 0 && pool_len % per_block == 0,
              "decoder_use_paged_cache: pool of %zu elems is not a whole number of %zu-elem blocks",
              pool_len, per_block);
    KVB_CHECK(max_blocks * block_size >= (size_t)c.max_seq,
              "decoder_use_paged_cache: %zu blocks of %zu hold fewer than max_seq %d positions",
              max_blocks, block_size, c.max_seq);
    if (!(c.head_dim == 64 && block_size % 64 == 0))
        return kvb::fail(KVB_ERR_UNSUPPORTED,
                         "decoder_use_paged_cache: needs head_dim 64 and block_size a multiple of 64");
    d->kpool = static_cast<uint8_t*>(k_pools);
    d->vpool = static_cast<uint8_t*>(v_pools);
    d->pool_len = pool_len;
    d->block_table = block_table;
    d->max_blocks = max_blocks;
    d->block_size = block_size;
    drop_graph(d);  // the next step records the paged step
    return KVB_OK;
}

int kvb_decoder_set_sampling(kvb_decoder_t d, float temperature, float top_p, uint64_t seed) {
    KVB_CHECK(d, "decoder_set_sampling: null decoder");
    KVB_CHECK(temperature == temperature && top_p == top_p,
              "decoder_set_sampling: temperature and top_p must be numbers");
    d->temperature = temperature;
    d->top_p = top_p;
    d->seed = seed;
    drop_graph(d);
    return KVB_OK;
}

int kvb_decoder_set_fused_lm_head(kvb_decoder_t d, int enable) {
    KVB_CHECK(d, "decoder_set_fused_lm_head: null decoder");
    d->fused_lm_head = enable != 0;
    drop_graph(d);
    return KVB_OK;
}

int kvb_decoder_set_row_projections(kvb_decoder_t d, int enable) {
    KVB_CHECK(d, "decoder_set_row_projections: null decoder");
    d->row_projections = enable != 0;
    drop_graph(d);
    return KVB_OK;
}

int kvb_decoder_set_lm_head(kvb_decoder_t d, const void* lm_head) {
    KVB_CHECK(d, "decoder_set_lm_head: null decoder");
    d->lm_head = lm_head;
    drop_graph(d);
    return KVB_OK;
}

int kvb_decoder_set_lengths(kvb_decoder_t d, kvb_stream_t s, const int32_t* cur_len_host) {
    KVB_CHECK(d && cur_len_host, "decoder_set_lengths: null argument");
    const int B = d->cfg.n_seq;
    std::vector<int32_t> pos(cur_len_host, cur_len_host + B), lens(B);
    for (int b = 0; b < B; ++b) {
        KVB_CHECK(pos[b] >= 0 && pos[b] < d->cfg.max_seq,
                  "decoder_set_lengths: length %d of sequence %d outside [0, %d)", pos[b], b,
                  d->cfg.max_seq);
        lens[b] = pos[b] + 1;
    }
    cudaError_t e = cudaMemcpyAsync(d->at(d->lay.pos), pos.data(), B * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d->at(d->lay.lens), lens.data(), B * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_set_lengths");
    return KVB_OK;
}

int32_t* kvb_decoder_ids_in(kvb_decoder_t d) { return d ? d->at<int32_t>(d->lay.ids_in) : nullptr; }
int32_t* kvb_decoder_ids_out(kvb_decoder_t d) { return d ? d->at<int32_t>(d->lay.ids_out) : nullptr; }
const float* kvb_decoder_logits(kvb_decoder_t d) { return d ? d->at<float>(d->lay.logits) : nullptr; }

// Runs each projection shape of the step once, eagerly on `s`, so that the
// autotuned GEMMs are chosen before the step is captured (a capture cannot time
// anything).  Inputs and outputs are the step's own scratch buffers, all fully
// rewritten by every step before they are read.
static int tune_projections(kvb_decoder_s* d, kvb_stream_t s) {
    const kvb_decoder_config& c = d->cfg;
    const size_t B = (size_t)c.n_seq, H = (size_t)c.hidden, I = (size_t)c.inter;
    const size_t qd = (size_t)c.n_q * c.head_dim, qkvd = qd + 2 * (size_t)c.n_kv * c.head_dim;
    const size_t V = (size_t)c.vocab;
    const int dt = c.dtype;
    const Layout& L = d->lay;
    int st = kvb_linear(d->blas, s, d->at(L.h), B * H, d->w_qkv[0], qkvd * H, d->at(L.qkv), B * qkvd,
                        B, H, qkvd, dt, 0);
    if (st == KVB_OK)
        st = kvb_linear(d->blas, s, d->at(L.attn), B * qd, d->w_o[0], H * qd, d->at(L.o), B * H, B,
                        qd, H, dt, 0);
    if (st == KVB_OK)
        st = kvb_linear(d->blas, s, d->at(L.h), B * H, d->w_gu[0], 2 * I * H, d->at(L.gu), B * 2 * I,
                        B, H, 2 * I, dt, 0);
    if (st == KVB_OK)
        st = kvb_linear(d->blas, s, d->at(L.act), B * I, d->w_down[0], H * I, d->at(L.o), B * H, B,
                        I, H, dt, 0);
    if (st == KVB_OK)
        st = kvb_linear(d->blas, s, d->at(L.h), B * H, d->lm_head ? d->lm_head : d->embed, V * H,
                        d->at<float>(L.logits), B * V, B, H, V, dt, 1);
    if (st != KVB_OK) return st;
    const cudaError_t e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? KVB_OK : kvb::cuda_fail(e, "decoder: projection tuning");
}

int kvb_decoder_step(kvb_decoder_t d, kvb_stream_t s) {
    KVB_CHECK(d != nullptr, "decoder_step: null decoder");
    if (!d->exec) {
        const int tst = tune_projections(d, s);
        if (tst != KVB_OK) return tst;
        kvb::sample_prepare();
        // Record the step once on the private capture stream (recording runs
        // nothing); host-side work (argument checks, tensor-map encoding)
        // happens only here, every step is then one graph launch on `s`.
        cudaStream_t cs = d->capture_stream;
        cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_step: begin capture");
        const int st = record_step(d, cs);
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(cs, &g);
        if (st != KVB_OK) {
            if (g) cudaGraphDestroy(g);
            return st;
        }
        if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_step: end capture");
        e = cudaGraphInstantiate(&d->exec, g, 0);
        if (e != cudaSuccess) {
            cudaGraphDestroy(g);
            return kvb::cuda_fail(e, "decoder_step: instantiate");
        }
        d->graph = g;
    }
    cudaError_t e = cudaGraphLaunch(d->exec, s);
    if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_step: graph launch");
    return KVB_OK;
}

int kvb_decoder_step_host(kvb_decoder_t d, kvb_stream_t s, const int32_t* ids_host_in,
                          int32_t* ids_host_out) {
    KVB_CHECK(d && ids_host_in && ids_host_out, "decoder_step_host: null argument");
    const size_t bytes = (size_t)d->cfg.n_seq * 4;
    cudaError_t e = cudaMemcpyAsync(d->at(d->lay.ids_in), ids_host_in, bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_step_host: ids upload");
    const int st = kvb_decoder_step(d, s);
    if (st != KVB_OK) return st;
    e = cudaMemcpyAsync(ids_host_out, d->at(d->lay.ids_out), bytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return kvb::cuda_fail(e, "decoder_step_host: ids download");
    return KVB_OK;
}

int kvb_decoder_launches_per_step(kvb_decoder_t d, int* own, int* library) {
    KVB_CHECK(d && own && library, "decoder_launches_per_step: null argument");
    *own = d->own_launches;
    *library = d->lib_launches;
    return KVB_OK;
}

}  // extern "C"
