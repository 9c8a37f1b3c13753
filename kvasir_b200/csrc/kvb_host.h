// kvb_host.h -- host-side helpers shared by the C-ABI translation units:
// thread-local error messages, shape-check macros, device properties and
// TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "kvasir_b200.h"  // include/ (on the compiler's include path)

namespace kvb {

// Records a message for kvb_last_error() and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char* what);

inline bool fits_i32(size_t x) { return x <= 0x7fffffffull; }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline bool valid_dtype(int d) { return d == KVB_BF16 || d == KVB_F16; }

// Streaming multiprocessors of the current device (cached per device).
int num_sms();
// kvb_embedding_rmsnorm runs as one launch (else as the gather and the norm): the
// rows kvb_rmsnorm normalises with its per-row kernel, buffers 16-byte aligned.
inline bool embedding_rmsnorm_fused(size_t rows, size_t hidden, const void* table, const void* w,
                                    const void* x, const void* out) {
    return hidden % 8 == 0 && (hidden / 8) % 32 == 0 && hidden / 8 <= 32 * 16 &&
           rows <= (size_t)num_sms() * 4 && aligned(table, 16) && aligned(w, 16) &&
           aligned(x, 16) && aligned(out, 16);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// dims / box are innermost-first; strides_bytes has rank-1 entries (the
// strides of dims 1..rank-1).  128-byte swizzle, zero fill out of bounds.
int encode_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int dtype);

// Sets the sampler's kernel attributes and decides its cluster size for the
// current device, outside any stream capture (kvb_sample_f32 then makes no
// attribute or occupancy call while a step is being recorded).
void sample_prepare();

// kvb_rope_attention_decode(_paged) for the decode-step driver.  Inside its step
// the cache rows before each sequence's new key are final: no kernel that can
// still be running when the launch starts writes them (each layer's cache is
// written only by its own attention launch, and steps are separate graph
// launches).  The decode kernel may then request its first K/V tiles before it
// waits for the preceding kernel (griddepcontrol.wait).
int rope_attention_decode_in_step(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                  const float* cos_t, const float* sin_t, size_t table_len,
                                  void* kc, void* vc, size_t seq_stride, size_t cache_len,
                                  const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                                  size_t n_kv, size_t head_dim, size_t max_seq, float scale,
                                  void* out, size_t out_row_stride, void* workspace,
                                  size_t workspace_len, int dtype);
int rope_attention_decode_paged_in_step(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                        const float* cos_t, const float* sin_t, size_t table_len,
                                        void* k_pool, void* v_pool, size_t pool_len,
                                        const int32_t* block_table, size_t max_blocks,
                                        size_t block_size, const int32_t* lens, size_t n_seq,
                                        size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                        float scale, void* out, size_t out_row_stride,
                                        void* workspace, size_t workspace_len, int dtype);

// Launches of a split-KV combine pass (0 or 1) that a split-KV decode call of this
// shape and workspace makes after its decode kernel (head_dim 64, aligned buffers).
int decode_combine_launches(size_t n_seq, size_t max_len, size_t n_q, size_t n_kv,
                            size_t head_dim, const void* workspace, size_t workspace_len);

}  // namespace kvb

#define KVB_CHECK(cond, ...)                                         \
    do {                                                             \
        if (!(cond)) return ::kvb::fail(KVB_ERR_SHAPE, __VA_ARGS__); \
    } while (0)

#define KVB_CHECK_DTYPE(d) KVB_CHECK(::kvb::valid_dtype(d), "unknown dtype tag %d", (int)(d))

#define KVB_CHECK_LAUNCH(what)                                      \
    do {                                                            \
        cudaError_t e_ = cudaGetLastError();                        \
        if (e_ != cudaSuccess) return ::kvb::cuda_fail(e_, (what)); \
    } while (0)
