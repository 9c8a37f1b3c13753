/*
 * kvasir_b200.h -- C ABI of libkvasir_b200.so, the sm_100a (B200) kernel
 * chain that replaces the launch wrappers of kvasir's engine/src/gpu.
 *
 * Conventions (mirroring the reference's `impl Gpu` methods in
 * engine/src/gpu/kernels.rs:58-372 and engine/src/gpu/gemm.rs:63-115):
 *   - every buffer is a device pointer plus its length in ELEMENTS, exactly
 *     the (ptr, len) pair a cudarc CudaView carries;
 *   - every entry point validates every dimension and length before it
 *     launches anything and returns KVB_ERR_SHAPE with a message (read with
 *     kvb_last_error) instead of launching (reference ensure_shape!,
 *     engine/src/error.rs:23-30); dimensions must fit in int32
 *     (reference i32_of, kernels.rs:48-50);
 *   - launches are asynchronous on the caller's stream; no entry point
 *     synchronises, allocates device memory or frees it (reference
 *     DESIGN.md:30-33).  Kernels that need scratch take a caller-provided
 *     workspace sized by the matching *_workspace_bytes function;
 *   - 16-bit element arrays carry a dtype tag: KVB_BF16 (primary) or KVB_F16
 *     (the reference's own element type).
 */
#ifndef KVASIR_B200_H
#define KVASIR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* kvb_stream_t;

enum kvb_status {
    KVB_OK = 0,
    KVB_ERR_SHAPE = 1,       /* a size or length check failed; nothing launched */
    KVB_ERR_CUDA = 2,        /* a CUDA runtime / driver / cuBLAS call failed */
    KVB_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
    KVB_ERR_DEVICE = 4,      /* a kernel reported a device-side error (kvb_device_error) */
    KVB_ERR_CONFIG = 5,      /* checkpoint content: missing tensor, bad header, bad values
                                (reference KvasirError::Config, engine/src/error.rs) */
    KVB_ERR_IO = 6           /* a checkpoint file could not be opened or mapped
                                (reference KvasirError::Io) */
};

enum kvb_dtype { KVB_BF16 = 0, KVB_F16 = 1 };

/* Message describing the last non-OK status returned on this host thread. */
const char* kvb_last_error(void);
const char* kvb_version(void);

/* Reads and clears the device-side error word of the current device
 * (bit 1: a bounded wait timed out; 2: a sequence length out of range;
 * 4: a position outside the cache or RoPE table).  Synchronises the device. */
int kvb_device_error(uint32_t* code);

/* ---------------------------------------------------------------------------
 * Kernels with a reference counterpart (one entry per `Gpu` method).
 * ------------------------------------------------------------------------- */

/* Replaces Gpu::embedding_gather (engine/src/gpu/kernels.rs:59-88;
 * kernel engine/kernels/embedding.cu:3-10).  out[t,:] = table[ids[t],:];
 * ids outside [0, table_len/hidden) produce a zero row. */
int kvb_embedding_gather(kvb_stream_t stream, const int32_t* ids, size_t t, const void* table,
                         size_t table_len, void* out, size_t out_len, size_t hidden, int dtype);

/* Replaces Gpu::rmsnorm (kernels.rs:90-121; engine/kernels/rmsnorm.cu:3-17).
 * out = x * rsqrt(mean(x^2) + eps) * w, f32 accumulation, one rounding. */
int kvb_rmsnorm(kvb_stream_t stream, const void* x, size_t x_len, const void* w, size_t w_len,
                void* out, size_t out_len, size_t rows, size_t hidden, float eps, int dtype);

/* Replaces Gpu::rope_inplace (kernels.rs:124-169; engine/kernels/rope.cu:3-19).
 * rotate_half RoPE on the n_q + n_kv leading heads of each qkv row, token t at
 * position pos0 + t; cos/sin are f32 [max_pos, head_dim/2]. */
int kvb_rope_inplace(kvb_stream_t stream, void* qkv, size_t qkv_len, const float* cos_t,
                     size_t cos_len, const float* sin_t, size_t sin_len, size_t t, size_t pos0,
                     size_t n_q, size_t n_kv, size_t head_dim, int dtype);

/* Replaces Gpu::silu_mul (kernels.rs:171-194; engine/kernels/silu_mul.cu:3-12).
 * out[t,i] = silu(gu[t,i]) * gu[t,inter+i]. */
int kvb_silu_mul(kvb_stream_t stream, const void* gu, size_t gu_len, void* out, size_t out_len,
                 size_t t, size_t inter, int dtype);

/* Replaces Gpu::add_inplace (kernels.rs:196-209; engine/kernels/elementwise.cu:4-9). */
int kvb_add_inplace(kvb_stream_t stream, void* x, size_t x_len, const void* y, size_t y_len,
                    int dtype);

/* Replaces Gpu::bf16_to_f16 (kernels.rs:211-235; engine/kernels/elementwise.cu:11-20).
 * Adds to *bad the number of values with !(|v| <= 65504). */
int kvb_bf16_to_f16(kvb_stream_t stream, const void* src, size_t src_len, void* dst,
                    size_t dst_len, uint32_t* bad, size_t bad_len);

/* Replaces Gpu::kv_append (kernels.rs:238-291; engine/kernels/elementwise.cu:22-34).
 * Copies the k and v slices of T qkv rows to kc/vc[h, pos0+t, :] of the
 * contiguous per-layer cache [n_kv, max_seq, head_dim]. */
int kvb_kv_append(kvb_stream_t stream, const void* qkv, size_t qkv_len, void* kc, size_t kc_len,
                  void* vc, size_t vc_len, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                  size_t head_dim, size_t max_seq, int dtype);

/* Replaces Gpu::attention (kernels.rs:294-371; engine/kernels/attention.cu:5-57).
 * Causal GQA attention of T query rows (read from the qkv buffer) against the
 * contiguous cache, scale 1/sqrt(head_dim).  T == 1 runs the split-KV decode
 * kernel, T > 1 the tcgen05 prefill kernel (head_dim 64) or, for other head
 * sizes, a general kernel.  workspace may be NULL (no KV split); a workspace
 * of kvb_attention_workspace_bytes(...) bytes lets long contexts split across
 * CTAs.  Unlike the reference there is no 48 KiB / ~11.9k-key limit. */
int kvb_attention(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                  size_t kc_len, const void* vc, size_t vc_len, void* out, size_t out_len,
                  size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                  void* workspace, size_t workspace_len, int dtype);
size_t kvb_attention_workspace_bytes(size_t t, size_t pos0, size_t n_q, size_t n_kv,
                                     size_t head_dim);

/* Replaces gemm::linear_f16 / gemm::linear_f32 (engine/src/gpu/gemm.rs:17-115):
 * y[t,out] = x[t,in] * w[out,in]^T through cublasGemmEx, f32 accumulate; y is
 * 16-bit (y_f32 = 0) or f32 (y_f32 = 1).  The handle owns a cuBLAS handle. */
typedef struct kvb_blas_s* kvb_blas_t;
int kvb_blas_create(kvb_blas_t* out);
int kvb_blas_destroy(kvb_blas_t blas);
int kvb_linear(kvb_blas_t blas, kvb_stream_t stream, const void* x, size_t x_len, const void* w,
               size_t w_len, void* y, size_t y_len, size_t t, size_t in_dim, size_t out_dim,
               int dtype, int y_f32);
/* Hands cuBLAS a caller-owned device workspace (cublasSetWorkspace) so that
 * GEMMs recorded into a CUDA graph never allocate. */
int kvb_blas_set_workspace(kvb_blas_t blas, void* workspace, size_t workspace_len);
/* Autotuned projections (off by default; the decode-step driver turns it on).
 * Still cuBLAS GEMMs, same f32 accumulation: the first kvb_linear call of each
 * (device, shape, dtype, output type, workspace size) outside stream capture
 * times cublasGemmEx against the cuBLASLt algorithms the heuristic offers
 * within the handle's workspace (split-K included, in-place atomic reductions
 * excluded) and the fastest serves every later call of that shape in the
 * process.  That first call overwrites y several times and synchronises the
 * stream.  Inside a capture an untuned shape uses cublasGemmEx. */
int kvb_blas_set_autotune(kvb_blas_t blas, int enable);

/* New: linear_f16 (engine/src/gpu/gemm.rs:63-88) for decode-sized batches on
 * this library's own tensor-core kernel, no cuBLAS handle: y[rows,out] =
 * x[rows,in] * w[out,in]^T, f32 accumulate, 16-bit y.  W is streamed from HBM
 * once; the in dimension is cut into `splits` slices per 128-row tile of w
 * (0: chosen for the shape; at most 8 and at most ceil(in / 64)), whose
 * partial tiles are added in a fixed order, so a call gives the same bits on
 * every run.  The launch is a programmatic dependent of the kernel before it on
 * the stream: it reads x and writes y only after that kernel has completed, but
 * starts reading w as soon as it runs, which can be while the kernels in front
 * of it that were themselves launched that way (this library's row-norm,
 * decode-attention, combine and kvb_linear_rows / kvb_linear_silu_mul kernels)
 * are still running -- w must not be the output of such a kernel still in
 * flight.  Supported: rows <= 128, in a multiple of 8, out a multiple of 4, x
 * and w 16-byte aligned, y 8-byte aligned; otherwise KVB_ERR_UNSUPPORTED
 * (kvb_linear serves every shape). */
int kvb_linear_rows(kvb_stream_t stream, const void* x, size_t x_len, const void* w, size_t w_len,
                    void* y, size_t y_len, size_t rows, size_t in_dim, size_t out_dim, int splits,
                    int dtype);
/* New: the gate/up projection and SiLU*mul in one pass: act[rows,inter] =
 * silu(G) * U with [G | U] = x[rows,hidden] * w_gu[2*inter,hidden]^T (w_gu rows
 * 0..inter-1 gate, inter..2*inter-1 up, the layout of engine/src/model/weights.rs).
 * G and U are rounded to the 16-bit type before the SiLU*mul, as in kvb_linear
 * followed by kvb_silu_mul; the [rows, 2*inter] intermediate is never stored.
 * Splits, ordering and support as kvb_linear_rows (inter a multiple of 4). */
int kvb_linear_silu_mul(kvb_stream_t stream, const void* x, size_t x_len, const void* w_gu,
                        size_t w_len, void* act, size_t act_len, size_t rows, size_t hidden,
                        size_t inter, int splits, int dtype);

/* Host-side RoPE table (engine/src/model/rope.rs:3-39): f64 inverse
 * frequencies with optional llama3 scaling, f32 cos/sin [max_pos, head_dim/2]
 * written to HOST arrays cos_t/sin_t of max_pos*head_dim/2 floats. */
int kvb_rope_table(size_t head_dim, double theta, int llama3_scaling, double factor,
                   double low_freq_factor, double high_freq_factor, double orig_max_pos,
                   size_t max_pos, float* cos_t, float* sin_t);

/* ---------------------------------------------------------------------------
 * Fused and batched kernels (no single reference counterpart; each equals a
 * composition of the entries above, bit for bit).
 * ------------------------------------------------------------------------- */

/* kvb_rope_inplace followed by kvb_kv_append, in one pass over qkv
 * (kernels.rs:124-169 + :238-291): q and k heads rotated in place, rotated k
 * and raw v written to the cache. */
int kvb_rope_kv_append(kvb_stream_t stream, void* qkv, size_t qkv_len, const float* cos_t,
                       const float* sin_t, size_t table_len, void* kc, void* vc, size_t cache_len,
                       size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim,
                       size_t max_seq, int dtype);

/* Batched decode form: row b of qkv belongs to sequence b at position pos[b]
 * (device int32 array).  Sequence b's cache starts at kc/vc + b*seq_stride
 * elements and is laid out [n_kv, max_seq, head_dim]. */
int kvb_rope_kv_append_batched(kvb_stream_t stream, void* qkv, size_t n_seq, const int32_t* pos,
                               const float* cos_t, const float* sin_t, size_t table_len,
                               void* kc, void* vc, size_t seq_stride, size_t cache_len,
                               size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                               int dtype);

/* Batched prefill form, one launch for n_seq sequences of t rows each, all
 * starting at pos0 (the layout kvb_attention_prefill reads): qkv is
 * [n_seq * t, (n_q + 2 n_kv) * head_dim]; sequence b's cache is kc/vc +
 * b * n_kv * max_seq * head_dim, cache_len = n_seq * n_kv * max_seq * head_dim.
 * Equal, bit for bit, to kvb_rope_kv_append on each sequence in turn. */
int kvb_rope_kv_append_prefill(kvb_stream_t stream, void* qkv, size_t qkv_len,
                               const float* cos_t, const float* sin_t, size_t table_len, void* kc,
                               void* vc, size_t cache_len, size_t n_seq, size_t t, size_t pos0,
                               size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                               int dtype);

/* kvb_embedding_gather(ids, table, x) followed by kvb_rmsnorm(x, w, out) (the
 * first norm of a decode step: Gpu::embedding_gather, kernels.rs:59-88, then
 * Gpu::rmsnorm, kernels.rs:90-121), in one launch for decode-sized batches;
 * x and out are bit-equal to the two calls.  x is [t, hidden] (the residual
 * stream), out [t, hidden]; ids outside the table give zero rows. */
int kvb_embedding_rmsnorm(kvb_stream_t stream, const int32_t* ids, size_t t, const void* table,
                          size_t table_len, const void* w, size_t w_len, void* x, size_t x_len,
                          void* out, size_t out_len, size_t hidden, float eps, int dtype);
/* kvb_add_inplace(x, y) followed by kvb_rmsnorm(x, w, out): the residual
 * stream x is updated in place and its normalised copy written to out. */
int kvb_add_rmsnorm(kvb_stream_t stream, void* x, size_t x_len, const void* y, size_t y_len,
                    const void* w, size_t w_len, void* out, size_t out_len, size_t rows,
                    size_t hidden, float eps, int dtype);

/* Batched single-query decode attention, one query row per sequence:
 * q row b at q + b*q_row_stride (head h at h*head_dim), sequence b attends
 * keys [0, lens[b]) of its cache (kc/vc + b*seq_stride, laid out
 * [n_kv, max_seq, head_dim]); out row b at out + b*out_row_stride.  lens is a
 * device int32 array with 0 <= lens[b] <= max_len <= max_seq (lens[b] == 0
 * gives a zero row).  Split-KV over CTAs with a combine pass when the
 * workspace (kvb_attention_decode_workspace_bytes) allows. */
int kvb_attention_decode(kvb_stream_t stream, const void* q, size_t q_row_stride, const void* kc,
                         const void* vc, size_t seq_stride, size_t cache_len,
                         const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                         size_t n_kv, size_t head_dim, size_t max_seq, float scale, void* out,
                         size_t out_row_stride, void* workspace, size_t workspace_len,
                         int dtype);
size_t kvb_attention_decode_workspace_bytes(size_t n_seq, size_t max_len, size_t n_q,
                                            size_t n_kv, size_t head_dim);

/* Paged KV cache -- the reference's planned stage-3 layout (kvasir
 * DESIGN.md:66-70: "[block, kv_head, block_size, head_dim]"; only the address
 * computation of attention / kv_append changes).  Per layer, K and V are pools
 * of n_blocks = pool_len / (n_kv * block_size * head_dim) blocks laid out
 * [n_blocks][n_kv][block_size][head_dim]; block_table is a device int32 array
 * [n_seq][max_blocks], and position p of sequence b lives in block
 * block_table[b * max_blocks + p / block_size] at offset p % block_size.  A
 * table entry outside [0, n_blocks) sets kvb_device_error code 4 (the row is
 * not written / those keys read as zeros); nothing faults.
 *
 * RoPE + KV append into the pools: qkv rows b*t .. b*t+t-1 belong to sequence b
 * at positions pos[b] .. pos[b]+t-1 (pos: device int32 [n_seq]); q and k heads
 * rotated in place, rotated k and raw v written to the blocks.  Equal, bit for
 * bit, to kvb_rope_kv_append into a contiguous cache holding the same rows. */
int kvb_rope_kv_append_paged(kvb_stream_t stream, void* qkv, size_t n_seq, size_t t,
                             const int32_t* pos, const float* cos_t, const float* sin_t,
                             size_t table_len, void* k_pool, void* v_pool, size_t pool_len,
                             const int32_t* block_table, size_t max_blocks, size_t block_size,
                             size_t n_q, size_t n_kv, size_t head_dim, int dtype);

/* kvb_attention_prefill over the pools: causal prefill of n_seq sequences of t
 * query rows (qkv rows as for kvb_attention_prefill) at positions pos0 .. pos0+t-1,
 * keys 0 .. pos0+t-1 read through the block table (pos0 + t <= max_blocks *
 * block_size).  Requires head_dim 64 and block_size a multiple of 32 (else
 * KVB_ERR_UNSUPPORTED).  Pool slots past a sequence's last key are never used,
 * whatever they hold.  Equal, bit for bit, to kvb_attention_prefill on a
 * contiguous cache holding the same keys. */
int kvb_attention_prefill_paged(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                const void* k_pool, const void* v_pool, size_t pool_len,
                                const int32_t* block_table, size_t max_blocks, size_t block_size,
                                void* out, size_t out_len, size_t n_seq, size_t t, size_t pos0,
                                size_t n_q, size_t n_kv, size_t head_dim, int dtype);

/* kvb_attention_decode over the pools: sequence b attends keys [0, lens[b]),
 * lens[b] <= max_len <= max_blocks * block_size.  Requires head_dim 64,
 * block_size a multiple of 64 and n_q / n_kv <= 16 (else KVB_ERR_UNSUPPORTED);
 * the workspace is sized by kvb_attention_decode_workspace_bytes.  Equal, bit for
 * bit, to kvb_attention_decode on a contiguous cache holding the same keys. */
int kvb_attention_decode_paged(kvb_stream_t stream, const void* q, size_t q_row_stride,
                               const void* k_pool, const void* v_pool, size_t pool_len,
                               const int32_t* block_table, size_t max_blocks, size_t block_size,
                               const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                               size_t n_kv, size_t head_dim, float scale, void* out,
                               size_t out_row_stride, void* workspace, size_t workspace_len,
                               int dtype);

/* No counterpart in the reference: an addition for callers that cannot
 * allocate device memory.  Same arguments and result as kvb_attention_decode
 * minus the workspace: the split-KV partials go to a scratch array that the
 * library itself holds in device memory (a file-scope __device__ array of
 * KVB_NOALLOC_SCRATCH_BYTES, present on every GPU that loads the library until
 * the process exits).  It serves callers that own no spare device buffer and
 * may not call cudaMalloc -- for example a host engine whose device memory
 * all belongs to long-lived weight / cache structs (the reference's own rule
 * for its launch wrappers), or code running where an allocation's implicit
 * device synchronisation is not acceptable.  The call allocates and frees
 * nothing.  Its output equals kvb_attention_decode's, bit for bit, when that
 * call is given a workspace of kvb_attention_decode_workspace_bytes.  Calls
 * that take the split-KV kernel (head_dim 64, n_q / n_kv <= 16, 16-byte aligned
 * q / kc / vc, row strides multiples of 8 elements, seq_stride a multiple of
 * 64) and whose partials need more than KVB_NOALLOC_SCRATCH_BYTES
 * (kvb_attention_decode_workspace_bytes) return KVB_ERR_SHAPE; other shapes run
 * kvb_attention_decode's general kernel, which needs no scratch.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current and keeps it with the id of the device's CUDA context;
 * when that context changes (a cudaDeviceReset and a new context) the next call
 * looks it up again.  Make the first call on a device, and the first after a
 * reset, outside any stream capture: inside one it returns KVB_ERR_UNSUPPORTED.
 * All calls on a device share the one array: calls that may overlap on the GPU
 * (different streams, or graphs replayed concurrently) race on it. */
#define KVB_NOALLOC_SCRATCH_BYTES (8u << 20)
int kvb_attention_decode_noalloc(kvb_stream_t stream, const void* q, size_t q_row_stride,
                                 const void* kc, const void* vc, size_t seq_stride,
                                 size_t cache_len, const int32_t* lens, size_t n_seq,
                                 size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                 size_t max_seq, float scale, void* out, size_t out_row_stride,
                                 int dtype);

/* Causal prefill attention for n_seq sequences of t tokens each (uniform
 * length, positions pos0 .. pos0+t-1): qkv rows [n_seq*t, (n_q+2n_kv)*hd],
 * caches [n_seq][n_kv][max_seq][hd] already holding keys [0, pos0+t); out
 * [n_seq*t, n_q*hd].  tcgen05/TMEM kernel for head_dim 64. */
int kvb_attention_prefill(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                          const void* vc, size_t cache_len, void* out, size_t out_len,
                          size_t n_seq, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                          size_t head_dim, size_t max_seq, int dtype);

/* kvb_attention_prefill with f32 output rows: the kernel's results before the
 * one rounding to the 16-bit type (rounding them to nearest even gives
 * kvb_attention_prefill's output bit for bit).  For callers that feed
 * attention into f32 work, and for measuring the kernel's own error.  head_dim
 * 64 and 16-byte aligned buffers only (else KVB_ERR_UNSUPPORTED).  New: the
 * reference's attention (engine/src/gpu/kernels.rs:294-371) writes 16-bit rows. */
int kvb_attention_prefill_f32(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                              const void* vc, size_t cache_len, float* out, size_t out_len,
                              size_t n_seq, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                              size_t head_dim, size_t max_seq, int dtype);

/* Decode step of the attention block in one launch: kvb_rope_kv_append_batched
 * followed by kvb_attention_decode, bit for bit, where the new token of
 * sequence b sits at position lens[b] - 1 (the decode convention: it is the
 * last key attended to).  qkv [n_seq, (n_q + 2 n_kv) * head_dim] stays
 * unrotated (the q heads are rotated in registers); the rotated k and the v
 * of each sequence are written to its cache row lens[b] - 1.  The reference
 * runs rope_inplace, kv_append and attention (kernels.rs:124-371) as three
 * launches.  head_dim 64, n_q/n_kv <= 16, contiguous caches, 16-byte aligned
 * buffers; otherwise KVB_ERR_UNSUPPORTED.  Workspace as for
 * kvb_attention_decode. */
int kvb_rope_attention_decode(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                              const float* cos_t, const float* sin_t, size_t table_len, void* kc,
                              void* vc, size_t seq_stride, size_t cache_len, const int32_t* lens,
                              size_t n_seq, size_t max_len, size_t n_q, size_t n_kv,
                              size_t head_dim, size_t max_seq, float scale, void* out,
                              size_t out_row_stride, void* workspace, size_t workspace_len,
                              int dtype);

/* The same on the paged cache: kvb_rope_kv_append_paged (one row per sequence,
 * at position lens[b] - 1) followed by kvb_attention_decode_paged, bit for bit,
 * in one launch.  Requirements and errors as kvb_attention_decode_paged. */
int kvb_rope_attention_decode_paged(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                    const float* cos_t, const float* sin_t, size_t table_len,
                                    void* k_pool, void* v_pool, size_t pool_len,
                                    const int32_t* block_table, size_t max_blocks,
                                    size_t block_size, const int32_t* lens, size_t n_seq,
                                    size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                    float scale, void* out, size_t out_row_stride, void* workspace,
                                    size_t workspace_len, int dtype);

/* Greedy sampling: ids[r] = first index of the maximum of logits[r, 0:vocab)
 * (NaN never wins; a row with no value above -inf gives 0).  If advance is
 * non-NULL, advance[r] += 1 for every r and, if advance2 is non-NULL,
 * advance2[r] += 1 (position / length counters of the decode loop). */
int kvb_argmax_f32(kvb_stream_t stream, const float* logits, size_t rows, size_t vocab,
                   int32_t* ids, int32_t* advance, int32_t* advance2);

/* The tied LM head and greedy argmax in one pass, f32 logits never stored
 * (replaces gemm::linear_f32 of the LM head, engine/src/gpu/gemm.rs:90-115,
 * followed by kvb_argmax_f32).  ids[r] = the first index of the maximum over
 * v < vocab of sum_k x[r, k] w[v, k] (f32 accumulation on the tensor cores),
 * with kvb_argmax_f32's rule: NaN never wins, a -inf never wins a tie, a row
 * with nothing above -inf gives 0; advance / advance2 as for kvb_argmax_f32.
 * x [rows, hidden], w [vocab, hidden] (16-bit, dtype).  rows <= 32, hidden a
 * multiple of 64 with rows <= 16 ? hidden <= 4096 : hidden <= 2048, 16-byte
 * aligned buffers, else KVB_ERR_UNSUPPORTED.  The workspace
 * (kvb_lm_head_argmax_workspace_bytes(rows)) holds per-CTA partials; its
 * contents need no initialisation.  Two launches, both programmatic dependents
 * of the kernel before them: x is read after that kernel completes, w as soon
 * as the pass runs (as for kvb_linear_rows, w must not be the output of one of
 * this library's kernels still in flight). */
size_t kvb_lm_head_argmax_workspace_bytes(size_t rows);
int kvb_lm_head_argmax(kvb_stream_t stream, const void* x, size_t x_len, const void* w,
                       size_t w_len, size_t rows, size_t hidden, size_t vocab, void* workspace,
                       size_t workspace_len, int32_t* ids, int32_t* advance, int32_t* advance2,
                       int dtype);

/* Temperature / top-p sampling on the device (the reference plans it on the
 * host over copied logits: kvasir DESIGN.md:24,109, "greedy / temperature /
 * top-p", seeded).  Per row: integer weights w_i = floor(2^32 * exp((l_i -
 * max l) / temperature)) (0 for NaN and -inf; a +inf logit takes the row, as
 * in the argmax); the kept set is every token whose logit is at least the
 * largest value K* with  sum_{l_j >= K*} w_j >= ceil(top_p * sum_j w_j)  (ties
 * at K* kept; top_p >= 1 keeps all); u24 = the top 24 bits of SplitMix64(seed +
 * SplitMix64(counter << 32 | row)) with counter = counters[row] (0 if counters
 * is NULL); ids[row] = the first index whose running kept weight, in
 * vocabulary order, exceeds floor(u24 * (kept weight) / 2^24).  All sums are
 * exact: the same seed, counter and logits give the same id.  temperature <= 0
 * is kvb_argmax_f32.  vocab at most 327680.  advance / advance2 as for
 * kvb_argmax_f32 (they may be the counters array: each row reads its counter
 * before advancing it).  One cluster of 8 CTAs per row, or of 16 when rows * 16
 * CTAs fit one per SM; the ids are the same either way. */
int kvb_sample_f32(kvb_stream_t stream, const float* logits, size_t rows, size_t vocab,
                   float temperature, float top_p, uint64_t seed, const int32_t* counters,
                   int32_t* ids, int32_t* advance, int32_t* advance2);

/* ---------------------------------------------------------------------------
 * Decode-step driver: the reference's planned Llama forward pass
 * (reference DESIGN.md:36-74, engine/src/model/weights.rs:13-27 for the
 * weight layout) for n_seq independent sequences, one token each, captured
 * in a CUDA graph on first use.  Weights, KV cache and workspace are
 * caller-owned device buffers; the driver allocates nothing on the device
 * after kvb_decoder_create (which creates its cuBLAS handle).
 * ------------------------------------------------------------------------- */
typedef struct {
    int32_t hidden, inter, n_layers, n_q, n_kv, head_dim, vocab;
    int32_t max_seq;  /* KV capacity per sequence */
    int32_t n_seq;    /* sequences decoded per step */
    float eps;
    int32_t dtype;
} kvb_decoder_config;

typedef struct {
    const void* embed;      /* [vocab, hidden]; tied LM head */
    const void* final_norm; /* [hidden] */
    const void* const* attn_norm; /* host array of n_layers device pointers, [hidden] each */
    const void* const* w_qkv;     /* [q_dim + 2 kv_dim, hidden] */
    const void* const* w_o;       /* [hidden, q_dim] */
    const void* const* mlp_norm;  /* [hidden] */
    const void* const* w_gu;      /* [2 inter, hidden] */
    const void* const* w_down;    /* [hidden, inter] */
} kvb_decoder_weights;

typedef struct kvb_decoder_s* kvb_decoder_t;

/* Bytes of device workspace the driver needs (activations, logits, split-KV
 * partials, position counters). */
size_t kvb_decoder_workspace_bytes(const kvb_decoder_config* cfg);
/* kc/vc: [n_layers][n_seq][n_kv][max_seq][head_dim] each; cos/sin: f32
 * [max_seq, head_dim/2] device tables. */
int kvb_decoder_create(kvb_decoder_t* out, const kvb_decoder_config* cfg,
                       const kvb_decoder_weights* w, void* kc, void* vc, const float* cos_t,
                       const float* sin_t, void* workspace, size_t workspace_len);
int kvb_decoder_destroy(kvb_decoder_t dec);
/* Switches the driver to a paged KV cache (see kvb_attention_decode_paged):
 * k_pools / v_pools hold n_layers pools of pool_len elements each
 * ([n_layers][n_blocks][n_kv][block_size][head_dim]); block_table ([n_seq]
 * [max_blocks] int32, device) is shared by all layers and must cover max_seq
 * positions.  The kc / vc given to kvb_decoder_create are no longer used.
 * Requires head_dim 64 and block_size a multiple of 64.  The next step records
 * the paged step; call it outside any stream capture. */
int kvb_decoder_use_paged_cache(kvb_decoder_t dec, void* k_pools, void* v_pools, size_t pool_len,
                                const int32_t* block_table, size_t max_blocks, size_t block_size);
/* Sets the per-sequence cache fill (tokens already in the cache) from a host
 * array; the next step writes position cur_len[b]. */
int kvb_decoder_set_lengths(kvb_decoder_t dec, kvb_stream_t stream, const int32_t* cur_len_host);
/* Device pointers of the step's input ids and output ids ([n_seq] int32 each).
 * The step reads ids_in and writes the greedy ids to ids_out; each step also
 * copies ids_out to ids_in so consecutive steps continue generation. */
int32_t* kvb_decoder_ids_in(kvb_decoder_t dec);
int32_t* kvb_decoder_ids_out(kvb_decoder_t dec);
const float* kvb_decoder_logits(kvb_decoder_t dec);
/* One decode step on the device (graph replay after the first call). */
int kvb_decoder_step(kvb_decoder_t dec, kvb_stream_t stream);
/* One decode step from host to host: copies ids_host_in (pinned or pageable)
 * to the device, runs the step, copies the greedy ids back to ids_host_out
 * and synchronises the stream. */
int kvb_decoder_step_host(kvb_decoder_t dec, kvb_stream_t stream, const int32_t* ids_host_in,
                          int32_t* ids_host_out);
/* Number of kernels (own + cuBLAS) one step launches. */
int kvb_decoder_launches_per_step(kvb_decoder_t dec, int* own, int* library);
/* Sampling of the step: temperature <= 0 is greedy (the default); otherwise
 * kvb_sample_f32 with the given top_p and seed, each sequence's counter being
 * its position, so every step draws afresh and a rerun from the same state
 * repeats.  The next step re-records its graph. */
int kvb_decoder_set_sampling(kvb_decoder_t dec, float temperature, float top_p, uint64_t seed);
/* enable != 0: greedy steps (temperature <= 0) end with kvb_lm_head_argmax (the
 * LM head and the argmax in one pass) where it applies (n_seq <= 32 and its
 * hidden / alignment limits), so kvb_decoder_logits is not written by those
 * steps; otherwise, and by default, the LM head is kvb_linear (f32 logits kept)
 * and kvb_argmax_f32.  The ids agree except where two logits of a row are within
 * the f32 rounding of their sums.  The next step re-records its graph.  New: the
 * fusion the reference's plan lists after its GEMM (engine/src/gpu/gemm.rs:90-115). */
int kvb_decoder_set_fused_lm_head(kvb_decoder_t dec, int enable);
/* enable != 0: the qkv, o and down projections run on kvb_linear_rows and the
 * gate/up projection with SiLU*mul on kvb_linear_silu_mul, where they apply
 * (n_seq <= 128 and their shape limits); otherwise, and by default, cuBLAS
 * (kvb_linear) and kvb_silu_mul.  Both accumulate in f32; the 16-bit results
 * agree within one rounding.  The next step re-records its graph. */
int kvb_decoder_set_row_projections(kvb_decoder_t dec, int enable);
/* Untied checkpoints (reference Weights::head, engine/src/model/weights.rs:29-32):
 * the LM head [vocab, hidden] used instead of the embedding table.  NULL goes
 * back to the tied head.  The next step re-records its graph. */
int kvb_decoder_set_lm_head(kvb_decoder_t dec, const void* lm_head);

/* ---------------------------------------------------------------------------
 * Weight load path (reference Weights::load, engine/src/model/weights.rs:47-230):
 * every *.safetensors file of a directory is memory-mapped (sorted by name; a
 * tensor name in a later file replaces an earlier one, as the reference's map
 * insertion does) and its header parsed.  kvb_checkpoint_load_rows copies named
 * tensors, concatenated by rows (the reference's fused w_qkv rows q|k|v and
 * w_gu rows gate|up, Loader::load_into), into a caller-owned device buffer in
 * the compute type:
 *   BF16 -> BF16, F16 -> F16: copied as they are (F16 checked finite);
 *   BF16 -> F16: on the device by kvb_bf16_to_f16, values that are not finite
 *                or outside the FP16 range counted in *bad (device u32), as
 *                the reference's Loader::convert_to;
 *   F16 -> BF16, F32 -> BF16, F32 -> F16: rounded to nearest even on the host;
 *                a non-finite result is KVB_ERR_CONFIG (reference check_finite).
 * Host staging is pinned and double-buffered; copies run on `stream`, and the
 * call returns once every source byte has been staged (the last copies may
 * still be in flight on the stream).  The loader allocates its own staging
 * (pinned host, and device memory for BF16 -> F16); nothing else.
 * ------------------------------------------------------------------------- */
typedef struct kvb_checkpoint_s* kvb_checkpoint_t;

enum kvb_ckpt_dtype { KVB_CKPT_BF16 = 0, KVB_CKPT_F16 = 1, KVB_CKPT_F32 = 2, KVB_CKPT_OTHER = 3 };

/* Maps and indexes every *.safetensors file of dir.  KVB_ERR_CONFIG if there is
 * none or a header is malformed, KVB_ERR_IO if a file cannot be read. */
int kvb_checkpoint_open(kvb_checkpoint_t* out, const char* dir);
/* Waits for the loader's copies still in flight, then unmaps and frees. */
int kvb_checkpoint_close(kvb_checkpoint_t ck);
/* Number of distinct tensor names. */
size_t kvb_checkpoint_num_tensors(kvb_checkpoint_t ck);
/* dtype (kvb_ckpt_dtype), rank and up to 8 dims of a tensor; KVB_ERR_CONFIG if
 * the name is missing. */
int kvb_checkpoint_tensor(kvb_checkpoint_t ck, const char* name, int* dtype, int* ndim,
                          uint64_t* dims);
/* Copies n_parts tensors into dst (dst_len elements of dst_dtype): part i must
 * have shape [rows[i], cols], or [cols] when rows[i] == 0 (a vector, counted as
 * one row).  Errors: a missing name or unsupported dtype is KVB_ERR_CONFIG, a
 * shape other than the expected one KVB_ERR_SHAPE ("<name>: shape [..],
 * expected [..]"), dst_len other than the parts' total KVB_ERR_SHAPE.  `bad`
 * (device, one u32) is required when a BF16 part goes to F16. */
int kvb_checkpoint_load_rows(kvb_checkpoint_t ck, kvb_stream_t stream, const char* const* names,
                             const uint64_t* rows, size_t n_parts, uint64_t cols, void* dst,
                             size_t dst_len, int dst_dtype, uint32_t* bad);

/* ---------------------------------------------------------------------------
 * Self test of the bounded-wait machinery: launches one CTA that waits on an
 * mbarrier nobody completes, with a time limit of limit_ms; returns
 * KVB_ERR_DEVICE once the kernel has given up (the device stays usable).
 * ------------------------------------------------------------------------- */
int kvb_selftest_wait_timeout(kvb_stream_t stream, uint32_t limit_ms);

#ifdef __cplusplus
}
#endif
#endif /* KVASIR_B200_H */
