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
