// kvb_blas.cpp -- the projections: cuBLAS GEMMs behind the reference's
// gemm::linear_f16 / linear_f32 (engine/src/gpu/gemm.rs:17-115), timed but not
// rewritten.  Row-major y[t,out] = x[t,in] * w[out,in]^T is issued as the
// column-major C[out x t] = op_T(W[in x out]) * X[in x t] (gemm.rs:263-305 form:
// OP_T / OP_N, lda = ldb = in, ldc = out), 16-bit inputs, f32 compute.
#include <cublas_v2.h>

#include <cmath>
#include <cstdlib>

#include "kvb_host.h"

struct kvb_blas_s {
    cublasHandle_t handle = nullptr;
    void* workspace = nullptr;  // optional caller-provided cuBLAS workspace
    size_t workspace_len = 0;
};

static int blas_fail(cublasStatus_t s, const char* what) {
    return kvb::fail(KVB_ERR_CUDA, "%s: cuBLAS status %d", what, (int)s);
}

extern "C" {

int kvb_blas_create(kvb_blas_t* out) {
    KVB_CHECK(out != nullptr, "blas_create: null output pointer");
    kvb_blas_s* b = new kvb_blas_s();
    cublasStatus_t s = cublasCreate(&b->handle);
    if (s != CUBLAS_STATUS_SUCCESS) {
        delete b;
        return blas_fail(s, "cublasCreate");
    }
    *out = b;
    return KVB_OK;
}

int kvb_blas_destroy(kvb_blas_t b) {
    if (!b) return KVB_OK;
    if (b->handle) cublasDestroy(b->handle);
    delete b;
    return KVB_OK;
}

// Internal: lets the decode driver hand cuBLAS a slice of its workspace so that
// a captured step never makes cuBLAS allocate.
int kvb_blas_set_workspace(kvb_blas_t b, void* ws, size_t len) {
    KVB_CHECK(b != nullptr, "blas_set_workspace: null handle");
    cublasStatus_t s = cublasSetWorkspace(b->handle, ws, len);
    if (s != CUBLAS_STATUS_SUCCESS) return blas_fail(s, "cublasSetWorkspace");
    b->workspace = ws;
    b->workspace_len = len;
    return KVB_OK;
}

int kvb_linear(kvb_blas_t b, kvb_stream_t stream, const void* x, size_t x_len, const void* w,
               size_t w_len, void* y, size_t y_len, size_t t, size_t in_dim, size_t out_dim,
               int dtype, int y_f32) {
    KVB_CHECK(b != nullptr, "linear: null cuBLAS handle");
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == t * in_dim, "linear: x has %zu elems, want %zux%zu", x_len, t, in_dim);
    KVB_CHECK(w_len == out_dim * in_dim, "linear: w has %zu elems, want %zux%zu", w_len, out_dim,
              in_dim);
    KVB_CHECK(y_len == t * out_dim, "linear: y has %zu elems, want %zux%zu", y_len, t, out_dim);
    KVB_CHECK(kvb::fits_i32(t) && kvb::fits_i32(in_dim) && kvb::fits_i32(out_dim),
              "linear: a dimension does not fit in i32");
    if (t == 0 || out_dim == 0) return KVB_OK;
    cublasStatus_t s = cublasSetStream(b->handle, stream);
    if (s != CUBLAS_STATUS_SUCCESS) return blas_fail(s, "cublasSetStream");
    const float alpha = 1.0f, beta = 0.0f;
    const cudaDataType_t ab = dtype == KVB_BF16 ? CUDA_R_16BF : CUDA_R_16F;
    const cudaDataType_t ct = y_f32 ? CUDA_R_32F : ab;
    s = cublasGemmEx(b->handle, CUBLAS_OP_T, CUBLAS_OP_N, (int)out_dim, (int)t, (int)in_dim, &alpha,
                     w, ab, (int)in_dim, x, ab, (int)in_dim, &beta, y, ct, (int)out_dim,
                     CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (s != CUBLAS_STATUS_SUCCESS) return blas_fail(s, "cublasGemmEx");
    return KVB_OK;
}

// ------------------------------------------------------------------ host RoPE tables
// engine/src/model/rope.rs:3-39: inverse frequencies 1/theta^(2j/hd) in f64
// with optional llama3 scaling, then cos/sin(p * inv_freq) rounded to f32.
int kvb_rope_table(size_t head_dim, double theta, int llama3_scaling, double factor,
                   double low_freq_factor, double high_freq_factor, double orig_max_pos,
                   size_t max_pos, float* cos_t, float* sin_t) {
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope_table: odd head_dim %zu", head_dim);
    KVB_CHECK(cos_t != nullptr && sin_t != nullptr, "rope_table: null output array");
    KVB_CHECK(!llama3_scaling || (high_freq_factor != low_freq_factor && factor > 0),
              "rope_table: degenerate llama3 scaling parameters");
    const size_t half = head_dim / 2;
    const double two_pi = 6.283185307179586476925286766559;
    double* inv = static_cast<double*>(malloc(sizeof(double) * half));
    if (!inv) return kvb::fail(KVB_ERR_CUDA, "rope_table: host allocation failed");
    for (size_t j = 0; j < half; ++j) {
        double f = 1.0 / pow(theta, 2.0 * (double)j / (double)head_dim);
        if (llama3_scaling) {
            const double wavelen = two_pi / f;
            const double low_wavelen = orig_max_pos / low_freq_factor;
            const double high_wavelen = orig_max_pos / high_freq_factor;
            if (wavelen > low_wavelen) {
                f = f / factor;
            } else if (wavelen >= high_wavelen) {
                const double smooth = (orig_max_pos / wavelen - low_freq_factor) /
                                      (high_freq_factor - low_freq_factor);
                f = (1.0 - smooth) * f / factor + smooth * f;
            }
        }
        inv[j] = f;
    }
    for (size_t p = 0; p < max_pos; ++p)
        for (size_t j = 0; j < half; ++j) {
            const double a = (double)p * inv[j];
            cos_t[p * half + j] = (float)cos(a);
            sin_t[p * half + j] = (float)sin(a);
        }
    free(inv);
    return KVB_OK;
}

}  // extern "C"
