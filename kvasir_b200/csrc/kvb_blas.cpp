// kvb_blas.cpp -- the projections: cuBLAS GEMMs behind the reference's
// gemm::linear_f16 / linear_f32 (engine/src/gpu/gemm.rs:17-115), timed but not
// rewritten.  Row-major y[t,out] = x[t,in] * w[out,in]^T is issued as the
// column-major C[out x t] = op_T(W[in x out]) * X[in x t] (gemm.rs:263-305 form:
// OP_T / OP_N, lda = ldb = in, ldc = out), 16-bit inputs, f32 compute.
#include <cublasLt.h>
#include <cublas_v2.h>

#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "kvb_host.h"

struct kvb_blas_s {
    cublasHandle_t handle = nullptr;
    cublasLtHandle_t lt = nullptr;
    void* workspace = nullptr;  // optional caller-provided cuBLAS workspace
    size_t workspace_len = 0;
    int autotune = 0;
};

static int blas_fail(cublasStatus_t s, const char* what) {
    return kvb::fail(KVB_ERR_CUDA, "%s: cuBLAS status %d", what, (int)s);
}

namespace {

// Autotuned projections: for each GEMM shape the cuBLASLt algorithms the
// heuristic offers (split-K ones included, those reducing in place with atomics
// excluded so results stay reproducible) are timed once against cublasGemmEx and
// the fastest is kept for the process, so every handle on a device issues the
// same algorithm for the same shape.
struct TunedGemm {
    bool use_lt = false;  // false: cublasGemmEx was fastest
    cublasLtMatmulAlgo_t algo;
    size_t ws = 0;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
};
using TuneKey = std::tuple<int, int, int, int, int, int, size_t>;  // dev, t, in, out, dtype, f32, ws
std::mutex g_tune_mu;
std::map<TuneKey, TunedGemm> g_tuned;

cublasStatus_t gemm_ex(kvb_blas_s* b, const void* x, const void* w, void* y, int t, int in_dim,
                       int out_dim, int dtype, int y_f32) {
    const float alpha = 1.0f, beta = 0.0f;
    const cudaDataType_t ab = dtype == KVB_BF16 ? CUDA_R_16BF : CUDA_R_16F;
    const cudaDataType_t ct = y_f32 ? CUDA_R_32F : ab;
    return cublasGemmEx(b->handle, CUBLAS_OP_T, CUBLAS_OP_N, out_dim, t, in_dim, &alpha, w, ab,
                        in_dim, x, ab, in_dim, &beta, y, ct, out_dim, CUBLAS_COMPUTE_32F,
                        CUBLAS_GEMM_DEFAULT);
}

cublasStatus_t gemm_lt(kvb_blas_s* b, const TunedGemm& g, const void* x, const void* w, void* y,
                       cudaStream_t s) {
    const float alpha = 1.0f, beta = 0.0f;
    return cublasLtMatmul(b->lt, g.op, &alpha, w, g.a, x, g.b, &beta, y, g.c, y, g.c, &g.algo,
                          b->workspace, g.ws, s);
}

// Times the candidates on the caller's buffers (outputs are overwritten) and
// returns the winner.  Runs outside stream capture only.
int tune_gemm(kvb_blas_s* b, cudaStream_t s, const void* x, const void* w, void* y, int t,
              int in_dim, int out_dim, int dtype, int y_f32, TunedGemm& out) {
    const cudaDataType_t ab = dtype == KVB_BF16 ? CUDA_R_16BF : CUDA_R_16F;
    const cudaDataType_t ct = y_f32 ? CUDA_R_32F : ab;
    TunedGemm g;
    cublasStatus_t st = cublasLtMatmulDescCreate(&g.op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
    const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasLtMatmulDescSetAttribute(g.op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof ta);
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasLtMatmulDescSetAttribute(g.op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof tb);
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasLtMatrixLayoutCreate(&g.a, ab, in_dim, out_dim, in_dim);
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasLtMatrixLayoutCreate(&g.b, ab, in_dim, t, in_dim);
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasLtMatrixLayoutCreate(&g.c, ct, out_dim, t, out_dim);
    cublasLtMatmulPreference_t pref = nullptr;
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasLtMatmulPreferenceCreate(&pref);
    const uint64_t wsmax = b->workspace_len;
    const uint32_t schemes = CUBLASLT_REDUCTION_SCHEME_COMPUTE_TYPE |
                             CUBLASLT_REDUCTION_SCHEME_OUTPUT_TYPE;  // no in-place (atomic) split-K
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES,
                                                  &wsmax, sizeof wsmax);
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_REDUCTION_SCHEME_MASK,
                                                  &schemes, sizeof schemes);
    cublasLtMatmulHeuristicResult_t res[32];
    int n = 0;
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasLtMatmulAlgoGetHeuristic(b->lt, g.op, g.a, g.b, g.c, g.c, pref, 32, res, &n);
    if (pref) cublasLtMatmulPreferenceDestroy(pref);
    if (st != CUBLAS_STATUS_SUCCESS) n = 0;  // no candidates: cublasGemmEx stays

    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    constexpr int kReps = 5;
    auto time_it = [&](auto&& run) -> float {  // ms per run, or -1 if a run failed
        if (run() != CUBLAS_STATUS_SUCCESS) return -1.f;  // warm-up
        cudaEventRecord(e0, s);
        for (int r = 0; r < kReps; ++r)
            if (run() != CUBLAS_STATUS_SUCCESS) return -1.f;
        cudaEventRecord(e1, s);
        if (cudaEventSynchronize(e1) != cudaSuccess) return -1.f;
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        return ms / kReps;
    };
    float best = time_it([&] { return gemm_ex(b, x, w, y, t, in_dim, out_dim, dtype, y_f32); });
    g.use_lt = false;
    auto try_algo = [&](const cublasLtMatmulAlgo_t& algo, size_t ws) {
        TunedGemm cand = g;
        cand.algo = algo;
        cand.ws = ws;
        const float ms = time_it([&] { return gemm_lt(b, cand, x, w, y, s); });
        if (ms > 0.f && (best < 0.f || ms < best)) {
            best = ms;
            g.use_lt = true;
            g.algo = algo;
            g.ws = ws;
        }
    };
    for (int i = 0; i < n; ++i) {
        if (res[i].state != CUBLAS_STATUS_SUCCESS || res[i].workspaceSize > b->workspace_len)
            continue;
        try_algo(res[i].algo, res[i].workspaceSize);
        // the same tile configuration with the K dimension split 2 .. 32 ways, the
        // partial products reduced in a separate pass (no atomics)
        if (i < 8) {
            for (int splitk : {2, 4, 8, 16, 32}) {
                cublasLtMatmulAlgo_t a2 = res[i].algo;
                const int32_t sk = splitk;
                const uint32_t scheme = CUBLASLT_REDUCTION_SCHEME_COMPUTE_TYPE;
                if (cublasLtMatmulAlgoConfigSetAttribute(&a2, CUBLASLT_ALGO_CONFIG_SPLITK_NUM, &sk,
                                                         sizeof sk) != CUBLAS_STATUS_SUCCESS ||
                    cublasLtMatmulAlgoConfigSetAttribute(&a2, CUBLASLT_ALGO_CONFIG_REDUCTION_SCHEME,
                                                         &scheme, sizeof scheme) !=
                        CUBLAS_STATUS_SUCCESS)
                    continue;
                cublasLtMatmulHeuristicResult_t chk;
                if (cublasLtMatmulAlgoCheck(b->lt, g.op, g.a, g.b, g.c, g.c, &a2, &chk) !=
                        CUBLAS_STATUS_SUCCESS ||
                    chk.state != CUBLAS_STATUS_SUCCESS || chk.workspaceSize > b->workspace_len)
                    continue;
                try_algo(a2, chk.workspaceSize);
            }
        }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGetLastError();  // a failed candidate must not leave a sticky runtime error behind
    if (best < 0.f) return kvb::fail(KVB_ERR_CUDA, "linear autotune: no GEMM ran");
    out = g;
    return KVB_OK;
}

}  // namespace

extern "C" {

int kvb_blas_create(kvb_blas_t* out) {
    KVB_CHECK(out != nullptr, "blas_create: null output pointer");
    kvb_blas_s* b = new kvb_blas_s();
    cublasStatus_t s = cublasCreate(&b->handle);
    if (s == CUBLAS_STATUS_SUCCESS) s = cublasLtCreate(&b->lt);
    if (s != CUBLAS_STATUS_SUCCESS) {
        if (b->handle) cublasDestroy(b->handle);
        delete b;
        return blas_fail(s, "cublasCreate");
    }
    *out = b;
    return KVB_OK;
}

int kvb_blas_destroy(kvb_blas_t b) {
    if (!b) return KVB_OK;
    if (b->lt) cublasLtDestroy(b->lt);
    if (b->handle) cublasDestroy(b->handle);
    delete b;
    return KVB_OK;
}

int kvb_blas_set_autotune(kvb_blas_t b, int enable) {
    KVB_CHECK(b != nullptr, "blas_set_autotune: null handle");
    b->autotune = enable ? 1 : 0;
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
    if (b->autotune) {
        int dev = 0;
        cudaGetDevice(&dev);
        const TuneKey key{dev, (int)t, (int)in_dim, (int)out_dim, dtype, y_f32, b->workspace_len};
        const TunedGemm* g = nullptr;
        {
            std::lock_guard<std::mutex> lock(g_tune_mu);
            auto it = g_tuned.find(key);
            if (it != g_tuned.end()) g = &it->second;
        }
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(stream, &cap);
        if (!g && cap == cudaStreamCaptureStatusNone) {  // tune now (never inside a capture)
            TunedGemm tg;
            const int st = tune_gemm(b, stream, x, w, y, (int)t, (int)in_dim, (int)out_dim, dtype,
                                     y_f32, tg);
            if (st != KVB_OK) return st;
            std::lock_guard<std::mutex> lock(g_tune_mu);
            g = &g_tuned.emplace(key, tg).first->second;  // an earlier winner stays if one raced
        }
        if (g && g->use_lt) {
            s = gemm_lt(b, *g, x, w, y, stream);
            if (s != CUBLAS_STATUS_SUCCESS) return blas_fail(s, "cublasLtMatmul");
            return KVB_OK;
        }
    }
    s = gemm_ex(b, x, w, y, (int)t, (int)in_dim, (int)out_dim, dtype, y_f32);
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
