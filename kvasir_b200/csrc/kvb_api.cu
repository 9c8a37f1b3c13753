// kvb_api.cu -- the kernels of libkvasir_b200 and their C-ABI launchers.
//
// Each kvb_* entry point validates its arguments exactly where the matching
// reference wrapper does (engine/src/gpu/kernels.rs, ensure_shape!), then picks
// the fast path (16-byte vectors, TMA, tensor cores) when shapes and
// alignment allow it, else a general kernel -- always on the GPU.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "attn_decode.cuh"
#include "attn_generic.cuh"
#include "attn_prefill.cuh"
#include "elementwise.cuh"
#include "kvb_host.h"
#include "linear_rows.cuh"
#include "lm_head.cuh"
#include "norm.cuh"
#include "rope.cuh"
#include "sample.cuh"

namespace kvb {

// ---------------------------------------------------------------- host helpers
static thread_local std::string t_err;

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // reset the runtime's last error so later checks do not see it again
    return fail(KVB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int dtype) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(KVB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    const CUresult r = fn(map,
                          dtype == KVB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                          (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return KVB_OK;
}

// Grid size for grid-stride loops: enough CTAs to fill every SM several times.
static unsigned grid_for(size_t work, int block) {
    size_t g = (work + block - 1) / block;
    const size_t cap = (size_t)num_sms() * 16;
    if (g > cap) g = cap;
    return g ? (unsigned)g : 1u;
}

// Raises a kernel's dynamic shared-memory limit once per (device, kernel), so
// that launches recorded into a CUDA graph make no attribute calls.
template <typename F>
static void set_max_smem(F* kernel, int bytes) {
    static std::mutex mu;
    static std::vector<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    const void* key = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == dev && d.second == key) return;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done.emplace_back(dev, key);
}

// Launches `kernel` as a programmatic dependent of the kernel before it on the
// stream: its CTAs may be scheduled while that kernel drains.  The kernel
// executes griddepcontrol.wait before its first access to memory that earlier
// kernels write or read.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- sampler launcher
// sample_kernel<kCluster>: one cluster of kCluster CTAs per row, each CTA staging
// its slice of the row in shared memory.
template <int kCluster>
static cudaError_t launch_sample(cudaStream_t stream, const float* logits, size_t rows,
                                 size_t vocab, float inv_temp, float top_p, uint64_t seed,
                                 const int32_t* counters, int32_t* ids, int32_t* adv,
                                 int32_t* adv2, int vec4) {
    const size_t slice = ((vocab + kCluster - 1) / kCluster + 3) & ~(size_t)3;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * kCluster));
    cfg.blockDim = dim3(kSampleThreads);
    cfg.dynamicSmemBytes = slice * 4;
    cfg.stream = stream;
    cudaLaunchAttribute attr = {};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = kCluster;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, sample_kernel<kCluster>, logits, (int)vocab, inv_temp, top_p,
                              seed, counters, ids, adv, adv2, vec4);
}

// Sets the sampler's kernel attributes once per device, and reports whether the
// device keeps a 16-CTA cluster of it resident (16 is a non-portable cluster size:
// the kernel must allow it, and the occupancy query must find room for one).
// While `stream` is being captured the query is not made: 8-CTA clusters, and the
// answer is left for a later call (the decode-step driver asks before it captures).
static bool sample_attrs_and_wide_ok(cudaStream_t stream) {
    static std::mutex mu;
    static int state[64];  // 0 unknown, 1 wide clusters run, 2 they do not
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (!state[dev] && stream != nullptr && cudaStreamIsCapturing(stream, &cap) == cudaSuccess &&
        cap != cudaStreamCaptureStatusNone) {
        set_max_smem(sample_kernel<kSampleCluster>, kSampleStageMax);
        return false;
    }
    if (!state[dev]) {
        cudaFuncSetAttribute(sample_kernel<kSampleCluster>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSampleStageMax);
        const size_t wide_smem =
            (((size_t)kSampleCluster * kSampleMaxSlice / kSampleClusterWide + 3) & ~(size_t)3) * 4;
        cudaError_t e = cudaFuncSetAttribute(sample_kernel<kSampleClusterWide>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)wide_smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(sample_kernel<kSampleClusterWide>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        int clusters = 0;
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(kSampleClusterWide);
            cfg.blockDim = dim3(kSampleThreads);
            cfg.dynamicSmemBytes = wide_smem;
            cudaLaunchAttribute attr = {};
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = kSampleClusterWide;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&clusters, sample_kernel<kSampleClusterWide>, &cfg);
        }
        if (e != cudaSuccess) cudaGetLastError();  // not an error of the caller's: 8-CTA clusters
        state[dev] = (e == cudaSuccess && clusters >= 1) ? 1 : 2;
    }
    return state[dev] == 1;
}

void sample_prepare() { sample_attrs_and_wide_ok(nullptr); }

// ---------------------------------------------------------------- rope / kv append launcher
// Persistent bulk-copy RoPE: 16 consumer warps when two 16-row stages fit in
// 200 KB of shared memory, else 8 or 4; as many CTAs per SM as fit, at most 2.
// Returns false when even 4 rows per stage do not fit (the caller falls back).
template <typename T, int CPR>
static bool launch_rope_bulk(kvb_stream_t stream, const RopeArgs& a, int rows) {
    const int rb = rope_bulk_row_bytes(a);
    int warps = 16;
    while (warps > 4 && 2 * warps * rb > 200 * 1024) warps /= 2;
    const int smem = rope_bulk_smem_bytes(a, warps);
    if (smem > 227 * 1024) return false;
    int per_sm = (228 * 1024) / (smem + 1024);
    per_sm = per_sm < 1 ? 1 : per_sm > 2 ? 2 : per_sm;
    if (warps == 16) per_sm = 1;
    const int cap = num_sms() * per_sm;
    const unsigned grid = (unsigned)(rows < cap ? rows : cap);
    const unsigned threads = 32u * (warps + 1);
    switch (warps) {
        case 16:
            set_max_smem(rope_append_bulk_kernel<T, CPR, 16>, 227 * 1024);
            rope_append_bulk_kernel<T, CPR, 16><<<grid, threads, smem, stream>>>(a, rows);
            break;
        case 8:
            set_max_smem(rope_append_bulk_kernel<T, CPR, 8>, 227 * 1024);
            rope_append_bulk_kernel<T, CPR, 8><<<grid, threads, smem, stream>>>(a, rows);
            break;
        default:
            set_max_smem(rope_append_bulk_kernel<T, CPR, 4>, 227 * 1024);
            rope_append_bulk_kernel<T, CPR, 4><<<grid, threads, smem, stream>>>(a, rows);
            break;
    }
    return true;
}

static int launch_rope(kvb_stream_t stream, const RopeArgs& a, int rows, int dtype, bool vec) {
    if (rows == 0) return KVB_OK;
    // Many rows (prefill): persistent bulk-copy CTAs.  Few rows (decode batches): a
    // CTA per row, which puts more loads in flight per row.
    const bool many = vec && a.do_rope && (a.hd == 64 || a.hd == 128) && rows >= num_sms() * 8;
    bool done = false;
    if (many && (a.row_stride * 2) % 16 == 0) {
        if (a.hd == 64)
            done = dtype == KVB_BF16 ? launch_rope_bulk<__nv_bfloat16, 4>(stream, a, rows)
                                     : launch_rope_bulk<__half, 4>(stream, a, rows);
        else
            done = dtype == KVB_BF16 ? launch_rope_bulk<__nv_bfloat16, 8>(stream, a, rows)
                                     : launch_rope_bulk<__half, 8>(stream, a, rows);
    }
    if (done) {
        // launched by launch_rope_bulk
    } else if (many) {  // rows too wide for the ring: a warp per row
        const unsigned grid = (unsigned)((rows + 3) / 4);
        if (a.hd == 64) {
            if (dtype == KVB_BF16)
                rope_append_warp_kernel<__nv_bfloat16, 4><<<grid, 128, 0, stream>>>(a, rows);
            else
                rope_append_warp_kernel<__half, 4><<<grid, 128, 0, stream>>>(a, rows);
        } else {
            if (dtype == KVB_BF16)
                rope_append_warp_kernel<__nv_bfloat16, 8><<<grid, 128, 0, stream>>>(a, rows);
            else
                rope_append_warp_kernel<__half, 8><<<grid, 128, 0, stream>>>(a, rows);
        }
    } else if (vec) {
        if (dtype == KVB_BF16)
            rope_append_vec_kernel<__nv_bfloat16><<<rows, 256, 0, stream>>>(a);
        else
            rope_append_vec_kernel<__half><<<rows, 256, 0, stream>>>(a);
    } else {
        if (dtype == KVB_BF16)
            rope_append_scalar_kernel<__nv_bfloat16><<<rows, 256, 0, stream>>>(a);
        else
            rope_append_scalar_kernel<__half><<<rows, 256, 0, stream>>>(a);
    }
    KVB_CHECK_LAUNCH("rope/kv_append launch");
    return KVB_OK;
}

// ---------------------------------------------------------------- decode attention launcher
// Keys per CTA: aim for ~5 waves of 3 resident CTAs per SM over the worst-case
// work (every sequence at max_len), at least one 64-key tile per warp -- four
// per warp once the (sequence, kv head) pairs alone fill every SM, where short
// chunks only add combine work (measured: batch 32 at context 1088 and config 2
// gain 1-3 %; one sequence, 8 pairs, needs the smaller chunks' parallelism).
// Measured at context 16384 on 32 / 64 / 256 sequences: 5 waves 163.3 / 307.4 /
// 1174.7 us per launch, 8 waves 167.5 / 310.6 / 1188.5, 3 and 4 waves in between,
// 2 and 16 waves slower (fewer, longer chunks pay fewer CTA start-ups and less
// combine work, until the last wave's shortfall outweighs that).
static int decode_chunk_keys(size_t n_seq, size_t n_kv, size_t max_len) {
    const size_t tiles = (max_len + 63) / 64;
    const size_t target = (size_t)num_sms() * 3 * 5;
    size_t per_cta = (n_seq * n_kv * tiles + target - 1) / target;
    const size_t min_tiles = n_seq * n_kv >= (size_t)num_sms() ? 16 : 4;
    if (per_cta < min_tiles) per_cta = min_tiles;
    per_cta = (per_cta + 3) / 4 * 4;
    if (per_cta > tiles) per_cta = (tiles + 3) / 4 * 4;
    return (int)(per_cta * 64);
}

// kvb_attention_decode takes the split-KV tensor-core kernel (and its workspace)
// for these shapes and buffers; every other valid call runs the general kernel,
// which uses no workspace.
static bool decode_fast_path(const void* q, size_t q_row_stride, const void* kc, const void* vc,
                             size_t seq_stride, size_t n_seq, size_t n_q, size_t n_kv,
                             size_t head_dim, size_t max_seq, size_t out_row_stride) {
    if (n_seq == 0 || n_kv == 0 || n_q % n_kv != 0) return false;
    const size_t per_seq = n_kv * max_seq * head_dim;
    const size_t total_rows = ((n_seq - 1) * seq_stride + per_seq) / 64;
    return head_dim == 64 && n_q / n_kv <= 16 && n_seq <= 65535 && n_kv <= 65535 &&
           seq_stride % 64 == 0 && q_row_stride % 8 == 0 && out_row_stride % 8 == 0 &&
           aligned(q, 16) && aligned(kc, 16) && aligned(vc, 16) && fits_i32(total_rows);
}

static size_t decode_ws_bytes(size_t n_seq, size_t max_len, size_t n_q, size_t n_kv) {
    if (max_len == 0 || n_kv == 0) return 0;
    const size_t ck = (size_t)decode_chunk_keys(n_seq, n_kv, max_len);
    const size_t chunks = (max_len + ck - 1) / ck;
    if (chunks <= 1) return 0;
    const size_t group = n_q / n_kv;
    return n_seq * n_kv * chunks * group * 66 * sizeof(float);
}

// How a split-KV decode call runs, from its shape and workspace:
//   kSingle  one CTA per (sequence, kv head), no workspace (none given, or too small);
//   kChunks  fixed-size chunks, partials in the workspace, a combine pass;
//   kFold    the same chunks folded in the kernel through a cluster (small grids).
enum DecodeMode { kSingle, kChunks, kFold };
struct DecodePlan {
    DecodeMode mode;
    int chunk_keys, max_chunks;
};
static DecodePlan decode_plan(size_t n_seq, size_t max_len, size_t n_q, size_t n_kv,
                              const void* ws, size_t ws_len) {
    DecodePlan p;
    int ck = decode_chunk_keys(n_seq, n_kv, max_len);
    const size_t need = decode_ws_bytes(n_seq, max_len, n_q, n_kv);
    const bool chunk_ws = need > 0 && ws != nullptr && ws_len >= need && aligned(ws, 16);
    if (!chunk_ws) {
        ck = (int)(((max_len + 255) / 256) * 256);  // one chunk: no workspace
        if (ck == 0) ck = 256;
    }
    // chunks are the grid's z extent: at most 65535 (wider chunks need less workspace)
    if ((max_len + ck - 1) / ck > 65535) ck = (int)(((max_len + 65534) / 65535 + 255) / 256 * 256);
    p.chunk_keys = ck;
    p.max_chunks = (int)((max_len + ck - 1) / ck);
    if (p.max_chunks < 1) p.max_chunks = 1;
    // Small split grids (every CTA resident at once, at most 8 chunks per sequence):
    // the chunks of a (sequence, kv head) form a cluster and fold in the kernel, with
    // no combine pass.  Measured on the one-sequence decode step: the combine launch
    // and its programmatic boundary cost ~3.6 us per layer.
    const size_t n_ctas = n_kv * n_seq * (size_t)p.max_chunks;
    if (chunk_ws && p.max_chunks >= 2 && p.max_chunks <= 8 && n_ctas <= (size_t)num_sms() * 3) {
        p.mode = kFold;
        return p;
    }
    p.mode = chunk_ws && p.max_chunks > 1 ? kChunks : kSingle;
    return p;
}

struct DecodeLaunch {
    const void* q;
    size_t q_row_stride;
    const void* kc;
    const void* vc;
    size_t seq_stride;  // elements
    size_t total_rows;  // rows of 64 elements covered by the caches
    const int32_t* lens;
    int len_const;
    size_t n_seq, max_len, n_q, n_kv, max_seq;
    float scale;
    void* out;
    size_t out_row_stride;
    void* ws;
    size_t ws_len;
    int dtype;
    // paged cache: pools [n_blocks][n_kv][block_size][64]; nullptr = contiguous
    const int32_t* block_table = nullptr;
    size_t max_blocks = 0, block_size = 0, n_blocks = 0;
    // fused RoPE + KV append (kvb_rope_attention_decode); nullptr = none
    const float* rope_cos = nullptr;
    const float* rope_sin = nullptr;
    size_t rope_max_pos = 0;
    bool kv_ready = false;  // DecodeArgs::kv_ready
};

static int launch_decode_mma(kvb_stream_t stream, const DecodeLaunch& L) {
    CUtensorMap kmap, vmap;
    const uint64_t dims[2] = {64, L.total_rows};
    const uint64_t strides[1] = {128};
    const uint32_t box[2] = {64, 64};
    int st = encode_tmap(&kmap, L.kc, 2, dims, strides, box, L.dtype);
    if (st) return st;
    st = encode_tmap(&vmap, L.vc, 2, dims, strides, box, L.dtype);
    if (st) return st;

    DecodeArgs a;
    a.q = static_cast<const uint16_t*>(L.q);
    a.q_row_stride = (long long)L.q_row_stride;
    a.lens = L.lens;
    a.len_const = L.len_const;
    a.max_len = (int)L.max_len;
    a.n_kv = (int)L.n_kv;
    a.group = (int)(L.n_q / L.n_kv);
    a.max_seq = (int)L.max_seq;
    a.seq_rows = (long long)(L.seq_stride / 64);
    a.scale_log2 = L.scale * 1.4426950408889634f;
    a.out = static_cast<uint16_t*>(L.out);
    a.out_row_stride = (long long)L.out_row_stride;
    a.block_table = L.block_table;
    a.max_blocks = (int)L.max_blocks;
    a.block_size = (int)L.block_size;
    a.n_blocks = (int)L.n_blocks;
    a.rope_cos = L.rope_cos;
    a.rope_sin = L.rope_sin;
    a.rope_max_pos = (int)L.rope_max_pos;
    a.kc_w = static_cast<uint16_t*>(const_cast<void*>(L.kc));
    a.vc_w = static_cast<uint16_t*>(const_cast<void*>(L.vc));
    a.cache_seq_stride = (long long)L.seq_stride;
    a.kv_ready = L.kv_ready ? 1 : 0;
    const DecodePlan plan = decode_plan(L.n_seq, L.max_len, L.n_q, L.n_kv, L.ws, L.ws_len);
    a.ws = plan.mode == kSingle ? nullptr : static_cast<float*>(L.ws);
    a.chunk_keys = plan.chunk_keys;
    a.max_chunks = plan.max_chunks;
    a.fold = plan.mode == kFold ? 1 : 0;

    cudaLaunchConfig_t dcfg = {};
    dcfg.gridDim = a.fold ? dim3((unsigned)a.max_chunks, (unsigned)L.n_kv, (unsigned)L.n_seq)
                          : dim3((unsigned)L.n_kv, (unsigned)L.n_seq, (unsigned)a.max_chunks);
    dcfg.blockDim = dim3(128);
    dcfg.dynamicSmemBytes = kDecSmemBytes;
    dcfg.stream = stream;
    cudaLaunchAttribute dattr[2];
    dattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    dattr[0].val.programmaticStreamSerializationAllowed = 1;
    dattr[1].id = cudaLaunchAttributeClusterDimension;
    dattr[1].val.clusterDim.x = (unsigned)a.max_chunks;
    dattr[1].val.clusterDim.y = 1;
    dattr[1].val.clusterDim.z = 1;
    dcfg.attrs = dattr;
    dcfg.numAttrs = a.fold ? 2 : 1;
#define KVB_DECODE_LAUNCH(T, ROPE)                                                   \
    do {                                                                             \
        set_max_smem(attn_decode_kernel<T, ROPE>, kDecSmemBytes);                    \
        const cudaError_t le = cudaLaunchKernelEx(&dcfg, attn_decode_kernel<T, ROPE>,  \
                                                  kmap, vmap, a);                    \
        if (le != cudaSuccess) return cuda_fail(le, "attention decode launch");       \
    } while (0)
    if (L.dtype == KVB_BF16) {
        if (L.rope_cos) KVB_DECODE_LAUNCH(__nv_bfloat16, true);
        else KVB_DECODE_LAUNCH(__nv_bfloat16, false);
    } else {
        if (L.rope_cos) KVB_DECODE_LAUNCH(__half, true);
        else KVB_DECODE_LAUNCH(__half, false);
    }
#undef KVB_DECODE_LAUNCH
    KVB_CHECK_LAUNCH("attention decode launch");
    if (plan.mode == kChunks) {
        // programmatic dependent launch: set-up overlaps the decode kernel's tail
        const int per_bytes = a.group * 66 * 4;
        const int cap = kCombineSmemBytes / per_bytes;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)L.n_kv, (unsigned)L.n_seq);
        cfg.blockDim = dim3(kCombineThreads);
        cfg.dynamicSmemBytes = (size_t)(a.max_chunks < cap ? a.max_chunks : cap) * per_bytes;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = L.dtype == KVB_BF16
                                  ? cudaLaunchKernelEx(&cfg, attn_combine_kernel<__nv_bfloat16>, a)
                                  : cudaLaunchKernelEx(&cfg, attn_combine_kernel<__half>, a);
        if (e != cudaSuccess) return cuda_fail(e, "attention combine launch");
    }
    return KVB_OK;
}

static int launch_generic_attn(kvb_stream_t stream, const GenericAttnArgs& a, size_t rows,
                               int dtype) {
    if (rows == 0) return KVB_OK;
    dim3 grid((unsigned)rows, (unsigned)((a.n_q + 3) / 4));
    if (dtype == KVB_BF16)
        attn_generic_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(a);
    else
        attn_generic_kernel<__half><<<grid, 128, 0, stream>>>(a);
    KVB_CHECK_LAUNCH("attention (general kernel) launch");
    return KVB_OK;
}

// Paged form when block_table != nullptr: kc / vc are pools of pool_len elements.
static int launch_prefill(kvb_stream_t stream, const void* qkv, const void* kc, const void* vc,
                          void* out, size_t n_seq, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                          size_t max_seq, int dtype, const int32_t* block_table = nullptr,
                          size_t max_blocks = 0, size_t block_size = 0, size_t pool_len = 0,
                          bool out_f32 = false) {
    const size_t stride = (n_q + 2 * n_kv) * 64;
    CUtensorMap qmap, kmap, vmap;
    {
        const uint64_t dims[3] = {stride, t, n_seq};
        const uint64_t strides[2] = {stride * 2, t * stride * 2};
        const uint32_t box[3] = {64, (uint32_t)kPfRows, 1};
        int st = encode_tmap(&qmap, qkv, 3, dims, strides, box, dtype);
        if (st) return st;
    }
    if (!block_table) {
        const uint64_t dims[3] = {64, pos0 + t, n_seq * n_kv};
        const uint64_t strides[2] = {128, max_seq * 128};
        const uint32_t box[3] = {64, (uint32_t)kPfKeys, 1};
        int st = encode_tmap(&kmap, kc, 3, dims, strides, box, dtype);
        if (st) return st;
        st = encode_tmap(&vmap, vc, 3, dims, strides, box, dtype);
        if (st) return st;
    } else {
        const uint64_t dims[2] = {64, pool_len / 64};
        const uint64_t strides[1] = {128};
        const uint32_t box[2] = {64, (uint32_t)kPfPagedPiece};
        int st = encode_tmap(&kmap, kc, 2, dims, strides, box, dtype);
        if (st) return st;
        st = encode_tmap(&vmap, vc, 2, dims, strides, box, dtype);
        if (st) return st;
    }
    PrefillArgs a;
    a.block_table = block_table;
    a.max_blocks = (int)max_blocks;
    a.block_size = (int)block_size;
    a.n_blocks = block_table ? (int)(pool_len / (n_kv * block_size * 64)) : 0;
    a.t = (int)t;
    a.pos0 = (int)pos0;
    a.n_q = (int)n_q;
    a.n_kv = (int)n_kv;
    a.group = (int)(n_q / n_kv);
    const size_t rows_per_block = (size_t)kPfRows;
    a.n_qblocks = (int)((t + rows_per_block - 1) / rows_per_block);
    a.scale_log2 = (1.0f / sqrtf(64.0f)) * 1.4426950408889634f;
    a.out = static_cast<uint16_t*>(out);
    a.out_row_stride = (long long)(n_q * 64);
    dim3 grid((unsigned)n_q, (unsigned)n_seq, (unsigned)a.n_qblocks);
#define KVB_PREFILL_LAUNCH(T, F32)                                                       \
    do {                                                                                 \
        set_max_smem(attn_prefill_kernel<T, F32>, kPfSmemBytes);                         \
        attn_prefill_kernel<T, F32><<<grid, kPfThreads, kPfSmemBytes, stream>>>(qmap, kmap, \
                                                                                vmap, a); \
    } while (0)
    if (dtype == KVB_BF16) {
        if (out_f32) KVB_PREFILL_LAUNCH(__nv_bfloat16, true);
        else KVB_PREFILL_LAUNCH(__nv_bfloat16, false);
    } else {
        if (out_f32) KVB_PREFILL_LAUNCH(__half, true);
        else KVB_PREFILL_LAUNCH(__half, false);
    }
#undef KVB_PREFILL_LAUNCH
    KVB_CHECK_LAUNCH("attention prefill launch");
    return KVB_OK;
}

// ---------------------------------------------------------------- norm launcher
// Persistent bulk-copy RMSNorm: kNormBulkPerSm CTAs per SM, fewer if the
// instantiation's registers or shared memory do not allow that many.
template <typename K>
static void launch_norm_bulk(K* kernel, int smem_cap, int smem, kvb_stream_t stream, void* x,
                             const void* y, const void* w, void* out, size_t rows, size_t chunks,
                             float ih, float eps) {
    set_max_smem(kernel, smem_cap);
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, const void*>, std::pair<int, int>>> seen;
    int dev = 0;
    cudaGetDevice(&dev);
    const void* key = reinterpret_cast<const void*>(kernel);
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& e : seen)
            if (e.first.first == dev && e.first.second == key && e.second.first == smem)
                per_sm = e.second.second;
        if (!per_sm) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kNormBulkThreads,
                                                              smem) != cudaSuccess ||
                per_sm < 1)
                per_sm = 1;
            seen.push_back({{dev, key}, {smem, per_sm}});
        }
    }
    const size_t cap = (size_t)num_sms() * (per_sm < kNormBulkPerSm ? per_sm : kNormBulkPerSm);
    const unsigned grid = (unsigned)(rows < cap ? rows : cap);
    kernel<<<grid, kNormBulkThreads, smem, stream>>>((uint4*)x, (const uint4*)y, (const uint4*)w,
                                                      (uint4*)out, (int)rows, (int)chunks, ih, eps);
}

template <bool kAdd>
static int launch_rmsnorm(kvb_stream_t stream, void* x, const void* y, const void* w, void* out,
                          size_t rows, size_t hidden, float eps, int dtype) {
    if (rows == 0) return KVB_OK;
    const size_t chunks = hidden / 8;
    const bool vec = hidden % 8 == 0 && aligned(x, 16) && aligned(w, 16) && aligned(out, 16) &&
                     (!kAdd || aligned(y, 16)) && chunks <= 32 * 16;
    // Decode-sized batches (fewer rows than 4 per SM): a CTA per row.
    const bool per_row = vec && chunks % 32 == 0 && chunks <= 1024 &&
                         rows <= (size_t)num_sms() * 4;
    if (per_row) {
        const float ih = 1.0f / (float)hidden;
        const cudaError_t le =
            dtype == KVB_BF16
                ? launch_pdl(rmsnorm_row_kernel<__nv_bfloat16, kAdd>, dim3((unsigned)rows),
                             dim3((unsigned)chunks), 0, stream, (uint4*)x, (const uint4*)y,
                             (const uint4*)w, (uint4*)out, (int)chunks, ih, eps)
                : launch_pdl(rmsnorm_row_kernel<__half, kAdd>, dim3((unsigned)rows),
                             dim3((unsigned)chunks), 0, stream, (uint4*)x, (const uint4*)y,
                             (const uint4*)w, (uint4*)out, (int)chunks, ih, eps);
        if (le != cudaSuccess) return cuda_fail(le, "rmsnorm launch");
    } else if (vec) {
        const float ih = 1.0f / (float)hidden;
        const int nv = chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : chunks <= 256 ? 8 : 16;
        const int smem = norm_bulk_smem_bytes((int)chunks, kAdd);
#define KVB_NORM_LAUNCH(T, NV, FULL)                                                               \
    launch_norm_bulk(rmsnorm_bulk_kernel<T, NV, kAdd, FULL>, norm_bulk_smem_cap(NV, kAdd), smem,    \
                     stream, x, y, w, out, rows, chunks, ih, eps)
#define KVB_NORM_CASE(NV)                                                                          \
    case NV:                                                                                       \
        if (dtype == KVB_BF16) {                                                                   \
            if (chunks == 32 * NV) KVB_NORM_LAUNCH(__nv_bfloat16, NV, true);                       \
            else KVB_NORM_LAUNCH(__nv_bfloat16, NV, false);                                        \
        } else {                                                                                   \
            if (chunks == 32 * NV) KVB_NORM_LAUNCH(__half, NV, true);                              \
            else KVB_NORM_LAUNCH(__half, NV, false);                                               \
        }                                                                                          \
        break;
        switch (nv) {
            KVB_NORM_CASE(1)
            KVB_NORM_CASE(2)
            KVB_NORM_CASE(4)
            KVB_NORM_CASE(8)
            KVB_NORM_CASE(16)
        }
#undef KVB_NORM_CASE
#undef KVB_NORM_LAUNCH
    } else {
        if (dtype == KVB_BF16)
            rmsnorm_generic_kernel<__nv_bfloat16, kAdd><<<(unsigned)rows, 256, 0, stream>>>(
                (__nv_bfloat16*)x, (const __nv_bfloat16*)y, (const __nv_bfloat16*)w,
                (__nv_bfloat16*)out, (int)hidden, eps);
        else
            rmsnorm_generic_kernel<__half, kAdd><<<(unsigned)rows, 256, 0, stream>>>(
                (__half*)x, (const __half*)y, (const __half*)w, (__half*)out, (int)hidden, eps);
    }
    KVB_CHECK_LAUNCH("rmsnorm launch");
    return KVB_OK;
}

// ---------------------------------------------------------------- projections of few rows
// linear_rows_kernel<N, kGlu, T>: a grid of n_tiles x splits CTAs in clusters of
// `splits`, launched as a programmatic dependent of the preceding kernel.
template <int N, bool kGlu, typename T>
static cudaError_t launch_linear_rows(cudaStream_t stream, const CUtensorMap& wmap,
                                      const CUtensorMap& xmap, const LinearRowsArgs& a,
                                      int n_tiles, uint32_t fmt) {
    auto* kernel = linear_rows_kernel<N, kGlu, T>;
    set_max_smem(kernel, lr_smem_bytes(N));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n_tiles * a.splits));
    cfg.blockDim = dim3(kLrThreads);
    cfg.dynamicSmemBytes = lr_smem_bytes(N);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n_attr = 0;
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr++].val.programmaticStreamSerializationAllowed = 1;
    if (a.splits > 1) {
        attr[n_attr].id = cudaLaunchAttributeClusterDimension;
        attr[n_attr].val.clusterDim.x = (unsigned)a.splits;
        attr[n_attr].val.clusterDim.y = 1;
        attr[n_attr++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
    return cudaLaunchKernelEx(&cfg, kernel, wmap, xmap, a, fmt);
}

template <bool kGlu, typename T>
static cudaError_t launch_linear_rows_n(int n, cudaStream_t stream, const CUtensorMap& wmap,
                                        const CUtensorMap& xmap, const LinearRowsArgs& a,
                                        int n_tiles, uint32_t fmt) {
    switch (n) {
        case 16: return launch_linear_rows<16, kGlu, T>(stream, wmap, xmap, a, n_tiles, fmt);
        case 32: return launch_linear_rows<32, kGlu, T>(stream, wmap, xmap, a, n_tiles, fmt);
        case 64: return launch_linear_rows<64, kGlu, T>(stream, wmap, xmap, a, n_tiles, fmt);
        default: return launch_linear_rows<128, kGlu, T>(stream, wmap, xmap, a, n_tiles, fmt);
    }
}

// Shared body of kvb_linear_rows (glu false: W has out rows) and
// kvb_linear_silu_mul (glu true: W_gu has 2 * out rows, Y is [rows, out]).
// The caller has checked the lengths; rows and out are positive.
static int linear_rows_launch(cudaStream_t stream, const void* x, const void* w, void* y,
                              size_t rows, size_t in_dim, size_t out, bool glu, int splits,
                              int dtype, const char* name) {
    const size_t w_rows = glu ? 2 * out : out;
    if (!(rows <= (size_t)kLrMaxRows && in_dim > 0 && in_dim % 8 == 0 && out % 4 == 0 &&
          fits_i32(in_dim) && fits_i32(w_rows) && aligned(x, 16) && aligned(w, 16) &&
          aligned(y, 8)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "%s: needs rows <= %d, in a multiple of 8, out a multiple of 4, 16-byte "
                    "aligned x and w, 8-byte aligned output (use kvb_linear)",
                    name, kLrMaxRows);
    const int n = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
    const int kchunks = (int)((in_dim + kLrK - 1) / kLrK);
    const int n_tiles = (int)(glu ? (out + 63) / 64 : (out + kLrTile - 1) / kLrTile);
    int s = splits;
    if (s == 0) {
        // about 8 chunks (160 KB of W) per CTA, which the ring requests at once;
        // clusters of at most 6 and at most two thirds of the SMs.  Measured on B200
        // at the Llama-3.2-1B shapes: 8-CTA clusters and wider grids finish later
        // (cluster placement, and the next projection finds no SMs to start on)
        s = kchunks / 8;
        if (s > 6) s = 6;
        const int by_sms = (num_sms() * 2 / 3) / n_tiles;
        if (s > by_sms) s = by_sms;
    }
    if (s > kchunks) s = kchunks;
    if (s < 1) s = 1;
    KVB_CHECK((size_t)n_tiles * (size_t)s <= 0x7fffffffu, "%s: too many tiles", name);
    CUtensorMap wmap, xmap;
    {
        const uint64_t dims[2] = {in_dim, w_rows};
        const uint64_t strides[1] = {in_dim * 2};
        const uint32_t box[2] = {(uint32_t)kLrK, (uint32_t)(glu ? 64 : kLrTile)};
        const int st = encode_tmap(&wmap, w, 2, dims, strides, box, dtype);
        if (st) return st;
    }
    {
        const uint64_t dims[2] = {in_dim, rows};
        const uint64_t strides[1] = {in_dim * 2};
        const uint32_t box[2] = {(uint32_t)kLrK, (uint32_t)n};  // rows past `rows` read as 0
        const int st = encode_tmap(&xmap, x, 2, dims, strides, box, dtype);
        if (st) return st;
    }
    LinearRowsArgs a;
    a.rows = (int)rows;
    a.out = (int)out;
    a.glu_up = glu ? (int)out : 0;
    a.kchunks = kchunks;
    a.splits = s;
    a.y = y;
    const uint32_t fmt = dtype == KVB_BF16 ? 1u : 0u;
    cudaError_t e;
    if (dtype == KVB_BF16)
        e = glu ? launch_linear_rows_n<true, __nv_bfloat16>(n, stream, wmap, xmap, a, n_tiles, fmt)
                : launch_linear_rows_n<false, __nv_bfloat16>(n, stream, wmap, xmap, a, n_tiles, fmt);
    else
        e = glu ? launch_linear_rows_n<true, __half>(n, stream, wmap, xmap, a, n_tiles, fmt)
                : launch_linear_rows_n<false, __half>(n, stream, wmap, xmap, a, n_tiles, fmt);
    if (e != cudaSuccess) return cuda_fail(e, name);
    return KVB_OK;
}

// ---------------------------------------------------------------- self test
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        // Nothing ever arrives on this barrier: the bounded wait must give up.
        mbar_wait(&bar, 0, limit_ns, kDevErrSelfTest);
        mbar_inval(&bar);
    }
}

}  // namespace kvb

using namespace kvb;

// =====================================================================================
extern "C" {

const char* kvb_last_error(void) { return t_err.c_str(); }
const char* kvb_version(void) { return "kvasir_b200 0.1 (sm_100a)"; }

int kvb_device_error(uint32_t* code) {
    KVB_CHECK(code != nullptr, "kvb_device_error: null output pointer");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "kvb_device_error: synchronize");
    uint32_t v = 0, zero = 0;
    e = cudaMemcpyFromSymbol(&v, g_dev_error, sizeof v);
    if (e != cudaSuccess) return cuda_fail(e, "kvb_device_error: read");
    e = cudaMemcpyToSymbol(g_dev_error, &zero, sizeof zero);
    if (e != cudaSuccess) return cuda_fail(e, "kvb_device_error: clear");
    *code = v;
    return KVB_OK;
}

// ------------------------------------------------------------------ embedding gather
int kvb_embedding_gather(kvb_stream_t stream, const int32_t* ids, size_t t, const void* table,
                         size_t table_len, void* out, size_t out_len, size_t hidden, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(hidden > 0, "embedding: hidden must be > 0");
    KVB_CHECK(out_len == t * hidden, "embedding: out has %zu elems, want %zux%zu", out_len, t, hidden);
    KVB_CHECK(table_len % hidden == 0, "embedding: table len %zu not a multiple of hidden %zu",
              table_len, hidden);
    KVB_CHECK(fits_i32(hidden), "hidden=%zu does not fit in i32", hidden);
    KVB_CHECK(fits_i32(t), "t=%zu does not fit in i32", t);
    const size_t vocab = table_len / hidden;
    KVB_CHECK(fits_i32(vocab), "vocab=%zu does not fit in i32", vocab);
    if (t == 0) return KVB_OK;
    if (hidden % 8 == 0 && aligned(table, 16) && aligned(out, 16)) {
        embedding_gather_vec_kernel<<<(unsigned)((t + 3) / 4), 128, 0, stream>>>(
            ids, (const uint4*)table, (uint4*)out, (int)t, (int)(hidden / 8), (int)vocab);
    } else {
        embedding_gather_scalar_kernel<<<(unsigned)t, 256, 0, stream>>>(
            ids, (const uint16_t*)table, (uint16_t*)out, (int)hidden, (int)vocab);
    }
    KVB_CHECK_LAUNCH("embedding launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ rmsnorm
int kvb_rmsnorm(kvb_stream_t stream, const void* x, size_t x_len, const void* w, size_t w_len,
                void* out, size_t out_len, size_t rows, size_t hidden, float eps, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == rows * hidden, "rmsnorm: x has %zu elems, want %zux%zu", x_len, rows, hidden);
    KVB_CHECK(out_len == rows * hidden, "rmsnorm: out has %zu elems, want %zux%zu", out_len, rows,
              hidden);
    KVB_CHECK(w_len == hidden, "rmsnorm: w has %zu elems, want %zu", w_len, hidden);
    KVB_CHECK(fits_i32(hidden), "hidden=%zu does not fit in i32", hidden);
    KVB_CHECK(fits_i32(rows), "rows=%zu does not fit in i32", rows);
    KVB_CHECK(hidden > 0 || rows == 0, "rmsnorm: hidden must be > 0");
    return launch_rmsnorm<false>(stream, const_cast<void*>(x), nullptr, w, out, rows, hidden, eps,
                                 dtype);
}

int kvb_embedding_rmsnorm(kvb_stream_t stream, const int32_t* ids, size_t t, const void* table,
                          size_t table_len, const void* w, size_t w_len, void* x, size_t x_len,
                          void* out, size_t out_len, size_t hidden, float eps, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(hidden > 0, "embedding_rmsnorm: hidden must be > 0");
    KVB_CHECK(x_len == t * hidden, "embedding_rmsnorm: x has %zu elems, want %zux%zu", x_len, t,
              hidden);
    KVB_CHECK(out_len == t * hidden, "embedding_rmsnorm: out has %zu elems, want %zux%zu", out_len,
              t, hidden);
    KVB_CHECK(w_len == hidden, "embedding_rmsnorm: w has %zu elems, want %zu", w_len, hidden);
    KVB_CHECK(table_len % hidden == 0,
              "embedding_rmsnorm: table len %zu not a multiple of hidden %zu", table_len, hidden);
    KVB_CHECK(fits_i32(hidden) && fits_i32(t), "embedding_rmsnorm: a dimension does not fit in i32");
    const size_t vocab = table_len / hidden;
    KVB_CHECK(fits_i32(vocab), "embedding_rmsnorm: vocab=%zu does not fit in i32", vocab);
    if (t == 0) return KVB_OK;
    const size_t chunks = hidden / 8;
    // the rows kvb_rmsnorm normalises with rmsnorm_row_kernel: one launch
    const bool fused = embedding_rmsnorm_fused(t, hidden, table, w, x, out);
    if (!fused) {  // the same two kernels as the unfused calls
        const int st = kvb_embedding_gather(stream, ids, t, table, table_len, x, x_len, hidden,
                                            dtype);
        if (st) return st;
        return kvb_rmsnorm(stream, x, x_len, w, w_len, out, out_len, t, hidden, eps, dtype);
    }
    const float ih = 1.0f / (float)hidden;
    const cudaError_t le =
        dtype == KVB_BF16
            ? launch_pdl(embedding_rmsnorm_row_kernel<__nv_bfloat16>, dim3((unsigned)t),
                         dim3((unsigned)chunks), 0, stream, ids, (const uint4*)table,
                         (const uint4*)w, (uint4*)x, (uint4*)out, (int)chunks, (int)vocab, ih, eps)
            : launch_pdl(embedding_rmsnorm_row_kernel<__half>, dim3((unsigned)t),
                         dim3((unsigned)chunks), 0, stream, ids, (const uint4*)table,
                         (const uint4*)w, (uint4*)x, (uint4*)out, (int)chunks, (int)vocab, ih, eps);
    if (le != cudaSuccess) return cuda_fail(le, "embedding_rmsnorm launch");
    return KVB_OK;
}

int kvb_add_rmsnorm(kvb_stream_t stream, void* x, size_t x_len, const void* y, size_t y_len,
                    const void* w, size_t w_len, void* out, size_t out_len, size_t rows,
                    size_t hidden, float eps, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == rows * hidden && y_len == x_len && out_len == x_len,
              "add_rmsnorm: x/y/out have %zu/%zu/%zu elems, want %zux%zu", x_len, y_len, out_len,
              rows, hidden);
    KVB_CHECK(w_len == hidden, "add_rmsnorm: w has %zu elems, want %zu", w_len, hidden);
    KVB_CHECK(fits_i32(hidden) && fits_i32(rows), "add_rmsnorm: rows/hidden do not fit in i32");
    KVB_CHECK(hidden > 0 || rows == 0, "add_rmsnorm: hidden must be > 0");
    KVB_CHECK(x != out, "add_rmsnorm: out must not alias the residual x");
    return launch_rmsnorm<true>(stream, x, y, w, out, rows, hidden, eps, dtype);
}

// ------------------------------------------------------------------ rope / kv append
static RopeArgs rope_args(void* qkv, size_t n_q, size_t n_kv, size_t hd) {
    RopeArgs a;
    memset(&a, 0, sizeof a);
    a.qkv = static_cast<uint16_t*>(qkv);
    a.n_q = (int)n_q;
    a.n_kv = (int)n_kv;
    a.hd = (int)hd;
    a.row_stride = (int)((n_q + 2 * n_kv) * hd);
    return a;
}

int kvb_rope_inplace(kvb_stream_t stream, void* qkv, size_t qkv_len, const float* cos_t,
                     size_t cos_len, const float* sin_t, size_t sin_len, size_t t, size_t pos0,
                     size_t n_q, size_t n_kv, size_t head_dim, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope: odd head_dim %zu", head_dim);
    KVB_CHECK(qkv_len == t * stride, "rope: qkv has %zu elems, want %zux%zu", qkv_len, t, stride);
    KVB_CHECK(cos_len == sin_len && cos_len % (head_dim / 2) == 0, "rope: bad cos/sin table sizes");
    const size_t max_pos = cos_len / (head_dim / 2);
    KVB_CHECK(pos0 + t <= max_pos, "rope: positions up to %zu exceed table of %zu", pos0 + t, max_pos);
    KVB_CHECK(fits_i32(pos0) && fits_i32(n_q) && fits_i32(n_kv) && fits_i32(head_dim) &&
                  fits_i32(stride) && fits_i32(t) && fits_i32(max_pos),
              "rope: a dimension does not fit in i32");
    if (t == 0) return KVB_OK;
    RopeArgs a = rope_args(qkv, n_q, n_kv, head_dim);
    a.rows_per_seq = (int)t;
    a.pos0 = (int)pos0;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.max_pos = (int)max_pos;
    a.max_seq = (int)max_pos;
    a.do_rope = 1;
    const bool vec = head_dim % 16 == 0 && aligned(qkv, 16) && aligned(cos_t, 16) && aligned(sin_t, 16);
    return launch_rope(stream, a, (int)t, dtype, vec);
}

int kvb_kv_append(kvb_stream_t stream, const void* qkv, size_t qkv_len, void* kc, size_t kc_len,
                  void* vc, size_t vc_len, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                  size_t head_dim, size_t max_seq, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(qkv_len == t * stride, "kv_append: qkv has %zu elems, want %zux%zu", qkv_len, t, stride);
    KVB_CHECK(kc_len == n_kv * max_seq * head_dim && vc_len == kc_len, "kv_append: bad cache sizes");
    KVB_CHECK(pos0 + t <= max_seq, "kv_append: positions up to %zu exceed max_seq %zu", pos0 + t,
              max_seq);
    KVB_CHECK(fits_i32(pos0) && fits_i32(n_kv) && fits_i32(head_dim) && fits_i32(max_seq) &&
                  fits_i32(n_q * head_dim) && fits_i32(stride) && fits_i32(t),
              "kv_append: a dimension does not fit in i32");
    if (t == 0) return KVB_OK;
    RopeArgs a = rope_args(const_cast<void*>(qkv), n_q, n_kv, head_dim);
    a.rows_per_seq = (int)t;
    a.pos0 = (int)pos0;
    a.kc = static_cast<uint16_t*>(kc);
    a.vc = static_cast<uint16_t*>(vc);
    a.seq_stride = 0;
    a.max_seq = (int)max_seq;
    a.do_append = 1;
    const bool vec = head_dim % 16 == 0 && aligned(qkv, 16) && aligned(kc, 16) && aligned(vc, 16);
    return launch_rope(stream, a, (int)t, dtype, vec);
}

// n_seq sequences of t rows each, all starting at pos0; sequence b's cache is
// kc/vc + b * n_kv * max_seq * head_dim.
static int rope_kv_append_seqs(kvb_stream_t stream, void* qkv, size_t qkv_len, const float* cos_t,
                               const float* sin_t, size_t table_len, void* kc, void* vc,
                               size_t cache_len, size_t n_seq, size_t t, size_t pos0, size_t n_q,
                               size_t n_kv, size_t head_dim, size_t max_seq, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope: odd head_dim %zu", head_dim);
    KVB_CHECK(qkv_len == n_seq * t * stride, "rope_kv_append: qkv has %zu elems, want %zux%zux%zu",
              qkv_len, n_seq, t, stride);
    KVB_CHECK(table_len % (head_dim / 2) == 0, "rope: bad cos/sin table sizes");
    const size_t max_pos = table_len / (head_dim / 2);
    KVB_CHECK(pos0 + t <= max_pos, "rope: positions up to %zu exceed table of %zu", pos0 + t, max_pos);
    const size_t per_seq = n_kv * max_seq * head_dim;
    KVB_CHECK(cache_len == n_seq * per_seq, "kv_append: bad cache sizes");
    KVB_CHECK(pos0 + t <= max_seq, "kv_append: positions up to %zu exceed max_seq %zu", pos0 + t,
              max_seq);
    KVB_CHECK(fits_i32(pos0) && fits_i32(stride) && fits_i32(t) && fits_i32(n_seq * t) &&
                  fits_i32(max_seq) && fits_i32(max_pos),
              "rope_kv_append: a dimension does not fit in i32");
    if (t == 0 || n_seq == 0) return KVB_OK;
    RopeArgs a = rope_args(qkv, n_q, n_kv, head_dim);
    a.rows_per_seq = (int)t;
    a.pos0 = (int)pos0;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.max_pos = (int)max_pos;
    a.kc = static_cast<uint16_t*>(kc);
    a.vc = static_cast<uint16_t*>(vc);
    a.seq_stride = (long long)per_seq;
    a.max_seq = (int)max_seq;
    a.do_rope = 1;
    a.do_append = 1;
    const bool vec = head_dim % 16 == 0 && aligned(qkv, 16) && aligned(cos_t, 16) &&
                     aligned(sin_t, 16) && aligned(kc, 16) && aligned(vc, 16);
    return launch_rope(stream, a, (int)(n_seq * t), dtype, vec);
}

int kvb_rope_kv_append(kvb_stream_t stream, void* qkv, size_t qkv_len, const float* cos_t,
                       const float* sin_t, size_t table_len, void* kc, void* vc, size_t cache_len,
                       size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim,
                       size_t max_seq, int dtype) {
    return rope_kv_append_seqs(stream, qkv, qkv_len, cos_t, sin_t, table_len, kc, vc, cache_len, 1,
                               t, pos0, n_q, n_kv, head_dim, max_seq, dtype);
}

int kvb_rope_kv_append_prefill(kvb_stream_t stream, void* qkv, size_t qkv_len,
                               const float* cos_t, const float* sin_t, size_t table_len, void* kc,
                               void* vc, size_t cache_len, size_t n_seq, size_t t, size_t pos0,
                               size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                               int dtype) {
    return rope_kv_append_seqs(stream, qkv, qkv_len, cos_t, sin_t, table_len, kc, vc, cache_len,
                               n_seq, t, pos0, n_q, n_kv, head_dim, max_seq, dtype);
}

int kvb_rope_kv_append_batched(kvb_stream_t stream, void* qkv, size_t n_seq, const int32_t* pos,
                               const float* cos_t, const float* sin_t, size_t table_len,
                               void* kc, void* vc, size_t seq_stride, size_t cache_len,
                               size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                               int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    const size_t per_seq = n_kv * max_seq * head_dim;
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope: odd head_dim %zu", head_dim);
    KVB_CHECK(pos != nullptr, "rope_kv_append_batched: null position array");
    KVB_CHECK(table_len % (head_dim / 2) == 0, "rope: bad cos/sin table sizes");
    KVB_CHECK(seq_stride >= per_seq, "rope_kv_append_batched: seq_stride %zu < cache of %zu",
              seq_stride, per_seq);
    KVB_CHECK(n_seq == 0 || cache_len >= (n_seq - 1) * seq_stride + per_seq,
              "rope_kv_append_batched: cache of %zu elems is too small", cache_len);
    KVB_CHECK(fits_i32(n_seq) && fits_i32(stride) && fits_i32(max_seq) &&
                  fits_i32(table_len / (head_dim / 2)),
              "rope_kv_append_batched: a dimension does not fit in i32");
    if (n_seq == 0) return KVB_OK;
    RopeArgs a = rope_args(qkv, n_q, n_kv, head_dim);
    a.rows_per_seq = 1;
    a.pos_arr = pos;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.max_pos = (int)(table_len / (head_dim / 2));
    a.kc = static_cast<uint16_t*>(kc);
    a.vc = static_cast<uint16_t*>(vc);
    a.seq_stride = (long long)seq_stride;
    a.max_seq = (int)max_seq;
    a.do_rope = 1;
    a.do_append = 1;
    const bool vec = head_dim % 16 == 0 && seq_stride % 8 == 0 && aligned(qkv, 16) &&
                     aligned(cos_t, 16) && aligned(sin_t, 16) && aligned(kc, 16) && aligned(vc, 16);
    return launch_rope(stream, a, (int)n_seq, dtype, vec);
}

// Paged form: sequence b's t rows (qkv rows b*t .. b*t+t-1) go to positions
// pos[b] .. pos[b]+t-1 of its blocks (block_table row b).
int kvb_rope_kv_append_paged(kvb_stream_t stream, void* qkv, size_t n_seq, size_t t,
                             const int32_t* pos, const float* cos_t, const float* sin_t,
                             size_t table_len, void* k_pool, void* v_pool, size_t pool_len,
                             const int32_t* block_table, size_t max_blocks, size_t block_size,
                             size_t n_q, size_t n_kv, size_t head_dim, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope: odd head_dim %zu", head_dim);
    KVB_CHECK(pos != nullptr && block_table != nullptr,
              "rope_kv_append_paged: null position array or block table");
    KVB_CHECK(table_len % (head_dim / 2) == 0, "rope: bad cos/sin table sizes");
    KVB_CHECK(block_size > 0 && n_kv > 0, "rope_kv_append_paged: block_size and n_kv must be > 0");
    const size_t per_block = n_kv * block_size * head_dim;
    KVB_CHECK(pool_len % per_block == 0,
              "rope_kv_append_paged: pool of %zu elems is not a whole number of %zu-elem blocks",
              pool_len, per_block);
    const size_t n_blocks = pool_len / per_block;
    const size_t max_seq = max_blocks * block_size;
    KVB_CHECK(fits_i32(n_seq * t) && fits_i32((n_q + 2 * n_kv) * head_dim) && fits_i32(max_seq) &&
                  fits_i32(n_blocks) && fits_i32(table_len / (head_dim / 2)),
              "rope_kv_append_paged: a dimension does not fit in i32");
    if (n_seq == 0 || t == 0) return KVB_OK;
    RopeArgs a = rope_args(qkv, n_q, n_kv, head_dim);
    a.rows_per_seq = (int)t;
    a.pos_arr = pos;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.max_pos = (int)(table_len / (head_dim / 2));
    a.kc = static_cast<uint16_t*>(k_pool);
    a.vc = static_cast<uint16_t*>(v_pool);
    a.max_seq = (int)max_seq;
    a.block_table = block_table;
    a.max_blocks = (int)max_blocks;
    a.block_size = (int)block_size;
    a.n_blocks = (int)n_blocks;
    a.do_rope = 1;
    a.do_append = 1;
    const bool vec = head_dim % 16 == 0 && aligned(qkv, 16) && aligned(cos_t, 16) &&
                     aligned(sin_t, 16) && aligned(k_pool, 16) && aligned(v_pool, 16);
    return launch_rope(stream, a, (int)(n_seq * t), dtype, vec);
}

// ------------------------------------------------------------------ silu_mul
int kvb_silu_mul(kvb_stream_t stream, const void* gu, size_t gu_len, void* out, size_t out_len,
                 size_t t, size_t inter, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(gu_len == t * 2 * inter, "silu_mul: gu has %zu elems, want %zux%zu", gu_len, t,
              2 * inter);
    KVB_CHECK(out_len == t * inter, "silu_mul: out has %zu elems, want %zux%zu", out_len, t, inter);
    KVB_CHECK(fits_i32(inter) && fits_i32(t), "silu_mul: a dimension does not fit in i32");
    if (t == 0 || inter == 0) return KVB_OK;
    const unsigned gy = (unsigned)(t < 65535 ? t : 65535);
    if (inter % 8 == 0 && aligned(gu, 16) && aligned(out, 16)) {
        const int chunks = (int)(inter / 8);
        dim3 grid((unsigned)((chunks + 255) / 256), gy);
        if (dtype == KVB_BF16)
            silu_mul_vec_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const uint4*)gu, (uint4*)out,
                                                                       chunks, (int)t);
        else
            silu_mul_vec_kernel<__half><<<grid, 256, 0, stream>>>((const uint4*)gu, (uint4*)out, chunks,
                                                                (int)t);
    } else {
        dim3 grid((unsigned)((inter + 255) / 256 < 64 ? (inter + 255) / 256 : 64), gy);
        if (dtype == KVB_BF16)
            silu_mul_scalar_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
                (const __nv_bfloat16*)gu, (__nv_bfloat16*)out, (int)inter, (int)t);
        else
            silu_mul_scalar_kernel<__half><<<grid, 256, 0, stream>>>((const __half*)gu, (__half*)out,
                                                                   (int)inter, (int)t);
    }
    KVB_CHECK_LAUNCH("silu_mul launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ add_inplace
int kvb_add_inplace(kvb_stream_t stream, void* x, size_t x_len, const void* y, size_t y_len,
                    int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == y_len, "add: lengths differ (%zu vs %zu)", x_len, y_len);
    if (x_len == 0) return KVB_OK;
    if (x_len % 8 == 0 && aligned(x, 16) && aligned(y, 16)) {
        const size_t nvec = x_len / 8;
        if (dtype == KVB_BF16)
            add_vec_kernel<__nv_bfloat16><<<grid_for(nvec, 256), 256, 0, stream>>>((uint4*)x,
                                                                                  (const uint4*)y, nvec);
        else
            add_vec_kernel<__half><<<grid_for(nvec, 256), 256, 0, stream>>>((uint4*)x, (const uint4*)y,
                                                                           nvec);
    } else {
        if (dtype == KVB_BF16)
            add_scalar_kernel<__nv_bfloat16><<<grid_for(x_len, 256), 256, 0, stream>>>(
                (__nv_bfloat16*)x, (const __nv_bfloat16*)y, x_len);
        else
            add_scalar_kernel<__half><<<grid_for(x_len, 256), 256, 0, stream>>>(
                (__half*)x, (const __half*)y, x_len);
    }
    KVB_CHECK_LAUNCH("add launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ bf16 -> f16
int kvb_bf16_to_f16(kvb_stream_t stream, const void* src, size_t src_len, void* dst,
                    size_t dst_len, uint32_t* bad, size_t bad_len) {
    KVB_CHECK(src_len == dst_len, "bf16_to_f16: lengths differ (%zu vs %zu)", src_len, dst_len);
    KVB_CHECK(bad_len == 1, "bf16_to_f16: bad counter must hold exactly one u32");
    if (src_len == 0) return KVB_OK;
    bf16_to_f16_kernel<<<grid_for(src_len, 256), 256, 0, stream>>>((const __nv_bfloat16*)src,
                                                                   (__half*)dst, src_len, bad);
    KVB_CHECK_LAUNCH("bf16_to_f16 launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ attention
size_t kvb_attention_workspace_bytes(size_t t, size_t pos0, size_t n_q, size_t n_kv,
                                     size_t head_dim) {
    if (t != 1 || head_dim != 64 || n_kv == 0) return 0;
    return decode_ws_bytes(1, pos0 + 1, n_q, n_kv);
}

int kvb_attention(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                  size_t kc_len, const void* vc, size_t vc_len, void* out, size_t out_len,
                  size_t t, size_t pos0, size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                  void* workspace, size_t workspace_len, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0, "attention: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(head_dim > 0 && 128 % head_dim == 0, "attention: head_dim %zu must divide 128",
              head_dim);
    KVB_CHECK(qkv_len == t * stride, "attention: qkv has %zu elems, want %zux%zu", qkv_len, t, stride);
    KVB_CHECK(kc_len == n_kv * max_seq * head_dim && vc_len == kc_len, "attention: bad cache sizes");
    KVB_CHECK(out_len == t * n_q * head_dim, "attention: out has %zu elems, want %zux%zu", out_len, t,
              n_q * head_dim);
    KVB_CHECK(pos0 + t <= max_seq, "attention: kv length %zu exceeds max_seq %zu", pos0 + t, max_seq);
    KVB_CHECK(fits_i32(pos0) && fits_i32(n_q) && fits_i32(n_kv) && fits_i32(head_dim) &&
                  fits_i32(max_seq) && fits_i32(stride) && fits_i32(t),
              "attention: a dimension does not fit in i32");
    if (t == 0) return KVB_OK;
    const size_t group = n_q / n_kv;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const bool fast = head_dim == 64 && aligned(qkv, 16) && aligned(kc, 16) && aligned(vc, 16) &&
                      aligned(out, 16) && fits_i32(n_kv * max_seq);
    if (fast && t == 1 && group <= 16) {
        DecodeLaunch L;
        L.q = qkv;
        L.q_row_stride = stride;
        L.kc = kc;
        L.vc = vc;
        L.seq_stride = n_kv * max_seq * 64;
        L.total_rows = n_kv * max_seq;
        L.lens = nullptr;
        L.len_const = (int)(pos0 + 1);
        L.n_seq = 1;
        L.max_len = pos0 + 1;
        L.n_q = n_q;
        L.n_kv = n_kv;
        L.max_seq = max_seq;
        L.scale = scale;
        L.out = out;
        L.out_row_stride = n_q * 64;
        L.ws = workspace;
        L.ws_len = workspace_len;
        L.dtype = dtype;
        return launch_decode_mma(stream, L);
    }
    if (fast && t > 1)
        return launch_prefill(stream, qkv, kc, vc, out, 1, t, pos0, n_q, n_kv, max_seq, dtype);
    GenericAttnArgs a;
    a.q = static_cast<const uint16_t*>(qkv);
    a.q_row_stride = (long long)stride;
    a.kc = static_cast<const uint16_t*>(kc);
    a.vc = static_cast<const uint16_t*>(vc);
    a.seq_stride = 0;
    a.rows_per_seq = (int)t;
    a.lens = nullptr;
    a.pos0 = (int)pos0;
    a.max_len = (int)(pos0 + t);
    a.n_q = (int)n_q;
    a.n_kv = (int)n_kv;
    a.hd = (int)head_dim;
    a.max_seq = (int)max_seq;
    a.scale = scale;
    a.out = static_cast<uint16_t*>(out);
    a.out_row_stride = (long long)(n_q * head_dim);
    return launch_generic_attn(stream, a, t, dtype);
}

size_t kvb_attention_decode_workspace_bytes(size_t n_seq, size_t max_len, size_t n_q,
                                            size_t n_kv, size_t head_dim) {
    if (head_dim != 64 || n_kv == 0) return 0;
    return decode_ws_bytes(n_seq, max_len, n_q, n_kv);
}

int kvb_attention_decode(kvb_stream_t stream, const void* q, size_t q_row_stride, const void* kc,
                         const void* vc, size_t seq_stride, size_t cache_len,
                         const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                         size_t n_kv, size_t head_dim, size_t max_seq, float scale, void* out,
                         size_t out_row_stride, void* workspace, size_t workspace_len,
                         int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t per_seq = n_kv * max_seq * head_dim;
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0, "attention_decode: n_q %zu not a multiple of n_kv %zu",
              n_q, n_kv);
    KVB_CHECK(head_dim > 0 && head_dim <= 256, "attention_decode: head_dim %zu unsupported",
              head_dim);
    KVB_CHECK(lens != nullptr, "attention_decode: null lengths array");
    KVB_CHECK(max_len <= max_seq, "attention_decode: max_len %zu exceeds max_seq %zu", max_len,
              max_seq);
    KVB_CHECK(seq_stride >= per_seq, "attention_decode: seq_stride %zu < per-sequence cache %zu",
              seq_stride, per_seq);
    KVB_CHECK(n_seq == 0 || cache_len >= (n_seq - 1) * seq_stride + per_seq,
              "attention_decode: cache of %zu elems is too small", cache_len);
    KVB_CHECK(q_row_stride >= n_q * head_dim, "attention_decode: q_row_stride too small");
    KVB_CHECK(out_row_stride >= n_q * head_dim, "attention_decode: out_row_stride too small");
    KVB_CHECK(fits_i32(n_seq) && fits_i32(max_seq) && fits_i32(max_len),
              "attention_decode: a dimension does not fit in i32");
    if (n_seq == 0) return KVB_OK;
    const size_t total_rows = ((n_seq - 1) * seq_stride + per_seq) / 64;
    if (decode_fast_path(q, q_row_stride, kc, vc, seq_stride, n_seq, n_q, n_kv, head_dim, max_seq,
                         out_row_stride)) {
        DecodeLaunch L;
        L.q = q;
        L.q_row_stride = q_row_stride;
        L.kc = kc;
        L.vc = vc;
        L.seq_stride = seq_stride;
        L.total_rows = total_rows;
        L.lens = lens;
        L.len_const = 0;
        L.n_seq = n_seq;
        L.max_len = max_len;
        L.n_q = n_q;
        L.n_kv = n_kv;
        L.max_seq = max_seq;
        L.scale = scale;
        L.out = out;
        L.out_row_stride = out_row_stride;
        L.ws = workspace;
        L.ws_len = workspace_len;
        L.dtype = dtype;
        return launch_decode_mma(stream, L);
    }
    GenericAttnArgs a;
    a.q = static_cast<const uint16_t*>(q);
    a.q_row_stride = (long long)q_row_stride;
    a.kc = static_cast<const uint16_t*>(kc);
    a.vc = static_cast<const uint16_t*>(vc);
    a.seq_stride = (long long)seq_stride;
    a.rows_per_seq = 1;
    a.lens = lens;
    a.pos0 = 0;
    a.max_len = (int)max_len;
    a.n_q = (int)n_q;
    a.n_kv = (int)n_kv;
    a.hd = (int)head_dim;
    a.max_seq = (int)max_seq;
    a.scale = scale;
    a.out = static_cast<uint16_t*>(out);
    a.out_row_stride = (long long)out_row_stride;
    return launch_generic_attn(stream, a, n_seq, dtype);
}

static int rope_attention_decode_impl(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                      const float* cos_t, const float* sin_t, size_t table_len,
                                      void* kc, void* vc, size_t seq_stride, size_t cache_len,
                                      const int32_t* lens, size_t n_seq, size_t max_len,
                                      size_t n_q, size_t n_kv, size_t head_dim, size_t max_seq,
                                      float scale, void* out, size_t out_row_stride,
                                      void* workspace, size_t workspace_len, int dtype,
                                      bool kv_ready) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    const size_t per_seq = n_kv * max_seq * head_dim;
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0,
              "rope_attention_decode: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(qkv_len == n_seq * stride, "rope_attention_decode: qkv has %zu elems, want %zux%zu",
              qkv_len, n_seq, stride);
    KVB_CHECK(cos_t != nullptr && sin_t != nullptr && lens != nullptr,
              "rope_attention_decode: null table or lengths array");
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0 && table_len % (head_dim / 2) == 0,
              "rope_attention_decode: bad cos/sin table sizes");
    KVB_CHECK(max_len <= max_seq, "rope_attention_decode: max_len %zu exceeds max_seq %zu",
              max_len, max_seq);
    KVB_CHECK(seq_stride >= per_seq, "rope_attention_decode: seq_stride %zu < per-sequence cache %zu",
              seq_stride, per_seq);
    KVB_CHECK(n_seq == 0 || cache_len >= (n_seq - 1) * seq_stride + per_seq,
              "rope_attention_decode: cache of %zu elems is too small", cache_len);
    KVB_CHECK(out_row_stride >= n_q * head_dim, "rope_attention_decode: out_row_stride too small");
    KVB_CHECK(fits_i32(n_seq) && fits_i32(max_seq) && fits_i32(max_len) &&
                  fits_i32(table_len / (head_dim / 2)),
              "rope_attention_decode: a dimension does not fit in i32");
    if (n_seq == 0) return KVB_OK;
    const size_t group = n_q / n_kv;
    const size_t total_rows = ((n_seq - 1) * seq_stride + per_seq) / 64;
    const bool fast = head_dim == 64 && group <= 16 && n_seq <= 65535 && n_kv <= 65535 &&
                      seq_stride % 64 == 0 && out_row_stride % 8 == 0 && aligned(qkv, 16) &&
                      aligned(kc, 16) && aligned(vc, 16) && fits_i32(total_rows);
    if (!fast)
        return fail(KVB_ERR_UNSUPPORTED,
                    "rope_attention_decode: needs head_dim 64, n_q/n_kv <= 16, 16-byte aligned "
                    "buffers and seq_stride a multiple of 64 (use kvb_rope_kv_append_batched + "
                    "kvb_attention_decode)");
    DecodeLaunch L;
    L.q = qkv;
    L.q_row_stride = stride;
    L.kc = kc;
    L.vc = vc;
    L.seq_stride = seq_stride;
    L.total_rows = total_rows;
    L.lens = lens;
    L.len_const = 0;
    L.n_seq = n_seq;
    L.max_len = max_len;
    L.n_q = n_q;
    L.n_kv = n_kv;
    L.max_seq = max_seq;
    L.scale = scale;
    L.out = out;
    L.out_row_stride = out_row_stride;
    L.ws = workspace;
    L.ws_len = workspace_len;
    L.dtype = dtype;
    L.rope_cos = cos_t;
    L.rope_sin = sin_t;
    L.rope_max_pos = table_len / (head_dim / 2);
    L.kv_ready = kv_ready;
    return launch_decode_mma(stream, L);
}

int kvb_rope_attention_decode(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                              const float* cos_t, const float* sin_t, size_t table_len, void* kc,
                              void* vc, size_t seq_stride, size_t cache_len, const int32_t* lens,
                              size_t n_seq, size_t max_len, size_t n_q, size_t n_kv,
                              size_t head_dim, size_t max_seq, float scale, void* out,
                              size_t out_row_stride, void* workspace, size_t workspace_len,
                              int dtype) {
    return rope_attention_decode_impl(stream, qkv, qkv_len, cos_t, sin_t, table_len, kc, vc,
                                      seq_stride, cache_len, lens, n_seq, max_len, n_q, n_kv,
                                      head_dim, max_seq, scale, out, out_row_stride, workspace,
                                      workspace_len, dtype, false);
}

int kvb_attention_prefill(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                          const void* vc, size_t cache_len, void* out, size_t out_len,
                          size_t n_seq, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                          size_t head_dim, size_t max_seq, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(qkv_len == n_seq * t * (n_q + 2 * n_kv) * head_dim,
              "attention_prefill: qkv has %zu elems, want %zux%zu", qkv_len, n_seq * t,
              (n_q + 2 * n_kv) * head_dim);
    KVB_CHECK(cache_len == n_seq * n_kv * max_seq * head_dim, "attention_prefill: bad cache sizes");
    KVB_CHECK(out_len == n_seq * t * n_q * head_dim, "attention_prefill: out has %zu elems, want %zux%zu",
              out_len, n_seq * t, n_q * head_dim);
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0, "attention_prefill: n_q %zu not a multiple of n_kv %zu",
              n_q, n_kv);
    KVB_CHECK(head_dim > 0 && head_dim <= 256, "attention_prefill: head_dim %zu unsupported", head_dim);
    KVB_CHECK(pos0 + t <= max_seq, "attention_prefill: kv length %zu exceeds max_seq %zu", pos0 + t,
              max_seq);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(fits_i32(n_seq * t) && fits_i32(pos0 + t) && fits_i32(stride) &&
                  fits_i32(n_seq * n_kv),
              "attention_prefill: a dimension does not fit in i32");
    if (n_seq == 0 || t == 0) return KVB_OK;
    const bool fast = head_dim == 64 && n_seq <= 65535 && aligned(qkv, 16) && aligned(kc, 16) &&
                      aligned(vc, 16) && aligned(out, 16);
    if (fast) return launch_prefill(stream, qkv, kc, vc, out, n_seq, t, pos0, n_q, n_kv, max_seq, dtype);
    GenericAttnArgs a;
    a.q = static_cast<const uint16_t*>(qkv);
    a.q_row_stride = (long long)stride;
    a.kc = static_cast<const uint16_t*>(kc);
    a.vc = static_cast<const uint16_t*>(vc);
    a.seq_stride = (long long)(n_kv * max_seq * head_dim);
    a.rows_per_seq = (int)t;
    a.lens = nullptr;
    a.pos0 = (int)pos0;
    a.max_len = (int)(pos0 + t);
    a.n_q = (int)n_q;
    a.n_kv = (int)n_kv;
    a.hd = (int)head_dim;
    a.max_seq = (int)max_seq;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.out = static_cast<uint16_t*>(out);
    a.out_row_stride = (long long)(n_q * head_dim);
    return launch_generic_attn(stream, a, n_seq * t, dtype);
}

int kvb_attention_prefill_f32(kvb_stream_t stream, const void* qkv, size_t qkv_len, const void* kc,
                              const void* vc, size_t cache_len, float* out, size_t out_len,
                              size_t n_seq, size_t t, size_t pos0, size_t n_q, size_t n_kv,
                              size_t head_dim, size_t max_seq, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(qkv_len == n_seq * t * (n_q + 2 * n_kv) * head_dim,
              "attention_prefill_f32: qkv has %zu elems, want %zux%zu", qkv_len, n_seq * t,
              (n_q + 2 * n_kv) * head_dim);
    KVB_CHECK(cache_len == n_seq * n_kv * max_seq * head_dim,
              "attention_prefill_f32: bad cache sizes");
    KVB_CHECK(out_len == n_seq * t * n_q * head_dim,
              "attention_prefill_f32: out has %zu elems, want %zux%zu", out_len, n_seq * t,
              n_q * head_dim);
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0,
              "attention_prefill_f32: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(pos0 + t <= max_seq, "attention_prefill_f32: kv length %zu exceeds max_seq %zu",
              pos0 + t, max_seq);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(fits_i32(n_seq * t) && fits_i32(pos0 + t) && fits_i32(stride) &&
                  fits_i32(n_seq * n_kv),
              "attention_prefill_f32: a dimension does not fit in i32");
    if (n_seq == 0 || t == 0) return KVB_OK;
    if (!(head_dim == 64 && n_seq <= 65535 && aligned(qkv, 16) && aligned(kc, 16) &&
          aligned(vc, 16) && aligned(out, 16)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "attention_prefill_f32: needs head_dim 64 and 16-byte aligned buffers");
    return launch_prefill(stream, qkv, kc, vc, out, n_seq, t, pos0, n_q, n_kv, max_seq, dtype,
                          nullptr, 0, 0, 0, true);
}

int kvb_attention_prefill_paged(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                const void* k_pool, const void* v_pool, size_t pool_len,
                                const int32_t* block_table, size_t max_blocks, size_t block_size,
                                void* out, size_t out_len, size_t n_seq, size_t t, size_t pos0,
                                size_t n_q, size_t n_kv, size_t head_dim, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0,
              "attention_prefill_paged: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(block_table != nullptr, "attention_prefill_paged: null block table");
    KVB_CHECK(block_size > 0 && head_dim > 0, "attention_prefill_paged: block_size must be > 0");
    KVB_CHECK(qkv_len == n_seq * t * stride,
              "attention_prefill_paged: qkv has %zu elems, want %zux%zux%zu", qkv_len, n_seq, t,
              stride);
    KVB_CHECK(out_len == n_seq * t * n_q * head_dim,
              "attention_prefill_paged: out has %zu elems, want %zux%zux%zu", out_len, n_seq, t,
              n_q * head_dim);
    const size_t per_block = n_kv * block_size * head_dim;
    KVB_CHECK(pool_len % per_block == 0,
              "attention_prefill_paged: pool of %zu elems is not a whole number of %zu-elem blocks",
              pool_len, per_block);
    KVB_CHECK(pos0 + t <= max_blocks * block_size,
              "attention_prefill_paged: positions up to %zu exceed %zu blocks of %zu", pos0 + t,
              max_blocks, block_size);
    KVB_CHECK(fits_i32(n_seq * t) && fits_i32(pos0 + t) && fits_i32(stride) &&
                  fits_i32(n_seq * max_blocks) && fits_i32(pool_len / 64 + 64),
              "attention_prefill_paged: a dimension does not fit in i32");
    if (n_seq == 0 || t == 0) return KVB_OK;
    if (!(head_dim == 64 && block_size % 32 == 0 && n_q <= 65535 && n_seq <= 65535 &&
          aligned(qkv, 16) && aligned(k_pool, 16) && aligned(v_pool, 16) && aligned(out, 16)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "attention_prefill_paged: needs head_dim 64, block_size a multiple of 32 and "
                    "16-byte aligned buffers");
    return launch_prefill(stream, qkv, k_pool, v_pool, out, n_seq, t, pos0, n_q, n_kv,
                          max_blocks * block_size, dtype, block_table, max_blocks, block_size,
                          pool_len);
}

// kvb_rope_kv_append_paged (one row per sequence, at position lens[b] - 1) and
// kvb_attention_decode_paged in one launch.
static int rope_attention_decode_paged_impl(
    kvb_stream_t stream, const void* qkv, size_t qkv_len, const float* cos_t, const float* sin_t,
    size_t table_len, void* k_pool, void* v_pool, size_t pool_len, const int32_t* block_table,
    size_t max_blocks, size_t block_size, const int32_t* lens, size_t n_seq, size_t max_len,
    size_t n_q, size_t n_kv, size_t head_dim, float scale, void* out, size_t out_row_stride,
    void* workspace, size_t workspace_len, int dtype, bool kv_ready) {
    KVB_CHECK_DTYPE(dtype);
    const size_t stride = (n_q + 2 * n_kv) * head_dim;
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0,
              "rope_attention_decode_paged: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(qkv_len == n_seq * stride,
              "rope_attention_decode_paged: qkv has %zu elems, want %zux%zu", qkv_len, n_seq, stride);
    KVB_CHECK(cos_t != nullptr && sin_t != nullptr && lens != nullptr && block_table != nullptr,
              "rope_attention_decode_paged: null table, lengths array or block table");
    KVB_CHECK(head_dim > 0 && head_dim % 2 == 0 && table_len % (head_dim / 2) == 0,
              "rope_attention_decode_paged: bad cos/sin table sizes");
    KVB_CHECK(block_size > 0, "rope_attention_decode_paged: block_size must be > 0");
    const size_t per_block = n_kv * block_size * head_dim;
    KVB_CHECK(pool_len % per_block == 0,
              "rope_attention_decode_paged: pool of %zu elems is not a whole number of %zu-elem blocks",
              pool_len, per_block);
    KVB_CHECK(max_len <= max_blocks * block_size,
              "rope_attention_decode_paged: max_len %zu exceeds %zu blocks of %zu", max_len,
              max_blocks, block_size);
    KVB_CHECK(out_row_stride >= n_q * head_dim, "rope_attention_decode_paged: out_row_stride too small");
    const size_t n_blocks = pool_len / per_block;
    const size_t total_rows = pool_len / 64;
    KVB_CHECK(fits_i32(n_seq) && fits_i32(max_len) && fits_i32(max_blocks) && fits_i32(n_blocks) &&
                  fits_i32(n_seq * max_blocks) && fits_i32(table_len / (head_dim / 2)),
              "rope_attention_decode_paged: a dimension does not fit in i32");
    if (n_seq == 0) return KVB_OK;
    const size_t group = n_q / n_kv;
    if (!(head_dim == 64 && block_size % 64 == 0 && group <= 16 && n_seq <= 65535 &&
          n_kv <= 65535 && out_row_stride % 8 == 0 && aligned(qkv, 16) && aligned(k_pool, 16) &&
          aligned(v_pool, 16) && fits_i32(total_rows + 64)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "rope_attention_decode_paged: needs head_dim 64, block_size a multiple of 64, "
                    "n_q/n_kv <= 16 and 16-byte aligned buffers");
    DecodeLaunch L;
    L.q = qkv;
    L.q_row_stride = stride;
    L.kc = k_pool;
    L.vc = v_pool;
    L.seq_stride = 0;
    L.total_rows = total_rows;
    L.lens = lens;
    L.len_const = 0;
    L.n_seq = n_seq;
    L.max_len = max_len;
    L.n_q = n_q;
    L.n_kv = n_kv;
    L.max_seq = max_blocks * block_size;
    L.scale = scale;
    L.out = out;
    L.out_row_stride = out_row_stride;
    L.ws = workspace;
    L.ws_len = workspace_len;
    L.dtype = dtype;
    L.block_table = block_table;
    L.max_blocks = max_blocks;
    L.block_size = block_size;
    L.n_blocks = n_blocks;
    L.rope_cos = cos_t;
    L.rope_sin = sin_t;
    L.rope_max_pos = table_len / (head_dim / 2);
    L.kv_ready = kv_ready;
    return launch_decode_mma(stream, L);
}

int kvb_rope_attention_decode_paged(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                    const float* cos_t, const float* sin_t, size_t table_len,
                                    void* k_pool, void* v_pool, size_t pool_len,
                                    const int32_t* block_table, size_t max_blocks,
                                    size_t block_size, const int32_t* lens, size_t n_seq,
                                    size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                    float scale, void* out, size_t out_row_stride, void* workspace,
                                    size_t workspace_len, int dtype) {
    return rope_attention_decode_paged_impl(stream, qkv, qkv_len, cos_t, sin_t, table_len, k_pool,
                                            v_pool, pool_len, block_table, max_blocks, block_size,
                                            lens, n_seq, max_len, n_q, n_kv, head_dim, scale, out,
                                            out_row_stride, workspace, workspace_len, dtype, false);
}

int kvb_attention_decode_paged(kvb_stream_t stream, const void* q, size_t q_row_stride,
                               const void* k_pool, const void* v_pool, size_t pool_len,
                               const int32_t* block_table, size_t max_blocks, size_t block_size,
                               const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                               size_t n_kv, size_t head_dim, float scale, void* out,
                               size_t out_row_stride, void* workspace, size_t workspace_len,
                               int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(n_kv > 0 && n_q % n_kv == 0,
              "attention_decode_paged: n_q %zu not a multiple of n_kv %zu", n_q, n_kv);
    KVB_CHECK(lens != nullptr && block_table != nullptr,
              "attention_decode_paged: null lengths array or block table");
    KVB_CHECK(block_size > 0, "attention_decode_paged: block_size must be > 0");
    const size_t per_block = n_kv * block_size * head_dim;
    KVB_CHECK(head_dim > 0 && pool_len % per_block == 0,
              "attention_decode_paged: pool of %zu elems is not a whole number of %zu-elem blocks",
              pool_len, per_block);
    KVB_CHECK(max_len <= max_blocks * block_size,
              "attention_decode_paged: max_len %zu exceeds %zu blocks of %zu", max_len, max_blocks,
              block_size);
    KVB_CHECK(q_row_stride >= n_q * head_dim, "attention_decode_paged: q_row_stride too small");
    KVB_CHECK(out_row_stride >= n_q * head_dim, "attention_decode_paged: out_row_stride too small");
    const size_t n_blocks = pool_len / per_block;
    const size_t total_rows = pool_len / 64;
    KVB_CHECK(fits_i32(n_seq) && fits_i32(max_len) && fits_i32(max_blocks) && fits_i32(n_blocks) &&
                  fits_i32(n_seq * max_blocks),
              "attention_decode_paged: a dimension does not fit in i32");
    if (n_seq == 0) return KVB_OK;
    const size_t group = n_q / n_kv;
    if (!(head_dim == 64 && block_size % 64 == 0 && group <= 16 && n_seq <= 65535 &&
          n_kv <= 65535 && q_row_stride % 8 == 0 && out_row_stride % 8 == 0 && aligned(q, 16) &&
          aligned(k_pool, 16) && aligned(v_pool, 16) && fits_i32(total_rows + 64)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "attention_decode_paged: needs head_dim 64, block_size a multiple of 64, "
                    "n_q/n_kv <= 16 and 16-byte aligned buffers");
    DecodeLaunch L;
    L.q = q;
    L.q_row_stride = q_row_stride;
    L.kc = k_pool;
    L.vc = v_pool;
    L.seq_stride = 0;
    L.total_rows = total_rows;
    L.lens = lens;
    L.len_const = 0;
    L.n_seq = n_seq;
    L.max_len = max_len;
    L.n_q = n_q;
    L.n_kv = n_kv;
    L.max_seq = max_blocks * block_size;
    L.scale = scale;
    L.out = out;
    L.out_row_stride = out_row_stride;
    L.ws = workspace;
    L.ws_len = workspace_len;
    L.dtype = dtype;
    L.block_table = block_table;
    L.max_blocks = max_blocks;
    L.block_size = block_size;
    L.n_blocks = n_blocks;
    return launch_decode_mma(stream, L);
}

}  // extern "C"

// ------------------------------------------------------------------ decode attention without allocation
// Scratch for kvb_attention_decode_noalloc: the split-KV partials of one call.
// It lives in the library's own device memory on every GPU that loads the
// library.  In host code this name is only a host-side stand-in for the
// device array; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[KVB_NOALLOC_SCRATCH_BYTES];

// Unique id of the calling thread's current CUDA context (cuCtxGetId, through
// the runtime's driver entry points as for the tensor maps); 0 if unavailable.
static unsigned long long current_context_id() {
    typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
    typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx &&
        get_id(ctx, &id) == CUDA_SUCCESS)
        return id;
    return 0;
}

// Device address of g_noalloc_scratch on the current device, looked up with
// that device current on the first call and cached together with the id of
// the device's context.  A new context on the device (after cudaDeviceReset)
// holds a new copy of the array, so a changed id repeats the look-up.  The
// look-up is refused while `stream` is being captured into a graph.
static void* noalloc_scratch_address(kvb_stream_t stream, int* status) {
    static std::mutex mu;
    static void* addr[64] = {};
    static unsigned long long ctx_id[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = cuda_fail(e, "attention_decode_noalloc: cudaGetDevice");
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        *status = fail(KVB_ERR_UNSUPPORTED, "attention_decode_noalloc: device ordinal %d > 63", dev);
        return nullptr;
    }
    const unsigned long long id = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx_id[dev] != id) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &cs);
        if (e != cudaSuccess) {
            *status = cuda_fail(e, "attention_decode_noalloc: cudaStreamIsCapturing");
            return nullptr;
        }
        if (cs != cudaStreamCaptureStatusNone) {
            *status = fail(KVB_ERR_UNSUPPORTED,
                           "attention_decode_noalloc: the first call on device %d runs inside a "
                           "stream capture; make one call before capturing (it looks up the "
                           "scratch array's device address)",
                           dev);
            return nullptr;
        }
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            *status = cuda_fail(e, "attention_decode_noalloc: cudaGetSymbolAddress");
            return nullptr;
        }
        addr[dev] = p;
        ctx_id[dev] = id;
    }
    return addr[dev];
}

extern "C" {

int kvb_attention_decode_noalloc(kvb_stream_t stream, const void* q, size_t q_row_stride,
                                 const void* kc, const void* vc, size_t seq_stride,
                                 size_t cache_len, const int32_t* lens, size_t n_seq,
                                 size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                 size_t max_seq, float scale, void* out, size_t out_row_stride,
                                 int dtype) {
    // Every partial the combine pass reads is written earlier in the same
    // call, so no part of the shared array has to start at zero.  Only the
    // split-KV kernel uses scratch; calls that kvb_attention_decode sends to
    // its general kernel pass none and meet no size limit.
    const size_t need =
        decode_fast_path(q, q_row_stride, kc, vc, seq_stride, n_seq, n_q, n_kv, head_dim, max_seq,
                         out_row_stride)
            ? kvb_attention_decode_workspace_bytes(n_seq, max_len, n_q, n_kv, head_dim)
            : 0;
    KVB_CHECK(need <= KVB_NOALLOC_SCRATCH_BYTES,
              "attention_decode_noalloc: the split-KV partials need %zu bytes, more than the "
              "%u-byte scratch array; use kvb_attention_decode with a workspace",
              need, (unsigned)KVB_NOALLOC_SCRATCH_BYTES);
    void* ws = nullptr;
    if (need > 0) {
        int st = KVB_OK;
        ws = noalloc_scratch_address(stream, &st);
        if (!ws) return st;
    }
    return kvb_attention_decode(stream, q, q_row_stride, kc, vc, seq_stride, cache_len, lens,
                                n_seq, max_len, n_q, n_kv, head_dim, max_seq, scale, out,
                                out_row_stride, ws, need, dtype);
}

// ------------------------------------------------------------------ argmax
int kvb_argmax_f32(kvb_stream_t stream, const float* logits, size_t rows, size_t vocab,
                   int32_t* ids, int32_t* advance, int32_t* advance2) {
    KVB_CHECK(vocab > 0 && fits_i32(vocab), "argmax: vocab %zu out of range", vocab);
    KVB_CHECK(rows <= 0x7fffffff / kArgmaxCluster, "argmax: rows %zu out of range", rows);
    if (rows == 0) return KVB_OK;
    const int vec4 = vocab % 4 == 0 && aligned(logits, 16);
    const size_t slice = ((vocab + kArgmaxCluster - 1) / kArgmaxCluster + 3) & ~(size_t)3;
    argmax_kernel<<<(unsigned)(rows * kArgmaxCluster), kArgmaxThreads, 0, stream>>>(
        logits, (int)vocab, (int)slice, ids, advance, advance2, vec4);
    KVB_CHECK_LAUNCH("argmax launch");
    return KVB_OK;
}

int kvb_sample_f32(kvb_stream_t stream, const float* logits, size_t rows, size_t vocab,
                   float temperature, float top_p, uint64_t seed, const int32_t* counters,
                   int32_t* ids, int32_t* advance, int32_t* advance2) {
    KVB_CHECK(vocab > 0 && vocab <= (size_t)kSampleCluster * kSampleMaxSlice,
              "sample: vocab %zu out of range (1 .. %d)", vocab, kSampleCluster * kSampleMaxSlice);
    KVB_CHECK(fits_i32(rows), "sample: rows %zu out of range", rows);
    KVB_CHECK(!(temperature != temperature) && !(top_p != top_p),
              "sample: temperature and top_p must be numbers");
    if (rows == 0) return KVB_OK;
    if (temperature <= 0.f)  // greedy
        return kvb_argmax_f32(stream, logits, rows, vocab, ids, advance, advance2);
    KVB_CHECK(rows <= 0x7fffffff / kSampleCluster, "sample: rows %zu out of range", rows);
    const int vec4 = vocab % 4 == 0 && aligned(logits, 16);
    // 16-CTA clusters when the rows' 16 CTAs each still get an SM of their own
    const bool wide =
        sample_attrs_and_wide_ok(stream) && rows * kSampleClusterWide <= (size_t)num_sms();
    const cudaError_t e =
        wide ? launch_sample<kSampleClusterWide>(stream, logits, rows, vocab, 1.0f / temperature,
                                                 top_p, seed, counters, ids, advance, advance2,
                                                 vec4)
             : launch_sample<kSampleCluster>(stream, logits, rows, vocab, 1.0f / temperature,
                                             top_p, seed, counters, ids, advance, advance2, vec4);
    if (e != cudaSuccess) return cuda_fail(e, "sample launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ LM head + argmax
size_t kvb_lm_head_argmax_workspace_bytes(size_t rows) {
    return rows * (size_t)kLmMaxCtas * (sizeof(float) + sizeof(int32_t));
}

int kvb_lm_head_argmax(kvb_stream_t stream, const void* x, size_t x_len, const void* w,
                       size_t w_len, size_t rows, size_t hidden, size_t vocab, void* workspace,
                       size_t workspace_len, int32_t* ids, int32_t* advance, int32_t* advance2,
                       int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == rows * hidden, "lm_head_argmax: x has %zu elems, want %zux%zu", x_len, rows,
              hidden);
    KVB_CHECK(w_len == vocab * hidden, "lm_head_argmax: w has %zu elems, want %zux%zu", w_len,
              vocab, hidden);
    KVB_CHECK(vocab > 0 && fits_i32(vocab) && fits_i32(hidden),
              "lm_head_argmax: vocab %zu / hidden %zu out of range", vocab, hidden);
    KVB_CHECK(ids != nullptr, "lm_head_argmax: null ids");
    if (rows == 0) return KVB_OK;
    const size_t need = kvb_lm_head_argmax_workspace_bytes(rows);
    KVB_CHECK(workspace != nullptr && workspace_len >= need,
              "lm_head_argmax: workspace of %zu bytes, need %zu", workspace_len, need);
    const int n = rows <= 16 ? 16 : 32;
    if (!(rows <= (size_t)kLmMaxRows && hidden > 0 && hidden % kLmK == 0 &&
          (size_t)n * hidden * 2 <= (size_t)kLmMaxXBytes && aligned(x, 16) && aligned(w, 16) &&
          aligned(workspace, 16)))
        return fail(KVB_ERR_UNSUPPORTED,
                    "lm_head_argmax: needs rows <= %d, hidden a multiple of 64 with rows' x in "
                    "128 KB, 16-byte aligned buffers (use kvb_linear + kvb_argmax_f32)",
                    kLmMaxRows);
    CUtensorMap wmap, xmap;
    {
        const uint64_t dims[2] = {hidden, vocab};
        const uint64_t strides[1] = {hidden * 2};
        const uint32_t box[2] = {(uint32_t)kLmK, (uint32_t)kLmRows};
        int st = encode_tmap(&wmap, w, 2, dims, strides, box, dtype);
        if (st) return st;
    }
    {
        const uint64_t dims[2] = {hidden, rows};
        const uint64_t strides[1] = {hidden * 2};
        const uint32_t box[2] = {(uint32_t)kLmK, (uint32_t)n};  // rows past `rows` read as 0
        int st = encode_tmap(&xmap, x, 2, dims, strides, box, dtype);
        if (st) return st;
    }
    LmArgs a;
    a.vocab = (int)vocab;
    a.hidden = (int)hidden;
    a.rows = (int)rows;
    a.n_tiles = (int)((vocab + kLmRows - 1) / kLmRows);
    int grid = num_sms();
    if (grid > a.n_tiles) grid = a.n_tiles;
    if (grid > kLmMaxCtas) grid = kLmMaxCtas;
    a.part_v = static_cast<float*>(workspace);
    a.part_i = reinterpret_cast<int32_t*>(static_cast<float*>(workspace) + (size_t)kLmMaxCtas * rows);
    const uint32_t fmt = dtype == KVB_BF16 ? 1u : 0u;
    const int smem = lm_smem_bytes(n, (int)hidden);
    cudaError_t e;
    if (n == 16) {
        set_max_smem(lm_head_argmax_kernel<16>, lm_smem_bytes(16, kLmMaxXBytes / 32));
        e = launch_pdl(lm_head_argmax_kernel<16>, dim3(grid), dim3(kLmThreads), smem, stream, wmap,
                       xmap, a, fmt);
    } else {
        set_max_smem(lm_head_argmax_kernel<32>, lm_smem_bytes(32, kLmMaxXBytes / 64));
        e = launch_pdl(lm_head_argmax_kernel<32>, dim3(grid), dim3(kLmThreads), smem, stream, wmap,
                       xmap, a, fmt);
    }
    if (e != cudaSuccess) return cuda_fail(e, "lm_head_argmax launch");
    e = launch_pdl(lm_head_argmax_finish_kernel, dim3((unsigned)rows), dim3(32), 0, stream,
                   (const float*)a.part_v, (const int32_t*)a.part_i, grid, (int)rows, ids, advance,
                   advance2);
    if (e != cudaSuccess) return cuda_fail(e, "lm_head_argmax finish launch");
    return KVB_OK;
}

// ------------------------------------------------------------------ projections of few rows
int kvb_linear_rows(kvb_stream_t stream, const void* x, size_t x_len, const void* w, size_t w_len,
                    void* y, size_t y_len, size_t rows, size_t in_dim, size_t out_dim, int splits,
                    int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == rows * in_dim, "linear_rows: x has %zu elems, want %zux%zu", x_len, rows,
              in_dim);
    KVB_CHECK(w_len == out_dim * in_dim, "linear_rows: w has %zu elems, want %zux%zu", w_len,
              out_dim, in_dim);
    KVB_CHECK(y_len == rows * out_dim, "linear_rows: y has %zu elems, want %zux%zu", y_len, rows,
              out_dim);
    KVB_CHECK(splits >= 0 && splits <= kLrMaxSplits, "linear_rows: splits %d outside [0, %d]",
              splits, kLrMaxSplits);
    if (rows == 0 || out_dim == 0) return KVB_OK;
    return linear_rows_launch(stream, x, w, y, rows, in_dim, out_dim, false, splits, dtype,
                              "linear_rows");
}

int kvb_linear_silu_mul(kvb_stream_t stream, const void* x, size_t x_len, const void* w_gu,
                        size_t w_len, void* act, size_t act_len, size_t rows, size_t hidden,
                        size_t inter, int splits, int dtype) {
    KVB_CHECK_DTYPE(dtype);
    KVB_CHECK(x_len == rows * hidden, "linear_silu_mul: x has %zu elems, want %zux%zu", x_len,
              rows, hidden);
    KVB_CHECK(w_len == 2 * inter * hidden, "linear_silu_mul: w_gu has %zu elems, want %zux%zu",
              w_len, 2 * inter, hidden);
    KVB_CHECK(act_len == rows * inter, "linear_silu_mul: act has %zu elems, want %zux%zu", act_len,
              rows, inter);
    KVB_CHECK(splits >= 0 && splits <= kLrMaxSplits, "linear_silu_mul: splits %d outside [0, %d]",
              splits, kLrMaxSplits);
    if (rows == 0 || inter == 0) return KVB_OK;
    return linear_rows_launch(stream, x, w_gu, act, rows, hidden, inter, true, splits, dtype,
                              "linear_silu_mul");
}

// ------------------------------------------------------------------ self test
int kvb_selftest_wait_timeout(kvb_stream_t stream, uint32_t limit_ms) {
    KVB_CHECK(limit_ms > 0 && limit_ms <= 10000, "selftest: limit %u ms out of range", limit_ms);
    selftest_wait_kernel<<<1, 32, 0, stream>>>((uint64_t)limit_ms * 1000000ull);
    KVB_CHECK_LAUNCH("selftest launch");
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "selftest synchronize");
    uint32_t code = 0;
    int st = kvb_device_error(&code);
    if (st) return st;
    if (code & kDevErrSelfTest)
        return fail(KVB_ERR_DEVICE, "bounded wait gave up after %u ms (device error word 0x%x)",
                    limit_ms, code);
    return fail(KVB_ERR_CUDA, "selftest: the wait completed although nothing arrived");
}

}  // extern "C"

// ------------------------------------------------------------------ decode-step forms
namespace kvb {

int rope_attention_decode_in_step(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                  const float* cos_t, const float* sin_t, size_t table_len,
                                  void* kc, void* vc, size_t seq_stride, size_t cache_len,
                                  const int32_t* lens, size_t n_seq, size_t max_len, size_t n_q,
                                  size_t n_kv, size_t head_dim, size_t max_seq, float scale,
                                  void* out, size_t out_row_stride, void* workspace,
                                  size_t workspace_len, int dtype) {
    return rope_attention_decode_impl(stream, qkv, qkv_len, cos_t, sin_t, table_len, kc, vc,
                                      seq_stride, cache_len, lens, n_seq, max_len, n_q, n_kv,
                                      head_dim, max_seq, scale, out, out_row_stride, workspace,
                                      workspace_len, dtype, true);
}

int rope_attention_decode_paged_in_step(kvb_stream_t stream, const void* qkv, size_t qkv_len,
                                        const float* cos_t, const float* sin_t, size_t table_len,
                                        void* k_pool, void* v_pool, size_t pool_len,
                                        const int32_t* block_table, size_t max_blocks,
                                        size_t block_size, const int32_t* lens, size_t n_seq,
                                        size_t max_len, size_t n_q, size_t n_kv, size_t head_dim,
                                        float scale, void* out, size_t out_row_stride,
                                        void* workspace, size_t workspace_len, int dtype) {
    return rope_attention_decode_paged_impl(stream, qkv, qkv_len, cos_t, sin_t, table_len, k_pool,
                                            v_pool, pool_len, block_table, max_blocks, block_size,
                                            lens, n_seq, max_len, n_q, n_kv, head_dim, scale, out,
                                            out_row_stride, workspace, workspace_len, dtype, true);
}

int decode_combine_launches(size_t n_seq, size_t max_len, size_t n_q, size_t n_kv,
                            size_t head_dim, const void* workspace, size_t workspace_len) {
    if (head_dim != 64 || n_kv == 0 || n_q % n_kv != 0 || n_q / n_kv > 16 || n_seq == 0) return 0;
    return decode_plan(n_seq, max_len, n_q, n_kv, workspace, workspace_len).mode == kChunks ? 1 : 0;
}

}  // namespace kvb
