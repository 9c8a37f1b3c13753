// kvb_checkpoint.cpp -- the weight load path (reference engine/src/model/weights.rs:47-230).
//
// A checkpoint is a directory of safetensors shards.  Each shard is a file of
//   u64 little-endian N | N bytes of JSON header | data
// where the header maps tensor names to {"dtype", "shape", "data_offsets":
// [begin, end)} relative to the start of the data (plus an optional
// "__metadata__" object).  The shards are memory-mapped; tensors are staged
// through pinned host buffers (two, alternating, so filling one overlaps the
// copy of the other) into caller-owned device buffers, converted to the compute
// type on the way.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "kvb_host.h"

namespace {

using kvb::fail;

// ------------------------------------------------------------------ JSON (header only)
struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    bool is_uint = false;  // a non-negative integer literal, held exactly in u
    uint64_t u = 0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JParser {
  public:
    JParser(const char* p, size_t n) : p_(p), e_(p + n) {}
    bool parse(JVal& v) {
        if (!value(v, 0)) return false;
        ws();
        return p_ == e_;
    }
    size_t offset(const char* base) const { return (size_t)(p_ - base); }

  private:
    const char* p_;
    const char* e_;
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* s) {
        const size_t n = strlen(s);
        if ((size_t)(e_ - p_) < n || memcmp(p_, s, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void put_utf8(std::string& out, uint32_t c) {
        if (c < 0x80) {
            out += (char)c;
        } else if (c < 0x800) {
            out += (char)(0xC0 | (c >> 6));
            out += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            out += (char)(0xE0 | (c >> 12));
            out += (char)(0x80 | ((c >> 6) & 0x3F));
            out += (char)(0x80 | (c & 0x3F));
        } else {
            out += (char)(0xF0 | (c >> 18));
            out += (char)(0x80 | ((c >> 12) & 0x3F));
            out += (char)(0x80 | ((c >> 6) & 0x3F));
            out += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& c) {
        if (e_ - p_ < 4) return false;
        c = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = *p_++;
            c <<= 4;
            if (h >= '0' && h <= '9') c |= (uint32_t)(h - '0');
            else if (h >= 'a' && h <= 'f') c |= (uint32_t)(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') c |= (uint32_t)(h - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string& out) {
        if (p_ >= e_ || *p_ != '"') return false;
        ++p_;
        while (p_ < e_ && *p_ != '"') {
            const unsigned char ch = (unsigned char)*p_;
            if (ch < 0x20) return false;
            if (ch != '\\') {
                out += (char)ch;
                ++p_;
                continue;
            }
            if (++p_ >= e_) return false;
            const char esc = *p_++;
            switch (esc) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t c;
                    if (!hex4(c)) return false;
                    if (c >= 0xD800 && c < 0xDC00) {  // surrogate pair
                        uint32_t lo;
                        if (!lit("\\u") || !hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        c = 0x10000 + ((c - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (c >= 0xDC00 && c < 0xE000) {
                        return false;
                    }
                    put_utf8(out, c);
                    break;
                }
                default: return false;
            }
        }
        if (p_ >= e_) return false;
        ++p_;
        return true;
    }
    bool number(JVal& v) {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') ++p_;
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        bool integral = true;
        while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                           *p_ == '+' || *p_ == '-')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integral = false;
            ++p_;
        }
        v.kind = JVal::kNum;
        if (integral && *s != '-') {
            uint64_t u = 0;
            for (const char* q = s; q < p_; ++q) {
                const uint64_t d = (uint64_t)(*q - '0');
                if (u > (UINT64_MAX - d) / 10) return false;  // does not fit 64 bits
                u = u * 10 + d;
            }
            v.is_uint = true;
            v.u = u;
        }
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > 64) return false;
        ws();
        if (p_ >= e_) return false;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = JVal::kObj;
            ws();
            if (p_ < e_ && *p_ == '}') {
                ++p_;
                return true;
            }
            while (true) {
                ws();
                std::string key;
                if (!string(key)) return false;
                ws();
                if (p_ >= e_ || *p_ != ':') return false;
                ++p_;
                v.obj.emplace_back(std::move(key), JVal());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p_ < e_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < e_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v.kind = JVal::kArr;
            ws();
            if (p_ < e_ && *p_ == ']') {
                ++p_;
                return true;
            }
            while (true) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p_ < e_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < e_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v.kind = JVal::kStr;
            return string(v.str);
        }
        if (lit("true")) {
            v.kind = JVal::kBool;
            return true;
        }
        if (lit("false")) {
            v.kind = JVal::kBool;
            return true;
        }
        if (lit("null")) return true;
        return number(v);
    }
};

// ------------------------------------------------------------------ shards and tensors
struct Tensor {
    int dtype = KVB_CKPT_OTHER;
    std::string dtype_name;
    std::vector<uint64_t> shape;
    const uint8_t* data = nullptr;
    uint64_t nbytes = 0;
    std::string file;
};

struct Mapping {
    void* base = nullptr;
    size_t len = 0;
};

int dtype_of(const std::string& s, int& tag, int& size) {
    static const struct {
        const char* name;
        int tag, size;
    } table[] = {{"BF16", KVB_CKPT_BF16, 2}, {"F16", KVB_CKPT_F16, 2}, {"F32", KVB_CKPT_F32, 4},
                 {"F64", KVB_CKPT_OTHER, 8},  {"I64", KVB_CKPT_OTHER, 8}, {"U64", KVB_CKPT_OTHER, 8},
                 {"I32", KVB_CKPT_OTHER, 4},  {"U32", KVB_CKPT_OTHER, 4}, {"I16", KVB_CKPT_OTHER, 2},
                 {"U16", KVB_CKPT_OTHER, 2},  {"I8", KVB_CKPT_OTHER, 1},  {"U8", KVB_CKPT_OTHER, 1},
                 {"BOOL", KVB_CKPT_OTHER, 1}, {"F8_E4M3", KVB_CKPT_OTHER, 1},
                 {"F8_E5M2", KVB_CKPT_OTHER, 1}};
    for (const auto& t : table)
        if (s == t.name) {
            tag = t.tag;
            size = t.size;
            return 0;
        }
    tag = KVB_CKPT_OTHER;
    size = 0;  // unknown element size: not checked, never loadable
    return 0;
}

// Parses one shard's header into `out` (later shards overwrite earlier names).
int index_shard(const std::string& path, const uint8_t* base, size_t len,
                std::map<std::string, Tensor>& out) {
    if (len < 8) return fail(KVB_ERR_CONFIG, "%s: shorter than the 8-byte header length", path.c_str());
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | base[i];
    if (n > len - 8) return fail(KVB_ERR_CONFIG, "%s: header length %llu exceeds the file (%zu bytes)",
                                 path.c_str(), (unsigned long long)n, len);
    const char* hdr = reinterpret_cast<const char*>(base + 8);
    JVal root;
    JParser jp(hdr, (size_t)n);
    if (!jp.parse(root) || root.kind != JVal::kObj)
        return fail(KVB_ERR_CONFIG, "%s: malformed header JSON (near byte %zu)", path.c_str(),
                    jp.offset(hdr));
    const uint8_t* data = base + 8 + n;
    const uint64_t data_len = len - 8 - n;
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal* dt = t.get("dtype");
        const JVal* shape = t.get("shape");
        const JVal* offs = t.get("data_offsets");
        if (t.kind != JVal::kObj || !dt || dt->kind != JVal::kStr || !shape ||
            shape->kind != JVal::kArr || !offs || offs->kind != JVal::kArr || offs->arr.size() != 2 ||
            !offs->arr[0].is_uint || !offs->arr[1].is_uint)
            return fail(KVB_ERR_CONFIG, "%s: tensor %s: malformed entry", path.c_str(), kv.first.c_str());
        Tensor ten;
        ten.dtype_name = dt->str;
        int esize = 0;
        dtype_of(dt->str, ten.dtype, esize);
        uint64_t numel = 1;
        for (const auto& d : shape->arr) {
            if (!d.is_uint)
                return fail(KVB_ERR_CONFIG, "%s: tensor %s: shape entries must be non-negative integers",
                            path.c_str(), kv.first.c_str());
            ten.shape.push_back(d.u);
            if (d.u && numel > UINT64_MAX / d.u)
                return fail(KVB_ERR_CONFIG, "%s: tensor %s: shape overflows", path.c_str(),
                            kv.first.c_str());
            numel *= d.u;
        }
        const uint64_t b = offs->arr[0].u, e = offs->arr[1].u;
        if (b > e || e > data_len)
            return fail(KVB_ERR_CONFIG, "%s: tensor %s: data_offsets [%llu, %llu) outside the %llu data bytes",
                        path.c_str(), kv.first.c_str(), (unsigned long long)b, (unsigned long long)e,
                        (unsigned long long)data_len);
        if (esize && (numel > UINT64_MAX / (uint64_t)esize || numel * (uint64_t)esize != e - b))
            return fail(KVB_ERR_CONFIG, "%s: tensor %s: %llu bytes for %llu %s elements", path.c_str(),
                        kv.first.c_str(), (unsigned long long)(e - b), (unsigned long long)numel,
                        dt->str.c_str());
        ten.data = data + b;
        ten.nbytes = e - b;
        ten.file = path;
        out[kv.first] = std::move(ten);
    }
    return KVB_OK;
}

std::string shape_str(const std::vector<uint64_t>& s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) {
        if (i) r += ", ";
        r += std::to_string((unsigned long long)s[i]);
    }
    return r + "]";
}

// ------------------------------------------------------------------ host conversions
// IEEE round-to-nearest-even narrowing, written from the formats' definitions.
inline float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    const uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {  // subnormal: value = man * 2^-24
        float f = (float)man * 5.9604644775390625e-08f;
        uint32_t u;
        memcpy(&u, &f, 4);
        bits = sign | u;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

inline uint16_t f32_to_f16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint16_t)(sign | 0x7C00 | (a > 0x7F800000u ? 0x200 : 0));
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00);  // rounds to >= 65520: overflow
    if (a >= 0x38800000u) {  // normal f16 range (>= 2^-14)
        const uint32_t exp = (a >> 23) - 112;
        uint32_t man = a & 0x7FFFFFu;
        uint32_t h = (exp << 10) | (man >> 13);
        const uint32_t rem = man & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    // subnormal or zero: value / 2^-24, rounded to nearest even
    float v;
    memcpy(&v, &a, 4);
    const float q = v * 16777216.0f;  // exact scaling by 2^24
    float r = std::nearbyint(q);      // default rounding mode: nearest even
    return (uint16_t)(sign | (uint16_t)r);
}

inline bool f16_finite(uint16_t h) { return (h & 0x7C00) != 0x7C00; }
inline bool bf16_finite(uint16_t h) { return (h & 0x7F80) != 0x7F80; }

}  // namespace

// ------------------------------------------------------------------ the checkpoint object
struct kvb_checkpoint_s {
    std::vector<Mapping> maps;
    std::map<std::string, Tensor> tensors;
    static constexpr size_t kStage = 32u << 20;  // bytes per staging buffer
    void* pinned[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    void* dev_stage = nullptr;  // bf16 source chunks for device conversion to f16
    int device = -1;

    int ensure_staging(bool need_dev) {
        if (!pinned[0]) {
            cudaGetDevice(&device);
            for (int i = 0; i < 2; ++i) {
                cudaError_t e = cudaHostAlloc(&pinned[i], kStage, cudaHostAllocDefault);
                if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: pinned staging");
                e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
                if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: staging event");
            }
        }
        if (need_dev && !dev_stage) {
            const cudaError_t e = cudaMalloc(&dev_stage, kStage);
            if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: device staging");
        }
        return KVB_OK;
    }
    ~kvb_checkpoint_s() {
        for (int i = 0; i < 2; ++i) {
            if (done[i]) {
                if (used[i]) cudaEventSynchronize(done[i]);
                cudaEventDestroy(done[i]);
            }
            if (pinned[i]) cudaFreeHost(pinned[i]);
        }
        if (dev_stage) cudaFree(dev_stage);
        for (auto& m : maps)
            if (m.base) munmap(m.base, m.len);
    }
};

extern "C" int kvb_checkpoint_open(kvb_checkpoint_t* out, const char* dir) {
    KVB_CHECK(out && dir, "checkpoint_open: null argument");
    *out = nullptr;
    DIR* d = opendir(dir);
    if (!d) return fail(KVB_ERR_IO, "%s: %s", dir, strerror(errno));
    std::vector<std::string> files;
    while (struct dirent* e = readdir(d)) {
        const std::string name = e->d_name;
        const std::string ext = ".safetensors";
        if (name.size() > ext.size() && name.compare(name.size() - ext.size(), ext.size(), ext) == 0)
            files.push_back(std::string(dir) + "/" + name);
    }
    closedir(d);
    std::sort(files.begin(), files.end());
    if (files.empty()) return fail(KVB_ERR_CONFIG, "no .safetensors files in %s", dir);
    auto* ck = new kvb_checkpoint_s();
    for (const auto& path : files) {
        const int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) {
            const int err = errno;
            delete ck;
            return fail(KVB_ERR_IO, "%s: %s", path.c_str(), strerror(err));
        }
        struct stat st;
        if (fstat(fd, &st) != 0) {
            const int err = errno;
            close(fd);
            delete ck;
            return fail(KVB_ERR_IO, "%s: %s", path.c_str(), strerror(err));
        }
        Mapping m;
        m.len = (size_t)st.st_size;
        if (m.len) {
            m.base = mmap(nullptr, m.len, PROT_READ, MAP_PRIVATE, fd, 0);
            if (m.base == MAP_FAILED) {
                const int err = errno;
                close(fd);
                delete ck;
                return fail(KVB_ERR_IO, "%s: mmap: %s", path.c_str(), strerror(err));
            }
        }
        close(fd);
        ck->maps.push_back(m);
        const int st2 = index_shard(path, static_cast<const uint8_t*>(m.base), m.len, ck->tensors);
        if (st2 != KVB_OK) {
            delete ck;
            return st2;
        }
    }
    *out = ck;
    return KVB_OK;
}

extern "C" int kvb_checkpoint_close(kvb_checkpoint_t ck) {
    delete ck;
    return KVB_OK;
}

extern "C" size_t kvb_checkpoint_num_tensors(kvb_checkpoint_t ck) {
    return ck ? ck->tensors.size() : 0;
}

extern "C" int kvb_checkpoint_tensor(kvb_checkpoint_t ck, const char* name, int* dtype, int* ndim,
                                     uint64_t* dims) {
    KVB_CHECK(ck && name, "checkpoint_tensor: null argument");
    const auto it = ck->tensors.find(name);
    if (it == ck->tensors.end()) return fail(KVB_ERR_CONFIG, "missing tensor %s", name);
    const Tensor& t = it->second;
    KVB_CHECK(t.shape.size() <= 8, "%s: rank %zu above 8", name, t.shape.size());
    if (dtype) *dtype = t.dtype;
    if (ndim) *ndim = (int)t.shape.size();
    if (dims)
        for (size_t i = 0; i < t.shape.size(); ++i) dims[i] = t.shape[i];
    return KVB_OK;
}

extern "C" int kvb_checkpoint_load_rows(kvb_checkpoint_t ck, kvb_stream_t stream,
                                        const char* const* names, const uint64_t* rows,
                                        size_t n_parts, uint64_t cols, void* dst, size_t dst_len,
                                        int dst_dtype, uint32_t* bad) {
    KVB_CHECK(ck && names && rows && dst, "checkpoint_load_rows: null argument");
    KVB_CHECK_DTYPE(dst_dtype);
    KVB_CHECK(n_parts > 0 && cols > 0, "checkpoint_load_rows: no parts or zero columns");
    // validate every part before the first copy (reference Loader::load_into)
    std::vector<const Tensor*> parts(n_parts);
    uint64_t total = 0;
    bool dev_convert = false;
    for (size_t i = 0; i < n_parts; ++i) {
        KVB_CHECK(names[i], "checkpoint_load_rows: null name");
        const auto it = ck->tensors.find(names[i]);
        if (it == ck->tensors.end()) return fail(KVB_ERR_CONFIG, "missing tensor %s", names[i]);
        const Tensor& t = it->second;
        std::vector<uint64_t> want;
        if (rows[i] == 0) want = {cols};
        else want = {rows[i], cols};
        KVB_CHECK(t.shape == want, "%s: shape %s, expected %s", names[i], shape_str(t.shape).c_str(),
                  shape_str(want).c_str());
        if (t.dtype == KVB_CKPT_OTHER)
            return fail(KVB_ERR_CONFIG, "%s: unsupported dtype %s", names[i], t.dtype_name.c_str());
        if (t.dtype == KVB_CKPT_BF16 && dst_dtype == KVB_F16) dev_convert = true;
        parts[i] = &t;
        total += (rows[i] ? rows[i] : 1) * cols;
    }
    KVB_CHECK(total == dst_len, "checkpoint_load_rows: the parts hold %llu elements, dst holds %zu",
              (unsigned long long)total, dst_len);
    KVB_CHECK(!dev_convert || bad, "checkpoint_load_rows: a BF16 -> F16 conversion needs the bad counter");
    int st = ck->ensure_staging(dev_convert);
    if (st != KVB_OK) return st;

    uint8_t* out = static_cast<uint8_t*>(dst);
    const size_t chunk = kvb_checkpoint_s::kStage / 4;  // elements per chunk (f32 sources fit)
    int slot = 0;
    for (size_t i = 0; i < n_parts; ++i) {
        const Tensor& t = *parts[i];
        const uint64_t n = (rows[i] ? rows[i] : 1) * cols;
        for (uint64_t off = 0; off < n; off += chunk) {
            const size_t m = (size_t)std::min<uint64_t>(chunk, n - off);
            if (ck->used[slot]) {
                const cudaError_t e = cudaEventSynchronize(ck->done[slot]);
                if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: staging wait");
            }
            uint16_t* stage = static_cast<uint16_t*>(ck->pinned[slot]);
            size_t non_finite = 0;
            bool on_device = false;
            if (t.dtype == KVB_CKPT_BF16 && dst_dtype == KVB_BF16) {
                memcpy(stage, t.data + off * 2, m * 2);
            } else if (t.dtype == KVB_CKPT_F16 && dst_dtype == KVB_F16) {
                memcpy(stage, t.data + off * 2, m * 2);
                for (size_t k = 0; k < m; ++k) non_finite += !f16_finite(stage[k]);
            } else if (t.dtype == KVB_CKPT_BF16) {  // -> F16 on the device
                memcpy(stage, t.data + off * 2, m * 2);
                on_device = true;
            } else if (t.dtype == KVB_CKPT_F16) {  // -> BF16
                const uint8_t* src = t.data + off * 2;
                for (size_t k = 0; k < m; ++k) {
                    uint16_t h;
                    memcpy(&h, src + 2 * k, 2);
                    non_finite += !f16_finite(h);
                    stage[k] = f32_to_bf16_rne(f16_bits_to_f32(h));
                }
            } else {  // F32 -> BF16 / F16
                const uint8_t* src = t.data + off * 4;
                for (size_t k = 0; k < m; ++k) {
                    float f;
                    memcpy(&f, src + 4 * k, 4);
                    const uint16_t h = dst_dtype == KVB_F16 ? f32_to_f16_rne(f) : f32_to_bf16_rne(f);
                    non_finite += dst_dtype == KVB_F16 ? !f16_finite(h) : !bf16_finite(h);
                    stage[k] = h;
                }
            }
            if (non_finite)
                return fail(KVB_ERR_CONFIG,
                            "%s: %zu values are non-finite or outside the %s range", names[i],
                            non_finite, dst_dtype == KVB_F16 ? "FP16" : "BF16");
            cudaError_t e;
            if (on_device) {
                e = cudaMemcpyAsync(ck->dev_stage, stage, m * 2, cudaMemcpyHostToDevice, stream);
                if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: staging copy");
                st = kvb_bf16_to_f16(stream, ck->dev_stage, m, out, m, bad, 1);
                if (st != KVB_OK) return st;
            } else {
                e = cudaMemcpyAsync(out, stage, m * 2, cudaMemcpyHostToDevice, stream);
                if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: copy");
            }
            e = cudaEventRecord(ck->done[slot], stream);
            if (e != cudaSuccess) return kvb::cuda_fail(e, "checkpoint: staging event");
            ck->used[slot] = true;
            out += m * 2;
            slot ^= 1;
        }
    }
    return KVB_OK;
}
