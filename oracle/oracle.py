"""ctypes/numpy front end of the CPU oracle (oracle/kvb_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py to check or time the CUDA path; the product
(kvasir_b200) never imports it.

16-bit tensors are numpy uint16 arrays holding bf16 or f16 bit patterns; the
dtype is given as "bf16" or "f16".
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libkvb_oracle.so")
DTYPES = {"bf16": 0, "f16": 1}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def _declare(L):
    L.kvo_to_f32_array.argtypes = [_u16p, _f32p, _sz, C.c_int]
    L.kvo_from_f32_array.argtypes = [_f32p, _u16p, _sz, C.c_int]
    L.kvo_set_threads.argtypes = [C.c_int]
    L.kvo_get_threads.restype = C.c_int
    L.kvo_fill_normal.argtypes = [_u16p, _sz, C.c_double, C.c_double, C.c_uint64, C.c_int]
    L.kvo_embedding_gather.argtypes = [_i32p, _sz, _u16p, _sz, _u16p, _sz]
    L.kvo_rmsnorm.argtypes = [_u16p, _u16p, _f32p, _sz, _sz, C.c_float, C.c_int]
    L.kvo_rope.argtypes = [_u16p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, C.c_int]
    L.kvo_kv_append.argtypes = [_u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _sz, _sz]
    L.kvo_attention.argtypes = [_u16p, _u16p, _u16p, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, C.c_int]
    L.kvo_attention_decode.argtypes = [_u16p, _sz, _u16p, _u16p, _i32p, _sz, _sz, _sz, _sz, _sz,
                                       C.c_double, _f32p, C.c_int]
    L.kvo_silu_mul.argtypes = [_u16p, _f32p, _sz, _sz, C.c_int]
    L.kvo_add.argtypes = [_u16p, _u16p, _u16p, _sz, C.c_int]
    L.kvo_bf16_to_f16.argtypes = [_u16p, _u16p, _sz]
    L.kvo_bf16_to_f16.restype = C.c_uint32
    L.kvo_linear.argtypes = [_u16p, _u16p, _f32p, _sz, _sz, _sz, C.c_int]
    L.kvo_argmax.argtypes = [_f32p, _sz, _sz, _i32p]
    L.kvo_inv_freq.argtypes = [_sz, C.c_double, C.c_int, C.c_double, C.c_double, C.c_double,
                               C.c_double, _f64p]
    L.kvo_cos_sin_table.argtypes = [_sz, C.c_double, C.c_int, C.c_double, C.c_double, C.c_double,
                                    C.c_double, _sz, _f32p, _f32p]
    L.kvo_set_round_dither.argtypes = [C.c_double, C.c_uint64]
    L.kvo_decode_step.argtypes = [C.POINTER(ModelDims), C.POINTER(ModelWeights), _f32p, _f32p,
                                  _u16p, _u16p, _i32p, _i32p, _sz, _f32p, _i32p, C.c_int]


class ModelDims(C.Structure):
    _fields_ = [("hidden", _sz), ("inter", _sz), ("n_layers", _sz), ("n_q", _sz), ("n_kv", _sz),
                ("head_dim", _sz), ("vocab", _sz), ("max_seq", _sz), ("eps", C.c_float)]


class ModelWeights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p),
                ("attn_norm", C.POINTER(C.c_void_p)), ("w_qkv", C.POINTER(C.c_void_p)),
                ("w_o", C.POINTER(C.c_void_p)), ("mlp_norm", C.POINTER(C.c_void_p)),
                ("w_gu", C.POINTER(C.c_void_p)), ("w_down", C.POINTER(C.c_void_p))]


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------- conversions
def to_f32(bits: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    bits = _c(bits, np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().kvo_to_f32_array(bits.ravel(), out.ravel(), bits.size, DTYPES[dtype])
    return out


def from_f32(x: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().kvo_from_f32_array(x.ravel(), out.ravel(), x.size, DTYPES[dtype])
    return out


def set_threads(n: int) -> None:
    lib().kvo_set_threads(int(n))


def get_threads() -> int:
    return int(lib().kvo_get_threads())


def fill_normal(n: int, mean: float, std: float, seed: int, dtype: str = "bf16") -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().kvo_fill_normal(out, n, mean, std, seed, DTYPES[dtype])
    return out


def uniform16(rng: np.random.Generator, n: int, amp: float, dtype: str = "bf16") -> np.ndarray:
    """Uniform(-amp, amp) rounded to 16 bits, like the reference's rand_f16
    (engine/tests/kernels.rs:9-11)."""
    return from_f32(rng.uniform(-amp, amp, n).astype(np.float32), dtype)


# ---------------------------------------------------------------- kernels
def embedding_gather(ids, table, hidden):
    ids = _c(ids, np.int32)
    table = _c(table, np.uint16)
    out = np.empty(ids.size * hidden, np.uint16)
    lib().kvo_embedding_gather(ids, ids.size, table.ravel(), table.size // hidden, out, hidden)
    return out


def rmsnorm(x, w, rows, hidden, eps, dtype="bf16"):
    out = np.empty(rows * hidden, np.float32)
    lib().kvo_rmsnorm(_c(x, np.uint16).ravel(), _c(w, np.uint16).ravel(), out, rows, hidden,
                      eps, DTYPES[dtype])
    return out


def rope(qkv, cos, sin, t, pos0, n_q, n_kv, hd, dtype="bf16"):
    qkv = _c(qkv, np.uint16).ravel()
    out = np.empty(qkv.size, np.float32)
    lib().kvo_rope(qkv, _c(cos, np.float32).ravel(), _c(sin, np.float32).ravel(), out, t, pos0,
                   n_q, n_kv, hd, DTYPES[dtype])
    return out


def kv_append(qkv, kc, vc, t, pos0, n_q, n_kv, hd, max_seq):
    """Returns new (kc, vc) arrays; inputs are not modified."""
    kc = _c(kc, np.uint16).ravel().copy()
    vc = _c(vc, np.uint16).ravel().copy()
    lib().kvo_kv_append(_c(qkv, np.uint16).ravel(), kc, vc, t, pos0, n_q, n_kv, hd, max_seq)
    return kc, vc


def attention(qkv, kc, vc, t, pos0, n_q, n_kv, hd, max_seq, dtype="bf16"):
    out = np.empty(t * n_q * hd, np.float32)
    lib().kvo_attention(_c(qkv, np.uint16).ravel(), _c(kc, np.uint16).ravel(),
                        _c(vc, np.uint16).ravel(), out, t, pos0, n_q, n_kv, hd, max_seq,
                        DTYPES[dtype])
    return out


def attention_decode(q, q_row_stride, kc, vc, lens, n_q, n_kv, hd, max_seq, scale,
                     dtype="bf16"):
    lens = _c(lens, np.int32)
    n_seq = lens.size
    out = np.empty(n_seq * n_q * hd, np.float32)
    lib().kvo_attention_decode(_c(q, np.uint16).ravel(), q_row_stride, _c(kc, np.uint16).ravel(),
                               _c(vc, np.uint16).ravel(), lens, n_seq, n_q, n_kv, hd, max_seq,
                               scale, out, DTYPES[dtype])
    return out


def silu_mul(gu, t, inter, dtype="bf16"):
    out = np.empty(t * inter, np.float32)
    lib().kvo_silu_mul(_c(gu, np.uint16).ravel(), out, t, inter, DTYPES[dtype])
    return out


def add(x, y, dtype="bf16"):
    x = _c(x, np.uint16).ravel()
    out = np.empty(x.size, np.uint16)
    lib().kvo_add(x, _c(y, np.uint16).ravel(), out, x.size, DTYPES[dtype])
    return out


def bf16_to_f16(src):
    src = _c(src, np.uint16).ravel()
    dst = np.empty(src.size, np.uint16)
    bad = lib().kvo_bf16_to_f16(src, dst, src.size)
    return dst, int(bad)


def linear(x, w, t, in_dim, out_dim, dtype="bf16"):
    y = np.empty(t * out_dim, np.float32)
    lib().kvo_linear(_c(x, np.uint16).ravel(), _c(w, np.uint16).ravel(), y, t, in_dim, out_dim,
                     DTYPES[dtype])
    return y


def argmax(logits, rows, vocab):
    out = np.empty(rows, np.int32)
    lib().kvo_argmax(_c(logits, np.float32).ravel(), rows, vocab, out)
    return out


_M64 = (1 << 64) - 1


def splitmix64(z: int) -> int:
    """SplitMix64 (Steele, Lea, Flood, OOPSLA 2014) on Python integers mod 2^64."""
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def sample_uniform(seed: int, row: int, counter: int) -> float:
    """24 random bits in [0, 1): the draw of kvb_sample_f32 for (seed, row, counter)."""
    z = splitmix64((seed + splitmix64(((counter & 0xFFFFFFFF) << 32) | row)) & _M64)
    return (z >> 40) / 16777216.0


def order_keys(l32: np.ndarray) -> np.ndarray:
    """The sampler's unsigned order of f32 values (monotone; -0.0 below +0.0)."""
    b = np.ascontiguousarray(l32, np.float32).view(np.uint32)
    return np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)


def sample(logits, temperature, top_p, seed, counters=None, target_scale=1.0, u_shift=0):
    """Restatement of kvb_sample_f32 (temperature > 0): per row the integer weights
    w = floor(2^32 * f32(exp((l - max) * (1/temperature)))) (difference and scaling
    in f32, as the kernel), the nucleus threshold K* over the order keys (ties
    kept), u24 from sample_uniform and the first index, in vocabulary order, whose
    running kept weight exceeds floor(u24 * kept / 2^24).  Sums are exact Python
    integers.  target_scale / u_shift (in units of 2^-24) perturb the nucleus
    target and the draw, so a test can tell a boundary case decided by the
    device's expf from an error.  The planned host sampler this stands for is in
    kvasir DESIGN.md:24,109."""
    logits = np.asarray(logits, np.float32)
    rows = logits.shape[0]
    inv = np.float32(1.0) / np.float32(temperature)
    out = np.zeros(rows, np.int32)
    for r in range(rows):
        l = logits[r]
        valid = l > -np.inf  # False for NaN
        if not valid.any():
            continue
        m = l[valid].max()
        if m == np.inf:  # the first +inf, as the argmax
            out[r] = int(np.nonzero(l == np.inf)[0][0])
            continue
        d = ((l - m).astype(np.float32) * inv).astype(np.float32)
        w32 = np.exp(d.astype(np.float64)).astype(np.float32)
        w = np.where(valid, np.floor(w32.astype(np.float64) * 2.0 ** 32), 0.0).astype(np.uint64)
        keys = order_keys(l)
        total = int(w.sum(dtype=np.uint64))
        if top_p < 1.0:
            target = int(np.ceil(float(np.float32(top_p)) * float(total) * target_scale))
            pos = w > 0
            uk, inv_idx = np.unique(keys[pos], return_inverse=True)  # ascending keys
            mass = np.zeros(uk.size, dtype=object)
            np.add.at(mass, inv_idx, w[pos].astype(object))
            cum = np.cumsum(mass[::-1])  # mass at or above each key, highest first
            hit = np.nonzero(cum >= target)[0]
            kstar = uk[::-1][hit[0]] if hit.size else uk[0]
            kept = keys >= kstar
        else:
            kept = np.ones_like(valid)
        wk = np.where(kept, w, np.uint64(0))
        kept_total = int(wk.sum(dtype=np.uint64))
        u = int(sample_uniform(seed, r, 0 if counters is None else int(counters[r])) * 16777216)
        u = min(max(u + u_shift, 0), (1 << 24) - 1)
        t = (kept_total * u) >> 24
        c = np.cumsum(wk.astype(object))
        idx = np.nonzero((c > t) & (wk > 0))[0]
        out[r] = idx[0] if idx.size else np.nonzero(wk > 0)[0][-1]
    return out


LLAMA3_ROPE = dict(theta=500000.0, scaled=True, factor=32.0, low=1.0, high=4.0, orig=8192.0)


def inv_freq(hd, theta, scaled, factor=32.0, low=1.0, high=4.0, orig=8192.0):
    out = np.empty(hd // 2, np.float64)
    lib().kvo_inv_freq(hd, theta, int(scaled), factor, low, high, orig, out)
    return out


def cos_sin_table(hd, max_pos, theta, scaled, factor=32.0, low=1.0, high=4.0, orig=8192.0):
    c = np.empty(max_pos * (hd // 2), np.float32)
    s = np.empty(max_pos * (hd // 2), np.float32)
    lib().kvo_cos_sin_table(hd, theta, int(scaled), factor, low, high, orig, max_pos, c, s)
    return c, s


def set_round_dither(rel: float, seed: int = 0) -> None:
    """Rounding dither of decode_step (kvo_set_round_dither); rel = 0 turns it off."""
    lib().kvo_set_round_dither(float(rel), int(seed) & 0xFFFFFFFFFFFFFFFF)


def decode_step(dims: dict, weights: dict, cos, sin, kc, vc, ids, pos, dtype="bf16"):
    """One decode step of the composed chain.  `weights` holds 'embed',
    'final_norm' and per-layer lists 'attn_norm', 'w_qkv', 'w_o', 'mlp_norm',
    'w_gu', 'w_down' (uint16 arrays).  kc/vc ([seq][layer][n_kv][max_seq][hd])
    are updated in place.  Returns (logits [n_seq, vocab] f32, ids [n_seq])."""
    d = ModelDims(**dims)
    keep = []

    def arr(lst):
        ptrs = (C.c_void_p * len(lst))()
        for i, a in enumerate(lst):
            a = _c(a, np.uint16)
            keep.append(a)
            ptrs[i] = a.ctypes.data
        keep.append(ptrs)
        return ptrs

    emb = _c(weights["embed"], np.uint16)
    fn = _c(weights["final_norm"], np.uint16)
    W = ModelWeights(emb.ctypes.data, fn.ctypes.data, arr(weights["attn_norm"]),
                     arr(weights["w_qkv"]), arr(weights["w_o"]), arr(weights["mlp_norm"]),
                     arr(weights["w_gu"]), arr(weights["w_down"]))
    ids = _c(ids, np.int32)
    pos = _c(pos, np.int32)
    n_seq = ids.size
    logits = np.empty(n_seq * dims["vocab"], np.float32)
    ids_out = np.empty(n_seq, np.int32)
    assert kc.dtype == np.uint16 and kc.flags.c_contiguous
    assert vc.dtype == np.uint16 and vc.flags.c_contiguous
    lib().kvo_decode_step(C.byref(d), C.byref(W), _c(cos, np.float32).ravel(),
                          _c(sin, np.float32).ravel(), kc.reshape(-1), vc.reshape(-1), ids, pos,
                          n_seq, logits, ids_out, DTYPES[dtype])
    return logits.reshape(n_seq, dims["vocab"]), ids_out


def ulp16(x: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    """Spacing of the 16-bit format at |x| (for values in the normal range;
    subnormal spacing below)."""
    mant = 7 if dtype == "bf16" else 10
    min_exp = -126 if dtype == "bf16" else -14
    ax = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0 ** min_exp)))
    return 2.0 ** (e - mant)
