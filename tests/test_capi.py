"""The C-ABI library: it loads without a GPU, exports every function the
header declares, the Python binding knows every one of them, and the argument
checks (reference ensure_shape!, engine/src/error.rs:23-30) reject bad shapes
before anything touches the device."""
import ctypes as C

import numpy as np
import pytest

from kvasir_b200 import _lib as L
from oracle import oracle as O


def test_library_exports_every_header_symbol():
    lib = L.lib()
    declared = L.header_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(L.SIGNATURES) == L.header_symbols()


def _status(fn, *args):
    st = fn(*args)
    msg = L.lib().kvb_last_error().decode()
    return st, msg


def test_shape_errors_are_reported_not_launched():
    """engine/tests/kernels.rs:366-374: a bad length is an error, not a panic."""
    lib = L.lib()
    fake = C.c_void_p(0x1000)  # never dereferenced: the checks fail first
    st, msg = _status(lib.kvb_rmsnorm, None, fake, 10, fake, 10, fake, 10, 2, 4, 1e-5, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "rmsnorm" in msg
    st, msg = _status(lib.kvb_add_inplace, None, fake, 10, fake, 5, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "lengths differ (10 vs 5)" in msg
    st, msg = _status(lib.kvb_linear, fake, None, fake, 10, fake, 10, fake, 10, 2, 4, 3,
                      L.KVB_BF16, 0)
    assert st == L.KVB_ERR_SHAPE and "linear" in msg
    st, msg = _status(lib.kvb_attention, None, fake, 12 * 64, fake, 2 * 16 * 64, fake,
                      2 * 16 * 64, fake, 8 * 64, 1, 20, 8, 2, 64, 16, None, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "max_seq" in msg
    st, msg = _status(lib.kvb_attention, None, fake, 12 * 48, fake, 2 * 16 * 48, fake,
                      2 * 16 * 48, fake, 8 * 48, 1, 0, 8, 2, 48, 16, None, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "divide 128" in msg
    st, msg = _status(lib.kvb_rope_inplace, None, fake, 5 * 768, fake, 32 * 32, fake, 32 * 32, 5,
                      30, 8, 2, 64, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "exceed table" in msg
    st, msg = _status(lib.kvb_kv_append, None, fake, 3 * 512, fake, 2 * 16 * 64, fake, 2 * 16 * 64,
                      3, 14, 4, 2, 64, 16, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "max_seq" in msg
    # prefill rope: 2 sequences x 3 rows need a cache of 2 * 2 * 16 * 64 elements
    st, msg = _status(lib.kvb_rope_kv_append_prefill, None, fake, 2 * 3 * 768, fake, fake, 16 * 32,
                      fake, fake, 2 * 16 * 64, 2, 3, 0, 8, 2, 64, 16, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "cache sizes" in msg
    st, msg = _status(lib.kvb_rope_kv_append_prefill, None, fake, 2 * 3 * 768, fake, fake, 16 * 32,
                      fake, fake, 2 * 2 * 16 * 64, 2, 3, 14, 8, 2, 64, 16, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "exceed" in msg
    # paged cache: the pool must be whole blocks of n_kv * block_size * head_dim
    st, msg = _status(lib.kvb_attention_decode_paged, None, fake, 32 * 64, fake, fake, 3 * 8 * 64 * 64 + 1,
                      fake, 4, 64, fake, 2, 100, 32, 8, 64, 0.125, fake, 32 * 64, None, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "whole number" in msg
    st, msg = _status(lib.kvb_attention_decode_paged, None, fake, 32 * 64, fake, fake, 3 * 8 * 64 * 64,
                      fake, 4, 64, fake, 2, 300, 32, 8, 64, 0.125, fake, 32 * 64, None, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "exceeds" in msg
    st, msg = _status(lib.kvb_attention_decode_paged, None, fake, 32 * 64, fake, fake, 3 * 8 * 32 * 64,
                      fake, 4, 32, fake, 2, 100, 32, 8, 64, 0.125, fake, 32 * 64, None, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_UNSUPPORTED and "multiple of 64" in msg
    st, msg = _status(lib.kvb_rope_kv_append_paged, None, fake, 2, 1, fake, fake, fake, 16 * 32,
                      fake, fake, 5 * 8 * 64 * 64 + 3, fake, 4, 64, 32, 8, 64, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "whole number" in msg
    st, msg = _status(lib.kvb_attention_prefill_paged, None, fake, 2 * 5 * 3072, fake, fake,
                      4 * 8 * 64 * 64, fake, 2, 64, fake, 2 * 5 * 2048, 2, 5, 130, 32, 8, 64,
                      L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "exceed" in msg
    st, msg = _status(lib.kvb_bf16_to_f16, None, fake, 10, fake, 10, fake, 2)
    assert st == L.KVB_ERR_SHAPE and "exactly one u32" in msg
    st, msg = _status(lib.kvb_embedding_gather, None, fake, 5, fake, 301, fake, 5 * 300, 300,
                      L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "multiple of hidden" in msg
    st, msg = _status(lib.kvb_silu_mul, None, fake, 3 * 2000, fake, 3 * 999, 3, 1000, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "silu_mul" in msg
    st, msg = _status(lib.kvb_rmsnorm, None, fake, 8, fake, 4, fake, 8, 2, 4, 1e-5, 7)
    assert st == L.KVB_ERR_SHAPE and "dtype" in msg
    # embedding + norm: w must be one row, x and out t rows, the table whole rows
    st, msg = _status(lib.kvb_embedding_rmsnorm, None, fake, 2, fake, 10 * 256, fake, 255, fake,
                      2 * 256, fake, 2 * 256, 256, 1e-5, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "w has 255" in msg
    st, msg = _status(lib.kvb_embedding_rmsnorm, None, fake, 2, fake, 10 * 256, fake, 256, fake,
                      3 * 256, fake, 2 * 256, 256, 1e-5, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "x has 768" in msg
    st, msg = _status(lib.kvb_embedding_rmsnorm, None, fake, 2, fake, 10 * 256 + 1, fake, 256,
                      fake, 2 * 256, fake, 2 * 256, 256, 1e-5, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "multiple of hidden" in msg
    # argmax: eight CTAs per row, so rows must keep the grid within 2^31 - 1 CTAs
    st, msg = _status(lib.kvb_argmax_f32, None, fake, 1 << 28, 10, fake, None, None)
    assert st == L.KVB_ERR_SHAPE and "rows" in msg


@pytest.mark.parametrize("scaled", [True, False])
def test_rope_table_matches_oracle_bitwise(scaled):
    """kvb_rope_table (product, engine/src/model/rope.rs:3-39) and the oracle's
    restatement evaluate the same f64 formula with the same libm."""
    lib = L.lib()
    max_pos, hd = 2048, 64
    c = np.empty(max_pos * 32, np.float32)
    s = np.empty(max_pos * 32, np.float32)
    st = lib.kvb_rope_table(hd, 500000.0, int(scaled), 32.0, 1.0, 4.0, 8192.0, max_pos,
                            c.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p))
    assert st == L.KVB_OK
    oc, os_ = O.cos_sin_table(hd, max_pos, 500000.0, scaled)
    np.testing.assert_array_equal(c, oc)
    np.testing.assert_array_equal(s, os_)


def test_noalloc_scratch_size_matches_header():
    import re
    with open(L.HEADER) as f:
        m = re.search(r"#define KVB_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", f.read())
    assert m and int(m.group(1)) << int(m.group(2)) == L.KVB_NOALLOC_SCRATCH_BYTES


def test_lm_head_argmax_and_prefill_f32_check_shapes_before_launch():
    lib = L.lib()
    fake = C.c_void_p(0x1000)
    st, msg = _status(lib.kvb_lm_head_argmax, None, fake, 4 * 64 - 1, fake, 100 * 64, 4, 64, 100,
                      fake, 1 << 20, fake, None, None, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "lm_head_argmax: x has" in msg
    st, msg = _status(lib.kvb_lm_head_argmax, None, fake, 4 * 64, fake, 100 * 64, 4, 64, 100,
                      fake, 16, fake, None, None, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "workspace" in msg
    st, msg = _status(lib.kvb_lm_head_argmax, None, fake, 4 * 64, fake, 100 * 64, 4, 64, 100,
                      fake, 1 << 20, None, None, None, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "null ids" in msg
    assert lib.kvb_lm_head_argmax_workspace_bytes(32) >= 32 * 8 * 148
    # one sequence of 2 tokens, 8 / 2 heads, max_seq 16: a cache one element short
    st, msg = _status(lib.kvb_attention_prefill_f32, None, fake, 2 * 768, fake, fake,
                      2 * 16 * 64 - 1, fake, 2 * 8 * 64, 1, 2, 0, 8, 2, 64, 16, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "bad cache sizes" in msg


def test_linear_rows_check_shapes_and_support_before_launch():
    """kvb_linear_rows / kvb_linear_silu_mul: length checks are KVB_ERR_SHAPE, shapes
    the kernel does not take are KVB_ERR_UNSUPPORTED, both before any CUDA call."""
    lib = L.lib()
    fake = C.c_void_p(0x1000)
    st, msg = _status(lib.kvb_linear_rows, None, fake, 4 * 64 - 1, fake, 128 * 64, fake, 4 * 128,
                      4, 64, 128, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "linear_rows: x has" in msg
    st, msg = _status(lib.kvb_linear_rows, None, fake, 4 * 64, fake, 128 * 64, fake, 4 * 128,
                      4, 64, 128, 9, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "splits" in msg
    st, msg = _status(lib.kvb_linear_rows, None, fake, 129 * 64, fake, 128 * 64, fake,
                      129 * 128, 129, 64, 128, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_UNSUPPORTED and "rows <= 128" in msg
    st, msg = _status(lib.kvb_linear_rows, None, fake, 4 * 60, fake, 128 * 60, fake, 4 * 128,
                      4, 60, 128, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_UNSUPPORTED
    st, msg = _status(lib.kvb_linear_silu_mul, None, fake, 4 * 64, fake, 2 * 100 * 64 - 1, fake,
                      4 * 100, 4, 64, 100, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE and "w_gu has" in msg
    st, msg = _status(lib.kvb_linear_silu_mul, None, fake, 4 * 64, fake, 2 * 102 * 64, fake,
                      4 * 102, 4, 64, 102, 0, L.KVB_BF16)
    assert st == L.KVB_ERR_UNSUPPORTED and "multiple of 4" in msg
    # nothing to do: OK without touching the pointers
    assert lib.kvb_linear_rows(None, fake, 0, fake, 128 * 64, fake, 0, 0, 64, 128, 0,
                               L.KVB_BF16) == L.KVB_OK
