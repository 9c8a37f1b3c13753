"""Parity of the elementwise / norm / RoPE / KV-append / GEMM kernels against
the CPU oracle, through the C ABI (kvasir_b200.Gpu -> libkvasir_b200.so).

Bars: bit-exact for embedding, KV append, add, bf16->f16 and argmax; within
1 ulp of the 16-bit format for RMSNorm and SiLU*mul against the f64 oracle;
RoPE bit-exact against the oracle's f32 evaluation rounded once.  Shapes: the
reference's own test shapes (engine/tests/kernels.rs) and BASELINE shapes."""
import numpy as np
import pytest
import torch

from gpu_util import assert_close, assert_within_ulp, dev, host_bits, host_f32, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = ["bf16", "f16"]


@pytest.fixture(scope="module")
def g():
    from kvasir_b200 import Gpu
    return Gpu(0)


# ------------------------------------------------------------------ embedding
@pytest.mark.parametrize("vocab,hidden,ids", [
    (50, 300, [7, 0, 49, 7, 23]),                          # reference shape (scalar path)
    (128256, 2048, [5]),                                    # batch-1 decode
    (128256, 2048, list(range(0, 128256, 4009))),           # 32 rows
])
def test_embedding_gather_is_exact(g, vocab, hidden, ids):
    rng = np.random.default_rng(1)
    table = normal16(rng, vocab * hidden, 0, 0.02)
    ids = np.array(ids, np.int32)
    out = torch.empty(len(ids) * hidden, dtype=torch.bfloat16, device="cuda")
    g.embedding_gather(torch.from_numpy(ids).cuda(), dev(table), out, hidden)
    np.testing.assert_array_equal(host_bits(out), O.embedding_gather(ids, table, hidden))


def test_embedding_out_of_range_ids_give_zero_rows(g):
    rng = np.random.default_rng(2)
    table = normal16(rng, 1000 * 64)
    ids = np.array([-1, 3, 1000, 999], np.int32)
    out = torch.full((4 * 64,), 7.0, dtype=torch.bfloat16, device="cuda")
    g.embedding_gather(torch.from_numpy(ids).cuda(), dev(table), out, 64)
    np.testing.assert_array_equal(host_bits(out), O.embedding_gather(ids, table, 64))


def test_embedding_prefill_rows(g):
    rng = np.random.default_rng(3)
    vocab, hidden, t = 128256, 2048, 8192
    table = normal16(rng, vocab * hidden, 0, 0.02)
    ids = rng.integers(0, vocab, t).astype(np.int32)
    out = torch.empty(t * hidden, dtype=torch.bfloat16, device="cuda")
    g.embedding_gather(torch.from_numpy(ids).cuda(), dev(table), out, hidden)
    np.testing.assert_array_equal(host_bits(out), O.embedding_gather(ids, table, hidden))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("vocab,hidden,ids", [
    (128256, 2048, [5]),                                    # batch-1 decode: one launch
    (128256, 2048, list(range(0, 128256, 4009))),           # 32 rows
    (1000, 256, [-1, 3, 1000, 999]),                        # ids outside the table: zero rows
    (300, 4096, [7, 0, 299]),                               # 512 chunks, the widest fused row
    (300, 4104, [7, 0, 299]),                               # wider: the two kernels
    (50, 300, [7, 0, 49]),                                  # odd width: the two kernels
    (40, 256, list(range(40)) * 16),                        # 640 rows: the two kernels
])
def test_embedding_rmsnorm_equals_gather_then_rmsnorm(g, dtype, vocab, hidden, ids):
    rng = np.random.default_rng(hidden + len(ids))
    table = O.uniform16(rng, vocab * hidden, 1.0, dtype)
    w = O.uniform16(rng, hidden, 1.5, dtype)
    ids = np.array(ids, np.int32)
    d_ids, d_table, d_w = torch.from_numpy(ids).cuda(), dev(table, dtype), dev(w, dtype)
    tdt = d_table.dtype
    n = len(ids) * hidden
    x_a, out_a = torch.full((n,), 3.0, dtype=tdt, device="cuda"), torch.empty(n, dtype=tdt, device="cuda")
    g.embedding_rmsnorm(d_ids, d_table, d_w, x_a, out_a, hidden, 1e-5)
    x_b, out_b = torch.empty(n, dtype=tdt, device="cuda"), torch.empty(n, dtype=tdt, device="cuda")
    g.embedding_gather(d_ids, d_table, x_b, hidden)
    g.rmsnorm(x_b, d_w, out_b, len(ids), hidden, 1e-5)
    np.testing.assert_array_equal(host_bits(x_a), O.embedding_gather(ids, table, hidden))
    np.testing.assert_array_equal(host_bits(x_a), host_bits(x_b))
    np.testing.assert_array_equal(host_bits(out_a), host_bits(out_b))


# ------------------------------------------------------------------ rmsnorm
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,hidden", [(5, 2048), (3, 100), (1, 2048), (7, 4096), (2, 8),
                                         (1000, 2048), (700, 4096), (2000, 512), (1500, 1032),
                                         (601, 256), (3, 136)])
def test_rmsnorm_within_one_ulp(g, dtype, rows, hidden):
    """reference shapes engine/tests/kernels.rs:50-82 (x ±3, w ±1.5), plus row counts
    above 4 per SM and widths of 1 … 16 chunks per lane, ragged ones included, for the
    persistent bulk-copy kernel (rows split unevenly over the CTAs)"""
    rng = np.random.default_rng(2)
    x = O.uniform16(rng, rows * hidden, 3.0, dtype)
    w = O.uniform16(rng, hidden, 1.5, dtype)
    out = torch.empty(rows * hidden, dtype=dev(x, dtype).dtype, device="cuda")
    g.rmsnorm(dev(x, dtype), dev(w, dtype), out, rows, hidden, 1e-5)
    want = O.rmsnorm(x, w, rows, hidden, 1e-5, dtype)
    assert_within_ulp(host_bits(out), want, dtype, name="rmsnorm")
    if dtype == "f16":  # the reference's own tolerance
        assert_close(host_f32(out, dtype), want, 1.5e-3, 1e-3, "rmsnorm")


def test_rmsnorm_prefill_shape(g):
    """BASELINE prefill: [8192, 2048] N(0,1), w = 1 + 0.02 N(0,1)"""
    rng = np.random.default_rng(4)
    rows, hidden = 8192, 2048
    x = normal16(rng, rows * hidden)
    w = normal16(rng, hidden, 1.0, 0.02)
    out = torch.empty(rows * hidden, dtype=torch.bfloat16, device="cuda")
    g.rmsnorm(dev(x), dev(w), out, rows, hidden, 1e-5)
    assert_within_ulp(host_bits(out), O.rmsnorm(x, w, rows, hidden, 1e-5), name="rmsnorm")


@pytest.mark.parametrize("rows,hidden", [(4, 2048), (3, 100), (1000, 2048), (700, 4096),
                                         (650, 520), (5, 16)])
def test_add_rmsnorm_equals_add_then_rmsnorm(g, rows, hidden):
    rng = np.random.default_rng(5)
    x, y = normal16(rng, rows * hidden), normal16(rng, rows * hidden)
    w = normal16(rng, hidden, 1.0, 0.02)
    xa, out_a = dev(x), torch.empty(rows * hidden, dtype=torch.bfloat16, device="cuda")
    g.add_rmsnorm(xa, dev(y), dev(w), out_a, rows, hidden, 1e-5)
    xb, out_b = dev(x), torch.empty_like(out_a)
    g.add_inplace(xb, dev(y))
    g.rmsnorm(xb, dev(w), out_b, rows, hidden, 1e-5)
    np.testing.assert_array_equal(host_bits(xa), host_bits(xb))
    np.testing.assert_array_equal(host_bits(out_a), host_bits(out_b))
    np.testing.assert_array_equal(host_bits(xa), O.add(x, y))


# ------------------------------------------------------------------ add / convert
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [10007, 8192 * 2048])
def test_add_inplace_is_exact(g, dtype, n):
    """engine/tests/kernels.rs:162-175 (n = 10007 takes the scalar path)"""
    rng = np.random.default_rng(5)
    x, y = O.uniform16(rng, n, 10.0, dtype), O.uniform16(rng, n, 10.0, dtype)
    dx = dev(x, dtype)
    g.add_inplace(dx, dev(y, dtype))
    np.testing.assert_array_equal(host_bits(dx), O.add(x, y, dtype))


def test_bf16_to_f16_converts_and_counts_overflow(g):
    """engine/tests/kernels.rs:177-194"""
    rng = np.random.default_rng(6)
    src = O.from_f32(rng.uniform(-4, 4, 5000).astype(np.float32), "bf16")
    src[10] = O.from_f32(np.array([1.0e6], np.float32), "bf16")[0]
    src[20] = O.from_f32(np.array([-7.0e4], np.float32), "bf16")[0]
    dst = torch.empty(5000, dtype=torch.float16, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.bf16_to_f16(dev(src), dst, bad)
    want, nbad = O.bf16_to_f16(src)
    assert int(bad.item()) == nbad == 2
    np.testing.assert_array_equal(host_bits(dst), want)


# ------------------------------------------------------------------ silu_mul
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("t,inter", [(3, 1000), (1, 8192), (5, 12)])
def test_silu_mul_within_one_ulp(g, dtype, t, inter):
    """engine/tests/kernels.rs:140-160 (±6)"""
    rng = np.random.default_rng(4)
    gu = O.uniform16(rng, t * 2 * inter, 6.0, dtype)
    out = torch.empty(t * inter, dtype=dev(gu, dtype).dtype, device="cuda")
    g.silu_mul(dev(gu, dtype), out, t, inter)
    want = O.silu_mul(gu, t, inter, dtype)
    assert_within_ulp(host_bits(out), want, dtype, name="silu_mul")
    if dtype == "f16":
        assert_close(host_f32(out, dtype), want, 2e-3, 1e-3, "silu_mul")


def test_silu_mul_prefill_shape(g):
    """BASELINE prefill: gate/up [8192, 8192] each, N(0,1)"""
    rng = np.random.default_rng(8)
    t, inter = 8192, 8192
    gu = normal16(rng, t * 2 * inter)
    out = torch.empty(t * inter, dtype=torch.bfloat16, device="cuda")
    g.silu_mul(dev(gu), out, t, inter)
    O.set_threads(8)
    want = O.silu_mul(gu, t, inter)
    O.set_threads(1)
    assert_within_ulp(host_bits(out), want, name="silu_mul")


# ------------------------------------------------------------------ rope / kv append
def _theta1e4_table(max_pos, hd):
    return O.cos_sin_table(hd, max_pos, 10000.0, False)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rope_matches_reference_test_and_leaves_v(g, dtype):
    """engine/tests/kernels.rs:98-138: n_q 8, n_kv 2, hd 64, T 5, pos0 3, theta 1e4"""
    rng = np.random.default_rng(3)
    n_q, n_kv, hd, t, pos0 = 8, 2, 64, 5, 3
    stride = (n_q + 2 * n_kv) * hd
    qkv = O.uniform16(rng, t * stride, 2.0, dtype)
    cos, sin = _theta1e4_table(32, hd)
    d = dev(qkv, dtype)
    g.rope_inplace(d, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), t, pos0, n_q,
                   n_kv, hd)
    want = O.rope(qkv, cos, sin, t, pos0, n_q, n_kv, hd, dtype)
    np.testing.assert_array_equal(host_bits(d), O.from_f32(want, dtype))
    got = host_bits(d).reshape(t, stride)
    np.testing.assert_array_equal(got[:, (n_q + n_kv) * hd:], qkv.reshape(t, stride)[:, (n_q + n_kv) * hd:])
    if dtype == "f16":
        assert_close(O.to_f32(got, dtype), want, 1e-3, 1e-3, "rope")


def test_rope_scalar_path_odd_head_dim(g):
    rng = np.random.default_rng(13)
    n_q, n_kv, hd, t, pos0 = 3, 1, 10, 4, 2
    stride = (n_q + 2 * n_kv) * hd
    qkv = O.uniform16(rng, t * stride, 2.0)
    cos, sin = _theta1e4_table(16, hd)
    d = dev(qkv)
    g.rope_inplace(d, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), t, pos0, n_q,
                   n_kv, hd)
    np.testing.assert_array_equal(host_bits(d),
                                  O.from_f32(O.rope(qkv, cos, sin, t, pos0, n_q, n_kv, hd)))


def test_rope_llama3_prefill_shape(g):
    """BASELINE prefill: qkv [2048, 3072] N(0,1), llama3 table, positions 0..2047"""
    rng = np.random.default_rng(9)
    n_q, n_kv, hd, t = 32, 8, 64, 2048
    qkv = normal16(rng, t * 3072)
    cos, sin = O.cos_sin_table(hd, t, **O.LLAMA3_ROPE)
    d = dev(qkv)
    g.rope_inplace(d, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), t, 0, n_q, n_kv,
                   hd)
    np.testing.assert_array_equal(host_bits(d), O.from_f32(O.rope(qkv, cos, sin, t, 0, n_q, n_kv, hd)))


def test_kv_append_places_k_and_v(g):
    """engine/tests/kernels.rs:196-234 (untouched slots stay zero)"""
    rng = np.random.default_rng(7)
    n_q, n_kv, hd, t, pos0, max_seq = 4, 2, 64, 3, 5, 16
    qkv = O.uniform16(rng, t * (n_q + 2 * n_kv) * hd, 2.0)
    kc = torch.zeros(n_kv * max_seq * hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    g.kv_append(dev(qkv), kc, vc, t, pos0, n_q, n_kv, hd, max_seq)
    z = np.zeros(n_kv * max_seq * hd, np.uint16)
    wk, wv = O.kv_append(qkv, z, z, t, pos0, n_q, n_kv, hd, max_seq)
    np.testing.assert_array_equal(host_bits(kc), wk)
    np.testing.assert_array_equal(host_bits(vc), wv)


def test_kv_append_odd_head_dim(g):
    rng = np.random.default_rng(17)
    n_q, n_kv, hd, t, pos0, max_seq = 2, 1, 7, 3, 1, 8
    qkv = O.uniform16(rng, t * (n_q + 2 * n_kv) * hd, 2.0)
    kc = torch.zeros(n_kv * max_seq * hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    g.kv_append(dev(qkv), kc, vc, t, pos0, n_q, n_kv, hd, max_seq)
    z = np.zeros(n_kv * max_seq * hd, np.uint16)
    wk, wv = O.kv_append(qkv, z, z, t, pos0, n_q, n_kv, hd, max_seq)
    np.testing.assert_array_equal(host_bits(kc), wk)
    np.testing.assert_array_equal(host_bits(vc), wv)


@pytest.mark.parametrize("t,pos0,max_seq", [(5, 3, 16), (2048, 0, 2048), (1, 512, 1024)])
def test_rope_kv_append_equals_rope_then_append(g, t, pos0, max_seq):
    rng = np.random.default_rng(10)
    n_q, n_kv, hd = 32, 8, 64
    qkv = normal16(rng, t * 3072)
    cos, sin = O.cos_sin_table(hd, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    a = dev(qkv)
    kc_a = torch.zeros(n_kv * max_seq * hd, dtype=torch.bfloat16, device="cuda")
    vc_a = torch.zeros_like(kc_a)
    g.rope_kv_append(a, c, s, kc_a, vc_a, t, pos0, n_q, n_kv, hd, max_seq)
    b = dev(qkv)
    kc_b, vc_b = torch.zeros_like(kc_a), torch.zeros_like(kc_a)
    g.rope_inplace(b, c, s, t, pos0, n_q, n_kv, hd)
    g.kv_append(b, kc_b, vc_b, t, pos0, n_q, n_kv, hd, max_seq)
    np.testing.assert_array_equal(host_bits(a), host_bits(b))
    np.testing.assert_array_equal(host_bits(kc_a), host_bits(kc_b))
    np.testing.assert_array_equal(host_bits(vc_a), host_bits(vc_b))
    rot = O.from_f32(O.rope(qkv, cos, sin, t, pos0, n_q, n_kv, hd))
    z = np.zeros(n_kv * max_seq * hd, np.uint16)
    wk, wv = O.kv_append(rot, z, z, t, pos0, n_q, n_kv, hd, max_seq)
    np.testing.assert_array_equal(host_bits(kc_a), wk)
    np.testing.assert_array_equal(host_bits(vc_a), wv)


def test_rope_kv_append_batched_per_sequence_positions(g):
    rng = np.random.default_rng(11)
    n_q, n_kv, hd, max_seq, n_seq = 32, 8, 64, 96, 5
    pos = np.array([0, 17, 63, 64, 95], np.int32)
    qkv = normal16(rng, n_seq * 3072)
    cos, sin = O.cos_sin_table(hd, max_seq, **O.LLAMA3_ROPE)
    per = n_kv * max_seq * hd
    kc = torch.zeros(n_seq * per, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    d = dev(qkv)
    g.rope_kv_append_batched(d, torch.from_numpy(pos).cuda(), torch.from_numpy(cos).cuda(),
                             torch.from_numpy(sin).cuda(), kc, vc, per, n_q, n_kv, hd, max_seq)
    assert g.device_error() == 0
    got_q, got_k, got_v = host_bits(d).reshape(n_seq, -1), host_bits(kc).reshape(n_seq, -1), \
        host_bits(vc).reshape(n_seq, -1)
    z = np.zeros(per, np.uint16)
    for b in range(n_seq):
        row = qkv.reshape(n_seq, -1)[b]
        rot = O.from_f32(O.rope(row, cos, sin, 1, int(pos[b]), n_q, n_kv, hd))
        np.testing.assert_array_equal(got_q[b], rot)
        wk, wv = O.kv_append(rot, z, z, 1, int(pos[b]), n_q, n_kv, hd, max_seq)
        np.testing.assert_array_equal(got_k[b], wk)
        np.testing.assert_array_equal(got_v[b], wv)


@pytest.mark.parametrize("n_seq,t,pos0,max_seq", [(3, 5, 2, 16), (4, 300, 0, 320), (2, 1, 7, 8)])
def test_rope_kv_append_prefill_equals_per_sequence(g, n_seq, t, pos0, max_seq):
    """One launch over n_seq sequences == kvb_rope_kv_append on each in turn == oracle."""
    rng = np.random.default_rng(21)
    n_q, n_kv, hd = 32, 8, 64
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, n_seq * t * stride)
    cos, sin = O.cos_sin_table(hd, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    per = n_kv * max_seq * hd
    a = dev(qkv)
    kc_a = torch.zeros(n_seq * per, dtype=torch.bfloat16, device="cuda")
    vc_a = torch.zeros_like(kc_a)
    g.rope_kv_append_prefill(a, c, s, kc_a, vc_a, n_seq, t, pos0, n_q, n_kv, hd, max_seq)
    assert g.device_error() == 0
    b = dev(qkv)
    kc_b, vc_b = torch.zeros_like(kc_a), torch.zeros_like(kc_a)
    for i in range(n_seq):
        g.rope_kv_append(b[i * t * stride:(i + 1) * t * stride], c, s, kc_b[i * per:(i + 1) * per],
                         vc_b[i * per:(i + 1) * per], t, pos0, n_q, n_kv, hd, max_seq)
    np.testing.assert_array_equal(host_bits(a), host_bits(b))
    np.testing.assert_array_equal(host_bits(kc_a), host_bits(kc_b))
    np.testing.assert_array_equal(host_bits(vc_a), host_bits(vc_b))
    z = np.zeros(per, np.uint16)
    for i in range(n_seq):
        rows = qkv[i * t * stride:(i + 1) * t * stride]
        rot = O.from_f32(O.rope(rows, cos, sin, t, pos0, n_q, n_kv, hd))
        np.testing.assert_array_equal(host_bits(a)[i * t * stride:(i + 1) * t * stride], rot)
        wk, wv = O.kv_append(rot, z, z, t, pos0, n_q, n_kv, hd, max_seq)
        np.testing.assert_array_equal(host_bits(kc_a)[i * per:(i + 1) * per], wk)
        np.testing.assert_array_equal(host_bits(vc_a)[i * per:(i + 1) * per], wv)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n_q,n_kv", [(16, 4), (32, 8), (64, 8)])
def test_rope_kv_append_prefill_head_dim_128(g, dtype, n_q, n_kv):
    """hd 128 (eight 8-pair chunks per head), 3 x 500 rows: the persistent bulk-copy
    kernel's wide-head form, in both 16-bit formats; rows of 6, 12 and 20 KB take
    16, 8 and 4 rows per ring stage."""
    rng = np.random.default_rng(23)
    hd, n_seq, t, pos0, max_seq = 128, 3, 500, 6, 512
    stride = (n_q + 2 * n_kv) * hd
    qkv = O.uniform16(rng, n_seq * t * stride, 2.0, dtype)
    cos, sin = O.cos_sin_table(hd, max_seq, **O.LLAMA3_ROPE)
    per = n_kv * max_seq * hd
    a = dev(qkv, dtype)
    kc = torch.zeros(n_seq * per, dtype=a.dtype, device="cuda")
    vc = torch.zeros_like(kc)
    g.rope_kv_append_prefill(a, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), kc, vc,
                             n_seq, t, pos0, n_q, n_kv, hd, max_seq)
    assert g.device_error() == 0
    z = np.zeros(per, np.uint16)
    for i in range(n_seq):
        rows = qkv[i * t * stride:(i + 1) * t * stride]
        rot = O.from_f32(O.rope(rows, cos, sin, t, pos0, n_q, n_kv, hd, dtype), dtype)
        np.testing.assert_array_equal(host_bits(a)[i * t * stride:(i + 1) * t * stride], rot)
        wk, wv = O.kv_append(rot, z, z, t, pos0, n_q, n_kv, hd, max_seq)
        np.testing.assert_array_equal(host_bits(kc)[i * per:(i + 1) * per], wk)
        np.testing.assert_array_equal(host_bits(vc)[i * per:(i + 1) * per], wv)


def test_rope_batched_rejects_position_outside_cache(g):
    """A position beyond the cache is skipped and flagged, never written."""
    n_q, n_kv, hd, max_seq = 4, 2, 64, 8
    per = n_kv * max_seq * hd
    kc = torch.zeros(2 * per, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    qkv = torch.ones(2 * (n_q + 2 * n_kv) * hd, dtype=torch.bfloat16, device="cuda")
    cos, sin = O.cos_sin_table(hd, max_seq, 10000.0, False)
    pos = torch.tensor([3, 8], dtype=torch.int32, device="cuda")
    g.device_error()  # clear
    g.rope_kv_append_batched(qkv, pos, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(),
                             kc, vc, per, n_q, n_kv, hd, max_seq)
    assert g.device_error() & 4
    assert not host_bits(kc)[per:].any()


# ------------------------------------------------------------------ argmax
def test_argmax_matches_oracle(g):
    rng = np.random.default_rng(12)
    rows, vocab = 33, 128256
    logits = rng.normal(0, 3, (rows, vocab)).astype(np.float32)
    logits[1, 100] = logits[1, 200] = 99.0          # tie: first index wins
    logits[2, :] = np.nan
    logits[2, 77] = 5.0                             # NaN never wins
    logits[3, :] = -np.inf                          # all -inf -> 0
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    g.argmax(torch.from_numpy(logits).cuda(), rows, vocab, ids)
    np.testing.assert_array_equal(ids.cpu().numpy(), O.argmax(logits, rows, vocab))


@pytest.mark.parametrize("vocab,offset", [(1, 0), (5, 0), (8, 0), (9, 0), (4003, 0),
                                          (128256, 0), (128256, 1), (128257, 0), (300001, 0)])
def test_argmax_slices_and_ties(g, vocab, offset):
    """Each row is scanned by several CTAs, one slice each: ties and maxima placed on
    and across slice boundaries, the scalar path (odd vocab, unaligned rows)."""
    rng = np.random.default_rng(vocab + offset)
    rows = 6
    logits = rng.normal(0, 3, (rows, vocab)).astype(np.float32)
    logits[0, -1] = 50.0                             # maximum in the last slice
    logits[1, vocab // 2:] = 60.0                    # tie spanning the later slices
    logits[2, :] = -np.inf
    logits[2, -1] = -1e30                            # the only finite value, at the end
    logits[3, ::2] = np.nan                          # NaN never wins
    logits[4, :] = 7.0                               # all equal: index 0
    logits[5, :] = -np.inf
    logits[5, 0] = np.nan                            # only NaN and -inf: index 0
    flat = torch.zeros(rows * vocab + offset, dtype=torch.float32, device="cuda")
    view = flat[offset:]
    view.copy_(torch.from_numpy(logits.ravel()).cuda())
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    g.argmax(view, rows, vocab, ids)
    want = O.argmax(logits, rows, vocab)
    np.testing.assert_array_equal(ids.cpu().numpy(), want)
    # argmax is one launch: repeated calls give the same ids
    g.argmax(view, rows, vocab, ids)
    np.testing.assert_array_equal(ids.cpu().numpy(), want)


def test_argmax_advances_counters(g):
    logits = torch.zeros(4, 10, device="cuda")
    ids = torch.empty(4, dtype=torch.int32, device="cuda")
    a = torch.tensor([1, 2, 3, 4], dtype=torch.int32, device="cuda")
    b = torch.tensor([5, 6, 7, 8], dtype=torch.int32, device="cuda")
    g.argmax(logits, 4, 10, ids, a, b)
    assert a.tolist() == [2, 3, 4, 5] and b.tolist() == [6, 7, 8, 9]


# ------------------------------------------------------------------ cuBLAS projections
@pytest.mark.parametrize("dtype", DTYPES)
def test_linear_16bit_out(g, dtype):
    """engine/tests/kernels.rs:328-345 (3 x 96 -> 50)"""
    rng = np.random.default_rng(8)
    t, i, o = 3, 96, 50
    x, w = O.uniform16(rng, t * i, 1.0, dtype), O.uniform16(rng, o * i, 1.0, dtype)
    y = torch.empty(t * o, dtype=dev(x, dtype).dtype, device="cuda")
    g.linear_f16(dev(x, dtype), dev(w, dtype), y, t, i, o)
    want = O.linear(x, w, t, i, o, dtype)
    assert_within_ulp(host_bits(y), want, dtype, ulps=1.0, name="linear")


def test_linear_f32_out(g):
    """engine/tests/kernels.rs:347-364 (1 x 2048 -> 777, f32 out)"""
    rng = np.random.default_rng(9)
    t, i, o = 1, 2048, 777
    x, w = O.uniform16(rng, t * i, 1.0), O.uniform16(rng, o * i, 0.1)
    y = torch.empty(t * o, dtype=torch.float32, device="cuda")
    g.linear_f32(dev(x), dev(w), y, t, i, o)
    assert_close(y.cpu().numpy(), O.linear(x, w, t, i, o), 1e-4, 1e-4, "linear_f32")


def test_shape_errors_are_reported_not_panics(g):
    """engine/tests/kernels.rs:366-374"""
    from kvasir_b200 import ShapeError
    x = torch.zeros(10, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(10, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(10, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ShapeError):
        g.linear_f16(x, w, y, 2, 4, 3)
    with pytest.raises(ShapeError):
        g.add_inplace(y, x[:5])
