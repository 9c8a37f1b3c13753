"""Parity of the attention kernels against the CPU oracle (f64 softmax
attention, engine/tests/kernels.rs:264-289), through the C ABI.

Tolerance: |got - want| <= 2e-3 + 2^-8 |want| -- the 2e-3 max-abs bar for
unit-scale inputs plus one rounding of the 16-bit output itself.  The f16
runs also meet the reference's own bound (rtol 2e-3, atol 1e-3)."""
import math

import numpy as np
import pytest
import torch

from gpu_util import assert_close, assert_within_ulp, dev, host_bits, host_f32, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 2.0 ** -8


@pytest.fixture(scope="module")
def g():
    from kvasir_b200 import Gpu
    return Gpu(0)


def _ref_inputs(rng, n_q, n_kv, hd, t, max_seq, dtype, amp=2.0):
    stride = (n_q + 2 * n_kv) * hd
    qkv = O.uniform16(rng, t * stride, amp, dtype)
    kc = O.uniform16(rng, n_kv * max_seq * hd, amp, dtype)
    vc = O.uniform16(rng, n_kv * max_seq * hd, amp, dtype)
    return qkv, kc, vc


# The reference's five attention cases (engine/tests/kernels.rs:293-316)
REF_CASES = [(8, 2, 64, 7, 0, 32), (8, 2, 64, 1, 12, 32), (8, 2, 64, 4, 5, 32),
             (32, 8, 64, 3, 397, 512), (4, 2, 128, 2, 20, 64)]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("case", REF_CASES)
def test_attention_reference_cases(g, dtype, case):
    n_q, n_kv, hd, t, pos0, max_seq = case
    rng = np.random.default_rng(100 + t * 31 + pos0)
    qkv, kc, vc = _ref_inputs(rng, n_q, n_kv, hd, t, max_seq, dtype)
    out = torch.empty(t * n_q * hd, dtype=dev(qkv, dtype).dtype, device="cuda")
    g.attention(dev(qkv, dtype), dev(kc, dtype), dev(vc, dtype), out, t, pos0, n_q, n_kv, hd,
                max_seq)
    want = O.attention(qkv, kc, vc, t, pos0, n_q, n_kv, hd, max_seq, dtype)
    got = host_f32(out, dtype)
    assert_close(got, want, RTOL, ATOL, f"attention{case}")
    if dtype == "f16":
        assert_close(got, want, 2e-3, 1e-3, f"attention{case}")


@pytest.mark.parametrize("pos0", [0, 63, 64, 255, 256, 511, 4095, 16383])
def test_attention_decode_single_sequence_split_and_unsplit(g, pos0):
    """T = 1 through the reference API, without and with a split-KV workspace."""
    n_q, n_kv, hd = 32, 8, 64
    max_seq = pos0 + 1
    rng = np.random.default_rng(pos0)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, stride)
    kc, vc = normal16(rng, n_kv * max_seq * hd), normal16(rng, n_kv * max_seq * hd)
    want = O.attention(qkv, kc, vc, 1, pos0, n_q, n_kv, hd, max_seq)
    out = torch.empty(n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention(dev(qkv), dev(kc), dev(vc), out, 1, pos0, n_q, n_kv, hd, max_seq)
    a = host_f32(out)
    assert_close(a, want, RTOL, ATOL, "decode/no-split")
    nbytes = g.attention_workspace_bytes(1, pos0, n_q, n_kv, hd)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
    g.attention(dev(qkv), dev(kc), dev(vc), out, 1, pos0, n_q, n_kv, hd, max_seq, workspace=ws)
    assert_close(host_f32(out), want, RTOL, ATOL, "decode/split")


def _batched_case(rng, lens, n_q=32, n_kv=8, hd=64, max_seq=None):
    n_seq = len(lens)
    max_seq = max_seq or max(max(lens), 1)
    q = normal16(rng, n_seq * n_q * hd)
    per = n_kv * max_seq * hd
    kc, vc = normal16(rng, n_seq * per), normal16(rng, n_seq * per)
    return q, kc, vc, max_seq, per


def _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per, use_ws=True, dtype="bf16"):
    n_seq = len(lens)
    out = torch.empty(n_seq * n_q * hd, dtype=torch.bfloat16 if dtype == "bf16" else torch.float16,
                      device="cuda")
    max_len = int(max(lens)) if len(lens) else 0
    nbytes = g.attention_decode_workspace_bytes(n_seq, max_len, n_q, n_kv, hd)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda") if use_ws else None
    g.attention_decode(dev(q, dtype), n_q * hd, dev(kc, dtype), dev(vc, dtype), per,
                       torch.tensor(lens, dtype=torch.int32, device="cuda"), max_len, n_q, n_kv,
                       hd, max_seq, out, n_q * hd, workspace=ws)
    return host_f32(out, dtype)


def test_decode_cluster_fold_equals_combine_pass(g):
    """Small split grids fold their chunks inside the decode kernel (a cluster per
    (sequence, kv head), distributed shared memory) instead of the workspace and the
    combine pass, with the combine's arithmetic: the rows are the same bits.  8
    sequences of 2000 keys are 8 chunks each, 512 CTAs (above one wave: workspace +
    combine); the first 5 of them, 320 CTAs, fold; both use 256-key chunks."""
    rng = np.random.default_rng(77)
    n_q, n_kv, hd = 32, 8, 64
    lens = [2000] * 8
    q, kc, vc, max_seq, per = _batched_case(rng, lens)
    q = O.from_f32(O.to_f32(q) * np.float32(3.0))  # peaked rows: the fold's weights matter
    split = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per)
    n5 = 5
    fold = _run_batched(g, q[:n5 * n_q * hd], kc[:n5 * per], vc[:n5 * per], lens[:n5], n_q,
                        n_kv, hd, max_seq, per)
    assert g.device_error() == 0
    np.testing.assert_array_equal(fold.view(np.uint32), split[:n5 * n_q * hd].view(np.uint32))
    want = O.attention_decode(q[:n5 * n_q * hd], n_q * hd, kc[:n5 * per], vc[:n5 * per],
                              np.array(lens[:n5], np.int32), n_q, n_kv, hd, max_seq, 1 / 8.0)
    err = np.abs(fold.astype(np.float64) - want)
    assert np.all(err <= 2e-3 + np.abs(want) * 2.0 ** -8), err.max()


def test_batched_decode_config2(g):
    """64 sequences, lengths U[1, 4096], 32/8 heads, hd 64,
    N(0,1) Q/K/V, scale 1/8."""
    rng = np.random.default_rng(2026)
    lens = rng.integers(1, 4097, 64).astype(np.int32)
    n_q, n_kv, hd = 32, 8, 64
    q, kc, vc, max_seq, per = _batched_case(rng, lens, max_seq=4096)
    got = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per)
    O.set_threads(8)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    O.set_threads(1)
    assert_close(got, want, RTOL, ATOL, "decode config 2")
    assert g.device_error() == 0


@pytest.mark.parametrize("length,q_std", [(16385, 1.0), (2000, 4.0)])
def test_decode_error_before_output_rounding(g, length, q_std):
    """The split-KV decode kernel's own error, before its output is rounded: 8
    sequences, each split over several chunks -- at the config-5 length with
    N(0,1) inputs (flat softmax, small outputs), and at 2000 keys with q scaled
    by 4 (peaked softmax: outputs of unit scale, where the bar bites).  Both
    grids are above one wave (33 and 8 chunks of 64 (sequence, kv head) pairs),
    so the chunks' partials go to the workspace rather than being folded in the
    kernel.
    Every chunk leaves f32 partials in the workspace -- per query head the
    unnormalised O row, the running max m (log2 units) and the sum l -- which
    are folded here in f64 (O = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c)
    and held to the plain 2e-3 max-abs bar against the f64 oracle.  The bf16
    rows of the same call are that fold rounded once (within one ulp: the
    combine kernel folds in f32)."""
    n_seq, n_q, n_kv, hd = 8, 32, 8, 64
    G = n_q // n_kv
    lens = np.full(n_seq, length, np.int32)
    rng = np.random.default_rng(length)
    q, kc, vc, max_seq, per = _batched_case(rng, lens, max_seq=length)
    q = O.from_f32(O.to_f32(q) * np.float32(q_std))
    nbytes = g.attention_decode_workspace_bytes(n_seq, length, n_q, n_kv, hd)
    chunks = nbytes // (n_seq * n_kv * G * 66 * 4)
    assert chunks >= 2 and nbytes == n_seq * n_kv * chunks * G * 66 * 4
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(n_seq * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention_decode(dev(q), n_q * hd, dev(kc), dev(vc), per,
                       torch.from_numpy(lens).cuda(), length, n_q, n_kv, hd, max_seq, out,
                       n_q * hd, workspace=ws)
    assert g.device_error() == 0
    part = ws.view(torch.float32).cpu().numpy().astype(np.float64)
    part = part.reshape(n_seq, n_kv, chunks, G * 66)
    o = part[..., :G * 64].reshape(n_seq, n_kv, chunks, G, hd)
    m = part[..., G * 64:G * 65]
    l = part[..., G * 65:G * 66]
    M = m.max(axis=2, keepdims=True)
    w = np.exp2(m - M)
    pre = (o * w[..., None]).sum(axis=2) / (l * w).sum(axis=2)[..., None]
    pre = pre.reshape(n_seq, n_q * hd)
    O.set_threads(8)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    O.set_threads(1)
    err = assert_close(pre, want, 0.0, 2e-3, "decode f32 partials folded")
    assert_within_ulp(host_bits(out), pre.ravel(), ulps=1.0, name="decode rows vs fold")
    print(f"decode 8 x {length} keys, q x {q_std:g}: max |err| before output rounding "
          f"{err:.2e} (max |out| {np.abs(want).max():.2f})")


def test_batched_decode_edge_lengths(g):
    """Empty sequence (zero row), single key, tile and chunk boundaries."""
    lens = np.array([0, 1, 2, 63, 64, 65, 255, 256, 257, 1000, 1023, 1024, 1025, 4096], np.int32)
    n_q, n_kv, hd = 32, 8, 64
    rng = np.random.default_rng(7)
    q, kc, vc, max_seq, per = _batched_case(rng, lens, max_seq=4096)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    want = want.reshape(len(lens), -1)
    want[0] = 0.0  # no keys: zero row by definition
    for use_ws in (True, False):
        got = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per, use_ws=use_ws)
        assert_close(got, want, RTOL, ATOL, f"decode edges ws={use_ws}")


@pytest.mark.parametrize("lens", [[1100], [0, 1, 70, 1100], [1, 2, 1100, 1099], [400, 1100]])
def test_batched_decode_few_sequences_five_chunks(g, lens):
    """Few sequences of ~1100 keys: five 256-key chunks each and the combine pass,
    beside sequences shorter than one chunk or one tile, and one with no keys."""
    lens = np.array(lens, np.int32)
    n_q, n_kv, hd = 32, 8, 64
    rng = np.random.default_rng(int(lens.sum()))
    q, kc, vc, max_seq, per = _batched_case(rng, lens, max_seq=1280)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    want = want.reshape(len(lens), -1)
    want[lens == 0] = 0.0
    got = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per)
    assert_close(got, want, RTOL, ATOL, "decode five chunks")
    assert g.device_error() == 0


@pytest.mark.parametrize("group", [1, 2, 8, 16])
def test_batched_decode_group_sizes(g, group):
    n_kv, hd = 2, 64
    n_q = n_kv * group
    lens = np.array([5, 300, 129], np.int32)
    rng = np.random.default_rng(group)
    q, kc, vc, max_seq, per = _batched_case(rng, lens, n_q=n_q, n_kv=n_kv, max_seq=320)
    got = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    assert_close(got, want, RTOL, ATOL, f"decode group {group}")


def test_batched_decode_general_kernel_head_dim_32(g):
    n_q, n_kv, hd = 8, 2, 32
    lens = np.array([1, 33, 100], np.int32)
    rng = np.random.default_rng(5)
    q, kc, vc, max_seq, per = _batched_case(rng, lens, n_q=n_q, n_kv=n_kv, hd=hd, max_seq=100)
    got = _run_batched(g, q, kc, vc, lens, n_q, n_kv, hd, max_seq, per)
    want = O.attention_decode(q, n_q * hd, kc, vc, lens, n_q, n_kv, hd, max_seq,
                              1 / math.sqrt(hd))
    assert_close(got, want, RTOL, ATOL, "decode hd 32")


def test_batched_decode_f16(g):
    lens = np.array([17, 1000, 64], np.int32)
    rng = np.random.default_rng(9)
    q, kc, vc, max_seq, per = _batched_case(rng, lens, max_seq=1024)
    q, kc, vc = (O.from_f32(O.to_f32(a), "f16") for a in (q, kc, vc))
    got = _run_batched(g, q, kc, vc, lens, 32, 8, 64, max_seq, per, dtype="f16")
    want = O.attention_decode(q, 32 * 64, kc, vc, lens, 32, 8, 64, max_seq, 1 / 8.0, "f16")
    assert_close(got, want, 2e-3, 1e-3, "decode f16")


@pytest.mark.parametrize("t,pos0", [(7, 0), (4, 5), (128, 0), (129, 0), (300, 17), (1000, 0)])
def test_prefill_tcgen05_against_oracle(g, t, pos0):
    """Causal prefill through the reference API (T > 1, head_dim 64)."""
    n_q, n_kv, hd = 8, 2, 64
    max_seq = pos0 + t
    rng = np.random.default_rng(t * 7 + pos0)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, t * stride)
    kc, vc = normal16(rng, n_kv * max_seq * hd), normal16(rng, n_kv * max_seq * hd)
    out = torch.empty(t * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention(dev(qkv), dev(kc), dev(vc), out, t, pos0, n_q, n_kv, hd, max_seq)
    O.set_threads(8)
    want = O.attention(qkv, kc, vc, t, pos0, n_q, n_kv, hd, max_seq)
    O.set_threads(1)
    assert_close(host_f32(out), want, RTOL, ATOL, f"prefill t={t} pos0={pos0}")
    assert g.device_error() == 0


@pytest.mark.parametrize("t,pos0", [(300, 17), (1000, 0)])
def test_prefill_f16_against_oracle(g, t, pos0):
    """f16 inputs: P enters the P.V product as one f16 (no remainder term); the
    reference's own f16 bound (rtol 2e-3, atol 1e-3) holds over many key tiles."""
    n_q, n_kv, hd = 8, 2, 64
    max_seq = pos0 + t
    rng = np.random.default_rng(t * 11 + pos0)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, t * stride, dtype="f16")
    kc = normal16(rng, n_kv * max_seq * hd, dtype="f16")
    vc = normal16(rng, n_kv * max_seq * hd, dtype="f16")
    out = torch.empty(t * n_q * hd, dtype=torch.float16, device="cuda")
    g.attention(dev(qkv, "f16"), dev(kc, "f16"), dev(vc, "f16"), out, t, pos0, n_q, n_kv, hd,
                max_seq)
    O.set_threads(8)
    want = O.attention(qkv, kc, vc, t, pos0, n_q, n_kv, hd, max_seq, "f16")
    O.set_threads(1)
    got = host_f32(out, "f16")
    assert_close(got, want, RTOL, ATOL, f"prefill f16 t={t} pos0={pos0}")
    assert_close(got, want, 2e-3, 1e-3, f"prefill f16 t={t} pos0={pos0}")
    assert g.device_error() == 0


def test_prefill_config3_shape(g):
    """4 sequences x 2048 tokens, 32/8 heads, hd 64, N(0,1),
    every (sequence, kv head) pair against the oracle (~69 GFLOP of f64 work,
    spread over all host cores).

    Two bars.  The 16-bit rows: 2e-3 + 2^-8 |want| (the 2e-3 bar plus their own
    rounding).  The kernel's f32 rows before that rounding
    (kvb_attention_prefill_f32): the plain 2e-3 max-abs bar; rounding them to
    bf16 must give the 16-bit rows bit for bit."""
    import os
    n_seq, t, n_q, n_kv, hd = 4, 2048, 32, 8, 64
    rng = np.random.default_rng(33)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, n_seq * t * stride)
    per = n_kv * t * hd
    kc, vc = normal16(rng, n_seq * per), normal16(rng, n_seq * per)
    out = torch.empty(n_seq * t * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention_prefill(dev(qkv), dev(kc), dev(vc), out, n_seq, t, 0, n_q, n_kv, hd, t)
    out32 = torch.empty(n_seq * t * n_q * hd, dtype=torch.float32, device="cuda")
    g.attention_prefill_f32(dev(qkv), dev(kc), dev(vc), out32, n_seq, t, 0, n_q, n_kv, hd, t)
    assert g.device_error() == 0
    got_bits = host_bits(out)
    got32 = out32.cpu().numpy()
    np.testing.assert_array_equal(O.from_f32(got32), got_bits)
    got = O.to_f32(got_bits).reshape(n_seq, t * n_q * hd)
    got32 = got32.reshape(n_seq, t * n_q * hd)
    O.set_threads(os.cpu_count() or 1)
    worst16 = worst32 = 0.0
    try:
        for seq in range(n_seq):
            want = O.attention(qkv[seq * t * stride:(seq + 1) * t * stride],
                               kc[seq * per:(seq + 1) * per], vc[seq * per:(seq + 1) * per], t, 0,
                               n_q, n_kv, hd, t)
            worst16 = max(worst16, assert_close(got[seq], want, RTOL, ATOL, f"prefill seq {seq}"))
            worst32 = max(worst32, assert_close(got32[seq], want, 0.0, 2e-3,
                                                f"prefill seq {seq}, f32 rows"))
    finally:
        O.set_threads(1)
    print(f"config 3 prefill: max |err| 16-bit rows {worst16:.2e}, f32 rows {worst32:.2e}")


def test_prefill_v_scale_is_exact(g):
    """V entries far outside the f16 range (up to ~2^19): scaling V by 2^17 (exact
    in bf16) must scale the prefill output by 2^17 bit for bit -- every product and
    sum scales exactly, so any overflow or change of rounding would show."""
    n_q, n_kv, hd, t = 8, 2, 64, 300
    rng = np.random.default_rng(55)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, t * stride)
    kc, vc = normal16(rng, n_kv * t * hd), normal16(rng, n_kv * t * hd)
    vbig = O.from_f32(O.to_f32(vc) * np.float32(2.0 ** 17))
    assert np.abs(O.to_f32(vbig)).max() > 2.0 ** 15
    a = torch.empty(t * n_q * hd, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    g.attention(dev(qkv), dev(kc), dev(vc), a, t, 0, n_q, n_kv, hd, t)
    g.attention(dev(qkv), dev(kc), dev(vbig), b, t, 0, n_q, n_kv, hd, t)
    assert g.device_error() == 0
    np.testing.assert_array_equal(host_f32(b), host_f32(a) * np.float32(2.0 ** 17))


def test_prefill_v_magnitudes_vary_by_key_tile(g):
    """V tiles up to 2^19 apart in magnitude within one sequence.  Per-row bar:
    2e-3 x the row's softmax-weighted mean |v| (the unit-scale bar, scaled) plus
    one rounding of the output."""
    n_q, n_kv, hd, t = 4, 1, 64, 600
    rng = np.random.default_rng(56)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, t * stride)
    kc = normal16(rng, t * hd)
    v = rng.normal(0, 1, (t, hd))
    for tile, e in enumerate([0, 17, 3, 19, 0]):
        v[tile * 128:(tile + 1) * 128] *= 2.0 ** e
    vc = O.from_f32(v.astype(np.float32).ravel())
    out = torch.empty(t * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention(dev(qkv), dev(kc), dev(vc), out, t, 0, n_q, n_kv, hd, t)
    assert g.device_error() == 0
    got = host_f32(out).reshape(t, n_q, hd).astype(np.float64)
    q = O.to_f32(qkv).reshape(t, n_q + 2, hd)[:, :n_q].astype(np.float64)
    k = O.to_f32(kc).reshape(t, hd).astype(np.float64)
    vv = O.to_f32(vc).reshape(t, hd).astype(np.float64)
    s = np.einsum("thd,kd->htk", q, k) / 8.0
    s = np.where(np.triu(np.ones((t, t), bool), 1)[None], -np.inf, s)
    p = np.exp(s - s.max(-1, keepdims=True))
    l = p.sum(-1, keepdims=True)
    want = np.einsum("htk,kd->htd", p, vv) / l
    scale = np.einsum("htk,kd->htd", p, np.abs(vv)) / l
    err = np.abs(got.transpose(1, 0, 2) - want)
    bound = 2e-3 * scale + 2.0 ** -8 * np.abs(want)
    assert (err <= bound).all(), float((err / bound).max())


def test_prefill_rows_are_prefix_consistent(g):
    """Size-independent property at full length: causal row i only depends on
    tokens <= i, so a prefill of the first 1000 tokens reproduces the first
    1000 rows of a 2048-token prefill bit for bit."""
    n_q, n_kv, hd, t = 32, 8, 64, 2048
    rng = np.random.default_rng(44)
    stride = (n_q + 2 * n_kv) * hd
    qkv = normal16(rng, t * stride)
    kc, vc = normal16(rng, n_kv * t * hd), normal16(rng, n_kv * t * hd)
    full = torch.empty(t * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention(dev(qkv), dev(kc), dev(vc), full, t, 0, n_q, n_kv, hd, t)
    k = 1024
    part = torch.empty(k * n_q * hd, dtype=torch.bfloat16, device="cuda")
    g.attention(dev(qkv[:k * stride]), dev(kc), dev(vc), part, k, 0, n_q, n_kv, hd, t)
    assert torch.equal(full[:k * n_q * hd], part)


def test_bounded_wait_selftest_keeps_context_usable(g):
    """A device-side wait on a barrier nobody completes gives up after its
    limit and reports KVB_ERR_DEVICE; later launches still work."""
    from kvasir_b200 import _lib as L
    st = g.selftest_wait_timeout(50)
    assert st == L.KVB_ERR_DEVICE
    assert g.device_error() == 0  # the self test read and cleared the word
    x = torch.ones(16, dtype=torch.bfloat16, device="cuda")
    g.add_inplace(x, x)
    assert float(x[0]) == 2.0


# ------------------------------------------------------------------ fused RoPE + append + decode
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("lens,n_q,n_kv,with_ws", [
    ([1, 64, 65, 300, 1000, 2049], 32, 8, True),
    ([7, 513], 32, 8, False),
    ([1024] * 32, 32, 8, True),
    ([5, 200, 4096], 8, 8, True),
    ([130, 1], 64, 4, True),
    ([1, 70, 1100], 32, 8, True),
])
def test_rope_attention_decode_equals_rope_then_decode(g, dtype, lens, n_q, n_kv, with_ws):
    """kvb_rope_attention_decode == kvb_rope_kv_append_batched (positions lens - 1) +
    kvb_attention_decode on the rotated qkv, bit for bit: the attention output and
    both caches (the new rows written, every other row untouched)."""
    rng = np.random.default_rng(sum(lens) + n_q)
    hd, max_seq = 64, 4160
    n_seq = len(lens)
    stride = (n_q + 2 * n_kv) * hd
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    qkv = normal16(rng, n_seq * stride, dtype=dtype)
    per = n_kv * max_seq * hd
    kc0 = normal16(rng, n_seq * per, dtype=dtype)
    vc0 = normal16(rng, n_seq * per, dtype=dtype)
    cos, sin = O.cos_sin_table(hd, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    lens_np = np.array(lens, np.int32)
    ld = torch.from_numpy(lens_np).cuda()
    pos = torch.from_numpy(lens_np - 1).cuda()
    max_len = int(lens_np.max())
    ws = None
    if with_ws:
        ws = torch.empty(max(16, g.attention_decode_workspace_bytes(n_seq, max_len, n_q, n_kv, hd)),
                         dtype=torch.uint8, device="cuda")
    # unfused: rotate + append, then decode over the rotated qkv
    qa, ka, va = dev(qkv, dtype), dev(kc0, dtype), dev(vc0, dtype)
    g.rope_kv_append_batched(qa, pos, c, s, ka, va, per, n_q, n_kv, hd, max_seq)
    want = torch.empty(n_seq * n_q * hd, dtype=tdt, device="cuda")
    g.attention_decode(qa, stride, ka, va, per, ld, max_len, n_q, n_kv, hd, max_seq, want, n_q * hd,
                       workspace=ws)
    # fused
    qb, kb, vb = dev(qkv, dtype), dev(kc0, dtype), dev(vc0, dtype)
    got = torch.empty_like(want)
    g.rope_attention_decode(qb, c, s, kb, vb, per, ld, max_len, n_q, n_kv, hd, max_seq, got,
                            n_q * hd, workspace=ws)
    assert g.device_error() == 0
    assert torch.equal(got, want)
    assert torch.equal(kb, ka) and torch.equal(vb, va)
    np.testing.assert_array_equal(host_bits(qb), qkv)  # qkv itself is not rotated


def test_rope_attention_decode_rejects_unsupported(g):
    from kvasir_b200.gpu import UnsupportedError
    n_seq, n_q, n_kv, hd, max_seq = 1, 4, 1, 32, 64
    qkv = torch.zeros(n_seq * (n_q + 2 * n_kv) * hd, dtype=torch.bfloat16, device="cuda")
    cos, sin = O.cos_sin_table(hd, max_seq, 10000.0, False)
    kc = torch.zeros(n_seq * n_kv * max_seq * hd, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(n_seq * n_q * hd, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(UnsupportedError, match="head_dim 64"):
        g.rope_attention_decode(qkv, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), kc,
                                kc.clone(), n_kv * max_seq * hd,
                                torch.ones(1, dtype=torch.int32, device="cuda"), 1, n_q, n_kv, hd,
                                max_seq, out, n_q * hd)
