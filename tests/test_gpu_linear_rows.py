"""kvb_linear_rows / kvb_linear_silu_mul: the decode-step projections on this
library's tensor-core kernel (reference linear_f16, engine/src/gpu/gemm.rs:63-88,
and silu_mul, engine/src/gpu/kernels.rs:171-194), through the C ABI, against the
oracle's f64 sums (engine/tests/kernels.rs:318-326 restated).

Bars.  The kernel multiplies 16-bit inputs exactly and accumulates in f32, then
rounds once to 16 bits.  Every element is therefore within
ulp(want) + K * 2^-24 * sum_k |x_k w_k| of the f64 sum (the final rounding plus
the f32 summation bound).  At small K that is the plain one-ulp bar; at the
Llama shapes (K up to 8192) the f32 error exceeds the bf16 spacing only for sums
near zero, so at least 99.5% of the elements must also be within one ulp.  A call
gives the same bits on every run; different splits of K agree within the bars.
SiLU*mul: the kernel rounds G and U to 16 bits and applies silu_mul_vec_kernel's
arithmetic, so its output is bounded through the derivatives of silu(g) * u by
the G and U bars above, and equals kvb_silu_mul of the kernel's own projection
bit for bit."""
import os

import numpy as np
import pytest
import torch

from gpu_util import TDT, dev, host_bits, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    from kvasir_b200 import Gpu
    O.set_threads(os.cpu_count() or 1)
    yield Gpu(0)
    O.set_threads(1)


def _inputs(seed, rows, k, n_w, dtype="bf16"):
    rng = np.random.default_rng(seed)
    x = normal16(rng, rows * k, 0.0, 1.0, dtype)
    w = normal16(rng, n_w * k, 0.0, 0.02, dtype)
    return x, w


def _sum_bound(x, w, rows, k, n_w, dtype="bf16"):
    """K * 2^-24 * sum_k |x_k w_k| for every (row, W row)."""
    xa = np.abs(O.to_f32(x, dtype).astype(np.float64).reshape(rows, k))
    wa = np.abs(O.to_f32(w, dtype).astype(np.float64).reshape(n_w, k))
    return k * 2.0 ** -24 * (xa @ wa.T)


def _rows(g, x, w, rows, k, out, splits=0, dtype="bf16"):
    y = torch.full((rows * out,), float("nan"), dtype=TDT[dtype], device="cuda")
    g.linear_rows(dev(x, dtype), dev(w, dtype), y, rows, k, out, splits)
    torch.cuda.synchronize()
    assert g.device_error() == 0
    return host_bits(y)


def _check_linear(got_bits, want, bound, dtype, strict, name):
    got = O.to_f32(got_bits, dtype).astype(np.float64)
    want = want.astype(np.float64).ravel()
    ulp = O.ulp16(want, dtype)
    err = np.abs(got - want)
    bad = np.nonzero(err > ulp + bound.ravel())[0]
    assert bad.size == 0, (f"{name}: {bad.size} beyond the summation bound; first {bad[0]}: "
                           f"got {got[bad[0]]} want {want[bad[0]]}")
    within = float((err <= ulp).mean())
    assert within >= (1.0 if strict else 0.995), f"{name}: {within:.4%} within one ulp"
    return within


SHAPES = [  # rows, in, out
    (3, 96, 52),        # the reference's 3 x 96 -> 50 shape, out rounded up to a multiple of 4
    (1, 2048, 3072),    # Llama-3.2-1B qkv, batch 1
    (7, 2048, 2048),    # o
    (16, 8192, 2048),   # down
    (17, 2048, 3072),
    (32, 8192, 2048),
    (33, 512, 384),
    (64, 2048, 512),
    (100, 200, 132),    # K and W-row tails inside the last chunk / tile
    (120, 512, 256),
    (128, 2048, 3072),
]


@pytest.mark.parametrize("rows,k,out", SHAPES)
def test_linear_rows_matches_oracle(g, rows, k, out):
    x, w = _inputs(rows * 7 + out, rows, k, out)
    got = _rows(g, x, w, rows, k, out)
    want = O.linear(x, w, rows, k, out)
    _check_linear(got, want, _sum_bound(x, w, rows, k, out), "bf16", k <= 256,
                  f"linear_rows {rows}x{k}->{out}")


def test_linear_rows_f16(g):
    rows, k, out = 9, 1024, 640
    x, w = _inputs(5, rows, k, out, "f16")
    got = _rows(g, x, w, rows, k, out, dtype="f16")
    want = O.linear(x, w, rows, k, out, "f16")
    _check_linear(got, want, _sum_bound(x, w, rows, k, out, "f16"), "f16", False, "f16")


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
def test_linear_rows_splits_and_repeatability(g, splits):
    """Every split of K meets the bars, and each gives the same bits on a rerun."""
    rows, k, out = 32, 8192, 2048
    x, w = _inputs(11, rows, k, out)
    want = O.linear(x, w, rows, k, out)
    bound = _sum_bound(x, w, rows, k, out)
    a = _rows(g, x, w, rows, k, out, splits)
    b = _rows(g, x, w, rows, k, out, splits)
    np.testing.assert_array_equal(a, b)
    _check_linear(a, want, bound, "bf16", False, f"splits {splits}")


def test_linear_rows_agrees_with_cublas(g):
    """Same inputs through kvb_linear (cuBLAS): both f32 sums, so the 16-bit
    results differ by at most one rounding and are mostly identical."""
    rows, k, out = 32, 2048, 3072
    x, w = _inputs(12, rows, k, out)
    a = _rows(g, x, w, rows, k, out)
    y = torch.empty(rows * out, dtype=torch.bfloat16, device="cuda")
    g.linear_f16(dev(x), dev(w), y, rows, k, out)
    b = host_bits(y)
    fa, fb = O.to_f32(a).astype(np.float64), O.to_f32(b).astype(np.float64)
    ulp = O.ulp16(np.maximum(np.abs(fa), np.abs(fb)))
    assert (np.abs(fa - fb) <= ulp + _sum_bound(x, w, rows, k, out).ravel() * 2).all()
    assert (a == b).mean() >= 0.95


def _silu_mul_bound(g64, u64, tol_g, tol_u, want, dtype):
    """First-order bound of |f(g', u') - f(g, u)| for f = silu(g) * u over
    |g' - g| <= tol_g, |u' - u| <= tol_u, plus the output rounding."""
    sig = 1.0 / (1.0 + np.exp(-g64))
    dfg = np.abs(u64 * sig * (1.0 + g64 * (1.0 - sig)))
    dfu = np.abs(g64 * sig)
    return dfg * tol_g + dfu * tol_u + O.ulp16(want, dtype) + 1e-7


GLU_SHAPES = [  # rows, hidden, inter
    (1, 2048, 8192),   # Llama-3.2-1B gate/up, batch 1
    (7, 2048, 8192),
    (32, 2048, 8192),
    (5, 96, 132),
    (64, 512, 256),
    (128, 256, 128),
]


@pytest.mark.parametrize("rows,h,inter", GLU_SHAPES)
def test_linear_silu_mul_matches_oracle(g, rows, h, inter):
    x, w = _inputs(rows * 3 + inter, rows, h, 2 * inter)
    act = torch.full((rows * inter,), float("nan"), dtype=torch.bfloat16, device="cuda")
    g.linear_silu_mul(dev(x), dev(w), act, rows, h, inter)
    torch.cuda.synchronize()
    assert g.device_error() == 0
    got = O.to_f32(host_bits(act)).astype(np.float64).reshape(rows, inter)
    gu = O.linear(x, w, rows, h, 2 * inter).reshape(rows, 2 * inter)
    bound = _sum_bound(x, w, rows, h, 2 * inter)
    g64, u64 = gu[:, :inter].astype(np.float64), gu[:, inter:].astype(np.float64)
    tol_g = O.ulp16(g64) + bound[:, :inter]
    tol_u = O.ulp16(u64) + bound[:, inter:]
    # the reference composition: 16-bit G and U, then SiLU*mul (kernels.rs:151-158 restated)
    want = O.silu_mul(O.from_f32(gu.astype(np.float32)).ravel(), rows, inter).astype(
        np.float64).reshape(rows, inter)
    err = np.abs(got - want)
    lim = _silu_mul_bound(g64, u64, tol_g, tol_u, want, "bf16")
    assert (err <= lim).all(), f"max err {err.max()}, worst ratio {(err / lim).max()}"
    assert (err <= O.ulp16(want)).mean() >= 0.99


@pytest.mark.parametrize("rows", [1, 32, 128])
def test_linear_silu_mul_equals_projection_then_silu_mul(g, rows):
    """One split each: the fused pass is kvb_linear_rows on W_gu followed by
    kvb_silu_mul, bit for bit (same f32 sums, same roundings)."""
    h, inter = 2048, 8192
    x, w = _inputs(20 + rows, rows, h, 2 * inter)
    xd, wd = dev(x), dev(w)
    act = torch.empty(rows * inter, dtype=torch.bfloat16, device="cuda")
    g.linear_silu_mul(xd, wd, act, rows, h, inter, splits=1)
    gu = torch.empty(rows * 2 * inter, dtype=torch.bfloat16, device="cuda")
    g.linear_rows(xd, wd, gu, rows, h, 2 * inter, splits=1)
    ref = torch.empty_like(act)
    g.silu_mul(gu, ref, rows, inter)
    torch.cuda.synchronize()
    assert torch.equal(act.view(torch.int16), ref.view(torch.int16))


def test_linear_rows_unsupported_and_shape_errors(g):
    from kvasir_b200.gpu import ShapeError, UnsupportedError
    x = torch.zeros(129 * 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64 * 64, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(129 * 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(UnsupportedError):  # rows > 128: unsupported (kvb_linear serves it)
        g.linear_rows(x, w, y, 129, 64, 64)
    with pytest.raises(ShapeError):
        g.linear_rows(x[:64 * 3], w, y[:64 * 2], 3, 64, 64)
    with pytest.raises(ShapeError):
        g.linear_rows(x[:64 * 2], w, y[:64 * 2], 2, 64, 64, splits=9)
    assert g.device_error() == 0
