"""kvb_lm_head_argmax: the LM head and greedy argmax in one pass (f32 logits never
stored; reference engine/src/gpu/gemm.rs:90-115 followed by the argmax), through
the C ABI, against the oracle's f64 logits (tests/kernels.rs:318-326 restated)
and against cuBLAS + kvb_argmax_f32.

The fused kernel sums in f32 on the tensor cores, so its logits differ from the
f64 ones by at most hidden * 2^-24 * sum_k |x_k w_k| (the worst case of an f32
sum of hidden products).  Its pick must be a token whose f64 logit is within
twice that of the row's best, and the f64 argmax wherever the top-2 margin
exceeds twice the bound.  Ties, NaN and infinities follow kvb_argmax_f32's rule:
the first index of the maximum, NaN never wins, -inf never wins a tie, a row with
nothing above -inf gives 0."""
import os

import numpy as np
import pytest
import torch

from gpu_util import dev, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    from kvasir_b200 import Gpu
    return Gpu(0)


def _fused(g, x_bits, w_bits, rows, hidden, vocab, dtype="bf16", adv=False):
    ids = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    a1 = torch.arange(rows, dtype=torch.int32, device="cuda") if adv else None
    a2 = (torch.arange(rows, dtype=torch.int32, device="cuda") * 3) if adv else None
    g.lm_head_argmax(dev(x_bits, dtype), dev(w_bits, dtype), rows, hidden, vocab, ids,
                     advance=a1, advance2=a2)
    torch.cuda.synchronize()
    assert g.device_error() == 0
    if adv:
        assert torch.equal(a1.cpu(), torch.arange(rows, dtype=torch.int32) + 1)
        assert torch.equal(a2.cpu(), torch.arange(rows, dtype=torch.int32) * 3 + 1)
    return ids.cpu().numpy()


def _cublas_argmax(g, x_bits, w_bits, rows, hidden, vocab):
    y = torch.empty(rows * vocab, dtype=torch.float32, device="cuda")
    g.linear_f32(dev(x_bits), dev(w_bits), y, rows, hidden, vocab)
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    g.argmax(y, rows, vocab, ids)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), y.cpu().numpy().reshape(rows, vocab)


@pytest.fixture(scope="module")
def llama_head():
    O.set_threads(os.cpu_count() or 1)
    try:
        return O.fill_normal(128256 * 2048, 0.0, 0.02, 77)
    finally:
        O.set_threads(1)


@pytest.mark.parametrize("rows", [1, 7, 16, 17, 32])
def test_lm_head_argmax_llama_shape_against_oracle(g, llama_head, rows):
    """hidden 2048, vocab 128256 (the tied Llama-3.2-1B LM head), x N(0,1) rows,
    W N(0,0.02)."""
    hidden, vocab = 2048, 128256
    rng = np.random.default_rng(rows)
    x = normal16(rng, rows * hidden)
    w = llama_head
    got = _fused(g, x, w, rows, hidden, vocab, adv=True)
    O.set_threads(os.cpu_count() or 1)
    try:
        want = O.linear(x, w, rows, hidden, vocab).reshape(rows, vocab).astype(np.float64)
    finally:
        O.set_threads(1)
    xf = O.to_f32(x).reshape(rows, hidden).astype(np.float64)
    best = want.argmax(axis=1)
    for r in range(rows):
        wr = O.to_f32(w.reshape(vocab, hidden)[[got[r], best[r]]]).astype(np.float64)
        bound = hidden * 2.0 ** -24 * (np.abs(xf[r]) * np.abs(wr)).sum(axis=1).max()
        assert want[r, got[r]] >= want[r, best[r]] - 2 * bound, (r, got[r], best[r])
        top2 = np.sort(want[r])[-2:]
        if top2[1] - top2[0] > 2 * bound:
            assert got[r] == best[r], (r, got[r], best[r])
    cub, _ = _cublas_argmax(g, x, w, rows, hidden, vocab)
    assert (cub == got).mean() >= 0.9  # the same picks but for near ties of the f32 sums


def test_lm_head_argmax_ties_nan_inf_and_partial_tile(g):
    """vocab 1000 (the last 128-row tile partial), hidden 64: two equal best rows
    (the first wins), a NaN row (never wins), +inf and -inf logits."""
    rows, hidden, vocab = 6, 64, 1000
    rng = np.random.default_rng(4)
    xf = rng.normal(0, 1, (rows, hidden)).astype(np.float32)
    xf[:, 0] = np.abs(xf[:, 0]) + 0.5  # x[r, 0] > 0 for r >= 1 ...
    xf[0, 0] = -xf[0, 0]               # ... and < 0 for row 0
    wf = rng.normal(0, 0.02, (vocab, hidden)).astype(np.float32)
    # row 0: rows 3 and 900 of W are equal and the largest logit for x row 0
    wf[3] = wf[900] = xf[0] * 0.5
    # NaN row everywhere
    wf[5] = np.nan
    # +inf at index 700 and 950 for rows with x[r, 0] > 0 (the first +inf wins), -inf
    # (never wins) for row 0
    wf[700, 0] = np.inf
    wf[950, 0] = np.inf
    x = O.from_f32(xf)
    w = O.from_f32(wf)
    got = _fused(g, x, w, rows, hidden, vocab, adv=True)
    cub, logits = _cublas_argmax(g, x, w, rows, hidden, vocab)
    np.testing.assert_array_equal(got, cub)
    assert got[0] == 3
    assert (got[1:] == 700).all()
    # -inf everywhere (or NaN): nothing above -inf gives 0
    x2f = np.abs(xf) + 0.1
    wf2 = rng.normal(0, 0.02, (vocab, hidden)).astype(np.float32)
    wf2[:, 0] = -np.inf
    wf2[7] = np.nan
    got2 = _fused(g, O.from_f32(x2f), O.from_f32(wf2), rows, hidden, vocab)
    assert (got2 == 0).all()
    cub2, _ = _cublas_argmax(g, O.from_f32(x2f), O.from_f32(wf2), rows, hidden, vocab)
    assert (cub2 == 0).all()
    # f16 inputs, the same rule
    got3 = _fused(g, O.from_f32(xf, "f16"), O.from_f32(np.nan_to_num(wf, nan=0.0, posinf=0.0), "f16"),
                  rows, hidden, vocab, dtype="f16")
    assert got3[0] == 3


@pytest.mark.parametrize("rows,hidden,vocab", [(3, 4096, 300), (16, 4096, 127), (2, 128, 5)])
def test_lm_head_argmax_shape_limits(g, rows, hidden, vocab):
    """hidden 4096 on the 16-column path (x fills its 128 KB), vocab below one tile."""
    rng = np.random.default_rng(rows + hidden + vocab)
    x = normal16(rng, rows * hidden)
    w = normal16(rng, vocab * hidden, std=0.05)
    got = _fused(g, x, w, rows, hidden, vocab, adv=True)
    cub, logits = _cublas_argmax(g, x, w, rows, hidden, vocab)
    top2 = np.sort(logits, axis=1)[:, -2:]
    clear = top2[:, 1] - top2[:, 0] > 1e-2
    np.testing.assert_array_equal(got[clear], cub[clear])
    assert ((got >= 0) & (got < vocab)).all()


def test_lm_head_argmax_rejects_unsupported(g):
    from kvasir_b200.gpu import UnsupportedError
    x = torch.zeros(33 * 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(256 * 64, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(33, dtype=torch.int32, device="cuda")
    with pytest.raises(UnsupportedError, match="rows <= 32"):
        g.lm_head_argmax(x, w, 33, 64, 256, ids)
    # 17 rows take the 32-column path: x of 32 x 4096 would not fit its 128 KB
    x2 = torch.zeros(17 * 4096, dtype=torch.bfloat16, device="cuda")
    w2 = torch.zeros(64 * 4096, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(UnsupportedError):
        g.lm_head_argmax(x2, w2, 17, 4096, 64, torch.zeros(17, dtype=torch.int32, device="cuda"))
