"""Helpers shared by the -m gpu parity tests: moving 16-bit bit patterns
between numpy (the oracle's format) and CUDA tensors (the C-ABI's buffers),
and the tolerance checks the tests state."""
import numpy as np
import torch

from oracle import oracle as O

TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


def dev(bits: np.ndarray, dtype: str = "bf16") -> torch.Tensor:
    b = np.ascontiguousarray(bits, np.uint16)
    return torch.from_numpy(b.view(np.int16).copy()).view(TDT[dtype]).cuda()


def host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def host_f32(t: torch.Tensor, dtype: str = "bf16") -> np.ndarray:
    return O.to_f32(host_bits(t), dtype)


def assert_within_ulp(got_bits, want_f32, dtype="bf16", ulps=1.0, name=""):
    """|got - want| <= ulps * spacing of the 16-bit format at |want|, i.e. the
    16-bit result is want rounded to one of its two neighbours."""
    got = O.to_f32(np.asarray(got_bits).ravel(), dtype).astype(np.float64)
    want = np.asarray(want_f32, np.float64).ravel()
    tol = ulps * O.ulp16(want, dtype)
    err = np.abs(got - want)
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, (f"{name}: {bad.size} of {want.size} beyond {ulps} ulp; first at "
                           f"{bad[0]}: got {got[bad[0]]}, want {want[bad[0]]}")
    return float(err.max()) if err.size else 0.0


def assert_close(got, want, rtol, atol, name=""):
    """|got - want| <= atol + rtol*|want| (reference tests/kernels.rs:17-29)."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want)
    bad = np.nonzero(err > atol + rtol * np.abs(want))[0]
    assert bad.size == 0, (f"{name}: {bad.size} of {want.size} outside tolerance; first at "
                           f"{bad[0]}: got {got[bad[0]]}, want {want[bad[0]]}")
    return float(err.max()) if err.size else 0.0


def normal16(rng, n, mean=0.0, std=1.0, dtype="bf16"):
    return O.from_f32(rng.normal(mean, std, n).astype(np.float32), dtype)


# Logit spread of the 16-layer Llama-3.2-1B decode step (random N(0, 0.02) weights)
# caused by bf16 rounding alone: an upper bound on the largest |logit| difference
# between the oracle's step and the same step with its rounding points dithered by a
# relative 2^-16 (measured 0.09-0.14 at logit rms 0.9; tests/test_gpu_decoder_full.py
# recomputes it on every run and checks this bound).  Two correct evaluations of the
# step agree within LOGIT_TOL_FACTOR times it.
LLAMA1B_LOGIT_SPREAD = 0.2
LOGIT_TOL_FACTOR = 2.0
