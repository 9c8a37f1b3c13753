"""kvb_attention_decode_noalloc: decode attention for callers that cannot
allocate device memory (no spare device buffer of their own and no cudaMalloc
allowed).  Its split-KV partials live in the library's own scratch array.  The
test calls it through the C ABI twice in a row with different inputs and
checks each result against kvb_attention_decode given a caller workspace: the
same kernel with the same chunking, so the outputs must be equal bit for bit.
Each result is also checked against the CPU oracle within the attention
tolerance of the other attention tests.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import assert_close, dev, host_bits, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 2.0 ** -8  # as in tests/test_gpu_attention.py


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _case(seed, lens, n_q=32, n_kv=8, hd=64, max_seq=4096):
    rng = np.random.default_rng(seed)
    n_seq = len(lens)
    per = n_kv * max_seq * hd
    q = normal16(rng, n_seq * n_q * hd)
    kc = normal16(rng, n_seq * per)
    vc = normal16(rng, n_seq * per)
    return q, kc, vc, per


def _run(lib, fn_name, q, kc, vc, lens_t, per, max_len, n_q, n_kv, hd, max_seq, ws=None):
    from kvasir_b200 import _lib as L
    n_seq = lens_t.numel()
    out = torch.full((n_seq * n_q * hd,), float("nan"), dtype=torch.bfloat16, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [s, _p(q), n_q * hd, _p(kc), _p(vc), per, kc.numel(), _p(lens_t), n_seq, max_len,
            n_q, n_kv, hd, max_seq, 1.0 / 8.0, _p(out), n_q * hd]
    if fn_name == "kvb_attention_decode":
        args += [_p(ws), ws.numel() if ws is not None else 0]
    st = getattr(lib, fn_name)(*args, L.KVB_BF16)
    assert st == L.KVB_OK, lib.kvb_last_error().decode()
    torch.cuda.synchronize()
    return host_bits(out)


def test_noalloc_decode_matches_workspace_decode_twice():
    from kvasir_b200 import _lib as L
    lib = L.lib()
    n_q, n_kv, hd, max_seq = 32, 8, 64, 4096
    cases = [
        (11, np.random.default_rng(1).integers(1, 4097, 48).astype(np.int32)),
        (12, np.array([0, 1, 64, 65, 2049, 4096, 333, 4000], np.int32)),
    ]
    for seed, lens in cases:
        qh, kh, vh, per = _case(seed, lens.tolist())
        q, kc, vc = dev(qh), dev(kh), dev(vh)
        lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
        max_len = int(lens.max())
        need = int(lib.kvb_attention_decode_workspace_bytes(len(lens), max_len, n_q, n_kv, hd))
        assert 0 < need <= L.KVB_NOALLOC_SCRATCH_BYTES  # the split path, within the array
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        want = _run(lib, "kvb_attention_decode", q, kc, vc, lens_t, per, max_len, n_q, n_kv, hd,
                    max_seq, ws)
        got = _run(lib, "kvb_attention_decode_noalloc", q, kc, vc, lens_t, per, max_len, n_q,
                   n_kv, hd, max_seq)
        np.testing.assert_array_equal(got, want, err_msg=f"noalloc vs workspace (seed {seed})")
        ref = O.attention_decode(qh, n_q * hd, kh, vh, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
        ref = ref.reshape(len(lens), -1)
        ref[lens == 0] = 0.0  # no keys: a zero row by definition
        assert_close(O.to_f32(got), ref, RTOL, ATOL, f"noalloc vs oracle (seed {seed})")


def test_noalloc_general_kernel_shape_needs_no_scratch():
    """A shape the split-KV kernel does not take (head_dim 32) runs the general
    kernel, which uses no scratch, even where the split path's partials would
    exceed the array."""
    from kvasir_b200 import _lib as L
    lib = L.lib()
    n_q, n_kv, hd, max_seq = 8, 2, 32, 96
    lens = np.array([1, 33, 96], np.int32)
    qh, kh, vh, per = _case(13, lens.tolist(), n_q=n_q, n_kv=n_kv, hd=hd, max_seq=max_seq)
    q, kc, vc = dev(qh), dev(kh), dev(vh)
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    want = _run(lib, "kvb_attention_decode", q, kc, vc, lens_t, per, max_seq, n_q, n_kv, hd,
                max_seq)
    got = _run(lib, "kvb_attention_decode_noalloc", q, kc, vc, lens_t, per, max_seq, n_q, n_kv,
               hd, max_seq)
    np.testing.assert_array_equal(got, want)


def test_noalloc_rejects_requests_beyond_its_scratch():
    from kvasir_b200 import _lib as L
    lib = L.lib()
    n_q, n_kv, hd, max_len = 128, 8, 64, 131072  # 16 query heads per kv head
    for n_seq in (64, 32, 128, 16, 256):
        need = int(lib.kvb_attention_decode_workspace_bytes(n_seq, max_len, n_q, n_kv, hd))
        if need > L.KVB_NOALLOC_SCRATCH_BYTES:
            break
    assert need > L.KVB_NOALLOC_SCRATCH_BYTES
    fake = C.c_void_p(0x1000)  # 16-byte aligned; rejected before anything touches these
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.kvb_attention_decode_noalloc(s, fake, n_q * hd, fake, fake, n_kv * max_len * hd,
                                          n_seq * n_kv * max_len * hd, fake, n_seq, max_len, n_q,
                                          n_kv, hd, max_len, 0.125, fake, n_q * hd, L.KVB_BF16)
    assert st == L.KVB_ERR_SHAPE
    assert "scratch" in lib.kvb_last_error().decode()
