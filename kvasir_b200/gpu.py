"""Host mirror of the reference's GPU launch-wrapper API (engine/src/gpu).

`Gpu` has one method per reference `impl Gpu` method
(engine/src/gpu/kernels.rs:58-372) with the same argument order and meaning,
plus `linear_f16` / `linear_f32` (engine/src/gpu/gemm.rs:63-115).  Buffers are
CUDA torch tensors standing in for cudarc's CudaView (a device pointer plus an
element count); every call goes through the C ABI of libkvasir_b200.so.  A
failed shape check raises `ShapeError` (the reference's KvasirError::Shape)
before anything is launched; launches are asynchronous on the Gpu's stream.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib as L


class KvasirError(RuntimeError):
    """Base error (reference engine/src/error.rs:3-19)."""


class ShapeError(KvasirError):
    pass


class CudaError(KvasirError):
    pass


class UnsupportedError(KvasirError):
    pass


class DeviceError(KvasirError):
    pass


class CheckpointError(KvasirError):
    """Checkpoint content (reference KvasirError::Config): a missing tensor, a
    malformed header, an unsupported dtype, values outside the target range."""


class CheckpointIoError(KvasirError):
    """A checkpoint file could not be opened or mapped (reference KvasirError::Io)."""


_ERRORS = {L.KVB_ERR_SHAPE: ShapeError, L.KVB_ERR_CUDA: CudaError,
           L.KVB_ERR_UNSUPPORTED: UnsupportedError, L.KVB_ERR_DEVICE: DeviceError,
           L.KVB_ERR_CONFIG: CheckpointError, L.KVB_ERR_IO: CheckpointIoError}


def check(status: int) -> None:
    if status != L.KVB_OK:
        msg = L.lib().kvb_last_error().decode(errors="replace")
        raise _ERRORS.get(status, KvasirError)(msg)


def dtype_tag(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return L.KVB_BF16
    if t.dtype == torch.float16:
        return L.KVB_F16
    raise ShapeError(f"unsupported element type {t.dtype} (bf16 or f16)")


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ShapeError("buffers must be CUDA tensors")
    if not t.is_contiguous():
        raise ShapeError("buffers must be contiguous")
    return C.c_void_p(t.data_ptr())


class Gpu:
    """One device, one stream, one cuBLAS handle (reference device.rs:10-31)."""

    def __init__(self, ordinal: int = 0, stream: torch.cuda.Stream | None = None):
        self.device = torch.device("cuda", ordinal)
        torch.cuda.set_device(self.device)
        self.stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        self._lib = L.lib()
        h = C.c_void_p()
        check(self._lib.kvb_blas_create(C.byref(h)))
        self._blas = h

    @classmethod
    def new(cls, ordinal: int = 0) -> "Gpu":
        return cls(ordinal)

    def __del__(self):
        try:
            if getattr(self, "_blas", None):
                self._lib.kvb_blas_destroy(self._blas)
                self._blas = None
        except Exception:
            pass

    @property
    def _s(self):
        return C.c_void_p(self.stream.cuda_stream)

    def synchronize(self) -> None:
        self.stream.synchronize()

    def device_error(self) -> int:
        code = C.c_uint32()
        check(self._lib.kvb_device_error(C.byref(code)))
        return code.value

    # ------------------------------------------------ reference kernels.rs methods
    def embedding_gather(self, ids, table, out, hidden):
        """kernels.rs:59-88"""
        check(self._lib.kvb_embedding_gather(self._s, _ptr(ids), ids.numel(), _ptr(table),
                                             table.numel(), _ptr(out), out.numel(), hidden,
                                             dtype_tag(table)))

    def rmsnorm(self, x, w, out, rows, hidden, eps):
        """kernels.rs:90-121"""
        check(self._lib.kvb_rmsnorm(self._s, _ptr(x), x.numel(), _ptr(w), w.numel(), _ptr(out),
                                    out.numel(), rows, hidden, eps, dtype_tag(x)))

    def embedding_rmsnorm(self, ids, table, w, x, out, hidden, eps):
        """kvb_embedding_rmsnorm: embedding_gather into x, then rmsnorm(x, w) into out,
        in one launch for decode-sized batches (bit-equal to the two calls)."""
        check(self._lib.kvb_embedding_rmsnorm(self._s, _ptr(ids), ids.numel(), _ptr(table),
                                              table.numel(), _ptr(w), w.numel(), _ptr(x),
                                              x.numel(), _ptr(out), out.numel(), hidden, eps,
                                              dtype_tag(table)))

    def rope_inplace(self, qkv, cos, sin, t, pos0, n_q, n_kv, head_dim):
        """kernels.rs:124-169"""
        check(self._lib.kvb_rope_inplace(self._s, _ptr(qkv), qkv.numel(), _ptr(cos), cos.numel(),
                                         _ptr(sin), sin.numel(), t, pos0, n_q, n_kv, head_dim,
                                         dtype_tag(qkv)))

    def silu_mul(self, gu, out, t, inter):
        """kernels.rs:171-194"""
        check(self._lib.kvb_silu_mul(self._s, _ptr(gu), gu.numel(), _ptr(out), out.numel(), t,
                                     inter, dtype_tag(gu)))

    def add_inplace(self, x, y):
        """kernels.rs:196-209"""
        check(self._lib.kvb_add_inplace(self._s, _ptr(x), x.numel(), _ptr(y), y.numel(),
                                        dtype_tag(x)))

    def bf16_to_f16(self, src, dst, bad):
        """kernels.rs:211-235"""
        check(self._lib.kvb_bf16_to_f16(self._s, _ptr(src), src.numel(), _ptr(dst), dst.numel(),
                                        _ptr(bad), bad.numel()))

    def kv_append(self, qkv, kc, vc, t, pos0, n_q, n_kv, head_dim, max_seq):
        """kernels.rs:238-291"""
        check(self._lib.kvb_kv_append(self._s, _ptr(qkv), qkv.numel(), _ptr(kc), kc.numel(),
                                      _ptr(vc), vc.numel(), t, pos0, n_q, n_kv, head_dim, max_seq,
                                      dtype_tag(qkv)))

    def attention(self, qkv, kc, vc, out, t, pos0, n_q, n_kv, head_dim, max_seq, workspace=None):
        """kernels.rs:294-371.  `workspace` (optional, a uint8 CUDA tensor of
        attention_workspace_bytes(...)) lets a long decode split across CTAs."""
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(self._lib.kvb_attention(self._s, _ptr(qkv), qkv.numel(), _ptr(kc), kc.numel(),
                                      _ptr(vc), vc.numel(), _ptr(out), out.numel(), t, pos0, n_q,
                                      n_kv, head_dim, max_seq, _ptr(workspace), ws_len,
                                      dtype_tag(qkv)))

    def attention_workspace_bytes(self, t, pos0, n_q, n_kv, head_dim) -> int:
        return int(self._lib.kvb_attention_workspace_bytes(t, pos0, n_q, n_kv, head_dim))

    # ------------------------------------------------ reference gemm.rs
    def linear_f16(self, x, w, y, t, in_dim, out_dim):
        """gemm.rs:63-88 (16-bit output; bf16 or f16 by the tensors' type)"""
        check(self._lib.kvb_linear(self._blas, self._s, _ptr(x), x.numel(), _ptr(w), w.numel(),
                                   _ptr(y), y.numel(), t, in_dim, out_dim, dtype_tag(x), 0))

    def linear_f32(self, x, w, y, t, in_dim, out_dim):
        """gemm.rs:90-115 (f32 output)"""
        if y.dtype != torch.float32:
            raise ShapeError("linear_f32: y must be float32")
        check(self._lib.kvb_linear(self._blas, self._s, _ptr(x), x.numel(), _ptr(w), w.numel(),
                                   _ptr(y), y.numel(), t, in_dim, out_dim, dtype_tag(x), 1))

    # ------------------------------------------------ fused / batched additions
    def rope_kv_append(self, qkv, cos, sin, kc, vc, t, pos0, n_q, n_kv, head_dim, max_seq):
        if cos.numel() != sin.numel():
            raise ShapeError("rope: bad cos/sin table sizes")
        if kc.numel() != vc.numel():
            raise ShapeError("kv_append: bad cache sizes")
        check(self._lib.kvb_rope_kv_append(self._s, _ptr(qkv), qkv.numel(), _ptr(cos), _ptr(sin),
                                           cos.numel(), _ptr(kc), _ptr(vc), kc.numel(), t, pos0,
                                           n_q, n_kv, head_dim, max_seq, dtype_tag(qkv)))

    def rope_kv_append_prefill(self, qkv, cos, sin, kc, vc, n_seq, t, pos0, n_q, n_kv, head_dim,
                               max_seq):
        """kvb_rope_kv_append_prefill: rope_kv_append over n_seq sequences of t rows
        each in one launch; caches [n_seq, n_kv, max_seq, head_dim]."""
        if cos.numel() != sin.numel():
            raise ShapeError("rope: bad cos/sin table sizes")
        if kc.numel() != vc.numel():
            raise ShapeError("kv_append: bad cache sizes")
        check(self._lib.kvb_rope_kv_append_prefill(
            self._s, _ptr(qkv), qkv.numel(), _ptr(cos), _ptr(sin), cos.numel(), _ptr(kc), _ptr(vc),
            kc.numel(), n_seq, t, pos0, n_q, n_kv, head_dim, max_seq, dtype_tag(qkv)))

    def rope_kv_append_batched(self, qkv, pos, cos, sin, kc, vc, seq_stride, n_q, n_kv, head_dim,
                               max_seq):
        if pos.dtype != torch.int32:
            raise ShapeError("positions must be int32")
        check(self._lib.kvb_rope_kv_append_batched(
            self._s, _ptr(qkv), pos.numel(), _ptr(pos), _ptr(cos), _ptr(sin), cos.numel(),
            _ptr(kc), _ptr(vc), seq_stride, kc.numel(), n_q, n_kv, head_dim, max_seq,
            dtype_tag(qkv)))

    def rope_kv_append_paged(self, qkv, n_seq, t, pos, cos, sin, k_pool, v_pool, block_table,
                             max_blocks, block_size, n_q, n_kv, head_dim):
        """kvb_rope_kv_append_paged: rows of sequence b at positions pos[b].. into the
        K/V block pools [n_blocks, n_kv, block_size, head_dim] via block_table
        [n_seq, max_blocks] (int32, device)."""
        if pos.dtype != torch.int32 or block_table.dtype != torch.int32:
            raise ShapeError("positions and block table must be int32")
        if cos.numel() != sin.numel() or k_pool.numel() != v_pool.numel():
            raise ShapeError("rope_kv_append_paged: cos/sin or pool sizes differ")
        check(self._lib.kvb_rope_kv_append_paged(
            self._s, _ptr(qkv), n_seq, t, _ptr(pos), _ptr(cos), _ptr(sin), cos.numel(),
            _ptr(k_pool), _ptr(v_pool), k_pool.numel(), _ptr(block_table), max_blocks, block_size,
            n_q, n_kv, head_dim, dtype_tag(qkv)))

    def attention_prefill_paged(self, qkv, k_pool, v_pool, block_table, max_blocks, block_size,
                                out, n_seq, t, pos0, n_q, n_kv, head_dim):
        """kvb_attention_prefill_paged: causal prefill reading K/V through block_table."""
        if block_table.dtype != torch.int32:
            raise ShapeError("block table must be int32")
        if k_pool.numel() != v_pool.numel():
            raise ShapeError("attention_prefill_paged: pool sizes differ")
        check(self._lib.kvb_attention_prefill_paged(
            self._s, _ptr(qkv), qkv.numel(), _ptr(k_pool), _ptr(v_pool), k_pool.numel(),
            _ptr(block_table), max_blocks, block_size, _ptr(out), out.numel(), n_seq, t, pos0,
            n_q, n_kv, head_dim, dtype_tag(qkv)))

    def attention_decode_paged(self, q, q_row_stride, k_pool, v_pool, block_table, max_blocks,
                               block_size, lens, max_len, n_q, n_kv, head_dim, out,
                               out_row_stride, scale=None, workspace=None):
        """kvb_attention_decode_paged: batched decode attention over K/V block pools."""
        if lens.dtype != torch.int32 or block_table.dtype != torch.int32:
            raise ShapeError("lengths and block table must be int32")
        if k_pool.numel() != v_pool.numel():
            raise ShapeError("attention_decode_paged: pool sizes differ")
        scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(self._lib.kvb_attention_decode_paged(
            self._s, _ptr(q), q_row_stride, _ptr(k_pool), _ptr(v_pool), k_pool.numel(),
            _ptr(block_table), max_blocks, block_size, _ptr(lens), lens.numel(), max_len, n_q,
            n_kv, head_dim, scale, _ptr(out), out_row_stride,
            _ptr(workspace) if workspace is not None else None, ws_len, dtype_tag(q)))

    def add_rmsnorm(self, x, y, w, out, rows, hidden, eps):
        check(self._lib.kvb_add_rmsnorm(self._s, _ptr(x), x.numel(), _ptr(y), y.numel(), _ptr(w),
                                        w.numel(), _ptr(out), out.numel(), rows, hidden, eps,
                                        dtype_tag(x)))

    def attention_decode_workspace_bytes(self, n_seq, max_len, n_q, n_kv, head_dim) -> int:
        return int(self._lib.kvb_attention_decode_workspace_bytes(n_seq, max_len, n_q, n_kv,
                                                                  head_dim))

    def attention_decode(self, q, q_row_stride, kc, vc, seq_stride, lens, max_len, n_q, n_kv,
                         head_dim, max_seq, out, out_row_stride, scale=None, workspace=None):
        if lens.dtype != torch.int32:
            raise ShapeError("lengths must be int32")
        scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(self._lib.kvb_attention_decode(
            self._s, _ptr(q), q_row_stride, _ptr(kc), _ptr(vc), seq_stride, kc.numel(),
            _ptr(lens), lens.numel(), max_len, n_q, n_kv, head_dim, max_seq, scale, _ptr(out),
            out_row_stride, _ptr(workspace), ws_len, dtype_tag(q)))

    def rope_attention_decode(self, qkv, cos, sin, kc, vc, seq_stride, lens, max_len, n_q, n_kv,
                              head_dim, max_seq, out, out_row_stride, scale=None, workspace=None):
        """kvb_rope_attention_decode: rope_kv_append_batched at positions lens - 1, then
        attention_decode, in one launch (qkv is left unrotated)."""
        if lens.dtype != torch.int32:
            raise ShapeError("lengths must be int32")
        scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(self._lib.kvb_rope_attention_decode(
            self._s, _ptr(qkv), qkv.numel(), _ptr(cos), _ptr(sin), cos.numel(), _ptr(kc),
            _ptr(vc), seq_stride, kc.numel(), _ptr(lens), lens.numel(), max_len, n_q, n_kv,
            head_dim, max_seq, scale, _ptr(out), out_row_stride, _ptr(workspace), ws_len,
            dtype_tag(qkv)))

    def rope_attention_decode_paged(self, qkv, cos, sin, k_pool, v_pool, block_table, max_blocks,
                                    block_size, lens, max_len, n_q, n_kv, head_dim, out,
                                    out_row_stride, scale=None, workspace=None):
        """kvb_rope_attention_decode_paged: rope_kv_append_paged at positions lens - 1,
        then attention_decode_paged, in one launch."""
        if lens.dtype != torch.int32 or block_table.dtype != torch.int32:
            raise ShapeError("lengths and block table must be int32")
        scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        check(self._lib.kvb_rope_attention_decode_paged(
            self._s, _ptr(qkv), qkv.numel(), _ptr(cos), _ptr(sin), cos.numel(), _ptr(k_pool),
            _ptr(v_pool), k_pool.numel(), _ptr(block_table), max_blocks, block_size, _ptr(lens),
            lens.numel(), max_len, n_q, n_kv, head_dim, scale, _ptr(out), out_row_stride,
            _ptr(workspace), ws_len, dtype_tag(qkv)))

    def attention_prefill(self, qkv, kc, vc, out, n_seq, t, pos0, n_q, n_kv, head_dim, max_seq):
        if vc.numel() != kc.numel():
            raise ShapeError("attention_prefill: bad cache sizes")
        check(self._lib.kvb_attention_prefill(self._s, _ptr(qkv), qkv.numel(), _ptr(kc), _ptr(vc),
                                              kc.numel(), _ptr(out), out.numel(), n_seq, t, pos0,
                                              n_q, n_kv, head_dim, max_seq, dtype_tag(qkv)))

    def attention_prefill_f32(self, qkv, kc, vc, out, n_seq, t, pos0, n_q, n_kv, head_dim,
                              max_seq):
        """kvb_attention_prefill_f32: the prefill rows as f32, before the one rounding."""
        if vc.numel() != kc.numel() or out.dtype != torch.float32:
            raise ShapeError("attention_prefill_f32: bad cache sizes or non-f32 output")
        check(self._lib.kvb_attention_prefill_f32(self._s, _ptr(qkv), qkv.numel(), _ptr(kc),
                                                  _ptr(vc), kc.numel(), _ptr(out), out.numel(),
                                                  n_seq, t, pos0, n_q, n_kv, head_dim, max_seq,
                                                  dtype_tag(qkv)))

    def lm_head_argmax(self, x, w, rows, hidden, vocab, ids, workspace=None, advance=None,
                       advance2=None):
        """kvb_lm_head_argmax: greedy ids of x @ w^T (f32 logits never stored)."""
        if ids.dtype != torch.int32 or ids.numel() != rows:
            raise ShapeError("lm_head_argmax: int32 ids of rows elements expected")
        if workspace is None:
            nb = int(self._lib.kvb_lm_head_argmax_workspace_bytes(rows))
            workspace = torch.empty(max(nb, 16), dtype=torch.uint8, device=x.device)
        ws_len = workspace.numel() * workspace.element_size()
        check(self._lib.kvb_lm_head_argmax(self._s, _ptr(x), x.numel(), _ptr(w), w.numel(), rows,
                                           hidden, vocab, _ptr(workspace), ws_len, _ptr(ids),
                                           _ptr(advance), _ptr(advance2), dtype_tag(x)))

    def linear_rows(self, x, w, y, rows, in_dim, out_dim, splits=0):
        """kvb_linear_rows: y = x @ w^T on this library's tensor-core kernel
        (rows <= 128; splits 0 = automatic)."""
        check(self._lib.kvb_linear_rows(self._s, _ptr(x), x.numel(), _ptr(w), w.numel(), _ptr(y),
                                        y.numel(), rows, in_dim, out_dim, splits, dtype_tag(x)))

    def linear_silu_mul(self, x, w_gu, act, rows, hidden, inter, splits=0):
        """kvb_linear_silu_mul: act = silu(G) * U with [G | U] = x @ w_gu^T."""
        check(self._lib.kvb_linear_silu_mul(self._s, _ptr(x), x.numel(), _ptr(w_gu), w_gu.numel(),
                                            _ptr(act), act.numel(), rows, hidden, inter, splits,
                                            dtype_tag(x)))

    def argmax(self, logits, rows, vocab, ids, advance=None, advance2=None):
        if logits.dtype != torch.float32 or ids.dtype != torch.int32:
            raise ShapeError("argmax: f32 logits and int32 ids expected")
        if logits.numel() != rows * vocab or ids.numel() != rows:
            raise ShapeError("argmax: bad sizes")
        check(self._lib.kvb_argmax_f32(self._s, _ptr(logits), rows, vocab, _ptr(ids),
                                       _ptr(advance), _ptr(advance2)))

    def sample(self, logits, rows, vocab, ids, temperature, top_p=1.0, seed=0, counters=None,
               advance=None, advance2=None):
        """kvb_sample_f32: temperature / top-p sampling, one id per row (temperature
        <= 0 is the argmax).  counters: int32 per row (None: 0)."""
        if logits.dtype != torch.float32 or ids.dtype != torch.int32:
            raise ShapeError("sample: f32 logits and int32 ids expected")
        if logits.numel() != rows * vocab or ids.numel() != rows:
            raise ShapeError("sample: bad sizes")
        if counters is not None and (counters.dtype != torch.int32 or counters.numel() != rows):
            raise ShapeError("sample: counters must be int32, one per row")
        check(self._lib.kvb_sample_f32(self._s, _ptr(logits), rows, vocab, temperature, top_p,
                                       seed & 0xFFFFFFFFFFFFFFFF, _ptr(counters), _ptr(ids),
                                       _ptr(advance), _ptr(advance2)))

    def selftest_wait_timeout(self, limit_ms: int) -> int:
        """Runs the bounded-wait self test; returns the status code."""
        return int(self._lib.kvb_selftest_wait_timeout(self._s, limit_ms))
