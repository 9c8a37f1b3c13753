"""Decode-step driver (the caller of the kernel chain): n_seq independent
sequences, one token each per step, through a Llama decoder with the
reference's weight layout (engine/src/model/weights.rs:13-27: fused w_qkv
rows q|k|v, fused w_gu rows gate|up, tied embedding / LM head).

The step itself is native: kvb_decoder_step in libkvasir_b200 records the
whole step (16 layers of cuBLAS projections + the kvb kernels + argmax) into
one CUDA graph and replays it.  This module owns the device buffers the driver
borrows -- weights, KV cache, RoPE tables, workspace -- as torch tensors.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L
from .config import LlamaConfig
from .gpu import ShapeError, check, dtype_tag
from .rope import cos_sin_table


def random_weights(cfg: LlamaConfig, device, dtype=torch.bfloat16, seed: int = 0,
                   std: float = 0.02) -> dict:
    """Random-init weights: projections and the tied embedding N(0, std),
    norm weights 1 + std*N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h, i = cfg.hidden_size, cfg.intermediate_size

    def normal(*shape):
        t = torch.empty(*shape, dtype=dtype, device=device)
        t.normal_(0.0, std, generator=g)
        return t

    def norm_w():
        t = torch.empty(h, dtype=dtype, device=device)
        t.normal_(1.0, std, generator=g)
        return t

    return {
        "embed": normal(cfg.vocab_size, h),
        "final_norm": norm_w(),
        "attn_norm": [norm_w() for _ in range(cfg.num_layers)],
        "w_qkv": [normal(cfg.qkv_dim, h) for _ in range(cfg.num_layers)],
        "w_o": [normal(h, cfg.q_dim) for _ in range(cfg.num_layers)],
        "mlp_norm": [norm_w() for _ in range(cfg.num_layers)],
        "w_gu": [normal(2 * i, h) for _ in range(cfg.num_layers)],
        "w_down": [normal(h, i) for _ in range(cfg.num_layers)],
    }


class Decoder:
    """Greedy decoding of n_seq sequences with KV capacity max_seq each.

    weights: the dict of random_weights or kvasir_b200.weights.load_weights
    ("lm_head" present for untied checkpoints).
    kc / vc: [n_layers, n_seq, n_kv, max_seq, head_dim], or with paged_block_size
    the block pools [n_layers, n_blocks, n_kv, paged_block_size, head_dim] that
    self.block_table ([n_seq, max_blocks], one table for all layers) indexes."""

    def __init__(self, cfg: LlamaConfig, n_seq: int, max_seq: int, device="cuda",
                 dtype=torch.bfloat16, weights: dict | None = None, seed: int = 0,
                 paged_block_size: int | None = None):
        self.cfg, self.n_seq, self.max_seq = cfg, n_seq, max_seq
        self.device = torch.device(device)
        self.dtype = dtype
        self.w = weights if weights is not None else random_weights(cfg, self.device, dtype, seed)
        shape = (cfg.num_layers, n_seq, cfg.num_kv_heads, max_seq, cfg.head_dim)
        if paged_block_size:
            # kc / vc are then block pools [n_layers, n_blocks, n_kv, block_size, head_dim]
            # with every sequence's blocks scattered through them by a seeded table
            bs = paged_block_size
            max_blocks = -(-max_seq // bs)
            n_blocks = n_seq * max_blocks
            shape = (cfg.num_layers, n_blocks, cfg.num_kv_heads, bs, cfg.head_dim)
            perm = np.random.default_rng(seed + 1).permutation(n_blocks).astype(np.int32)
            self.block_table = torch.from_numpy(perm.reshape(n_seq, max_blocks)).to(self.device)
        self.kc = torch.empty(shape, dtype=dtype, device=self.device)
        self.vc = torch.empty(shape, dtype=dtype, device=self.device)
        cos, sin = cos_sin_table(cfg, max_seq)
        self.cos = torch.from_numpy(cos).to(self.device)
        self.sin = torch.from_numpy(sin).to(self.device)
        c = L.DecoderConfig(cfg.hidden_size, cfg.intermediate_size, cfg.num_layers, cfg.num_heads,
                            cfg.num_kv_heads, cfg.head_dim, cfg.vocab_size, max_seq, n_seq,
                            cfg.rms_norm_eps, dtype_tag(self.kc))
        self._cfg = c
        lib = L.lib()
        nbytes = int(lib.kvb_decoder_workspace_bytes(C.byref(c)))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=self.device)

        def arr(lst):
            a = (C.c_void_p * len(lst))(*[t.data_ptr() for t in lst])
            return a

        self._ptr_arrays = {k: arr(self.w[k]) for k in
                            ("attn_norm", "w_qkv", "w_o", "mlp_norm", "w_gu", "w_down")}
        W = L.DecoderWeights(self.w["embed"].data_ptr(), self.w["final_norm"].data_ptr(),
                             *[C.cast(self._ptr_arrays[k], C.POINTER(C.c_void_p)) for k in
                               ("attn_norm", "w_qkv", "w_o", "mlp_norm", "w_gu", "w_down")])
        h = C.c_void_p()
        torch.cuda.synchronize(self.device)
        check(lib.kvb_decoder_create(C.byref(h), C.byref(c), C.byref(W), self.kc.data_ptr(),
                                     self.vc.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(),
                                     self.workspace.data_ptr(), nbytes))
        self._h = h
        self._lib = lib
        base = self.workspace.data_ptr()

        def view(ptr, n, dt):
            off = ptr - base
            esz = torch.tensor([], dtype=dt).element_size()
            return self.workspace[off:off + n * esz].view(dt)

        if "lm_head" in self.w:  # untied checkpoint (kvasir_b200.weights.load_weights)
            check(lib.kvb_decoder_set_lm_head(h, self.w["lm_head"].data_ptr()))
        if paged_block_size:
            self.use_paged_cache(self.kc, self.vc, self.block_table, max_blocks, paged_block_size)
        self.ids_in = view(lib.kvb_decoder_ids_in(h), n_seq, torch.int32)
        self.ids_out = view(lib.kvb_decoder_ids_out(h), n_seq, torch.int32)
        self.logits = view(lib.kvb_decoder_logits(h), n_seq * cfg.vocab_size,
                           torch.float32).view(n_seq, cfg.vocab_size)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.kvb_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ cache set-up
    def fill_kv_normal(self, seed: int = 1, std: float = 1.0, first_seq: int | None = None) -> None:
        """Fills the whole KV cache with N(0, std) (the synthetic context).

        first_seq=None: one generator over the whole cache.  first_seq=g: local
        sequence b is filled from generators seeded by (seed, g + b, layer, k|v)
        only, so a sequence's context does not depend on how the sequences are
        split over ranks (a paged cache gets the same contents through its
        block table)."""
        g = torch.Generator(device=self.device)
        if first_seq is None:
            g.manual_seed(seed)
            for l in range(self.cfg.num_layers):
                self.kc[l].normal_(0.0, std, generator=g)
                self.vc[l].normal_(0.0, std, generator=g)
            return
        nkv, hd = self.cfg.num_kv_heads, self.cfg.head_dim
        paged = getattr(self, "_paged", None)
        tmp = seq = None
        if paged is not None:
            bs = self.kc.shape[3]
            mb = self.block_table.shape[1]
            tmp = torch.zeros(nkv, mb * bs, hd, dtype=self.dtype, device=self.device)
            seq = torch.empty(nkv, self.max_seq, hd, dtype=self.dtype, device=self.device)
        for b in range(self.n_seq):
            for l in range(self.cfg.num_layers):
                for kind, cache in ((0, self.kc), (1, self.vc)):
                    s = (((seed * 1000003 + first_seq + b) * 1024 + l) * 2 + kind) & (2 ** 63 - 1)
                    g.manual_seed(s)
                    if paged is None:
                        cache[l, b].normal_(0.0, std, generator=g)
                    else:  # the contiguous contents, scattered into the pool's blocks
                        seq.normal_(0.0, std, generator=g)
                        tmp[:, :self.max_seq] = seq
                        blocks = tmp.view(nkv, mb, bs, hd).permute(1, 0, 2, 3)
                        cache[l][self.block_table[b].long()] = blocks

    def use_paged_cache(self, k_pools, v_pools, block_table, max_blocks: int,
                        block_size: int) -> None:
        """Switch to a paged KV cache (kvb_decoder_use_paged_cache).  k_pools / v_pools:
        [n_layers, n_blocks, n_kv, block_size, head_dim]; block_table: int32
        [n_seq, max_blocks], shared by all layers.  The tensors are kept alive here."""
        if block_table.dtype != torch.int32:
            raise ShapeError("block table must be int32")
        self._paged = (k_pools, v_pools, block_table)
        check(self._lib.kvb_decoder_use_paged_cache(self._h, k_pools.data_ptr(),
                                                    v_pools.data_ptr(), k_pools[0].numel(),
                                                    block_table.data_ptr(), max_blocks, block_size))

    def set_sampling(self, temperature: float, top_p: float = 1.0, seed: int = 0) -> None:
        """Temperature / top-p sampling for the following steps (kvb_decoder_set_sampling);
        temperature <= 0 goes back to greedy."""
        check(self._lib.kvb_decoder_set_sampling(self._h, temperature, top_p,
                                                 seed & 0xFFFFFFFFFFFFFFFF))

    def set_fused_lm_head(self, enable: bool = True) -> None:
        """Greedy steps through kvb_lm_head_argmax (LM head + argmax in one pass;
        self.logits is then not written by those steps)."""
        check(self._lib.kvb_decoder_set_fused_lm_head(self._h, 1 if enable else 0))

    def set_row_projections(self, enable: bool = True) -> None:
        """Projections on kvb_linear_rows and the gate/up projection + SiLU*mul on
        kvb_linear_silu_mul (decode-sized batches) instead of cuBLAS."""
        check(self._lib.kvb_decoder_set_row_projections(self._h, 1 if enable else 0))

    def set_lengths(self, cur_len) -> None:
        """Tokens already in each sequence's cache; the next step writes there."""
        arr = np.ascontiguousarray(np.broadcast_to(np.asarray(cur_len, np.int32), (self.n_seq,)))
        if arr.max() >= self.max_seq or arr.min() < 0:
            raise ShapeError("set_lengths: length outside [0, max_seq)")
        s = torch.cuda.current_stream(self.device)
        check(self._lib.kvb_decoder_set_lengths(self._h, C.c_void_p(s.cuda_stream),
                                                arr.ctypes.data_as(C.c_void_p)))

    # ------------------------------------------------------------ stepping
    def step(self, stream: torch.cuda.Stream | None = None) -> None:
        """One decode step on the device: reads ids_in, writes ids_out (and
        copies it to ids_in for the next step)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(self._lib.kvb_decoder_step(self._h, C.c_void_p(s.cuda_stream)))

    def step_host(self, ids_host_in: torch.Tensor, ids_host_out: torch.Tensor,
                  stream: torch.cuda.Stream | None = None) -> None:
        """One step from host ids to host ids (H2D copy, step, D2H copy, sync)."""
        for t in (ids_host_in, ids_host_out):
            if t.device.type != "cpu" or t.dtype != torch.int32 or t.numel() != self.n_seq:
                raise ShapeError("step_host: host int32 tensors of n_seq ids expected")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(self._lib.kvb_decoder_step_host(self._h, C.c_void_p(s.cuda_stream),
                                              C.c_void_p(ids_host_in.data_ptr()),
                                              C.c_void_p(ids_host_out.data_ptr())))

    def launches_per_step(self) -> tuple[int, int]:
        own, lib = C.c_int(), C.c_int()
        check(self._lib.kvb_decoder_launches_per_step(self._h, C.byref(own), C.byref(lib)))
        return own.value, lib.value

    def weight_bytes(self) -> int:
        return self.cfg.weight_params() * self.kc.element_size()
