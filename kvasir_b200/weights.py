"""Weight load path (reference engine/src/model/weights.rs:47-230): a directory
holding config.json and safetensors shards with HuggingFace Llama names, loaded
into device tensors with the reference's fused layout -- w_qkv rows q|k|v,
w_gu rows gate|up, the embedding as the tied LM head unless the checkpoint has
lm_head.weight -- in the compute type (bf16, or f16 as the reference).

The mapping, parsing and copies are native (kvb_checkpoint_* in
libkvasir_b200); this module names the tensors and owns the device buffers.
The dict it returns is the one Decoder takes (and random_weights makes), plus
"lm_head" for untied checkpoints.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib as L
from .config import LlamaConfig
from .gpu import CheckpointError, check

_DTYPE_NAMES = {L.KVB_CKPT_BF16: "BF16", L.KVB_CKPT_F16: "F16", L.KVB_CKPT_F32: "F32",
                L.KVB_CKPT_OTHER: "other"}


class Checkpoint:
    """The safetensors shards of one directory, memory-mapped (kvb_checkpoint_open)."""

    def __init__(self, directory: str):
        self._lib = L.lib()
        h = C.c_void_p()
        check(self._lib.kvb_checkpoint_open(C.byref(h), os.fsencode(directory)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.kvb_checkpoint_close(self._h)
            self._h = None

    __del__ = close

    def __enter__(self) -> "Checkpoint":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __len__(self) -> int:
        return int(self._lib.kvb_checkpoint_num_tensors(self._h))

    def info(self, name: str) -> tuple[str, tuple[int, ...]]:
        """(dtype name, shape) of a tensor; CheckpointError if it is missing."""
        dt, nd = C.c_int(), C.c_int()
        dims = (C.c_uint64 * 8)()
        check(self._lib.kvb_checkpoint_tensor(self._h, name.encode(), C.byref(dt), C.byref(nd),
                                              dims))
        return _DTYPE_NAMES[dt.value], tuple(int(dims[i]) for i in range(nd.value))

    def load_rows(self, parts: list[tuple[str, int]], cols: int, dst: torch.Tensor,
                  bad: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """Copies the named tensors, concatenated by rows, into dst (a contiguous
        bf16/f16 CUDA tensor).  parts: (name, rows), rows 0 for a [cols] vector.
        bad: int32 CUDA tensor of one element counting BF16 values outside the
        FP16 range when dst is f16 (reference Loader::convert_to)."""
        from .gpu import dtype_tag
        names = (C.c_char_p * len(parts))(*[n.encode() for n, _ in parts])
        rows = (C.c_uint64 * len(parts))(*[r for _, r in parts])
        if stream is None and dst.is_cuda:
            stream = torch.cuda.current_stream(dst.device)
        s = stream.cuda_stream if stream is not None else 0
        check(self._lib.kvb_checkpoint_load_rows(
            self._h, C.c_void_p(s), names, rows, len(parts), cols,
            C.c_void_p(dst.data_ptr()), dst.numel(), dtype_tag(dst),
            C.c_void_p(bad.data_ptr()) if bad is not None else None))


def load_weights(directory: str, cfg: LlamaConfig | None = None, device="cuda",
                 dtype=torch.bfloat16) -> tuple[LlamaConfig, dict]:
    """(config, weights) from a checkpoint directory (reference Weights::load).
    Raises CheckpointError for missing tensors, malformed shards or values the
    target type cannot hold, ShapeError for a tensor of the wrong shape."""
    if cfg is None:
        with open(os.path.join(directory, "config.json")) as f:
            cfg = LlamaConfig.from_json(f.read())
    device = torch.device(device)
    h, q, kv, inter, v = (cfg.hidden_size, cfg.q_dim, cfg.kv_dim, cfg.intermediate_size,
                          cfg.vocab_size)
    bad = torch.zeros(1, dtype=torch.int32, device=device)
    with Checkpoint(directory) as ck:
        def load(parts, cols):
            rows = sum(max(r, 1) for _, r in parts)
            shape = (rows, cols) if parts[0][1] else (cols,)
            t = torch.empty(shape, dtype=dtype, device=device)
            ck.load_rows(parts, cols, t, bad)
            return t

        w = {"embed": load([("model.embed_tokens.weight", v)], h),
             "final_norm": load([("model.norm.weight", 0)], h)}
        if not cfg.tie_word_embeddings:
            w["lm_head"] = load([("lm_head.weight", v)], h)
        for key in ("attn_norm", "w_qkv", "w_o", "mlp_norm", "w_gu", "w_down"):
            w[key] = []
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            w["attn_norm"].append(load([(p + "input_layernorm.weight", 0)], h))
            w["w_qkv"].append(load([(p + "self_attn.q_proj.weight", q),
                                    (p + "self_attn.k_proj.weight", kv),
                                    (p + "self_attn.v_proj.weight", kv)], h))
            w["w_o"].append(load([(p + "self_attn.o_proj.weight", h)], q))
            w["mlp_norm"].append(load([(p + "post_attention_layernorm.weight", 0)], h))
            w["w_gu"].append(load([(p + "mlp.gate_proj.weight", inter),
                                   (p + "mlp.up_proj.weight", inter)], h))
            w["w_down"].append(load([(p + "mlp.down_proj.weight", h)], inter))
        torch.cuda.current_stream(device).synchronize()
    n_bad = int(bad.item())
    if n_bad:
        raise CheckpointError(f"{n_bad} weights are non-finite or outside the FP16 range")
    return cfg, w
