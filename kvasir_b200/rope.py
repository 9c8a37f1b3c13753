"""RoPE cos/sin tables (reference engine/src/model/rope.rs:3-39), computed by
kvb_rope_table in libkvasir_b200 (f64 inverse frequencies with llama3
scaling, f32 tables [max_pos, head_dim/2])."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .config import LlamaConfig
from .gpu import check


def cos_sin_table(cfg: LlamaConfig, max_pos: int) -> tuple[np.ndarray, np.ndarray]:
    half = cfg.head_dim // 2
    cos = np.empty(max_pos * half, np.float32)
    sin = np.empty(max_pos * half, np.float32)
    rs = cfg.rope_scaling
    scaled = rs is not None
    check(L.lib().kvb_rope_table(
        cfg.head_dim, cfg.rope_theta, int(scaled),
        float(rs["factor"]) if scaled else 1.0,
        float(rs["low_freq_factor"]) if scaled else 1.0,
        float(rs["high_freq_factor"]) if scaled else 2.0,
        float(rs["original_max_position_embeddings"]) if scaled else 1.0,
        max_pos, cos.ctypes.data_as(C.c_void_p), sin.ctypes.data_as(C.c_void_p)))
    return cos, sin
