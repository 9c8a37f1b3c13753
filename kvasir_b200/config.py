"""Llama shapes (reference engine/src/model/config.rs).

Only what the kernel chain needs: the dimensions, their validation
(config.rs:184-206) and the derived sizes q_dim / kv_dim / qkv_dim
(config.rs:208-216).  `from_json` accepts a HuggingFace config.json text like
the reference and rejects rope types other than "llama3" (config.rs:146-158).
"""
from __future__ import annotations

import dataclasses
import json


class ConfigError(ValueError):
    pass


@dataclasses.dataclass
class LlamaConfig:
    hidden_size: int = 2048
    intermediate_size: int = 8192
    num_layers: int = 16
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 64
    vocab_size: int = 128256
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = dataclasses.field(default_factory=lambda: {
        "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    max_position_embeddings: int = 131072
    tie_word_embeddings: bool = True

    @classmethod
    def llama_3_2_1b(cls) -> "LlamaConfig":
        return cls()

    @classmethod
    def from_json(cls, text: str) -> "LlamaConfig":
        try:
            raw = json.loads(text)
            n_heads = raw["num_attention_heads"]
            rs = raw.get("rope_scaling")
            if rs is not None and rs.get("rope_type") != "llama3":
                raise ConfigError(f"unsupported rope_type {rs.get('rope_type')!r} (only \"llama3\")")
            cfg = cls(
                hidden_size=raw["hidden_size"], intermediate_size=raw["intermediate_size"],
                num_layers=raw["num_hidden_layers"], num_heads=n_heads,
                num_kv_heads=raw.get("num_key_value_heads") or n_heads,
                head_dim=raw.get("head_dim") or raw["hidden_size"] // n_heads,
                vocab_size=raw["vocab_size"], rms_norm_eps=float(raw["rms_norm_eps"]),
                rope_theta=float(raw["rope_theta"]), rope_scaling=rs,
                max_position_embeddings=raw["max_position_embeddings"],
                tie_word_embeddings=bool(raw.get("tie_word_embeddings", False)))
        except (KeyError, TypeError, json.JSONDecodeError) as e:
            raise ConfigError(f"config.json: {e}") from e
        cfg.validate()
        return cfg

    def validate(self) -> None:
        if self.num_kv_heads == 0 or self.num_heads % self.num_kv_heads:
            raise ConfigError(f"num_heads {self.num_heads} not a multiple of num_kv_heads "
                              f"{self.num_kv_heads}")
        if self.head_dim % 2 or 128 % self.head_dim:
            raise ConfigError(f"head_dim {self.head_dim} unsupported (must be even and divide 128)")
        if self.q_dim != self.hidden_size:
            raise ConfigError(f"num_heads*head_dim = {self.q_dim} != hidden_size {self.hidden_size}")

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def weight_params(self) -> int:
        """Parameters read per decode step (reference Weights::decode_bytes,
        engine/src/model/weights.rs:34-45, divided by 2 bytes)."""
        h, i = self.hidden_size, self.intermediate_size
        per_layer = 2 * h + self.qkv_dim * h + h * self.q_dim + 2 * i * h + h * i
        return self.num_layers * per_layer + h + self.vocab_size * h
