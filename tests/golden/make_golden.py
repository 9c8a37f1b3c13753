"""Generate the golden fixtures in tests/golden/ from HuggingFace transformers.

The reference (kvasir) ships no golden vectors and its Rust tests cannot run
here.  Its design names HuggingFace's Llama implementation as the numerical
target of the chain (reference DESIGN.md:57-64 for the rotate_half / llama3
RoPE convention, DESIGN.md:124-131 for logit matching against HF).  This
script runs transformers' own Llama modules -- LlamaRMSNorm,
LlamaRotaryEmbedding + apply_rotary_pos_emb, eager_attention_forward with
repeat_kv, the SiLU activation of LlamaMLP -- on small seeded inputs and
stores inputs (16-bit bit patterns) and HF outputs.  tests/test_oracle.py
checks the CPU oracle against them; the CUDA path is then checked against
the oracle.

Run from the repository root:  python tests/golden/make_golden.py
(needs transformers; the fixtures are committed, so test runs do not.)
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

LLAMA_3_2_1B = dict(
    hidden_size=2048, intermediate_size=8192, num_hidden_layers=16, num_attention_heads=32,
    num_key_value_heads=8, head_dim=64, vocab_size=128256, rms_norm_eps=1e-5,
    max_position_embeddings=131072, tie_word_embeddings=True,
    rope_theta=500000.0,
    rope_scaling={"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                  "original_max_position_embeddings": 8192, "rope_type": "llama3"},
)


def bits(t: torch.Tensor, dtype) -> np.ndarray:
    """Round to the 16-bit dtype and return the raw bit patterns as uint16."""
    return t.to(dtype).contiguous().view(torch.int16).numpy().view(np.uint16)


def up(b: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(b.view(np.int16).copy()).view(dtype).to(torch.float64)


def hf_config():
    from transformers import LlamaConfig
    cfg = LlamaConfig(**LLAMA_3_2_1B)
    return cfg


def gen_rope_tables(out):
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = hf_config()
    rot = LlamaRotaryEmbedding(cfg)
    inv = rot.inv_freq.detach().to(torch.float64).numpy()
    positions = np.array(list(range(64)) + [511, 512, 2047, 8191, 16383], np.int64)
    x = torch.zeros(1, len(positions), 64, dtype=torch.float32)
    cos, sin = rot(x, torch.from_numpy(positions)[None, :])
    out.update(
        rope_inv_freq=inv,
        rope_positions=positions,
        rope_cos=cos[0, :, :32].numpy().astype(np.float32),
        rope_sin=sin[0, :, :32].numpy().astype(np.float32),
    )


def gen_rmsnorm(out, rng):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm
    for name, rows, hidden in (("rmsnorm_llama", 4, 2048), ("rmsnorm_odd", 3, 100)):
        x = bits(torch.from_numpy(rng.normal(0, 1, (rows, hidden))), torch.bfloat16)
        w = bits(torch.from_numpy(1 + 0.02 * rng.normal(0, 1, hidden)), torch.bfloat16)
        norm = LlamaRMSNorm(hidden, eps=1e-5)
        with torch.no_grad():
            norm.weight.copy_(up(w, torch.bfloat16).to(torch.float32))
            y = norm(up(x, torch.bfloat16).to(torch.float32))
        out[f"{name}_x"] = x
        out[f"{name}_w"] = w
        out[f"{name}_y"] = y.numpy().astype(np.float32)


def gen_rope_apply(out, rng):
    """rotate_half RoPE on the q/k heads of qkv rows, HF formula in f64 with
    the cos/sin rows given explicitly (the table itself is pinned above)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    n_q, n_kv, hd, t, pos0 = 8, 2, 64, 5, 3
    qkv = bits(torch.from_numpy(rng.uniform(-2, 2, (t, (n_q + 2 * n_kv) * hd))), torch.bfloat16)
    # plain theta = 1e4 table, as the reference test builds it (tests/kernels.rs:84-96)
    half = hd // 2
    pos = np.arange(pos0 + t + 4, dtype=np.float64)
    freq = 1.0 / (10000.0 ** (2.0 * np.arange(half) / hd))
    ang = pos[:, None] * freq[None, :]
    cos_t = np.cos(ang).astype(np.float32)
    sin_t = np.sin(ang).astype(np.float32)
    v = up(qkv, torch.bfloat16).view(t, n_q + 2 * n_kv, hd)
    q = v[:, :n_q].transpose(0, 1)[None]          # [1, n_q, t, hd]
    k = v[:, n_q:n_q + n_kv].transpose(0, 1)[None]
    rows = slice(pos0, pos0 + t)
    c = torch.from_numpy(np.concatenate([cos_t[rows], cos_t[rows]], -1)).to(torch.float64)[None]
    s = torch.from_numpy(np.concatenate([sin_t[rows], sin_t[rows]], -1)).to(torch.float64)[None]
    qe, ke = apply_rotary_pos_emb(q, k, c, s)
    want = v.clone()
    want[:, :n_q] = qe[0].transpose(0, 1)
    want[:, n_q:n_q + n_kv] = ke[0].transpose(0, 1)
    out.update(rope_apply_qkv=qkv, rope_apply_cos=cos_t, rope_apply_sin=sin_t,
               rope_apply_want=want.reshape(t, -1).numpy().astype(np.float32),
               rope_apply_dims=np.array([n_q, n_kv, hd, t, pos0], np.int64))


class _Mod(torch.nn.Module):
    def __init__(self, groups):
        super().__init__()
        self.num_key_value_groups = groups


def gen_attention(out, rng):
    """Causal GQA attention with a KV prefix: HF eager attention in f64."""
    from transformers.models.llama.modeling_llama import eager_attention_forward
    cases = {"attn_prefill": (8, 2, 64, 7, 0, 32), "attn_prefix": (8, 2, 64, 4, 5, 32),
             "attn_decode": (32, 8, 64, 1, 40, 64)}
    for name, (n_q, n_kv, hd, t, pos0, max_seq) in cases.items():
        stride = (n_q + 2 * n_kv) * hd
        qkv = bits(torch.from_numpy(rng.normal(0, 1, (t, stride))), torch.bfloat16)
        kc = bits(torch.from_numpy(rng.normal(0, 1, (n_kv, max_seq, hd))), torch.bfloat16)
        vc = bits(torch.from_numpy(rng.normal(0, 1, (n_kv, max_seq, hd))), torch.bfloat16)
        L = pos0 + t
        q = up(qkv, torch.bfloat16).view(t, -1)[:, :n_q * hd].view(t, n_q, hd).transpose(0, 1)[None]
        k = up(kc, torch.bfloat16)[:, :L][None]
        v = up(vc, torch.bfloat16)[:, :L][None]
        qi = torch.arange(t)[:, None] + pos0
        kj = torch.arange(L)[None, :]
        mask = torch.where(kj <= qi, 0.0, float("-inf")).to(torch.float64)[None, None]
        o, _ = eager_attention_forward(_Mod(n_q // n_kv), q, k, v, mask, scaling=hd ** -0.5)
        out[f"{name}_qkv"] = qkv
        out[f"{name}_kc"] = kc
        out[f"{name}_vc"] = vc
        out[f"{name}_want"] = o[0].reshape(t, n_q * hd).numpy().astype(np.float32)
        out[f"{name}_dims"] = np.array([n_q, n_kv, hd, t, pos0, max_seq], np.int64)


def gen_silu(out, rng):
    t, inter = 3, 1000
    gu = bits(torch.from_numpy(rng.uniform(-6, 6, (t, 2 * inter))), torch.bfloat16)
    g = up(gu, torch.bfloat16)
    want = torch.nn.functional.silu(g[:, :inter]) * g[:, inter:]
    out.update(silu_gu=gu, silu_want=want.numpy().astype(np.float32),
               silu_dims=np.array([t, inter], np.int64))


def main():
    rng = np.random.default_rng(20261201)
    out: dict = {}
    gen_rope_tables(out)
    gen_rmsnorm(out, rng)
    gen_rope_apply(out, rng)
    gen_attention(out, rng)
    gen_silu(out, rng)
    path = os.path.join(HERE, "hf_llama_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
