"""Weight load path on the GPU (reference engine/src/model/weights.rs:47-230):
tensors land in device memory bit for bit as the conversions define them
(copy, IEEE round-to-nearest-even narrowing, the device bf16 -> f16 kernel with
its out-of-range counter), rows concatenate as the reference fuses q|k|v and
gate|up, and a decoder built from a loaded checkpoint equals one built from the
same weights directly."""
import json
import os

import numpy as np
import pytest
import torch

import st_util as S
from gpu_util import dev, host_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _values(rng, n):
    """N(0,1) plus edge values: signed zeros, f16 subnormals and their rounding
    ties, the f16 maximum and values just below the bf16 / f16 rounding points."""
    edge = np.array([0.0, -0.0, 1e-7, -3e-8, 5.9604645e-08, 2.9802322e-08, 6.1035156e-05,
                     65504.0, -65504.0, 65519.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, 3.14159265,
                     -2.5e-3, 1.0009765625, 1.00048828125], np.float32)
    return np.concatenate([rng.normal(0, 1, n - edge.size).astype(np.float32), edge])


def _f16_bits(x32):
    with np.errstate(over="ignore"):  # values above the FP16 range become inf, as on the device
        return np.asarray(x32, np.float32).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("src", ["BF16", "F16", "F32"])
@pytest.mark.parametrize("dst", ["bf16", "f16"])
def test_conversions_and_row_concat(tmp_path, src, dst):
    from kvasir_b200.weights import Checkpoint
    rng = np.random.default_rng(3)
    cols = 40
    a32, b32, v32 = _values(rng, 3 * cols), _values(rng, 5 * cols), _values(rng, cols)
    enc = {"BF16": lambda x, s: S.bf16(O.from_f32(x), s),
           "F16": lambda x, s: S.f16(x.astype(np.float16), s),
           "F32": lambda x, s: S.f32(x, s)}[src]
    S.write(tmp_path / "m.safetensors", {"a": enc(a32, (3, cols)), "b": enc(b32, (5, cols)),
                                         "v": enc(v32, (cols,))})
    # what each conversion defines, from the source values as stored
    stored = {"BF16": lambda x: O.to_f32(O.from_f32(x)), "F16": lambda x: x.astype(np.float16).astype(np.float32),
              "F32": lambda x: x}[src]
    want = lambda x: O.from_f32(stored(x)) if dst == "bf16" else _f16_bits(stored(x))
    tdt = torch.bfloat16 if dst == "bf16" else torch.float16
    out = torch.full((8 * cols,), float("nan"), dtype=tdt, device="cuda")
    vec = torch.empty(cols, dtype=tdt, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    with Checkpoint(str(tmp_path)) as ck:
        ck.load_rows([("a", 3), ("b", 5)], cols, out, bad)
        ck.load_rows([("v", 0)], cols, vec, bad)
        torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bits(out), np.concatenate([want(a32), want(b32)]))
    np.testing.assert_array_equal(host_bits(vec), want(v32))
    # 65504 and 65519 become 65536 in bf16: out of the FP16 range, counted on the device
    n_over = sum(int(np.sum(np.abs(stored(x)) > 65504.0)) for x in (a32, b32, v32))
    assert int(bad.item()) == (n_over if (src, dst) == ("BF16", "f16") else 0)


def test_bf16_to_f16_out_of_range_is_counted(tmp_path):
    """BF16 sources outside the FP16 range go through the device conversion and
    are counted (reference bf16_to_f16, engine/kernels/elementwise.cu:11-20)."""
    from kvasir_b200.weights import Checkpoint
    x = np.array([1.0, 7e4, -1e5, 65504.0, np.inf, np.nan, 2.0, 65536.0], np.float32)
    S.write(tmp_path / "m.safetensors", {"w": S.bf16(O.from_f32(x), (8,))})
    out = torch.empty(8, dtype=torch.float16, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    with Checkpoint(str(tmp_path)) as ck:
        ck.load_rows([("w", 0)], 8, out, bad)
        torch.cuda.synchronize()
    stored = O.to_f32(O.from_f32(x))
    assert int(bad.item()) == int(np.sum(~(np.abs(stored) <= 65504.0)))


def test_host_conversion_out_of_range_is_an_error(tmp_path):
    from kvasir_b200.gpu import CheckpointError
    from kvasir_b200.weights import Checkpoint
    S.write(tmp_path / "m.safetensors", {"w": S.f32(np.array([1.0, 7e4], np.float32), (2,)),
                                         "h": S.f16(np.array([1.0, np.inf], np.float16), (2,))})
    with Checkpoint(str(tmp_path)) as ck:
        with pytest.raises(CheckpointError, match="w: 1 values are non-finite or outside the FP16"):
            ck.load_rows([("w", 0)], 2, torch.empty(2, dtype=torch.float16, device="cuda"))
        with pytest.raises(CheckpointError, match="h: 1 values are non-finite"):
            ck.load_rows([("h", 0)], 2, torch.empty(2, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("src", ["BF16", "F32"])
def test_large_tensor_spans_staging_chunks(tmp_path, src):
    """9.4 M elements: more than one 8 M-element staging chunk, both buffers reused."""
    from kvasir_b200.weights import Checkpoint
    rng = np.random.default_rng(4)
    rows, cols = 4600, 2048
    bits = O.from_f32(rng.normal(0, 1, rows * cols).astype(np.float32))
    t = S.bf16(bits, (rows, cols)) if src == "BF16" else S.f32(O.to_f32(bits), (rows, cols))
    S.write(tmp_path / "m.safetensors", {"w": t})
    out = torch.empty(rows * cols, dtype=torch.bfloat16, device="cuda")
    with Checkpoint(str(tmp_path)) as ck:
        ck.load_rows([("w", rows)], cols, out)
        torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bits(out), bits)


def _tiny_cfg_json(tied: bool) -> dict:
    return {"hidden_size": 256, "intermediate_size": 512, "num_hidden_layers": 2,
            "num_attention_heads": 4, "num_key_value_heads": 1, "head_dim": 64,
            "vocab_size": 1000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
            "rope_scaling": {"factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                             "original_max_position_embeddings": 8192, "rope_type": "llama3"},
            "max_position_embeddings": 4096, "tie_word_embeddings": tied}


def _write_llama(tmp_path, cfg, rng, tied, split_files):
    """HuggingFace names, separate q/k/v and gate/up, over one or two shards."""
    h, i, q, kv, v = (cfg.hidden_size, cfg.intermediate_size, cfg.q_dim, cfg.kv_dim,
                      cfg.vocab_size)
    n = lambda k, s=0.05: O.from_f32(rng.normal(0, s, k).astype(np.float32))
    one = lambda: O.from_f32((1 + 0.02 * rng.normal(0, 1, h)).astype(np.float32))
    t = {"model.embed_tokens.weight": (n(v * h, 0.5), (v, h)), "model.norm.weight": (one(), (h,))}
    if not tied:
        t["lm_head.weight"] = (n(v * h, 0.5), (v, h))
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = (one(), (h,))
        t[p + "post_attention_layernorm.weight"] = (one(), (h,))
        t[p + "self_attn.q_proj.weight"] = (n(q * h), (q, h))
        t[p + "self_attn.k_proj.weight"] = (n(kv * h), (kv, h))
        t[p + "self_attn.v_proj.weight"] = (n(kv * h), (kv, h))
        t[p + "self_attn.o_proj.weight"] = (n(h * q), (h, q))
        t[p + "mlp.gate_proj.weight"] = (n(i * h), (i, h))
        t[p + "mlp.up_proj.weight"] = (n(i * h), (i, h))
        t[p + "mlp.down_proj.weight"] = (n(h * i), (h, i))
    names = sorted(t)
    shards = [names[: len(names) // 2], names[len(names) // 2:]] if split_files else [names]
    for k, part in enumerate(shards):
        S.write(tmp_path / f"model-{k:05d}.safetensors", {nm: S.bf16(*t[nm]) for nm in part},
                {"format": "pt"})
    (tmp_path / "config.json").write_text(json.dumps(_tiny_cfg_json(tied)))
    return {nm: bits for nm, (bits, _) in t.items()}


@pytest.mark.parametrize("tied", [True, False])
def test_decoder_from_checkpoint_equals_direct_weights(tmp_path, tied):
    from kvasir_b200.decoder import Decoder
    from kvasir_b200.weights import load_weights
    from kvasir_b200.config import LlamaConfig
    cfg0 = LlamaConfig.from_json(json.dumps(_tiny_cfg_json(tied)))
    raw = _write_llama(tmp_path, cfg0, np.random.default_rng(9), tied, split_files=not tied)
    cfg, w = load_weights(str(tmp_path))
    assert cfg.tie_word_embeddings == tied and ("lm_head" in w) == (not tied)
    h, i = cfg.hidden_size, cfg.intermediate_size
    # the fused layout, bit for bit
    np.testing.assert_array_equal(host_bits(w["embed"]).ravel(), raw["model.embed_tokens.weight"])
    np.testing.assert_array_equal(
        host_bits(w["w_qkv"][1]).ravel(),
        np.concatenate([raw[f"model.layers.1.self_attn.{x}_proj.weight"] for x in "qkv"]))
    np.testing.assert_array_equal(
        host_bits(w["w_gu"][0]).ravel(),
        np.concatenate([raw[f"model.layers.0.mlp.{x}_proj.weight"] for x in ("gate", "up")]))
    # the same weights handed over directly (untied: the LM head as a separate buffer)
    direct = {k: (x.clone() if torch.is_tensor(x) else [y.clone() for y in x]) for k, x in w.items()}
    n_seq, max_seq = 2, 64
    outs = []
    for weights in (w, direct):
        dec = Decoder(cfg, n_seq, max_seq, weights=weights)
        dec.fill_kv_normal(seed=5)
        dec.set_lengths([3, 17])
        dec.ids_in.copy_(torch.tensor([11, 500], dtype=torch.int32, device="cuda"))
        for _ in range(3):
            dec.step()
        torch.cuda.synchronize()
        outs.append((dec.logits.clone(), dec.ids_out.clone()))
        dec.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    if not tied:  # the head really is lm_head, not the embedding
        dec = Decoder(cfg, n_seq, max_seq, weights={k: x for k, x in w.items() if k != "lm_head"})
        dec.fill_kv_normal(seed=5)
        dec.set_lengths([3, 17])
        dec.ids_in.copy_(torch.tensor([11, 500], dtype=torch.int32, device="cuda"))
        for _ in range(3):
            dec.step()
        torch.cuda.synchronize()
        assert not torch.equal(dec.logits, outs[0][0])
        dec.close()


def test_load_weights_f16_target_counts_out_of_range(tmp_path):
    from kvasir_b200.config import LlamaConfig
    from kvasir_b200.gpu import CheckpointError
    from kvasir_b200.weights import load_weights
    cfg = LlamaConfig.from_json(json.dumps(_tiny_cfg_json(True)))
    raw = _write_llama(tmp_path, cfg, np.random.default_rng(2), True, split_files=False)
    _, w = load_weights(str(tmp_path), dtype=torch.float16)
    np.testing.assert_array_equal(host_bits(w["w_o"][0]).ravel(),
                                  _f16_bits(O.to_f32(raw["model.layers.0.self_attn.o_proj.weight"])))
    big = raw["model.norm.weight"].copy()
    big[:3] = O.from_f32(np.array([1e5, -7e4, np.inf], np.float32))
    S.write(tmp_path / "model-00001.safetensors", {"model.norm.weight": S.bf16(big, (cfg.hidden_size,))})
    with pytest.raises(CheckpointError, match="3 weights are non-finite or outside the FP16 range"):
        load_weights(str(tmp_path), dtype=torch.float16)
