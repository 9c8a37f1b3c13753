"""The decode-step driver (kvb_decoder_*) against the oracle's composed decode
step on a small Llama-shaped model: same weights, same prefilled KV cache,
several greedy steps.  Logits agree to within the bf16 activation rounding
that the two accumulation orders (cuBLAS f32 vs oracle f64) can flip;
greedy ids must agree wherever the oracle's top-2 margin is clear."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _tiny_cfg():
    from kvasir_b200.config import LlamaConfig
    return LlamaConfig(hidden_size=256, intermediate_size=512, num_layers=2, num_heads=4,
                       num_kv_heads=1, head_dim=64, vocab_size=1000, rms_norm_eps=1e-5,
                       rope_theta=500000.0, max_position_embeddings=4096)


def _weights_bits(rng, cfg):
    h, i = cfg.hidden_size, cfg.intermediate_size
    n = lambda k, s=0.05: O.from_f32(rng.normal(0, s, k).astype(np.float32))
    one = lambda: O.from_f32((1 + 0.02 * rng.normal(0, 1, h)).astype(np.float32))
    L = cfg.num_layers
    return dict(embed=n(cfg.vocab_size * h, 0.5), final_norm=one(),
                attn_norm=[one() for _ in range(L)], mlp_norm=[one() for _ in range(L)],
                w_qkv=[n(cfg.qkv_dim * h) for _ in range(L)], w_o=[n(h * cfg.q_dim) for _ in range(L)],
                w_gu=[n(2 * i * h) for _ in range(L)], w_down=[n(h * i) for _ in range(L)])


def _to_torch(wb, cfg):
    h, i = cfg.hidden_size, cfg.intermediate_size
    t = lambda b, *shape: dev(b).view(*shape)
    return dict(embed=t(wb["embed"], cfg.vocab_size, h), final_norm=t(wb["final_norm"], h),
                attn_norm=[t(b, h) for b in wb["attn_norm"]],
                mlp_norm=[t(b, h) for b in wb["mlp_norm"]],
                w_qkv=[t(b, cfg.qkv_dim, h) for b in wb["w_qkv"]],
                w_o=[t(b, h, cfg.q_dim) for b in wb["w_o"]],
                w_gu=[t(b, 2 * i, h) for b in wb["w_gu"]],
                w_down=[t(b, h, i) for b in wb["w_down"]])


@pytest.mark.parametrize("row_proj", [False, True])
def test_decoder_matches_oracle_steps(row_proj):
    """row_proj: the projections on kvb_linear_rows / kvb_linear_silu_mul instead of
    cuBLAS + kvb_silu_mul (same bars: both sum in f32)."""
    from kvasir_b200.decoder import Decoder
    from kvasir_b200.rope import cos_sin_table
    cfg = _tiny_cfg()
    rng = np.random.default_rng(21)
    n_seq, max_seq = 3, 96
    wb = _weights_bits(rng, cfg)
    dec = Decoder(cfg, n_seq, max_seq, weights=_to_torch(wb, cfg))
    dec.set_row_projections(row_proj)
    L, nkv, hd = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    # prefilled context: random K/V at positions < cur_len
    cur = np.array([5, 40, 64], np.int32)
    kv_shape = (L, n_seq, nkv, max_seq, hd)
    kc = O.from_f32(rng.normal(0, 1, int(np.prod(kv_shape))).astype(np.float32)).reshape(kv_shape)
    vc = O.from_f32(rng.normal(0, 1, int(np.prod(kv_shape))).astype(np.float32)).reshape(kv_shape)
    dec.kc.copy_(dev(kc).view(kv_shape))
    dec.vc.copy_(dev(vc).view(kv_shape))
    dec.set_lengths(cur)
    ids = np.array([3, 500, 999], np.int32)
    dec.ids_in.copy_(torch.from_numpy(ids).cuda())
    # oracle state, cache layout [seq][layer][...]
    okc = np.ascontiguousarray(kc.transpose(1, 0, 2, 3, 4))
    ovc = np.ascontiguousarray(vc.transpose(1, 0, 2, 3, 4))
    cos, sin = cos_sin_table(cfg, max_seq)
    dims = dict(hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_layers=L, n_q=cfg.num_heads,
                n_kv=nkv, head_dim=hd, vocab=cfg.vocab_size, max_seq=max_seq, eps=cfg.rms_norm_eps)
    pos = cur.copy()
    for step in range(4):
        dec.step()
        torch.cuda.synchronize()
        logits_want, ids_want = O.decode_step(dims, wb, cos, sin, okc, ovc, ids, pos)
        got = dec.logits.cpu().numpy()
        scale = np.abs(logits_want).max()
        assert np.abs(got - logits_want).max() <= 0.03 * scale + 0.02, f"step {step}"
        got_ids = dec.ids_out.cpu().numpy()
        top2 = np.sort(logits_want, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 0.1 * scale
        np.testing.assert_array_equal(got_ids[clear], ids_want[clear])
        # the cache slot of this step holds the rotated K / raw V of the new token
        new_k = host_bits(dec.kc).reshape(kv_shape)
        for b in range(n_seq):
            assert new_k[:, b, :, pos[b]].any()
        ids = got_ids.astype(np.int32)  # continue from the GPU's choice (drivers diverge otherwise)
        pos = pos + 1
    own, lib = dec.launches_per_step()
    # cuBLAS: qkv, o, gate/up, down per layer + the f32 LM head; rows: the LM head only
    assert own > 0 and lib == (1 if row_proj else 4 * L + 1)
    dec.close()


def test_decoder_step_host_equals_device_step():
    from kvasir_b200.decoder import Decoder
    cfg = _tiny_cfg()
    n_seq, max_seq = 4, 64
    a = Decoder(cfg, n_seq, max_seq, seed=5)
    b = Decoder(cfg, n_seq, max_seq, weights=a.w)
    for d in (a, b):
        d.kc.copy_(a.kc.normal_(0, 1) if d is a else a.kc)
        d.vc.copy_(a.vc.normal_(0, 1) if d is a else a.vc)
        d.set_lengths([10, 11, 12, 13])
    ids = torch.tensor([1, 2, 3, 4], dtype=torch.int32)
    a.ids_in.copy_(ids.cuda())
    outs_dev = []
    for _ in range(3):
        a.step()
        outs_dev.append(a.ids_out.cpu().clone())
    host_in = ids.clone().pin_memory()
    host_out = torch.empty(n_seq, dtype=torch.int32).pin_memory()
    outs_host = []
    for _ in range(3):
        b.step_host(host_in, host_out)
        outs_host.append(host_out.clone())
        host_in.copy_(host_out)
    for x, y in zip(outs_dev, outs_host):
        assert torch.equal(x, y)
    a.close()
    b.close()


@pytest.mark.parametrize("row_proj", [False, True])
def test_decoder_paged_cache_equals_contiguous(row_proj):
    """kvb_decoder_use_paged_cache: the same step over a shuffled pool of 64-key
    blocks (one block table for all layers) gives the same logits and ids, bit for
    bit, as the contiguous cache, step after step (the appended K/V included);
    with the cuBLAS projections and with kvb_linear_rows / kvb_linear_silu_mul."""
    from kvasir_b200.decoder import Decoder
    cfg = _tiny_cfg()
    rng = np.random.default_rng(23)
    n_seq, max_seq, bs = 3, 192, 64
    wb = _weights_bits(rng, cfg)
    L, nkv, hd = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    kv_shape = (L, n_seq, nkv, max_seq, hd)
    kc = dev(O.from_f32(rng.normal(0, 1, int(np.prod(kv_shape))).astype(np.float32))).view(kv_shape)
    vc = dev(O.from_f32(rng.normal(0, 1, int(np.prod(kv_shape))).astype(np.float32))).view(kv_shape)
    max_blocks = max_seq // bs
    n_blocks = n_seq * max_blocks + 2
    perm = torch.from_numpy(np.random.default_rng(5).permutation(n_blocks)[:n_seq * max_blocks]
                            .astype(np.int64)).cuda()
    table = perm.view(n_seq, max_blocks).to(torch.int32)
    kp = torch.zeros(L, n_blocks, nkv, bs, hd, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    blocks = lambda c: c.view(n_seq, nkv, max_blocks, bs, hd).permute(0, 2, 1, 3, 4).reshape(
        n_seq * max_blocks, nkv, bs, hd)
    for l in range(L):
        kp[l][perm] = blocks(kc[l])
        vp[l][perm] = blocks(vc[l])
    cur = np.array([5, 63, 120], np.int32)
    ids = torch.tensor([7, 300, 999], dtype=torch.int32, device="cuda")
    decs = []
    for paged in (False, True):
        d = Decoder(cfg, n_seq, max_seq, weights=_to_torch(wb, cfg))
        d.set_row_projections(row_proj)
        d.kc.copy_(kc)
        d.vc.copy_(vc)
        if paged:
            d.use_paged_cache(kp, vp, table, max_blocks, bs)
        d.set_lengths(cur)
        d.ids_in.copy_(ids)
        decs.append(d)
    for step in range(4):
        for d in decs:
            d.step()
        torch.cuda.synchronize()
        assert torch.equal(decs[0].logits, decs[1].logits), f"step {step}"
        assert torch.equal(decs[0].ids_out, decs[1].ids_out), f"step {step}"
    for d in decs:
        d.close()


def test_decoder_fused_lm_head_equals_unfused_ids():
    """kvb_decoder_set_fused_lm_head: greedy steps through kvb_lm_head_argmax give the
    unfused step's ids (kvb_linear's f32 logits + kvb_argmax_f32) wherever the
    unfused logits' top-2 margin exceeds twice the f32 rounding bound of the sums
    (hidden * 2^-24 * sum |x w|, at most ~1.2e-3 here); both decoders are fed the
    same ids every step.  The step launches one cuBLAS GEMM fewer and one kernel of
    this library more (the LM-head pass and the merge of its partials, in place of
    the argmax)."""
    from kvasir_b200.decoder import Decoder
    cfg = _tiny_cfg()
    n_seq, max_seq = 5, 64
    a = Decoder(cfg, n_seq, max_seq, seed=6)
    b = Decoder(cfg, n_seq, max_seq, weights=a.w)
    a.kc.normal_(0, 1)
    a.vc.normal_(0, 1)
    b.kc.copy_(a.kc)
    b.vc.copy_(a.vc)
    for d in (a, b):
        d.set_lengths([3, 20, 33, 40, 50])
    b.set_fused_lm_head(True)
    ids = torch.tensor([1, 22, 333, 444, 999], dtype=torch.int32, device="cuda")
    compared = 0
    for step in range(4):
        a.ids_in.copy_(ids)
        b.ids_in.copy_(ids)
        a.step()
        b.step()
        torch.cuda.synchronize()
        la = a.logits.cpu().numpy().astype(np.float64)
        top2 = np.sort(la, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 5e-3
        ia, ib = a.ids_out.cpu().numpy(), b.ids_out.cpu().numpy()
        np.testing.assert_array_equal(ib[clear], ia[clear])
        compared += int(clear.sum())
        ids = a.ids_out.clone()
    assert compared >= 15
    own_a, lib_a = a.launches_per_step()
    own_b, lib_b = b.launches_per_step()
    assert (own_b, lib_b) == (own_a + 1, lib_a - 1)
    a.close()
    b.close()


def test_fill_kv_by_global_index_is_the_same_paged_and_contiguous():
    """Decoder.fill_kv_normal(first_seq=g) gives each sequence the contents of its
    global index alone: a paged decoder (blocks scattered by its table) and a
    contiguous one seeded alike step to the same logits, bit for bit, and a decoder
    holding only sequences 2.. (first_seq=2) holds exactly their caches."""
    from kvasir_b200.decoder import Decoder
    cfg = _tiny_cfg()
    n_seq, max_seq = 4, 192
    a = Decoder(cfg, n_seq, max_seq, seed=8)
    b = Decoder(cfg, n_seq, max_seq, weights=a.w, seed=8, paged_block_size=64)
    c = Decoder(cfg, n_seq - 2, max_seq, weights=a.w, seed=8)
    a.fill_kv_normal(seed=5, first_seq=0)
    b.fill_kv_normal(seed=5, first_seq=0)
    c.fill_kv_normal(seed=5, first_seq=2)
    torch.testing.assert_close(c.kc, a.kc[:, 2:], rtol=0, atol=0)
    lens = np.array([7, 64, 100, 150], np.int32)
    ids = torch.tensor([5, 50, 500, 900], dtype=torch.int32, device="cuda")
    for d in (a, b):
        d.set_lengths(lens)
        d.ids_in.copy_(ids)
        d.step()
    torch.cuda.synchronize()
    assert torch.equal(a.logits, b.logits)
    assert torch.equal(a.ids_out, b.ids_out)
    for d in (a, b, c):
        d.close()
