"""Pins the CPU oracle (oracle/kvb_oracle.c) before it is trusted as the checker.

Sources of truth, in order:
  * the known-answer tests the reference holds for this path
    (engine/src/model/rope.rs:56-74, engine/src/model/config.rs:156-171, the
    exactness checks in engine/tests/kernels.rs),
  * golden vectors from HuggingFace transformers' Llama modules
    (tests/golden/hf_llama_golden.npz, made by tests/golden/make_golden.py),
  * independent numpy restatements for the pure arithmetic.
No GPU is needed.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


# ------------------------------------------------------------------ rounding
@pytest.mark.parametrize("dtype,tdt", [("bf16", torch.bfloat16), ("f16", torch.float16)])
def test_rounding_matches_torch(dtype, tdt):
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.normal(0, 1, 20000), rng.normal(0, 1e4, 2000), rng.normal(0, 1e-5, 2000),
        rng.uniform(-70000, 70000, 2000),
        [0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e-8, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
         1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -9, np.inf, -np.inf],
    ]).astype(np.float32)
    want = _bits(torch.from_numpy(x).to(tdt))
    got = O.from_f32(x, dtype)
    np.testing.assert_array_equal(got, want)
    back = O.to_f32(got, dtype)
    np.testing.assert_array_equal(back, torch.from_numpy(x).to(tdt).to(torch.float32).numpy())


# ------------------------------------------------------------------ rope tables (rope.rs KATs)
def test_llama3_scaling_regimes():
    """engine/src/model/rope.rs:56-68"""
    scaled = O.inv_freq(64, 500000.0, True)
    base = O.inv_freq(64, 500000.0, False)
    assert scaled[0] == base[0]
    assert abs(scaled[-1] - base[-1] / 32.0) < 1e-18
    assert np.all(scaled <= base)
    assert np.all(scaled[:-1] > scaled[1:])


def test_position_zero_is_identity():
    """engine/src/model/rope.rs:70-74"""
    c, s = O.cos_sin_table(64, 4, 500000.0, True)
    assert np.all(c[:32] == 1.0) and np.all(s[:32] == 0.0)


def test_rope_table_matches_hf(golden):
    inv = O.inv_freq(64, **{k: v for k, v in O.LLAMA3_ROPE.items()})
    np.testing.assert_allclose(inv, golden["rope_inv_freq"], rtol=5e-7)  # HF computes it in f32
    pos = golden["rope_positions"]
    c, s = O.cos_sin_table(64, int(pos.max()) + 1, **O.LLAMA3_ROPE)
    c = c.reshape(-1, 32)[pos]
    s = s.reshape(-1, 32)[pos]
    # HF evaluates the angle p*inv_freq in f32; the reference (and oracle) in f64
    tol = 1e-6 + 1.2e-7 * pos[:, None].astype(np.float64)
    assert np.all(np.abs(c - golden["rope_cos"]) <= tol)
    assert np.all(np.abs(s - golden["rope_sin"]) <= tol)


# ------------------------------------------------------------------ exact kernels
def test_embedding_gather_is_exact():
    """engine/tests/kernels.rs:31-48 shapes; out-of-range ids give zero rows."""
    rng = np.random.default_rng(1)
    vocab, hidden = 50, 300
    table = O.uniform16(rng, vocab * hidden, 2.0)
    ids = np.array([7, 0, 49, 7, 23], np.int32)
    out = O.embedding_gather(ids, table, hidden).reshape(5, hidden)
    t2 = table.reshape(vocab, hidden)
    for i, idx in enumerate(ids):
        np.testing.assert_array_equal(out[i], t2[idx])
    out = O.embedding_gather(np.array([-1, 50, 3], np.int32), table, hidden).reshape(3, hidden)
    assert not out[:2].any()
    np.testing.assert_array_equal(out[2], t2[3])


@pytest.mark.parametrize("dtype,npdt", [("f16", np.float16), ("bf16", None)])
def test_add_is_exact(dtype, npdt):
    """engine/tests/kernels.rs:162-175"""
    rng = np.random.default_rng(5)
    n = 10007
    x, y = O.uniform16(rng, n, 10.0, dtype), O.uniform16(rng, n, 10.0, dtype)
    got = O.add(x, y, dtype)
    s = O.to_f32(x, dtype) + O.to_f32(y, dtype)
    want = s.astype(np.float16).view(np.uint16) if npdt else _bits(
        torch.from_numpy(s).to(torch.bfloat16))
    np.testing.assert_array_equal(got, want)


def test_bf16_to_f16_counts_overflow():
    """engine/tests/kernels.rs:177-194"""
    rng = np.random.default_rng(6)
    src = _bits(torch.from_numpy(rng.uniform(-4, 4, 5000).astype(np.float32)).to(torch.bfloat16))
    src = src.copy()
    src[10] = _bits(torch.tensor([1.0e6]).to(torch.bfloat16))[0]
    src[20] = _bits(torch.tensor([-7.0e4]).to(torch.bfloat16))[0]
    dst, bad = O.bf16_to_f16(src)
    assert bad == 2
    want = O.to_f32(src, "bf16").astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(dst, want)


def test_kv_append_places_k_and_v():
    """engine/tests/kernels.rs:196-234"""
    rng = np.random.default_rng(7)
    n_q, n_kv, hd, t, pos0, max_seq = 4, 2, 64, 3, 5, 16
    stride = (n_q + 2 * n_kv) * hd
    qkv = O.uniform16(rng, t * stride, 2.0)
    z = np.zeros(n_kv * max_seq * hd, np.uint16)
    kc, vc = O.kv_append(qkv, z, z, t, pos0, n_q, n_kv, hd, max_seq)
    kc = kc.reshape(n_kv, max_seq, hd)
    vc = vc.reshape(n_kv, max_seq, hd)
    q3 = qkv.reshape(t, stride)
    for h in range(n_kv):
        for p in range(max_seq):
            if pos0 <= p < pos0 + t:
                r = q3[p - pos0]
                np.testing.assert_array_equal(kc[h, p], r[n_q * hd + h * hd:n_q * hd + (h + 1) * hd])
                np.testing.assert_array_equal(
                    vc[h, p], r[(n_q + n_kv) * hd + h * hd:(n_q + n_kv) * hd + (h + 1) * hd])
            else:
                assert not kc[h, p].any() and not vc[h, p].any()


# ------------------------------------------------------------------ floating-point kernels vs HF
@pytest.mark.parametrize("name", ["rmsnorm_llama", "rmsnorm_odd"])
def test_rmsnorm_matches_hf(golden, name):
    x, w, y = golden[f"{name}_x"], golden[f"{name}_w"], golden[f"{name}_y"]
    got = O.rmsnorm(x, w, y.shape[0], y.shape[1], 1e-5).reshape(y.shape)
    np.testing.assert_allclose(got, y, rtol=3e-6, atol=1e-6)


def test_rope_matches_hf_and_leaves_v(golden):
    n_q, n_kv, hd, t, pos0 = (int(v) for v in golden["rope_apply_dims"])
    qkv = golden["rope_apply_qkv"]
    got = O.rope(qkv, golden["rope_apply_cos"], golden["rope_apply_sin"], t, pos0, n_q, n_kv, hd)
    got = got.reshape(t, -1)
    np.testing.assert_allclose(got, golden["rope_apply_want"], rtol=1e-6, atol=1e-6)
    v0 = (n_q + n_kv) * hd
    np.testing.assert_array_equal(got[:, v0:], O.to_f32(qkv.reshape(t, -1)[:, v0:]))


@pytest.mark.parametrize("name", ["attn_prefill", "attn_prefix", "attn_decode"])
def test_attention_matches_hf(golden, name):
    n_q, n_kv, hd, t, pos0, max_seq = (int(v) for v in golden[f"{name}_dims"])
    got = O.attention(golden[f"{name}_qkv"], golden[f"{name}_kc"], golden[f"{name}_vc"], t, pos0,
                      n_q, n_kv, hd, max_seq)
    np.testing.assert_allclose(got.reshape(t, -1), golden[f"{name}_want"], rtol=1e-5, atol=1e-6)


def test_silu_mul_matches_hf(golden):
    t, inter = (int(v) for v in golden["silu_dims"])
    got = O.silu_mul(golden["silu_gu"], t, inter).reshape(t, inter)
    np.testing.assert_allclose(got, golden["silu_want"], rtol=1e-6, atol=1e-7)


# ------------------------------------------------------------------ internal consistency
def test_decode_attention_equals_single_sequence_attention():
    rng = np.random.default_rng(11)
    n_q, n_kv, hd, max_seq = 8, 2, 64, 40
    lens = np.array([1, 17, 40], np.int32)
    stride = (n_q + 2 * n_kv) * hd
    q = O.uniform16(rng, 3 * stride, 2.0).reshape(3, stride)
    kc = O.uniform16(rng, 3 * n_kv * max_seq * hd, 2.0).reshape(3, -1)
    vc = O.uniform16(rng, 3 * n_kv * max_seq * hd, 2.0).reshape(3, -1)
    got = O.attention_decode(q, stride, kc, vc, lens, n_q, n_kv, hd, max_seq, 1 / 8.0)
    got = got.reshape(3, -1)
    for b in range(3):
        want = O.attention(q[b], kc[b], vc[b], 1, int(lens[b]) - 1, n_q, n_kv, hd, max_seq)
        np.testing.assert_array_equal(got[b], want)


def test_linear_matches_numpy():
    """engine/tests/kernels.rs:318-364 shapes"""
    rng = np.random.default_rng(8)
    for t, i, o in ((3, 96, 50), (1, 2048, 777)):
        x, w = O.uniform16(rng, t * i, 1.0), O.uniform16(rng, o * i, 1.0)
        got = O.linear(x, w, t, i, o).reshape(t, o)
        want = O.to_f32(x).reshape(t, i).astype(np.float64) @ O.to_f32(w).reshape(o, i).T.astype(
            np.float64)
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


def test_argmax_first_index_and_nan():
    logits = np.array([[1, 3, 3, 2], [np.nan, -1, -1, np.nan], [-np.inf] * 4,
                       [np.nan, -np.inf, -np.inf, np.nan], [-np.inf, -np.inf, -np.inf, -3e38]],
                      np.float32)
    # nothing above -inf: index 0, whatever the row holds
    np.testing.assert_array_equal(O.argmax(logits, 5, 4), [1, 1, 0, 0, 3])


def test_threads_do_not_change_results():
    rng = np.random.default_rng(9)
    x, w = O.uniform16(rng, 4 * 256, 1.0), O.uniform16(rng, 300 * 256, 1.0)
    O.set_threads(1)
    a = O.linear(x, w, 4, 256, 300)
    O.set_threads(4)
    b = O.linear(x, w, 4, 256, 300)
    O.set_threads(1)
    np.testing.assert_array_equal(a, b)


def test_fill_normal_moments_and_determinism():
    a = O.fill_normal(200001, 0.0, 1.0, 42)
    O.set_threads(3)
    b = O.fill_normal(200001, 0.0, 1.0, 42)
    O.set_threads(1)
    np.testing.assert_array_equal(a, b)
    f = O.to_f32(a)
    assert abs(f.mean()) < 0.01 and abs(f.std() - 1.0) < 0.01


# ------------------------------------------------------------------ decode step composition
def _np_round(x, dtype="bf16"):
    return O.to_f32(O.from_f32(np.asarray(x, np.float32), dtype)).astype(np.float64)


def test_decode_step_matches_numpy_restatement():
    """The composed step against an independent numpy restatement of the
    planned forward pass (reference DESIGN.md:36-74) with the same rounding
    points."""
    rng = np.random.default_rng(12)
    H, I, L, n_q, n_kv, hd, V, S = 64, 96, 2, 4, 2, 16, 100, 12
    qd, kvd = n_q * hd, n_kv * hd
    f = lambda n, s=0.2: O.from_f32(rng.normal(0, s, n).astype(np.float32))
    W = dict(embed=f(V * H, 0.5), final_norm=O.from_f32(1 + 0.02 * rng.normal(0, 1, H)),
             attn_norm=[O.from_f32(1 + 0.02 * rng.normal(0, 1, H)) for _ in range(L)],
             mlp_norm=[O.from_f32(1 + 0.02 * rng.normal(0, 1, H)) for _ in range(L)],
             w_qkv=[f((qd + 2 * kvd) * H) for _ in range(L)], w_o=[f(H * qd) for _ in range(L)],
             w_gu=[f(2 * I * H) for _ in range(L)], w_down=[f(H * I) for _ in range(L)])
    dims = dict(hidden=H, inter=I, n_layers=L, n_q=n_q, n_kv=n_kv, head_dim=hd, vocab=V,
                max_seq=S, eps=1e-5)
    cos, sin = O.cos_sin_table(hd, S, 10000.0, False)
    n_seq = 2
    kc = np.zeros((n_seq, L, n_kv, S, hd), np.uint16)
    vc = np.zeros_like(kc)
    kc_np = np.zeros((n_seq, L, n_kv, S, hd))
    vc_np = np.zeros_like(kc_np)
    F = lambda a: O.to_f32(a).astype(np.float64)
    c2, s2 = cos.reshape(S, hd // 2), sin.reshape(S, hd // 2)

    def rms(x, w):
        return _np_round(x / np.sqrt(np.mean(x * x) + 1e-5) * F(w))

    ids = np.array([3, 77], np.int32)
    for step in range(4):
        pos = np.array([step, step + 2], np.int32)
        logits, out_ids = O.decode_step(dims, W, cos, sin, kc, vc, ids, pos)
        for b in range(n_seq):
            p = int(pos[b])
            x = F(W["embed"]).reshape(V, H)[ids[b]].copy()
            for l in range(L):
                h = rms(x, W["attn_norm"][l])
                qkv = _np_round(F(W["w_qkv"][l]).reshape(-1, H) @ h)
                heads = qkv[:qd + kvd].reshape(-1, hd).astype(np.float32)
                x0, x1 = heads[:, :hd // 2].copy(), heads[:, hd // 2:].copy()
                c, s = c2[p], s2[p]
                heads[:, :hd // 2] = x0 * c - x1 * s
                heads[:, hd // 2:] = x1 * c + x0 * s
                qkv[:qd + kvd] = _np_round(heads.reshape(-1))
                kc_np[b, l, :, p] = qkv[qd:qd + kvd].reshape(n_kv, hd)
                vc_np[b, l, :, p] = qkv[qd + kvd:].reshape(n_kv, hd)
                att = np.zeros(qd)
                for hh in range(n_q):
                    kv = hh // (n_q // n_kv)
                    sc = kc_np[b, l, kv, :p + 1] @ qkv[hh * hd:(hh + 1) * hd] / np.sqrt(hd)
                    pr = np.exp(sc - sc.max())
                    att[hh * hd:(hh + 1) * hd] = pr @ vc_np[b, l, kv, :p + 1] / pr.sum()
                att = _np_round(att)
                o = _np_round(F(W["w_o"][l]).reshape(H, qd) @ att)
                x = _np_round(x + o)
                h = rms(x, W["mlp_norm"][l])
                gu = _np_round(F(W["w_gu"][l]).reshape(-1, H) @ h)
                a = _np_round(gu[:I] / (1 + np.exp(-gu[:I])) * gu[I:])
                d = _np_round(F(W["w_down"][l]).reshape(H, I) @ a)
                x = _np_round(x + d)
            h = rms(x, W["final_norm"])
            want = F(W["embed"]).reshape(V, H) @ h
            np.testing.assert_allclose(logits[b], want, rtol=2e-3, atol=2e-3)
            np.testing.assert_array_equal(kc[b, :, :, p], O.from_f32(kc_np[b, :, :, p]))
        ids = out_ids


# ------------------------------------------------------------------ sampling restatement
def test_splitmix64_known_answers():
    """The first outputs of SplitMix64 from state 0 (the generator's published
    reference sequence): state advances by the golden gamma, output = mix(state)."""
    gamma, m64 = 0x9E3779B97F4A7C15, (1 << 64) - 1
    got = [O.splitmix64((i * gamma) & m64) for i in range(3)]
    assert got == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def test_sample_restatement_properties():
    rng = np.random.default_rng(5)
    logits = rng.normal(0, 2, (6, 500)).astype(np.float32)
    # a nucleus of ~0 mass keeps only the top token: the argmax
    np.testing.assert_array_equal(O.sample(logits, 1.0, 1e-9, 7), O.argmax(logits, 6, 500))
    # same seed and counters: same ids; the draw depends on the counter
    a = O.sample(logits, 0.8, 0.9, 11, counters=[1, 2, 3, 4, 5, 6])
    np.testing.assert_array_equal(a, O.sample(logits, 0.8, 0.9, 11, counters=[1, 2, 3, 4, 5, 6]))
    us = {O.sample_uniform(11, 0, c) for c in range(50)}
    assert len(us) == 50 and all(0.0 <= u < 1.0 for u in us)
    # ids stay inside the nucleus: the kept tokens' mass reaches top_p
    l = logits[0]
    w = np.exp((l - l.max()).astype(np.float64))
    order = np.argsort(-l)
    top = set(order[: int(np.searchsorted(np.cumsum(w[order]) / w.sum(), 0.5)) + 1].tolist())
    ids = O.sample(np.repeat(logits[:1], 200, 0), 1.0, 0.5, 3)
    assert set(ids.tolist()) <= top
    # NaN and -inf never win; an all -inf row gives 0
    bad = logits[:2].copy()
    bad[0, ::2] = np.nan
    bad[1, :] = -np.inf
    ids = O.sample(bad, 1.0, 1.0, 1)
    assert ids[0] % 2 == 1 and ids[1] == 0
