"""Per-kernel measurements for BASELINE configs 1-4 (`bench.py --workload cfgN`).

Each config prints one JSON line per measured item.  Device times are CUDA
events on the launching stream after warm-up; HBM-bound kernels whose working
set fits in L2 are timed one launch at a time with an L2 flush between
launches (a 256 MB write, then a 256 MB read so that no dirty flush line is
left for the timed launch to write back; the flush is outside the timed
interval).  CPU numbers are the
oracle (oracle/, the reference's CPU-reference computations restated) on all
host cores, timed on the same inputs or a stated sample.
"""
from __future__ import annotations

import json
import math
import os
import time

import numpy as np
import torch

from kvasir_b200 import Gpu
from kvasir_b200.config import LlamaConfig
from kvasir_b200.rope import cos_sin_table

ROOT = os.path.dirname(os.path.abspath(__file__))


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class _Flusher:
    """L2 flush between timed launches: write a 256 MB buffer, then read another
    256 MB buffer.  The write evicts the previous launch's lines; the read leaves
    L2 holding clean lines only, so the timed launch does not pay for writing
    the flush's own dirty lines back to HBM."""

    def __init__(self):
        self.wbuf = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.rbuf = torch.ones(64 << 20, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.wbuf.zero_()
        torch.sum(self.rbuf)


def time_each(fn, reps: int, flush=None) -> float:
    """Mean ms of fn over reps launches, each bracketed by its own events
    (optionally after an L2 flush that is not timed)."""
    s = torch.cuda.current_stream()
    evs = []
    for _ in range(reps):
        if flush:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        evs.append((a, b))
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in evs]))


def time_loop(fn, reps: int) -> float:
    """Mean ms of reps back-to-back calls (for working sets far above L2)."""
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(s)
    for _ in range(reps):
        fn()
    b.record(s)
    b.synchronize()
    return a.elapsed_time(b) / reps


def _emit(d):
    print(json.dumps(d), flush=True)


def _cpu_threads():
    return os.cpu_count() or 1


def _bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


# ----------------------------------------------------------------------------- config 1
def cfg1(args):
    """One decoder layer's kernel chain at batch 1: embedding gather, RMSNorm,
    RoPE + KV append at position 512, GQA decode attention over 513 keys,
    SiLU*mul on one [1, 16384] gate/up row.  Launch-latency bound: reported as
    microseconds per chain, eager and as a CUDA graph."""
    from oracle import oracle as O
    cfg = LlamaConfig.llama_3_2_1b()
    g = Gpu(0)
    gen = torch.Generator(device="cuda").manual_seed(1)
    H, hd, nq, nkv, I, V = 2048, 64, 32, 8, 8192, 128256
    pos, max_seq = 512, 1024
    table = (torch.randn(V, H, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(H, generator=gen, device="cuda")).to(torch.bfloat16)
    ids = torch.randint(0, V, (1,), dtype=torch.int32, device="cuda", generator=gen)
    x = torch.empty(H, dtype=torch.bfloat16, device="cuda")
    h = torch.empty_like(x)
    qkv0 = torch.randn(cfg.qkv_dim, generator=gen, device="cuda").to(torch.bfloat16)
    qkv = qkv0.clone()
    kc = torch.randn(nkv * max_seq * hd, generator=gen, device="cuda").to(torch.bfloat16)
    vc = torch.randn(nkv * max_seq * hd, generator=gen, device="cuda").to(torch.bfloat16)
    c, s = cos_sin_table(cfg, max_seq)
    cos, sin = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    out = torch.empty(nq * hd, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(max(16, g.attention_workspace_bytes(1, pos, nq, nkv, hd)), dtype=torch.uint8,
                     device="cuda")
    gu = torch.randn(2 * I, generator=gen, device="cuda").to(torch.bfloat16)
    act = torch.empty(I, dtype=torch.bfloat16, device="cuda")

    def chain():
        g.embedding_gather(ids, table, x, H)
        g.rmsnorm(x, w, h, 1, H, 1e-5)
        g.rope_kv_append(qkv, cos, sin, kc, vc, 1, pos, nq, nkv, hd, max_seq)
        g.attention(qkv, kc, vc, out, 1, pos, nq, nkv, hd, max_seq, workspace=ws)
        g.silu_mul(gu, act, 1, I)

    # The same chain through the fused entry points: embedding + RMSNorm in one launch,
    # RoPE + KV append + decode attention in one (the new key at lens - 1 = pos).
    lens = torch.tensor([pos + 1], dtype=torch.int32, device="cuda")
    qkv_u = qkv0.clone()  # read unrotated by the fused attention, never modified
    dws = torch.empty(max(16, g.attention_decode_workspace_bytes(1, pos + 1, nq, nkv, hd)),
                      dtype=torch.uint8, device="cuda")

    def chain_fused():
        g.embedding_rmsnorm(ids, table, w, x, h, H, 1e-5)
        g.rope_attention_decode(qkv_u, cos, sin, kc, vc, nkv * max_seq * hd, lens, pos + 1, nq,
                                nkv, hd, max_seq, out, nq * hd, workspace=dws)
        g.silu_mul(gu, act, 1, I)

    def timed(fn):
        for _ in range(5):
            fn()
        eager = time_loop(fn, 200)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        g.stream = stream
        with torch.cuda.stream(stream):
            fn()  # warm on the capture stream
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=stream):
                fn()
        g.stream = torch.cuda.current_stream()
        for _ in range(5):
            graph.replay()
        return eager, time_loop(graph.replay, 500)

    eager_ms, graph_ms = timed(chain)
    fused_eager_ms, fused_graph_ms = timed(chain_fused)
    alg = (2 * H * 2) + (3 * H * 2) + (40 * hd * 2 * 2 + 8 * hd * 2 * 2 + 256 * 4) + \
          (513 * nkv * hd * 4 + 2 * nq * hd * 2) + (3 * I * 2)
    # CPU: the same chain through the oracle
    O.set_threads(_cpu_threads())
    tb, wb, qb = _bits(table), _bits(w), _bits(qkv0)
    kb, vb, gb = _bits(kc), _bits(vc), _bits(gu)
    idh = ids.cpu().numpy()
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 2.0 or n < 3:
        xb = O.embedding_gather(idh, tb, H)
        O.rmsnorm(xb, wb, 1, H, 1e-5)
        r = O.from_f32(O.rope(qb, c, s, 1, pos, nq, nkv, hd))
        k2, v2 = O.kv_append(r, kb, vb, 1, pos, nq, nkv, hd, max_seq)
        O.attention(r, k2, v2, 1, pos, nq, nkv, hd, max_seq)
        O.silu_mul(gb, 1, I)
        n += 1
    cpu_us = (time.perf_counter() - t0) / n * 1e6
    O.set_threads(1)
    _emit({"workload": "cfg1: one decoder layer chain, batch-1 decode at position 512 (513 keys)",
           "metric": "us per chain", "value": graph_ms * 1e3, "eager_us": eager_ms * 1e3,
           "graph_us": graph_ms * 1e3, "unit": "us", "higher_is_better": False,
           "launches_per_chain": 5 + (1 if ws.numel() > 16 else 0),
           "alg_bytes": alg, "gbs_informative": alg / (graph_ms * 1e-3) / 1e9,
           "cpu_oracle_us": cpu_us, "cpu_threads": _cpu_threads()})
    _emit({"workload": "cfg1 fused: the same chain through kvb_embedding_rmsnorm, "
                       "kvb_rope_attention_decode and kvb_silu_mul",
           "metric": "us per chain", "value": fused_graph_ms * 1e3,
           "eager_us": fused_eager_ms * 1e3, "graph_us": fused_graph_ms * 1e3, "unit": "us",
           "higher_is_better": False,
           "launches_per_chain": 3 + (1 if dws.numel() > 16 else 0),
           "alg_bytes": alg, "gbs_informative": alg / (fused_graph_ms * 1e-3) / 1e9})


# ----------------------------------------------------------------------------- config 2
def cfg2(args):
    """Batched decode attention: 64 sequences, lengths U[1, 4096], 32/8 heads,
    hd 64, N(0,1) Q/K/V, scale 1/8."""
    from oracle import oracle as O
    peaks, kind = _peaks()
    g = Gpu(0)
    rng = np.random.default_rng(2)
    n_seq, nq, nkv, hd, max_seq = 64, 32, 8, 64, 4096
    lens = rng.integers(1, max_seq + 1, n_seq).astype(np.int32)
    gen = torch.Generator(device="cuda").manual_seed(2)
    per = nkv * max_seq * hd
    q = torch.randn(n_seq * nq * hd, generator=gen, device="cuda").to(torch.bfloat16)
    kc = torch.empty(n_seq * per, dtype=torch.bfloat16, device="cuda").normal_(generator=gen)
    vc = torch.empty(n_seq * per, dtype=torch.bfloat16, device="cuda").normal_(generator=gen)
    out = torch.empty(n_seq * nq * hd, dtype=torch.bfloat16, device="cuda")
    lens_t = torch.from_numpy(lens).cuda()
    nb = g.attention_decode_workspace_bytes(n_seq, max_seq, nq, nkv, hd)
    ws = torch.empty(max(nb, 16), dtype=torch.uint8, device="cuda")

    def run():
        g.attention_decode(q, nq * hd, kc, vc, per, lens_t, max_seq, nq, nkv, hd, max_seq, out,
                           nq * hd, scale=0.125, workspace=ws)

    for _ in range(5):
        run()
    flush = _Flusher()
    ms = time_each(run, 50, flush)
    alg = int(lens.sum()) * nkv * hd * 2 * 2 + n_seq * nq * hd * 2 * 2
    gbs = alg / (ms * 1e-3) / 1e9
    O.set_threads(_cpu_threads())
    qb, kb, vb = _bits(q), _bits(kc), _bits(vc)
    t0 = time.perf_counter()
    O.attention_decode(qb, nq * hd, kb, vb, lens, nq, nkv, hd, max_seq, 0.125)
    cpu_s = time.perf_counter() - t0
    O.set_threads(1)
    _emit({"workload": "cfg2: batched decode attention, 64 seqs, lens U[1,4096], 32/8 heads, hd 64",
           "metric": "attention HBM GB/s", "value": gbs, "unit": "GB/s", "us": ms * 1e3,
           "alg_bytes": alg, "frac_of_peak": gbs / peaks["hbm_gbs"],
           "peak": f"{peaks['hbm_gbs']} GB/s ({kind})", "l2": "flushed between launches",
           "cpu_oracle_ms": cpu_s * 1e3, "cpu_threads": _cpu_threads(),
           "cpu_gbs": alg / cpu_s / 1e9})
    # The same keys in a paged cache: 64-key blocks of every sequence scattered
    # through one shuffled pool (kvb_attention_decode_paged); output checked equal.
    bs = 64
    max_blocks = max_seq // bs
    n_blocks = n_seq * max_blocks
    perm = torch.from_numpy(np.random.default_rng(3).permutation(n_blocks).astype(np.int64)).cuda()
    table = perm.view(n_seq, max_blocks).to(torch.int32)
    src = lambda c: c.view(n_seq, nkv, max_blocks, bs, hd).permute(0, 2, 1, 3, 4).reshape(
        n_blocks, nkv, bs, hd)
    kpool = torch.empty(n_blocks * nkv * bs * hd, dtype=torch.bfloat16, device="cuda")
    vpool = torch.empty_like(kpool)
    kpool.view(n_blocks, nkv, bs, hd)[perm] = src(kc)
    vpool.view(n_blocks, nkv, bs, hd)[perm] = src(vc)
    out_p = torch.empty_like(out)

    def run_paged():
        g.attention_decode_paged(q, nq * hd, kpool, vpool, table, max_blocks, bs, lens_t, max_seq,
                                 nq, nkv, hd, out_p, nq * hd, scale=0.125, workspace=ws)

    for _ in range(5):
        run_paged()
    ms_p = time_each(run_paged, 50, flush)
    gbs_p = alg / (ms_p * 1e-3) / 1e9
    _emit({"workload": "cfg2 paged: the same decode over a shuffled pool of 64-key blocks",
           "metric": "attention HBM GB/s", "value": gbs_p, "unit": "GB/s", "us": ms_p * 1e3,
           "alg_bytes": alg, "frac_of_peak": gbs_p / peaks["hbm_gbs"],
           "peak": f"{peaks['hbm_gbs']} GB/s ({kind})", "l2": "flushed between launches",
           "equal_to_contiguous": bool(torch.equal(out_p, out))})


# ----------------------------------------------------------------------------- config 3
def cfg3(args):
    """Prefill, batch 4 x 2048 tokens: RMSNorm [8192, 2048]; RoPE (llama3,
    positions 0..2047) fused with KV append into empty caches; causal GQA
    attention 32/8 heads hd 64 on tcgen05; SiLU*mul on [8192, 8192] gate/up."""
    from oracle import oracle as O
    peaks, kind = _peaks()
    cfg = LlamaConfig.llama_3_2_1b()
    g = Gpu(0)
    gen = torch.Generator(device="cuda").manual_seed(3)
    n_seq, T, H, hd, nq, nkv, I = 4, 2048, 2048, 64, 32, 8, 8192
    rows = n_seq * T
    flush = _Flusher()
    res = {}
    # RMSNorm
    x = torch.randn(rows * H, generator=gen, device="cuda").to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(H, generator=gen, device="cuda")).to(torch.bfloat16)
    y = torch.empty_like(x)
    f = lambda: g.rmsnorm(x, w, y, rows, H, 1e-5)
    f()
    ms = time_each(f, 30, flush)
    res["rmsnorm"] = (ms, rows * H * 2 * 2 + H * 2)
    # the same kernel on 4x the rows (268 MB in, 268 MB out: far above L2)
    x4 = torch.randn(4 * rows * H, generator=gen, device="cuda").to(torch.bfloat16)
    y4 = torch.empty_like(x4)
    f = lambda: g.rmsnorm(x4, w, y4, 4 * rows, H, 1e-5)
    f()
    res["rmsnorm [32768, 2048] (4x the rows)"] = (time_each(f, 30, flush), 4 * rows * H * 2 * 2 + H * 2)
    del x4, y4
    # RoPE + KV append (each sequence into its own empty cache)
    qkv = torch.randn(rows * cfg.qkv_dim, generator=gen, device="cuda").to(torch.bfloat16)
    qkv_work = qkv.clone()
    kc = torch.zeros(n_seq * nkv * T * hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    c, s = cos_sin_table(cfg, T)
    cos, sin = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    per_seq = T * cfg.qkv_dim

    def rope_all():  # one launch over the 4 sequences
        g.rope_kv_append_prefill(qkv_work, cos, sin, kc, vc, n_seq, T, 0, nq, nkv, hd, T)

    def rope_reset():
        qkv_work.copy_(qkv)
        flush()

    rope_all()
    ms = time_each(rope_all, 30, rope_reset)
    res["rope_kv_append"] = (ms, rows * ((nq + nkv) * hd * 2 * 2 + nkv * hd * 2 + 2 * nkv * hd * 2))
    # attention (tcgen05)
    out = torch.empty(rows * nq * hd, dtype=torch.bfloat16, device="cuda")
    att = lambda: g.attention_prefill(qkv_work, kc, vc, out, n_seq, T, 0, nq, nkv, hd, T)
    att()
    ms_att = time_each(att, 30, flush)
    flops = 4.0 * n_seq * nq * (T * (T + 1) / 2) * hd
    # The same prefill over a paged cache: 64-key blocks scattered through a pool.
    bs = 64
    max_blocks = T // bs
    n_blocks = n_seq * max_blocks
    perm = torch.from_numpy(np.random.default_rng(4).permutation(n_blocks).astype(np.int64)).cuda()
    table = perm.view(n_seq, max_blocks).to(torch.int32)
    blocks = lambda c: c.view(n_seq, nkv, max_blocks, bs, hd).permute(0, 2, 1, 3, 4).reshape(
        n_blocks, nkv, bs, hd)
    kpool = torch.empty_like(kc)
    vpool = torch.empty_like(vc)
    kpool.view(n_blocks, nkv, bs, hd)[perm] = blocks(kc)
    vpool.view(n_blocks, nkv, bs, hd)[perm] = blocks(vc)
    out_p = torch.empty_like(out)
    att_p = lambda: g.attention_prefill_paged(qkv_work, kpool, vpool, table, max_blocks, bs, out_p,
                                              n_seq, T, 0, nq, nkv, hd)
    att_p()
    ms_att_p = time_each(att_p, 30, flush)
    paged_equal = bool(torch.equal(out_p, out))
    # SiLU*mul
    gu = torch.randn(rows * 2 * I, generator=gen, device="cuda").to(torch.bfloat16)
    act = torch.empty(rows * I, dtype=torch.bfloat16, device="cuda")
    f = lambda: g.silu_mul(gu, act, rows, I)
    f()
    ms = time_each(f, 30, flush)
    res["silu_mul"] = (ms, rows * I * 2 * 3)
    for name, (ms, b) in res.items():
        gbs = b / (ms * 1e-3) / 1e9
        # A device-to-device copy moving the same bytes (b/2 read + b/2 written), timed the
        # same way: at working sets near the L2 size the launch and ramp of any kernel
        # are a large part of its time, and this copy is what the hardware gives there.
        src = torch.empty(b // 2, dtype=torch.uint8, device="cuda")
        dst = torch.empty_like(src)
        cp = lambda: dst.copy_(src)
        cp()
        cp_gbs = b / (time_each(cp, 30, flush) * 1e-3) / 1e9
        del src, dst
        _emit({"workload": f"cfg3: prefill 4 x 2048, {name}", "metric": "HBM GB/s", "value": gbs,
               "unit": "GB/s", "us": ms * 1e3, "alg_bytes": b, "frac_of_peak": gbs / peaks["hbm_gbs"],
               "peak": f"{peaks['hbm_gbs']} GB/s ({kind})", "l2": "flushed between launches",
               "same_bytes_copy_gbs": cp_gbs, "frac_of_same_bytes_copy": gbs / cp_gbs})
    tflops = flops / (ms_att * 1e-3) / 1e12
    # CPU: one (sequence, kv head) group of the causal attention, scaled to all 32
    O.set_threads(_cpu_threads())
    qb = _bits(qkv_work[:per_seq]).reshape(T, nq + 2 * nkv, hd)
    sub = np.ascontiguousarray(np.concatenate([qb[:, 0:4], qb[:, nq:nq + 1], qb[:, nq + nkv:nq + nkv + 1]], 1))
    kb = _bits(kc[:T * hd])
    vb = _bits(vc[:T * hd])
    t0 = time.perf_counter()
    O.attention(sub, kb, vb, T, 0, 4, 1, hd, T)
    cpu_s = (time.perf_counter() - t0) * (n_seq * nkv)
    O.set_threads(1)
    lib_ref = _library_prefill_reference(g, n_seq, T, nq, nkv, hd, flops, flush)
    _emit({"workload": "cfg3: prefill 4 x 2048, causal GQA attention 32/8 heads hd 64 (tcgen05)",
           "metric": "TFLOP/s", "value": tflops, "unit": "TFLOP/s", "us": ms_att * 1e3,
           "flops": flops, "frac_of_peak": tflops / peaks["bf16_tflops"],
           "peak": f"{peaks['bf16_tflops']} TFLOP/s ({kind}, burst)",
           "cpu_oracle_s_scaled": cpu_s, "cpu_sample": "1 of 32 (sequence, kv head) groups, x32",
           "cpu_threads": _cpu_threads(), "library_reference": lib_ref})
    tflops_p = flops / (ms_att_p * 1e-3) / 1e12
    _emit({"workload": "cfg3 paged: the same prefill attention over a shuffled pool of 64-key blocks",
           "metric": "TFLOP/s", "value": tflops_p, "unit": "TFLOP/s", "us": ms_att_p * 1e3,
           "flops": flops, "frac_of_peak": tflops_p / peaks["bf16_tflops"],
           "peak": f"{peaks['bf16_tflops']} TFLOP/s ({kind}, burst)",
           "equal_to_contiguous": paged_equal})


def _library_prefill_reference(g, n_seq, T, nq, nkv, hd, flops, flush):
    """torch SDPA with the cuDNN backend on the same shapes (causal, bf16), timed the
    same way: what NVIDIA's own attention reaches on this GPU at head_dim 64.  A
    comparison only; nothing of this library runs through it.  K and V are expanded
    to the query heads (cuDNN's GQA support varies by version).  Its accuracy is
    reported beside its speed: the largest difference from this library's f32 rows
    (kvb_attention_prefill_f32, within ~1e-5 of the f64 oracle on these shapes) and
    the share of its bf16 outputs outside this library's 16-bit attention bar,
    2e-3 + 2^-8 |want|."""
    import torch.nn.functional as F
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        gen = torch.Generator(device="cuda").manual_seed(5)
        q = torch.randn(n_seq, nq, T, hd, generator=gen, device="cuda").to(torch.bfloat16)
        k = torch.randn(n_seq, nkv, T, hd, generator=gen, device="cuda").to(torch.bfloat16)
        v = torch.randn(n_seq, nkv, T, hd, generator=gen, device="cuda").to(torch.bfloat16)
        k = k.repeat_interleave(nq // nkv, dim=1).contiguous()
        v = v.repeat_interleave(nq // nkv, dim=1).contiguous()
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            f = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True)
            for _ in range(3):
                f()
            ms = time_each(f, 30, flush)
            lib_out = f()
        # the same inputs through this library: q in the qkv rows, K / V as the caches
        stride = (nq + 2 * nkv) * hd
        qkv = torch.zeros(n_seq, T, stride, dtype=torch.bfloat16, device="cuda")
        qkv[:, :, :nq * hd] = q.permute(0, 2, 1, 3).reshape(n_seq, T, nq * hd)
        kc = k[:, ::nq // nkv].contiguous()
        vc = v[:, ::nq // nkv].contiguous()
        out32 = torch.empty(n_seq * T * nq * hd, dtype=torch.float32, device="cuda")
        g.attention_prefill_f32(qkv.reshape(-1), kc.reshape(-1), vc.reshape(-1), out32, n_seq, T,
                                0, nq, nkv, hd, T)
        want = out32.view(n_seq, T, nq, hd).permute(0, 2, 1, 3).double()
        err = (lib_out.double() - want).abs()
        outside = (err > 2e-3 + 2.0 ** -8 * want.abs()).double().mean()
        return {"impl": "torch SDPA, cuDNN backend (K/V expanded to 32 heads)",
                "tflops": flops / (ms * 1e-3) / 1e12, "us": ms * 1e3,
                "max_abs_err_vs_f32_rows": float(err.max()),
                "share_outside_16bit_attention_bar": float(outside)}
    except Exception as e:  # a torch build without the backend
        return {"impl": "torch SDPA, cuDNN backend", "unavailable": str(e).splitlines()[0][:200]}


# ----------------------------------------------------------------------------- config 4
def cfg4(args):
    """Full 16-layer decode, context 1024, batch 1 and 32, 256 greedy steps
    from uniform random prompt ids (random-init weights, N(0,1) context KV)."""
    from kvasir_b200.decoder import Decoder
    peaks, kind = _peaks()
    cfg = LlamaConfig.llama_3_2_1b()
    steps, ctx = 256, 1024
    weights = None
    for B in (1, 32):
        dec = Decoder(cfg, B, ctx + steps + 8, weights=weights, seed=0)
        weights = dec.w
        dec.fill_kv_normal(seed=4)
        dec.set_lengths(ctx)
        rng = np.random.default_rng(4)
        dec.ids_in.copy_(torch.from_numpy(rng.integers(0, cfg.vocab_size, B).astype(np.int32)).cuda())
        for _ in range(3):
            dec.step()
        dec.set_lengths(ctx)
        torch.cuda.synchronize()
        s = torch.cuda.current_stream()
        if getattr(args, "ncu_window", False) and B == 1:
            torch.cuda.profiler.start()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        for _ in range(steps):
            dec.step()
        b.record(s)
        b.synchronize()
        ms = a.elapsed_time(b)
        tps = B * steps / (ms * 1e-3)
        # bytes per step: weights + KV read at the mean context of the run
        kv = B * (ctx + steps / 2) * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * 2 * 2
        step_bytes = dec.weight_bytes() + kv + B * cfg.vocab_size * 4
        roof_tps = B / (step_bytes / (peaks["hbm_gbs"] * 1e9))
        own, lib = dec.launches_per_step()
        _emit({"workload": f"cfg4: 16-layer decode, batch {B}, context 1024, 256 greedy steps",
               "metric": "tokens/s", "value": tps, "unit": "tokens/s", "ms_per_step": ms / steps,
               "bytes_per_step": step_bytes, "hbm_roofline_tokens_s": roof_tps,
               "frac_of_roofline": tps / roof_tps, "peak": f"{peaks['hbm_gbs']} GB/s ({kind})",
               "lm_head": "cuBLAS f32 logits + kvb_argmax_f32",
               "launches_per_step": {"own": own, "cublas": lib}})
        # the same greedy steps with the LM head and the argmax in one pass, then also
        # with the projections on kvb_linear_rows / kvb_linear_silu_mul
        fused_bytes = step_bytes - B * cfg.vocab_size * 4
        for rows_proj in (False, True):
            dec.set_fused_lm_head(True)
            dec.set_row_projections(rows_proj)
            dec.set_lengths(ctx)
            for _ in range(3):
                dec.step()
            dec.set_lengths(ctx)
            torch.cuda.synchronize()
            a.record(s)
            for _ in range(steps):
                dec.step()
            b.record(s)
            b.synchronize()
            ms_f = a.elapsed_time(b)
            own, lib = dec.launches_per_step()
            _emit({"workload": f"cfg4: 16-layer decode, batch {B}, context 1024, 256 greedy steps, "
                               f"LM head + argmax fused" +
                               (", projections on kvb_linear_rows" if rows_proj else ""),
                   "metric": "tokens/s", "value": B * steps / (ms_f * 1e-3), "unit": "tokens/s",
                   "ms_per_step": ms_f / steps, "bytes_per_step": fused_bytes,
                   "frac_of_roofline": (B * steps / (ms_f * 1e-3)) /
                                       (B / (fused_bytes / (peaks["hbm_gbs"] * 1e9))),
                   "lm_head": "kvb_lm_head_argmax (f32 logits never stored)",
                   "projections": ("kvb_linear_rows + kvb_linear_silu_mul" if rows_proj
                                   else "cuBLAS (autotuned) + kvb_silu_mul"),
                   "launches_per_step": {"own": own, "cublas": lib}})
        dec.set_fused_lm_head(False)
        dec.set_row_projections(False)
        # the same steps with device-side temperature / top-p sampling in place of argmax,
        # and the two sampling kernels alone on this step's logits
        dec.set_sampling(0.8, 0.95, seed=1)
        dec.set_lengths(ctx)
        for _ in range(3):
            dec.step()
        dec.set_lengths(ctx)
        torch.cuda.synchronize()
        a.record(s)
        for _ in range(steps):
            dec.step()
        b.record(s)
        b.synchronize()
        ms_s = a.elapsed_time(b)
        g = Gpu(0)
        ids = torch.empty(B, dtype=torch.int32, device="cuda")
        lg = dec.logits.reshape(-1)
        us = {}
        for name, fn in (("argmax", lambda: g.argmax(lg, B, cfg.vocab_size, ids)),
                         ("sample", lambda: g.sample(lg, B, cfg.vocab_size, ids, 0.8, 0.95, 1))):
            for _ in range(3):
                fn()
            us[name] = time_loop(fn, 50) * 1e3
        _emit({"workload": f"cfg4: 16-layer decode, batch {B}, context 1024, 256 steps sampled "
                           f"on the device (temperature 0.8, top-p 0.95)",
               "metric": "tokens/s", "value": B * steps / (ms_s * 1e-3), "unit": "tokens/s",
               "ms_per_step": ms_s / steps, "greedy_ms_per_step": ms / steps,
               "kernel_us": {"argmax": us["argmax"], "top_p_sample": us["sample"]}})
        dec.close()
        del dec
        torch.cuda.empty_cache()


def sample(args):
    """kvb_sample_f32 alone: rows of 128,256 f32 logits drawn N(0, 5^2) (peaked) or
    N(0, 0.1^2) (flat), temperature 0.8, top_p 1.0 / 0.95 / 0.5; 1 row (16-CTA
    clusters) and 32 rows (8-CTA clusters).  The logits stay in L2 between the
    back-to-back calls, as the decoder's do between its LM head and the draw."""
    g = Gpu(0)
    vocab = 128256
    torch.manual_seed(0)
    for sd in (5.0, 0.1):
        for rows in (1, 32):
            x = (torch.randn(rows, vocab, device="cuda") * sd).reshape(-1)
            ids = torch.empty(rows, dtype=torch.int32, device="cuda")
            for _ in range(5):
                g.argmax(x, rows, vocab, ids)
            argmax_us = time_loop(lambda: g.argmax(x, rows, vocab, ids), 200) * 1e3
            us = {}
            for top_p in (1.0, 0.95, 0.5):
                fn = lambda: g.sample(x, rows, vocab, ids, 0.8, top_p, 7)
                for _ in range(5):
                    fn()
                us[str(top_p)] = time_loop(fn, 200) * 1e3
            _emit({"workload": f"sample: {rows} row(s) of {vocab} logits N(0, {sd}^2), "
                               "temperature 0.8", "metric": "us per call", "unit": "us",
                   "top_p_us": us, "argmax_us": argmax_us})



# ----------------------------------------------------------------------------- LM head + argmax
def lmhead(args):
    """The tied Llama-3.2-1B LM head (128256 x 2048 bf16, 525 MB) and greedy argmax
    for 1, 8 and 32 rows: kvb_lm_head_argmax (one pass, logits never stored)
    against kvb_linear (cuBLAS, f32 logits, autotuned) + kvb_argmax_f32.  The
    weights are far above L2, so back-to-back launches read them from HBM."""
    peaks, kind = _peaks()
    g = Gpu(0)
    H, V = 2048, 128256
    gen = torch.Generator(device="cuda").manual_seed(9)
    w = torch.empty(V * H, dtype=torch.bfloat16, device="cuda").normal_(0, 0.02, generator=gen)
    from kvasir_b200 import _lib as L
    import ctypes as C
    blas = C.c_void_p()
    L.lib().kvb_blas_create(C.byref(blas))
    L.lib().kvb_blas_set_autotune(blas, 1)
    for B in (1, 8, 32):
        x = torch.randn(B * H, generator=gen, device="cuda").to(torch.bfloat16)
        ids_f = torch.empty(B, dtype=torch.int32, device="cuda")
        ids_u = torch.empty(B, dtype=torch.int32, device="cuda")
        y = torch.empty(B * V, dtype=torch.float32, device="cuda")
        ws = torch.empty(int(L.lib().kvb_lm_head_argmax_workspace_bytes(B)), dtype=torch.uint8,
                         device="cuda")
        fused = lambda: g.lm_head_argmax(x, w, B, H, V, ids_f, workspace=ws)

        def unfused():
            s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            L.lib().kvb_linear(blas, s, C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(w.data_ptr()),
                               w.numel(), C.c_void_p(y.data_ptr()), y.numel(), B, H, V, L.KVB_BF16, 1)
            g.argmax(y, B, V, ids_u)

        for f in (fused, unfused):
            for _ in range(3):
                f()
        torch.cuda.synchronize()
        us_f = time_loop(fused, 30) * 1e3
        us_u = time_loop(unfused, 30) * 1e3
        wb = V * H * 2
        _emit({"workload": f"LM head + greedy argmax, {B} rows, vocab {V}, hidden {H}",
               "metric": "us", "value": us_f, "unit": "us", "fused_us": us_f,
               "cublas_plus_argmax_us": us_u, "fused_weight_gbs": wb / (us_f * 1e-6) / 1e9,
               "frac_of_peak": wb / (us_f * 1e-6) / 1e9 / peaks["hbm_gbs"],
               "ids_equal": bool(torch.equal(ids_f, ids_u)),
               "peak": f"{peaks['hbm_gbs']} GB/s ({kind})"})
    L.lib().kvb_blas_destroy(blas)


# ----------------------------------------------------------------------------- config 5 kernel
def attn5(args):
    """The config-5 step's dominant launch alone: RoPE + KV append + split-KV decode
    attention (kvb_rope_attention_decode, decode + combine) over one layer's cache of
    `--seqs` sequences at `--context` keys (+ the new one).  Sized by --seqs so that
    a profiler capture can run it on a small case (8 sequences: 269 MB of K/V, above
    L2)."""
    peaks, kind = _peaks()
    g = Gpu(0)
    n_seq, ctx = args.seqs, args.context
    nq, nkv, hd = 32, 8, 64
    max_seq = ctx + 8
    qkv_dim = (nq + 2 * nkv) * hd
    gen = torch.Generator(device="cuda").manual_seed(5)
    per = nkv * max_seq * hd
    kc = torch.empty(n_seq * per, dtype=torch.bfloat16, device="cuda").normal_(generator=gen)
    vc = torch.empty(n_seq * per, dtype=torch.bfloat16, device="cuda").normal_(generator=gen)
    qkv = torch.randn(n_seq * qkv_dim, generator=gen, device="cuda").to(torch.bfloat16)
    cos, sin = cos_sin_table(LlamaConfig.llama_3_2_1b(), max_seq)
    cos_t, sin_t = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    lens_host = np.full(n_seq, ctx + 1, np.int32)
    lens = torch.from_numpy(lens_host).cuda()
    out = torch.empty(n_seq * nq * hd, dtype=torch.bfloat16, device="cuda")
    nb = g.attention_decode_workspace_bytes(n_seq, max_seq, nq, nkv, hd)
    ws = torch.empty(max(nb, 16), dtype=torch.uint8, device="cuda")

    def run():
        g.rope_attention_decode(qkv, cos_t, sin_t, kc, vc, per, lens, max_seq, nq, nkv, hd,
                                max_seq, out, nq * hd, workspace=ws)

    for _ in range(3):
        run()
    reps = max(3, min(50, args.steps))
    ms = time_loop(run, reps) if n_seq * per * 4 > (1 << 30) else time_each(run, reps, _Flusher())
    alg = (int(lens_host.sum()) * nkv * hd * 2 * 2 + n_seq * qkv_dim * 2 +
           n_seq * 2 * nkv * hd * 2 + n_seq * nq * hd * 2)
    gbs = alg / (ms * 1e-3) / 1e9
    _emit({"workload": f"cfg5 attention launch: RoPE + KV append + split-KV decode, {n_seq} seqs "
                       f"x {ctx + 1} keys, 32/8 heads, hd 64, one layer",
           "metric": "attention HBM GB/s", "value": gbs, "unit": "GB/s", "us": ms * 1e3,
           "alg_bytes": alg, "frac_of_peak": gbs / peaks["hbm_gbs"],
           "peak": f"{peaks['hbm_gbs']} GB/s ({kind})",
           "l2": "K/V above L2" if n_seq * per * 4 > (1 << 30) else "flushed between launches"})


# ----------------------------------------------------------------------------- projections
def proj(args):
    """The decode step's four projections of Llama-3.2-1B for `--seqs` rows (qkv
    2048 -> 3072, o 2048 -> 2048, down 8192 -> 2048, gate/up 2048 -> 2 x 8192 +
    SiLU*mul): kvb_linear_rows / kvb_linear_silu_mul against kvb_linear (cuBLAS,
    autotuned) + kvb_silu_mul.  Each is timed as a chain of 24 calls on 24
    different weight matrices (together above L2) captured in one CUDA graph, as
    the decode step runs them, alone and with an RMSNorm launch in front of every
    call (the step's order).  `--steps 0` runs each form once, uncaptured (a
    profiler target)."""
    from kvasir_b200 import _lib as L
    import ctypes as C
    peaks, kind = _peaks()
    s = torch.cuda.Stream()
    g = Gpu(0, stream=s)
    lib = L.lib()
    blas_ws = torch.empty(32 << 20, dtype=torch.uint8, device="cuda")
    lib.kvb_blas_set_workspace(g._blas, C.c_void_p(blas_ws.data_ptr()), blas_ws.numel())
    lib.kvb_blas_set_autotune(g._blas, 1)
    rows, R = args.seqs, 24
    gen = torch.Generator(device="cuda").manual_seed(3)

    def graph_us(calls, reps=20):
        with torch.cuda.stream(s):
            for c in calls:
                c()
        s.synchronize()
        if args.steps == 0:
            return float("nan")
        G = torch.cuda.CUDAGraph()
        with torch.cuda.graph(G, stream=s):
            for c in calls:
                c()
        with torch.cuda.stream(s):
            G.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                G.replay()
            e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps / len(calls) * 1e3

    with torch.cuda.stream(s):
        for name, k, out, glu in (("qkv", 2048, 3072, False), ("o", 2048, 2048, False),
                                  ("down", 8192, 2048, False), ("gate/up + SiLU*mul", 2048, 8192, True)):
            n_w = 2 * out if glu else out
            ws = [torch.empty(n_w * k, dtype=torch.bfloat16, device="cuda").normal_(0, 0.02, generator=gen)
                  for _ in range(R)]
            x = torch.randn(rows * k, generator=gen, device="cuda").to(torch.bfloat16)
            nw = torch.ones(k, dtype=torch.bfloat16, device="cuda")
            h = torch.empty_like(x)
            y = torch.empty(rows * out, dtype=torch.bfloat16, device="cuda")
            gu = torch.empty(rows * 2 * out, dtype=torch.bfloat16, device="cuda") if glu else None

            def call(i, pre, mine):
                def f():
                    src = x
                    if pre:
                        g.rmsnorm(x, nw, h, rows, k, 1e-5)
                        src = h
                    if mine:
                        if glu:
                            g.linear_silu_mul(src, ws[i], y, rows, k, out)
                        else:
                            g.linear_rows(src, ws[i], y, rows, k, out)
                    elif glu:
                        g.linear_f16(src, ws[i], gu, rows, k, 2 * out)
                        g.silu_mul(gu, y, rows, out)
                    else:
                        g.linear_f16(src, ws[i], y, rows, k, out)
                return f

            res = {pre: {mine: graph_us([call(i, pre, mine) for i in range(R)]) for mine in (True, False)}
                   for pre in (False, True)}
            wb = n_w * k * 2
            _emit({"workload": f"{name} projection, {rows} rows, Llama-3.2-1B", "metric": "us",
                   "value": res[False][True], "unit": "us per call (graph chain)",
                   "linear_rows_us": res[False][True], "cublas_us": res[False][False],
                   "after_rmsnorm": {"linear_rows_us": res[True][True], "cublas_us": res[True][False]},
                   "weight_bytes": wb,
                   "weight_gbs": wb / (res[False][True] * 1e-6) / 1e9,
                   "frac_of_peak": wb / (res[False][True] * 1e-6) / 1e9 / peaks["hbm_gbs"],
                   "peak": f"{peaks['hbm_gbs']} GB/s ({kind})"})
            del ws
    assert g.device_error() == 0


def run(name, args):
    {"cfg1": cfg1, "cfg2": cfg2, "cfg3": cfg3, "cfg4": cfg4, "sample": sample,
     "attn5": attn5, "lmhead": lmhead, "proj": proj}[name](args)
