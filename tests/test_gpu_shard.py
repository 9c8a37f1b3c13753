"""Sharding by sequence changes nothing a sequence computes: two ranks, each
with its own decoder, weights and shard of the KV caches (as bench.py's
ranks), give every sequence the logits of a one-rank run within the bf16
rounding bar, and the id table gathered from the two ranks holds each
sequence's ids at its global index.

The ranks are gloo processes on the same GPU: the kernels of one rank never
wait on the other's, so they may share a device.  Each rank seeds its contexts
by global sequence index (Decoder.fill_kv_normal(first_seq=...)), runs the
host-facing step, and gathers its ids with gather_ids_checked after the
steps.  The full Llama-3.2-1B shape at a short context.

Every step is fed the one-rank run's ids of the previous step (teacher
forcing), so each (sequence, step) can be compared: greedy picks on random
weights are often near ties (top-2 margins average ~0.2 at logit rms 0.9),
and a near tie decided the other way would change all later inputs.  The
per-rank batch is a different GEMM shape, so cuBLAS may sum in another order:
logits agree within LOGIT_TOL_FACTOR * LLAMA1B_LOGIT_SPREAD (a wrongly seeded
or misplaced sequence differs by the logits' own scale), and ids are equal
wherever the one-rank margin exceeds twice the row's logit difference."""
import os
import socket

import numpy as np
import pytest
import torch

from gpu_util import LLAMA1B_LOGIT_SPREAD, LOGIT_TOL_FACTOR

pytestmark = pytest.mark.gpu

N_TOTAL, CTX, STEPS = 8, 192, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_shard(world, rank, forced=None):
    """bench.py's per-rank set-up and host-facing loop at a reduced size.
    forced: [STEPS, N_TOTAL] ids whose row s - 1 feeds step s (None: the
    rank's own picks).  Returns the ids table [STEPS, n_local] and the logits
    [STEPS, n_local, vocab]."""
    from kvasir_b200.config import LlamaConfig
    from kvasir_b200.decoder import Decoder
    from kvasir_b200.shard import shard_sequences
    cfg = LlamaConfig.llama_3_2_1b()
    first, n_local = shard_sequences(N_TOTAL, world, rank)
    dec = Decoder(cfg, n_local, CTX + STEPS + 2, seed=0)
    dec.fill_kv_normal(seed=1000, first_seq=first)
    dec.set_lengths(CTX)
    ids0 = np.random.default_rng(7).integers(0, cfg.vocab_size, N_TOTAL).astype(np.int32)
    h_in = torch.from_numpy(ids0[first:first + n_local].copy()).pin_memory()
    h_out = torch.empty(n_local, dtype=torch.int32).pin_memory()
    table = torch.empty((STEPS, n_local), dtype=torch.int32)
    logits = np.empty((STEPS, n_local, cfg.vocab_size), np.float32)
    for i in range(STEPS):
        if forced is not None and i > 0:
            h_in.copy_(torch.from_numpy(forced[i - 1, first:first + n_local].copy()))
        dec.step_host(h_in, h_out)
        h_in.copy_(h_out)
        table[i].copy_(h_out)
        logits[i] = dec.logits.cpu().numpy()
    dec.close()
    return table, logits


def _rank_worker(rank, world, port, forced, q):
    import datetime

    import torch.distributed as dist

    from kvasir_b200.shard import RankMonitor, gather_ids_checked
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    try:
        torch.cuda.set_device(0)
        mon = RankMonitor()
        with mon.guard():
            table, logits = _run_shard(world, rank, forced)
        full, st = gather_ids_checked(table, N_TOTAL, mon, timeout_s=300.0)
        q.put((rank, st.ok, st.reason, None if full is None else full.numpy(), table.numpy(),
               logits))
    except Exception as e:  # noqa: BLE001 -- reported to the test process
        q.put((rank, False, f"{type(e).__name__}: {e}", None, None, None))
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_equals_one_rank_table():
    import torch.multiprocessing as mp

    from kvasir_b200.shard import shard_sequences
    one, one_logits = _run_shard(1, 0)
    one = one.numpy()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, one, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        reports = {}
        for _ in procs:
            r = q.get(timeout=900)
            reports[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=120)
    for r in (0, 1):
        assert reports[r][1], reports[r][2]
    two = reports[0][3]
    assert two.shape == (STEPS, N_TOTAL)
    np.testing.assert_array_equal(reports[1][3], two)  # every rank holds the same table
    bar = LOGIT_TOL_FACTOR * LLAMA1B_LOGIT_SPREAD
    compared = 0
    for r in (0, 1):
        first, n = shard_sequences(N_TOTAL, 2, r)
        np.testing.assert_array_equal(two[:, first:first + n], reports[r][4])  # placement
        d = np.abs(reports[r][5].astype(np.float64) - one_logits[:, first:first + n])
        assert d.max() <= bar, (r, d.max(axis=2))
        ol = one_logits[:, first:first + n]
        top2 = np.sort(ol, axis=2)[:, :, -2:]
        clear = (top2[:, :, 1] - top2[:, :, 0]) > 2 * d.max(axis=2)
        np.testing.assert_array_equal(two[:, first:first + n][clear], one[:, first:first + n][clear])
        compared += int(clear.sum())
    print(f"two-rank ids equal on {compared} of {STEPS * N_TOTAL} clear (sequence, step) pairs")
