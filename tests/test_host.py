"""Host-side logic without a GPU: config shapes (reference
engine/src/model/config.rs:144-172), sequence sharding, and the id gather
across ranks as world-size-2 gloo process groups."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kvasir_b200.config import ConfigError, LlamaConfig
from kvasir_b200.shard import gather_ids, shard_sequences

LLAMA_3_2_1B = """{
  "bos_token_id": 128000, "eos_token_id": 128001, "head_dim": 64, "hidden_size": 2048,
  "intermediate_size": 8192, "max_position_embeddings": 131072, "num_attention_heads": 32,
  "num_hidden_layers": 16, "num_key_value_heads": 8, "rms_norm_eps": 1e-05,
  "rope_scaling": {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
    "original_max_position_embeddings": 8192, "rope_type": "llama3"},
  "rope_theta": 500000.0, "tie_word_embeddings": true, "vocab_size": 128256 }"""


def test_parses_llama_3_2_1b():
    """config.rs:156-165"""
    c = LlamaConfig.from_json(LLAMA_3_2_1B)
    assert (c.qkv_dim, c.kv_dim) == (3072, 512)
    assert c.tie_word_embeddings
    assert c.rope_scaling["factor"] == 32.0
    assert c.group == 4


def test_rejects_unknown_rope_type():
    """config.rs:167-171"""
    with pytest.raises(ConfigError):
        LlamaConfig.from_json(LLAMA_3_2_1B.replace("llama3", "yarn"))


def test_rejects_bad_head_layout():
    with pytest.raises(ConfigError):
        LlamaConfig.from_json(LLAMA_3_2_1B.replace('"num_key_value_heads": 8', '"num_key_value_heads": 5'))


def test_decode_bytes_formula():
    """engine/src/model/weights.rs:34-45: 1,235,814,400 params for Llama-3.2-1B."""
    assert LlamaConfig.llama_3_2_1b().weight_params() == 1235814400


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (7, 3), (2, 4)])
def test_shards_cover_every_sequence_once(n, world):
    seen = []
    for r in range(world):
        s, c = shard_sequences(n, world, r)
        seen.extend(range(s, s + c))
    assert seen == list(range(n))
    sizes = [shard_sequences(n, world, r)[1] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, n_total, steps, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s, c = shard_sequences(n_total, world, rank)
        local = torch.arange(s, s + c, dtype=torch.int32)[None, :].repeat(steps, 1)
        local += torch.arange(steps, dtype=torch.int32)[:, None] * 1000
        full = gather_ids(local, n_total)
        q.put((rank, full.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_total", [256, 5])
def test_gather_ids_world_2_gloo(n_total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    steps = 3
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, n_total, steps, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [[step * 1000 + i for i in range(n_total)] for step in range(steps)]
    assert results[0] == want and results[1] == want


# ------------------------------------------------------------------ failure detection
# A CPU stand-in for the per-rank decode loop: each step maps ids to new ids, as
# the decoder does on the device.  One rank is made to fail (raise) or stall
# between steps; the other must get an error status naming it from the checked
# gather within the stated limit, instead of waiting in the collective for good.
GATHER_LIMIT_S = 2.0


def _standin_step(ids: torch.Tensor) -> torch.Tensor:
    return (ids * 31 + 7) % 128256


def _failure_worker(rank, world, port, mode, q):
    from kvasir_b200.shard import RankFailure, RankMonitor, gather_ids_checked
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    mon = RankMonitor()
    n_total, steps = 8, 4
    s, c = shard_sequences(n_total, world, rank)
    ids = torch.arange(s, s + c, dtype=torch.int32)
    table = []
    try:
        with mon.guard():
            for step in range(steps):
                if rank == 1 and step == 2:
                    if mode == "raise":
                        raise RuntimeError("stand-in step failed on purpose")
                    if mode == "stall":
                        time.sleep(3600)  # the test process terminates this rank
                mon.check()
                ids = _standin_step(ids)
                table.append(ids.clone())
        t0 = time.monotonic()
        full, st = gather_ids_checked(torch.stack(table), n_total, mon, timeout_s=GATHER_LIMIT_S)
        q.put((rank, st.ok, st.rank, st.reason, time.monotonic() - t0,
               None if full is None else full.tolist()))
    except RankFailure as e:  # seen between steps, before the gather
        q.put((rank, False, e.rank, str(e), 0.0, None))
    except RuntimeError as e:  # this rank's own failure
        q.put((rank, False, rank, f"raised: {e}", 0.0, None))
    if mode == "none":
        dist.destroy_process_group()
    q.close()
    q.join_thread()  # flush the report before the hard exit
    os._exit(0)


def _run_failure_case(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failure_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    want_reports = 2 if mode != "stall" else 1
    try:
        reports = {}
        for _ in range(want_reports):
            r = q.get(timeout=120)
            reports[r[0]] = r
    finally:
        for p in procs:
            if mode == "stall" and p is procs[1]:
                p.terminate()
            p.join(timeout=60)
    return reports


def test_checked_gather_all_ranks_healthy():
    reports = _run_failure_case("none")
    want = []
    ids = torch.arange(8, dtype=torch.int32)
    for _ in range(4):
        ids = _standin_step(ids)
        want.append(ids.tolist())
    for r in (0, 1):
        assert reports[r][1], reports[r][3]
        assert reports[r][5] == want


def test_checked_gather_names_a_rank_that_raised():
    reports = _run_failure_case("raise")
    ok, bad_rank, reason, waited = reports[0][1:5]
    assert not ok and bad_rank == 1
    assert "rank 1 failed" in reason and "on purpose" in reason
    assert waited < GATHER_LIMIT_S + 1.0  # seen between steps (0 s) or at the gather
    assert reports[1][1] is False  # the failing rank itself reports its own error


def test_checked_gather_times_out_on_a_stalled_rank():
    reports = _run_failure_case("stall")
    ok, bad_rank, reason, waited = reports[0][1:5]
    assert not ok and bad_rank == 1
    assert "did not reach" in reason
    assert GATHER_LIMIT_S - 0.1 <= waited < GATHER_LIMIT_S + 2.0
