"""Independent-sequence sharding across ranks (one process per GPU).

Sequences are split into contiguous, as-equal-as-possible blocks; each rank
keeps a full weight replica and the KV cache of its block, and no data moves
between ranks during a step.  The only exchange is the gather of sampled token
ids, done on the host after the steps (`gather_ids`), over whatever
torch.distributed backend the process group uses (gloo on CPU tests, NCCL in
the bench).

Failure detection is host-side (the reference has typed errors only,
engine/src/error.rs:3-19).  A `RankMonitor` keeps a few keys in the process
group's key-value store: a rank that fails marks itself failed (its `guard()`
does this for any exception), and every rank marks its arrival at a gather.
`gather_ids_checked` waits for every rank's arrival mark with a time limit
before it enters the collective, so that a rank that raised, exited or stalled
between steps turns into an error status naming that rank, instead of a
collective that never completes.
"""
from __future__ import annotations

import contextlib
import dataclasses
import time

import torch


def shard_sequences(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(first sequence, count) owned by `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


@dataclasses.dataclass
class RankStatus:
    """Outcome of a checked wait: ok, or the first rank that failed (with its
    message) or did not arrive in time."""
    ok: bool
    rank: int | None = None
    reason: str = ""


class RankFailure(RuntimeError):
    def __init__(self, status: RankStatus):
        super().__init__(status.reason)
        self.status = status
        self.rank = status.rank


def _default_store():
    """The key-value store of the initialised default process group (under a prefix)."""
    import torch.distributed as dist
    from torch.distributed import distributed_c10d as c10d
    get = getattr(c10d, "_get_default_store", None)
    if get is None or not dist.is_initialized():
        raise RuntimeError("RankMonitor: no default process group store; pass store=")
    return dist.PrefixStore("kvb_monitor", get())


class RankMonitor:
    """Arrival and failure marks of this rank in a c10d store (by default the
    store of the initialised default process group)."""

    def __init__(self, store=None, rank: int | None = None, world: int | None = None):
        import torch.distributed as dist
        self.store = store if store is not None else _default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self._epoch = 0

    def _fkey(self, r: int) -> str:
        return f"failed/{r}"

    def report_failure(self, message: str) -> None:
        """Marks this rank failed; every later check on the other ranks sees it."""
        self.store.set(self._fkey(self.rank), message[:1000])

    @contextlib.contextmanager
    def guard(self):
        """Marks this rank failed if the body raises (the exception propagates)."""
        try:
            yield self
        except BaseException as e:  # noqa: BLE001 -- marked, then re-raised
            try:
                self.report_failure(f"{type(e).__name__}: {e}")
            finally:
                raise

    def failed_rank(self) -> RankStatus:
        """The lowest rank marked failed, if any (a cheap check between steps)."""
        for r in range(self.world):
            if r != self.rank and self.store.check([self._fkey(r)]):
                msg = self.store.get(self._fkey(r)).decode(errors="replace")
                return RankStatus(False, r, f"rank {r} failed: {msg}")
        return RankStatus(True)

    def check(self) -> None:
        """Raises RankFailure if another rank has marked itself failed."""
        st = self.failed_rank()
        if not st.ok:
            raise RankFailure(st)

    def wait_all(self, tag: str, timeout_s: float, poll_s: float = 0.02) -> RankStatus:
        """Marks this rank's arrival at `tag` and waits, at most timeout_s, for
        every other rank's mark.  Returns the first failed rank as soon as one
        is marked failed, or the first rank missing at the limit."""
        self.store.set(f"arrive/{tag}/{self.rank}", "1")
        deadline = time.monotonic() + timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            st = self.failed_rank()
            if not st.ok:
                return st
            pending = [r for r in pending if not self.store.check([f"arrive/{tag}/{r}"])]
            if not pending:
                return RankStatus(True)
            if time.monotonic() >= deadline:
                r = pending[0]
                return RankStatus(False, r, f"rank {r} did not reach '{tag}' within "
                                            f"{timeout_s:g} s")
            time.sleep(poll_s)

    def next_tag(self, name: str) -> str:
        self._epoch += 1
        return f"{name}/{self._epoch}"


def _all_gather_ids(local_ids: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    import torch.distributed as dist
    world = dist.get_world_size(group)
    steps = local_ids.shape[0]
    width = -(-n_total // world)  # ceil: pad every block to the same width
    dev = local_ids.device
    if dist.get_backend(group) == "nccl" and dev.type != "cuda":
        dev = torch.device("cuda", torch.cuda.current_device())
    pad = torch.full((steps, width), -1, dtype=torch.int32, device=dev)
    pad[:, :local_ids.shape[1]] = local_ids.to(dev)
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = torch.empty((steps, n_total), dtype=torch.int32)
    for r, p in enumerate(parts):
        s, c = shard_sequences(n_total, world, r)
        out[:, s:s + c] = p[:, :c].cpu()
    return out


def gather_ids(local_ids: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All ranks' [steps, local] int32 id blocks -> [steps, n_total] in
    sequence order (every rank receives the full table, on the host)."""
    return _all_gather_ids(local_ids, n_total, group)


def gather_ids_checked(local_ids: torch.Tensor, n_total: int, monitor: RankMonitor,
                       timeout_s: float = 30.0, group=None):
    """gather_ids behind an arrival check: every rank first marks its arrival
    in the store and waits at most timeout_s for the others.  Returns
    (table, RankStatus); the table is None when a rank failed or did not
    arrive, and then no collective was entered."""
    st = monitor.wait_all(monitor.next_tag("gather"), timeout_s)
    if not st.ok:
        return None, st
    return _all_gather_ids(local_ids, n_total, group), st
