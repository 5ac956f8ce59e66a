"""Row sharding across GPUs (one process per GPU, torch.distributed).

Token rows are independent in every layer op (the norms reduce within a row
only), so a job splits into contiguous row ranges with no data exchange:

* row ops ([rows, hidden]):  rows [r0, r1) per rank, balanced to within one row;
* RoPE ([batch, heads, seq, head_dim]): along batch when there are at least as
  many batches as ranks, otherwise along seq, where a rank's slice starting at
  s0 is rotated with position_offset + s0 -- the reference's own
  position_offset parameter (src/lib.rs:821-827) makes a mid-sequence shard
  exact.

The collectives here are for timing and verification only: the maximum of
per-rank times, and gathering shards (or their checksums) to compare against
an unsharded run.  They work on any backend (gloo on CPU tensors, NCCL on
CUDA tensors).

Failure detection is on the host (PeerMonitor): before a collective, every
rank publishes its step in the process group's key-value store and waits,
with a deadline, for its peers' heartbeats.  A rank that failed, or stopped,
is reported as PeerFailure before the survivors enter a collective that would
wait for it; no GPU work is involved.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


def row_range(total_rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `total_rows` for `rank`; sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world or total_rows < 0:
        raise ValueError("bad shard arguments")
    base, extra = divmod(total_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class RopeShard:
    b0: int
    b1: int
    s0: int
    s1: int
    position_offset: int  # offset to pass to rope_embed for this shard


def rope_shard(batch: int, seq: int, position_offset: int, world: int, rank: int) -> RopeShard:
    """Shard of a [batch, heads, seq, head_dim] RoPE call for `rank`."""
    if batch >= world:
        b0, b1 = row_range(batch, world, rank)
        return RopeShard(b0, b1, 0, seq, position_offset)
    s0, s1 = row_range(seq, world, rank)
    return RopeShard(0, batch, s0, s1, position_offset + s0)


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. a CUDA-event time) over all ranks."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(shard: torch.Tensor, total_rows: int) -> torch.Tensor:
    """All-gathers row shards (as split by row_range) into the full tensor on every rank."""
    world, rank = dist.get_world_size(), dist.get_rank()
    counts = [row_range(total_rows, world, r)[1] - row_range(total_rows, world, r)[0] for r in range(world)]
    if shard.shape[0] != counts[rank]:
        raise ValueError("shard does not match row_range")
    # move raw bytes: every backend can all_gather uint8 (gloo has no 16-bit ints)
    raw = shard.contiguous().reshape(shard.shape[0], -1).view(torch.uint8)
    pad = torch.zeros((max(counts), raw.shape[1]), dtype=torch.uint8, device=shard.device)
    pad[: raw.shape[0]] = raw
    parts: List[torch.Tensor] = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    full = torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
    return full.view(shard.dtype).reshape(total_rows, *shard.shape[1:])


def checksum(t: torch.Tensor) -> int:
    """Order-sensitive 64-bit checksum of a tensor's bytes (same on CPU and GPU)."""
    b = t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32).reshape(-1).to(torch.int64)
    idx = torch.arange(b.numel(), device=b.device, dtype=torch.int64)
    return int(((b & 0xFFFF if t.element_size() == 2 else b) * (idx % 65521 + 1)).sum().item())


class PeerFailure(RuntimeError):
    """One or more peer ranks failed or stopped publishing heartbeats."""

    def __init__(self, ranks: Sequence[int], reason: str):
        super().__init__(f"rank(s) {list(ranks)}: {reason}")
        self.ranks, self.reason = list(ranks), reason


class PeerMonitor:
    """Heartbeats through a c10d key-value store (host only).

    beat(step) publishes this rank's step; wait_peers(step, timeout_s) returns
    once every peer has published a step >= `step`, and raises PeerFailure as
    soon as a peer has declared a failure (fail(reason)), or when the deadline
    passes with peers missing, or when the store itself is unreachable (the rank
    that hosts it is gone).  Call wait_peers between steps, before the next
    collective, with no kernels or collectives in flight.
    """

    def __init__(self, store, rank: int, world: int, prefix: str = "hrm/peer"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    @classmethod
    def for_default_group(cls, prefix: str = "hrm/peer") -> "PeerMonitor":
        """A monitor on the default process group's own key-value store (the one
        its rendezvous created), so no extra port or server is needed.  torch
        exposes that store only through distributed_c10d._get_default_store;
        pass a store to the constructor where that helper is missing."""
        from torch.distributed import distributed_c10d as c10d

        get = getattr(c10d, "_get_default_store", None)
        if get is None:
            raise RuntimeError("this torch has no distributed_c10d._get_default_store: "
                               "construct PeerMonitor(store, rank, world) with a store of your own")
        return cls(get(), dist.get_rank(), dist.get_world_size(), prefix)

    def _hb(self, r: int) -> str:
        return f"{self.prefix}/hb/{r}"

    def _fail(self, r: int) -> str:
        return f"{self.prefix}/fail/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._hb(self.rank), str(int(step)))

    def fail(self, reason: str) -> None:
        """Declares this rank failed (best effort: the store may be gone too)."""
        try:
            self.store.set(self._fail(self.rank), reason)
        except Exception:  # noqa: BLE001 - nothing more to report through
            pass

    def wait_peers(self, step: int, timeout_s: float = 10.0, poll_s: float = 0.005) -> None:
        deadline = time.monotonic() + timeout_s
        pending = set(range(self.world)) - {self.rank}
        try:
            while pending:
                for r in sorted(pending):
                    if self.store.check([self._fail(r)]):
                        raise PeerFailure([r], self.store.get(self._fail(r)).decode(errors="replace"))
                    if self.store.check([self._hb(r)]) and int(self.store.get(self._hb(r))) >= step:
                        pending.discard(r)
                if pending and time.monotonic() > deadline:
                    raise PeerFailure(sorted(pending), f"no heartbeat for step {step} within {timeout_s:g} s")
                if pending:
                    time.sleep(poll_s)
        except PeerFailure:
            raise
        except Exception as e:  # noqa: BLE001 - an unreachable store is a failed peer
            raise PeerFailure(sorted(pending), f"store unreachable: {type(e).__name__}: {e}") from e

    def sync(self, step: int, timeout_s: float = 10.0) -> None:
        """beat(step) then wait_peers(step)."""
        self.beat(step)
        self.wait_peers(step, timeout_s)
