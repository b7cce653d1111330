"""Data parallelism over independent audio streams (one process per GPU).

The path shards without any exchange: streams are independent, weights are
replicated, so a rank computes its streams alone and the only cross-rank
traffic is on the host: the shard map, each rank's results, and the
timings. Nothing here touches a GPU; ranks talk through a
torch.distributed store (TCP) or a gloo/NCCL process group.

- ``shard(n, world, rank)``: the streams of a rank (stream s goes to rank
  s mod world, so every rank's load differs by at most one stream).
- ``gather_results(store, world, rank, results, timeout_s)``: every rank
  publishes its results; rank 0 collects them and reports the ranks whose
  shard never arrived (a rank that raised, exited or hung) instead of
  waiting forever.
- ``max_over_ranks(x, group)``: the max of a per-rank timing, as bench.py
  reports multi-GPU time.
"""

from __future__ import annotations

import json
import time
from dataclasses import dataclass, field


def shard(n: int, world: int, rank: int) -> list[int]:
    """Streams of `rank`: s with s mod world == rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"dp: rank {rank} of {world}")
    return list(range(rank, n, world))


@dataclass
class Gathered:
    """What rank 0 collected: results per stream, and the missing ranks."""

    results: dict[int, object] = field(default_factory=dict)
    missing_ranks: list[int] = field(default_factory=list)
    missing_streams: list[int] = field(default_factory=list)

    @property
    def complete(self) -> bool:
        return not self.missing_ranks


def publish(store, rank: int, results: dict[int, object]) -> None:
    """Rank `rank` puts its {stream: result} map in the store."""
    store.set(f"dp/result/{rank}", json.dumps({str(k): v for k, v in results.items()}))


def gather_results(store, world: int, rank: int, n: int, results: dict[int, object],
                   timeout_s: float = 30.0, poll_s: float = 0.05) -> Gathered | None:
    """Publishes this rank's results; on rank 0 collects every rank's until
    timeout_s and reports the ranks (and streams) that never arrived.
    Other ranks return None."""
    publish(store, rank, results)
    if rank != 0:
        return None
    out = Gathered()
    pending = set(range(world))
    deadline = time.monotonic() + timeout_s
    while pending and time.monotonic() < deadline:
        for r in sorted(pending):
            key = f"dp/result/{r}"
            if store.check([key]):
                for k, v in json.loads(store.get(key)).items():
                    out.results[int(k)] = v
                pending.discard(r)
        if pending:
            time.sleep(poll_s)
    out.missing_ranks = sorted(pending)
    out.missing_streams = sorted(s for r in pending for s in shard(n, world, r))
    return out


def max_over_ranks(x: float, group=None) -> float:
    """The maximum of x over the ranks of `group` (a single process: x)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return float(x)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
