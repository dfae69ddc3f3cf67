"""Batch sharding across GPUs: one process per GPU, weights replicated.

The spike-sparse convolution has no exchange step: every image (t, n) is an
independent unit, so N (dim 1 of a [T, N, C, H, W] tensor; dim 0 of a 4-D
one) is split into contiguous per-rank chunks and each rank runs its chunk on
its own GPU. No collective runs on the data path. The helpers here are the
host-side plumbing around that:

* ``shard_range`` / ``shard_batch``: the contiguous, balanced split.
* ``gather_shards``: collects every rank's output on all ranks (for
  verification or a host-side consumer; not part of a timed step).
* ``PeerMonitor``: step heartbeats through a ``torch.distributed`` store, so
  a rank learns on the host, between steps, that a peer stopped stepping
  (exited, crashed or hung) before it launches work that would wait on it.

The reference runs on one GPU; its benchmark shards nothing. The split over
N keeps each sample's T time steps (and LIF state) on one rank.
"""
from __future__ import annotations

import time
from typing import Dict, Optional, Tuple

import torch


def shard_range(n: int, world_size: int, rank: int) -> Tuple[int, int]:
    """[start, end) of rank's contiguous share of n units; sizes differ by at most one."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    if n < 0:
        raise ValueError("n must be non-negative")
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_dim(x: torch.Tensor) -> int:
    """The N dimension: 1 for [T, N, C, H, W], 0 for [N, C, H, W]."""
    if x.dim() == 5:
        return 1
    if x.dim() == 4:
        return 0
    raise ValueError(f"expected a 4-D or 5-D tensor, got {x.dim()}-D")


def shard_batch(x: torch.Tensor, world_size: int, rank: int) -> torch.Tensor:
    """This rank's slice of x along N (a view; no copy)."""
    d = batch_dim(x)
    s, e = shard_range(x.shape[d], world_size, rank)
    return x.narrow(d, s, e - s)


def gather_shards(y_local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather per-rank outputs (split by ``shard_range``) into the full tensor.

    Works on gloo (CPU tensors) and NCCL (CUDA tensors): shards are padded to
    the largest share, gathered, then trimmed and concatenated along N.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    d = batch_dim(y_local)
    sizes = [shard_range(n_total, world, r) for r in range(world)]
    longest = max(e - s for s, e in sizes)
    shape = list(y_local.shape)
    shape[d] = longest
    padded = torch.zeros(shape, dtype=y_local.dtype, device=y_local.device)
    padded.narrow(d, 0, y_local.shape[d]).copy_(y_local)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p.narrow(d, 0, e - s) for p, (s, e) in zip(parts, sizes)], dim=d)


class PeerFailure(RuntimeError):
    """A peer rank stopped advancing its step heartbeat within the timeout."""

    def __init__(self, ranks, step):
        super().__init__(f"rank(s) {sorted(ranks)} made no progress to step {step} within the timeout")
        self.ranks = sorted(ranks)
        self.step = step


class PeerMonitor:
    """Host-side liveness check between steps.

    Each rank calls ``beat(step)`` after finishing a step (no kernel or
    collective of that step still in flight on its side) and ``wait_peers(step)``
    before launching the next one. ``wait_peers`` returns once every peer has
    reported ``step`` and raises ``PeerFailure`` naming the ranks that did not
    within ``timeout_s`` of wall time, so a dead or hung peer is detected on
    the host instead of inside a collective or a spin on the GPU.
    """

    def __init__(self, store, rank: int, world_size: int, timeout_s: float = 5.0, prefix: str = "sf_hb",
                 poll_s: float = 0.01):
        self.store = store
        self.rank = rank
        self.world = world_size
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self.poll_s = poll_s

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), str(int(step)))

    def peer_steps(self) -> Dict[int, Optional[int]]:
        out: Dict[int, Optional[int]] = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            k = self._key(r)
            out[r] = int(self.store.get(k).decode()) if self.store.check([k]) else None
        return out

    def wait_peers(self, step: int) -> None:
        deadline = time.monotonic() + self.timeout_s
        while True:
            lagging = [r for r, s in self.peer_steps().items() if s is None or s < step]
            if not lagging:
                return
            if time.monotonic() >= deadline:
                raise PeerFailure(lagging, step)
            time.sleep(self.poll_s)
