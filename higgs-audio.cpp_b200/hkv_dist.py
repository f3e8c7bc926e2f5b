"""Multi-GPU placement for the paged KV engine: one process and one engine per GPU.

Two placements, neither of which exists in the reference (it runs every
request on CUDA device 0, src/higgs_pipeline.cpp:126):

* Slot sharding (independent requests).  A request lives on one rank for its
  whole life; every rank runs its own engine on its own slots and no data
  crosses GPUs.  ``shard_requests`` places request r on rank r % world;
  ``balanced_shards`` gives every rank the same number of requests with
  nearly the same total context (the step time of a rank is set by the K/V
  bytes it reads, so the slowest rank sets the job's).

* KV-head split (one long request).  Rank g of N holds KV heads
  [g*G/N, (g+1)*G/N) for all layers in its own engine (configured with
  n_head_kv = G/N and n_head = 4*G/N), so each rank reads only 1/N of the
  request's KV bytes.  Per layer every rank computes its query heads
  4*g*G/N .. and one all-gather assembles the head-major [n_head*head_dim]
  output in rank order, which is head order, before o_proj.
  ``HeadSplit`` does the slicing and the gather.

The collective runs through torch.distributed (NCCL on GPUs, gloo in the CPU
tests); every rank issues the same collectives in the same order.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence


def shard_requests(request_ids: Sequence[int], world: int, rank: int) -> List[int]:
    """Requests placed on `rank` (request id modulo world size)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return [r for r in request_ids if r % world == rank]


def balanced_shards(costs: Sequence[int], world: int) -> List[List[int]]:
    """Request indices grouped into `world` shards of equal size with nearly
    equal total cost (for decode attention the cost of a request is its
    context length: that many K/V rows are read per layer and step).  Longest
    first, each request to the lightest shard that still has room; ties go
    to the lower rank.  Deterministic, so every rank computes the same
    placement from the same list."""
    n = len(costs)
    if world <= 0 or n % world != 0:
        raise ValueError(f"{n} requests do not split into {world} equal shards")
    per = n // world
    order = sorted(range(n), key=lambda i: (-int(costs[i]), i))
    shards: List[List[int]] = [[] for _ in range(world)]
    total = [0] * world
    for i in order:
        r = min((r for r in range(world) if len(shards[r]) < per), key=lambda r: (total[r], r))
        shards[r].append(i)
        total[r] += int(costs[i])
    return [sorted(s) for s in shards]


def _contiguous(x):
    if hasattr(x, "contiguous"):
        return x.contiguous()  # torch
    import numpy as np
    return np.ascontiguousarray(x)


@dataclass(frozen=True)
class HeadSplit:
    """KV-head split of one request across `world` ranks."""

    world: int
    rank: int
    n_head_kv: int = 8
    gqa: int = 4
    head_dim: int = 128

    def __post_init__(self):
        if self.world <= 0 or self.n_head_kv % self.world != 0:
            raise ValueError(f"{self.n_head_kv} KV heads do not split over {self.world} ranks")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world of {self.world}")

    @property
    def local_kv_heads(self) -> int:
        return self.n_head_kv // self.world

    @property
    def local_q_heads(self) -> int:
        return self.local_kv_heads * self.gqa

    @property
    def kv_range(self) -> range:
        g = self.local_kv_heads
        return range(self.rank * g, (self.rank + 1) * g)

    @property
    def q_range(self) -> range:
        h = self.local_q_heads
        return range(self.rank * h, (self.rank + 1) * h)

    def engine_shape(self) -> dict:
        """n_head / n_head_kv for this rank's engine."""
        return {"n_head": self.local_q_heads, "n_head_kv": self.local_kv_heads}

    def slice_kv(self, x):
        """[..., n_head_kv, head_dim] -> this rank's KV heads (contiguous)."""
        r = self.kv_range
        return _contiguous(x[..., r.start:r.stop, :])

    def slice_q(self, x):
        """[..., n_head, head_dim] -> this rank's query heads (contiguous)."""
        r = self.q_range
        return _contiguous(x[..., r.start:r.stop, :])

    def gather_output(self, local_out, group=None):
        """All-gathers the per-rank [n, local_q_heads*head_dim] outputs into the
        head-major [n, n_head*head_dim] output (rank order == head order)."""
        import torch
        import torch.distributed as dist
        n = local_out.shape[0]
        width = self.local_q_heads * self.head_dim
        if self.world == 1:
            return local_out.reshape(n, width)
        flat = local_out.reshape(n, width).contiguous()
        full = torch.empty((self.world * n, width), dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(full, flat, group=group)
        return full.view(self.world, n, width).permute(1, 0, 2).reshape(n, self.world * width)
