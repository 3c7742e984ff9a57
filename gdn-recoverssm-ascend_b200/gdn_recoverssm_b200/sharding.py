"""Value-head sharding of the verify + commit path over ranks.

The path has no cross-head term: a unit is one (sequence row, value head)
pair, verify reads that head's checkpoint tile and writes that head's
records and output, the fold reads and writes that head's tiles.  Ranks
therefore own disjoint value-head ranges (and the key heads those value heads
read, preserving the GQA ratio), exactly like the reference's tensor-parallel
head split, and nothing in the path communicates.  The only collective is the
benchmark's MAX of per-rank timings, outside the timed region.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    """Half-open head ranges owned by one rank."""

    key_begin: int
    key_end: int
    value_begin: int
    value_end: int

    @property
    def key_heads(self) -> int:
        return self.key_end - self.key_begin

    @property
    def value_heads(self) -> int:
        return self.value_end - self.value_begin


def head_shard(key_heads: int, value_heads: int, world: int, rank: int) -> HeadShard:
    """Rank ``rank`` of ``world`` owns value heads ``[r*HV/n, (r+1)*HV/n)`` and
    key heads ``[r*H/n, (r+1)*H/n)``; value head ``hv`` reads key head
    ``hv // (HV/H)``, which this split keeps on the same rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"GDN RecoverSSM: rank {rank} outside world {world}")
    if key_heads <= 0 or value_heads % key_heads:
        raise ValueError(f"GDN RecoverSSM: {value_heads} value heads are not a multiple of {key_heads} key heads")
    if key_heads % world or value_heads % world:
        raise ValueError(f"GDN RecoverSSM: {key_heads} key / {value_heads} value heads do not shard over {world} ranks")
    kh, vh = key_heads // world, value_heads // world
    return HeadShard(rank * kh, (rank + 1) * kh, rank * vh, (rank + 1) * vh)


def max_over_ranks(values, device=None):
    """MAX over ranks of a list of floats (one all-reduce); the identity when
    no process group is initialised."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
