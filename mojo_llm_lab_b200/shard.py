"""Row sharding of the large matvecs over ranks (one process per GPU).

The fused gate/up and the Q6_K vocabulary projection split their rows into
contiguous, equal blocks, one per rank; each rank runs the matvec on its block
and an all-gather (NCCL over NVLink on GPUs, gloo in the CPU tests) collects
the fp32 outputs.  The gathered buffer is rank-major:
[world, outputs, rows_per_rank]; `assemble` turns it into [outputs, rows].

Rows that do not divide evenly are padded up to world * rows_per_rank; the
padding rows of the last rank are zero weights and their outputs are dropped.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RowShard:
    rows: int
    world: int
    rank: int

    @property
    def per_rank(self) -> int:
        return -(-self.rows // self.world)

    @property
    def start(self) -> int:
        return min(self.rows, self.rank * self.per_rank)

    @property
    def stop(self) -> int:
        return min(self.rows, (self.rank + 1) * self.per_rank)

    @property
    def local_rows(self) -> int:
        return self.stop - self.start

    def slice_weights(self, flat: torch.Tensor, row_bytes: int) -> torch.Tensor:
        """This rank's rows of a flat byte tensor, zero-padded to per_rank rows."""
        mine = flat[self.start * row_bytes:self.stop * row_bytes]
        if self.local_rows == self.per_rank:
            return mine.clone()
        out = torch.zeros(self.per_rank * row_bytes, dtype=flat.dtype, device=flat.device)
        out[:mine.numel()] = mine
        return out


def all_gather_rows(local: torch.Tensor, shard: RowShard, group=None) -> torch.Tensor:
    """local: [outputs, per_rank] -> gathered [world, outputs, per_rank] (rank-major)."""
    if local.shape[-1] != shard.per_rank:
        raise ValueError("local output has the wrong number of rows")
    out = torch.empty((shard.world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out.view(-1), local.contiguous().view(-1), group=group)
    return out


def assemble(gathered: torch.Tensor, shard: RowShard) -> torch.Tensor:
    """[world, outputs, per_rank] -> [outputs, rows] in global row order."""
    world, outputs, per = gathered.shape
    full = gathered.permute(1, 0, 2).reshape(outputs, world * per)
    return full[:, :shard.rows]
