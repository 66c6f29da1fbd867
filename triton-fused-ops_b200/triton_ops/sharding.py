"""Token-row sharding across GPUs (one process per GPU).

Every op on the hot path is independent per token row, so a batch
[batch, seq_len, hidden] is split into contiguous row slabs, one per rank,
with no collective on the data path. The only communication is a one-time
broadcast of the weights / RoPE tables from a source rank (NCCL over NVLink on
GPUs, gloo on CPU for tests). RoPE positions stay global: a slab that starts
at global row r0 uses position (r0 + i) % seq_len for its i-th row, so each
rank receives the cos/sin rows its slab needs.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, List

import torch


@dataclass(frozen=True)
class RowShard:
    rank: int
    world_size: int
    start: int  # first global row (inclusive)
    stop: int  # last global row (exclusive)

    @property
    def rows(self) -> int:
        return self.stop - self.start


def shard_rows(total_rows: int, world_size: int, rank: int) -> RowShard:
    """Contiguous, balanced slab of `total_rows` for `rank` (sizes differ by at most one)."""
    if world_size <= 0 or not (0 <= rank < world_size):
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    if total_rows < 0:
        raise ValueError("total_rows must be non-negative")
    base, extra = divmod(total_rows, world_size)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return RowShard(rank, world_size, start, stop)


def shard_positions(shard: RowShard, seq_len: int) -> torch.Tensor:
    """Global RoPE positions ((start + i) % seq_len) of a slab's rows."""
    return torch.arange(shard.start, shard.stop, dtype=torch.int64) % seq_len


def slab_tables(cos: torch.Tensor, sin: torch.Tensor, shard: RowShard, seq_len: int):
    """cos/sin rows for a slab whose rows are fed to the kernel as one sequence.

    When the slab starts on a sequence boundary and covers whole sequences, the
    original tables are used unchanged (batch = rows // seq_len). Otherwise the
    per-row positions are gathered so the slab can run as a single sequence of
    `shard.rows` tokens.
    """
    if shard.start % seq_len == 0 and shard.rows % seq_len == 0:
        return cos, sin, shard.rows // seq_len, seq_len
    pos = shard_positions(shard, seq_len).to(cos.device)
    return cos.index_select(0, pos).contiguous(), sin.index_select(0, pos).contiguous(), 1, shard.rows


def broadcast_tensors(tensors: Iterable[torch.Tensor], src: int = 0, group=None) -> List[torch.Tensor]:
    """In-place broadcast of each tensor from `src` (setup only, never on the hot path)."""
    import torch.distributed as dist

    out = []
    for t in tensors:
        dist.broadcast(t, src=src, group=group)
        out.append(t)
    return out
