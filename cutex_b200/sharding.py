"""N-sharding of one MXFP8 GEMM across the GPUs of a node (one process per GPU).

Rank r of g holds all of A[M,K] + SFA and the contiguous slice
B[n0:n1, :] + its SFB rows, and computes D[:, n0:n1]. There is no exchange in
the compute; slice boundaries are multiples of 256 rows of B so that every
slice starts on a 128-row scale block and on a 256-wide output tile. The
optional ``allgather_columns`` assembles the full row-major D[M, N] from the
slices with one NCCL all-gather plus a local re-layout.
"""

from __future__ import annotations

from dataclasses import dataclass

SHARD_ALIGN = 256


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    n0: int
    n1: int

    @property
    def n(self) -> int:
        return self.n1 - self.n0


def shard_bounds(n: int, world: int, rank: int, align: int = SHARD_ALIGN) -> Shard:
    """Contiguous, ``align``-aligned split of N over ``world`` ranks (last slice takes the rest)."""

    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n % align:
        raise ValueError(f"N={n} must be a multiple of {align} to shard on scale-block/tile boundaries")
    blocks = n // align
    if blocks < world:
        raise ValueError(f"N={n} has only {blocks} blocks of {align} for {world} ranks")
    base, extra = divmod(blocks, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return Shard(rank, world, start * align, stop * align)


def scale_rows_slice(shard: Shard, k: int) -> tuple[int, int]:
    """Byte range of a 128x4-swizzled scale buffer that holds rows [n0, n1) (whole 128-row blocks)."""

    per_block = 128 * (k // 32)
    return (shard.n0 // 128) * per_block, (shard.n1 // 128) * per_block


def allgather_columns(d_local, world: int, group=None):
    """All-gather column slices D[:, n0:n1] (equal widths) into a row-major D[M, N] (torch.distributed)."""

    import torch
    import torch.distributed as dist

    m, n_local = d_local.shape
    gathered = torch.empty((world * m, n_local), dtype=d_local.dtype, device=d_local.device)
    dist.all_gather_into_tensor(gathered, d_local.contiguous(), group=group)
    return gathered.view(world, m, n_local).permute(1, 0, 2).reshape(m, world * n_local)


__all__ = ["SHARD_ALIGN", "Shard", "allgather_columns", "scale_rows_slice", "shard_bounds"]
