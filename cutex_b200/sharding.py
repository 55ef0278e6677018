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


class FusedAllGatherGemm:
    """N-sharded GEMM whose epilogue also writes each finished tile into every peer's full D.

    Every rank holds a full ``d_full`` [M, N] (bf16). Rank r computes
    ``d_full[:, n0:n1]`` from all of A and its B slice; the kernel stores each
    finished chunk into its own copy and, over NVLink, into the same place of
    every peer's copy (``cutex_mxfp8_gemm_allgather``), so the gather overlaps
    the GEMM. The peer copies are mapped once with CUDA IPC (handles exchanged
    through ``group``). A call ends with a one-element all-reduce on the
    current stream; after it every rank's ``d_full`` is complete.
    """

    def __init__(self, m: int, n: int, k: int, group=None, config=None, device=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        from .kernels.dense_gemm import GemmConfig

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world < 2 or self.world > 8:
            raise ValueError("the fused all-gather needs 2..8 ranks on one node")
        self.shard = shard_bounds(n, self.world, self.rank)
        self.m, self.n, self.k = m, n, k
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.d_full = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        lib = _lib.load()
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_int64(0)
        _lib.check(lib.cutex_ipc_export(self.d_full.data_ptr(), handle, ctypes.byref(offset)), "cutex_ipc_export")
        entries = [None] * self.world
        dist.all_gather_object(entries, (handle.raw, offset.value), group=group)
        self._mappings = []
        peers = []
        for r, (h, off) in enumerate(entries):
            if r == self.rank:
                continue
            ptr, mapping = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(lib.cutex_ipc_import(h, off, ctypes.byref(ptr), ctypes.byref(mapping)), "cutex_ipc_import")
            self._mappings.append(mapping.value)
            peers.append(ptr.value + self.shard.n0 * 2)  # this rank's columns in peer r's copy
        self._peers = (ctypes.c_void_p * len(peers))(*peers)
        self._maps = torch.empty(128 * len(peers), dtype=torch.uint8, device=dev)
        self._cfg = (config or GemmConfig()).to_c()
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def __call__(self, a, b_local, sfa, sfb_local, stream=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        from .kernels.dense_gemm import _stream_handle

        handle = _stream_handle(stream)
        status = _lib.load().cutex_mxfp8_gemm_allgather(
            a.data_ptr(), b_local.data_ptr(), sfa.data_ptr(), sfb_local.data_ptr(),
            self.d_full.data_ptr() + self.shard.n0 * 2, self.m, self.shard.n, self.k, self.n, self._peers,
            len(self._peers), self._maps.data_ptr(), self._maps.numel(), ctypes.byref(self._cfg), handle)
        _lib.check(status, "cutex_mxfp8_gemm_allgather")
        # Cross-rank barrier in stream order: every rank's pushes have landed.
        s = stream if stream is not None and not isinstance(stream, int) else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            dist.all_reduce(self._flag, group=self.group)
        return self.d_full

    def close(self) -> None:
        from . import _lib

        lib = _lib.load()
        for mapping in self._mappings:
            lib.cutex_ipc_close(mapping)
        self._mappings = []


__all__ = ["SHARD_ALIGN", "FusedAllGatherGemm", "Shard", "allgather_columns", "scale_rows_slice", "shard_bounds"]
