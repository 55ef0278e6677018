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

    Every rank holds full [M, N] bf16 result buffers. Rank r computes its
    columns ``[n0, n1)`` from all of A and its B slice; the kernel stores each
    finished chunk into its own buffer and, over NVLink, into the same place of
    every peer's buffer (``cutex_mxfp8_gemm_allgather``), so the gather overlaps
    the GEMM. The peers' buffers are mapped once with CUDA IPC (handles
    exchanged through ``group``). A call ends with a one-element all-reduce on
    the call's stream; after it every rank's result is complete.

    Two result buffers alternate between calls. Call k+1's peer stores go to
    the other buffer, and call k+2's (into this buffer again) start only after
    every rank has reached call k+1's closing all-reduce on its stream. So the
    result of a call may be read by work enqueued on the stream before the next
    call is made; work enqueued later may see it overwritten. ``d_full`` is the
    buffer the last call wrote.
    """

    BUFFERS = 2

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
        lib = _lib.load()
        self._buffers = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(self.BUFFERS)]
        mine = []
        for buf in self._buffers:
            handle = ctypes.create_string_buffer(64)
            offset = ctypes.c_int64(0)
            _lib.check(lib.cutex_ipc_export(buf.data_ptr(), handle, ctypes.byref(offset)), "cutex_ipc_export")
            mine.append((handle.raw, offset.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._mappings = []
        self._maps = []
        self.num_peers = self.world - 1
        for i in range(self.BUFFERS):
            peers = []
            # Peers in rotated order (rank + 1, rank + 2, ...): each chunk's j-th peer
            # store goes to a different GPU on every rank, so no GPU's ingress gets
            # every rank's first store at once.
            for j in range(1, self.world):
                r = (self.rank + j) % self.world
                h, off = everyone[r][i]
                ptr, mapping = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.check(lib.cutex_ipc_import(h, off, ctypes.byref(ptr), ctypes.byref(mapping)),
                           "cutex_ipc_import")
                self._mappings.append(mapping.value)
                peers.append(ptr.value + self.shard.n0 * 2)  # this rank's columns in peer r's buffer i
            ptrs = (ctypes.c_void_p * len(peers))(*peers)
            maps = torch.empty(128 * len(peers), dtype=torch.uint8, device=dev)
            # The peers' TMA store descriptors, written once (a host copy that waits
            # for the stream would otherwise serialise every call).
            _lib.check(lib.cutex_mxfp8_allgather_maps(ptrs, len(peers), m, self.shard.n, n, maps.data_ptr(),
                                                      maps.numel(), torch.cuda.current_stream().cuda_stream),
                       "cutex_mxfp8_allgather_maps")
            self._maps.append(maps)
        torch.cuda.current_stream().synchronize()  # descriptors in place before any stream's GEMM reads them
        self._cfg = (config or GemmConfig()).to_c()
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        self._calls = 0
        self.d_full = self._buffers[-1]

    def __call__(self, a, b_local, sfa, sfb_local, stream=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib

        if stream is None:
            s = torch.cuda.current_stream()
        elif isinstance(stream, int):
            s = torch.cuda.ExternalStream(stream)
        else:
            s = stream
        i = self._calls % self.BUFFERS
        out = self._buffers[i]
        status = _lib.load().cutex_mxfp8_gemm_allgather(
            a.data_ptr(), b_local.data_ptr(), sfa.data_ptr(), sfb_local.data_ptr(),
            out.data_ptr() + self.shard.n0 * 2, self.m, self.shard.n, self.k, self.n, self._maps[i].data_ptr(),
            self.num_peers, ctypes.byref(self._cfg), s.cuda_stream)
        _lib.check(status, "cutex_mxfp8_gemm_allgather")
        self._calls += 1
        self.d_full = out
        # Cross-rank barrier in the call's stream order: every rank's pushes have landed.
        with torch.cuda.stream(s):
            dist.all_reduce(self._flag, group=self.group)
        return out

    def close(self) -> None:
        from . import _lib

        lib = _lib.load()
        for mapping in self._mappings:
            lib.cutex_ipc_close(mapping)
        self._mappings = []


class ShardedHostGemm:
    """N-sharded GEMM from pinned host buffers, with A's host-to-device copy split across the ranks.

    Every rank needs all of A, but A is the same on every rank: each rank copies
    only its ``rows`` (M / world rows of A and their scale rows) over its own host
    link, and one NCCL all-gather over NVLink assembles A on every GPU. Each rank
    copies its B slice in on a second stream meanwhile, runs the GEMM of its
    D[:, n0:n1] in row blocks and copies each finished block back to the host
    while the next one computes. Host link traffic per rank: 1/world of A plus its
    own B slice and D slice. M must be a multiple of 128 * world.
    """

    def __init__(self, m: int, n: int, k: int, group=None, config=None, device=None, blocks: int = 4):
        import torch
        import torch.distributed as dist

        from .kernels.dense_gemm import GemmConfig
        from .kernels.dense_gemm_contract import scale_buffer_bytes

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if m % (128 * self.world):
            raise ValueError(f"M={m} must be a multiple of 128 * world = {128 * self.world}")
        self.cols = shard_bounds(n, self.world, self.rank)
        self.rows = shard_bounds(m, self.world, self.rank, align=128)
        self.m, self.n, self.k = m, n, k
        self.config = config or GemmConfig()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        u8 = torch.uint8
        n_loc, m_loc = self.cols.n, self.rows.n
        self.sf_row = k // 32
        self.a = torch.empty(m * k, dtype=u8, device=dev)
        self.sfa = torch.empty(scale_buffer_bytes(m, k), dtype=u8, device=dev)
        self.a_part = torch.empty(m_loc * k, dtype=u8, device=dev)
        self.sfa_part = torch.empty(m_loc * self.sf_row, dtype=u8, device=dev)
        self.b = torch.empty(n_loc, k, dtype=u8, device=dev)
        self.sfb = torch.empty(scale_buffer_bytes(n_loc, k), dtype=u8, device=dev)
        self.d = torch.empty(m, n_loc, dtype=torch.bfloat16, device=dev)
        blk = -(-m // blocks)
        blk = -(-blk // 256) * 256
        self.row_blocks = [(r0, min(m, r0 + blk)) for r0 in range(0, m, blk)]
        self._b_stream = torch.cuda.Stream(dev)
        self._d_stream = torch.cuda.Stream(dev)

    def host_bytes(self) -> tuple[int, int]:
        """(host-to-device, device-to-host) bytes this rank moves per call."""

        h2d = self.a_part.numel() + self.sfa_part.numel() + self.b.numel() + self.sfb.numel()
        return h2d, self.d.numel() * 2

    def __call__(self, a_rows_host, sfa_rows_host, b_host, sfb_host, d_host, stream=None):
        """a_rows_host: this rank's ``rows`` of A [m_loc, K] and sfa_rows_host their scale rows
        (whole 128-row blocks of the swizzled buffer); b_host / sfb_host: this rank's B slice and
        its scales; d_host [M, n_loc]: D[:, n0:n1]. Pinned host tensors. Asynchronous on ``stream``."""

        import torch
        import torch.distributed as dist

        from .kernels.dense_gemm import dense_gemm

        s = torch.cuda.current_stream() if stream is None else stream
        self._b_stream.wait_stream(s)
        with torch.cuda.stream(self._b_stream):
            self.b.copy_(b_host, non_blocking=True)
            self.sfb.copy_(sfb_host.reshape(-1), non_blocking=True)
        with torch.cuda.stream(s):
            self.a_part.copy_(a_rows_host.reshape(-1), non_blocking=True)
            self.sfa_part.copy_(sfa_rows_host.reshape(-1), non_blocking=True)
            dist.all_gather_into_tensor(self.a, self.a_part, group=self.group)
            dist.all_gather_into_tensor(self.sfa[: self.m * self.sf_row], self.sfa_part, group=self.group)
            s.wait_stream(self._b_stream)
            a2 = self.a.view(self.m, self.k)
            for r0, r1 in self.row_blocks:
                dense_gemm(a2[r0:r1], self.b, self.sfa[r0 * self.sf_row:], self.sfb, self.d[r0:r1], stream=s,
                           config=self.config)
                ev = torch.cuda.Event()
                ev.record(s)
                self._d_stream.wait_event(ev)
                with torch.cuda.stream(self._d_stream):
                    d_host[r0:r1].copy_(self.d[r0:r1], non_blocking=True)
            s.wait_stream(self._d_stream)


__all__ = ["SHARD_ALIGN", "FusedAllGatherGemm", "Shard", "ShardedHostGemm", "allgather_columns",
           "scale_rows_slice", "shard_bounds"]
