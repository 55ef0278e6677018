"""Python API of the B200 MXFP8 GEMM, over the C ABI of libcutex_mxfp8.so.

* ``dense_gemm(a, b, sfa, sfb, out, stream=None, config=None)``: torch tensors.
* ``dense_gemm_v13(a_ptr, b_ptr, sfa_ptr, sfb_ptr, c_ptr, max_active_clusters,
  stream)``: the reference's fixed 16384^3 pointer interface
  (``cutex/kernels/dense_gemm_v13.py:947-956``), raw device addresses.
* ``mxfp8_gemm_launch``: the autotunable launcher (``@autotune`` search space
  over native configurations, keyed by shape and device target) for
  ``cutex_b200.compile``.
* ``query(m, n, k, config)``: what a launch would do (grid, SMEM, stages).
* ``HostGemm(m, n, k)`` / ``dense_gemm_host``: the same GEMM from host buffers
  to a host buffer, H2D copies, block GEMMs and D2H copies overlapped
  (``cutex_mxfp8_gemm_host``).

Operands: ``a`` [M, K] and ``b`` [N, K] E4M3 (``torch.float8_e4m3fn`` or
``uint8``), K-major and contiguous; ``sfa``/``sfb`` flat 128x4-swizzled E8M0
buffers (``torch.float8_e8m0fnu`` or ``uint8``) of at least
``scale_buffer_bytes(rows, K)`` bytes; ``out`` [M, N] bf16 with unit column
stride and a row stride that is a multiple of 8 elements.
"""

from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass
from typing import Any

from .. import _lib
from ..autotune import Config, autotune
from ..compiler import DEVICE_STATUS_ATTRIBUTE
from .dense_gemm_contract import scale_buffer_bytes, validate_mxfp8_gemm_shape


@dataclass(frozen=True)
class GemmConfig:
    """Native configuration (``cutex_gemm_config``); 0 = library heuristic for that field."""

    kernel: int = 0
    tile_n: int = 0
    stages: int = 0
    raster_group: int = 0
    raster_along_n: int = 0
    split_k: int = 0
    max_ctas: int = 0
    epi_buffers: int = 0
    sf_buffers: int = 0
    scheduler: int = 0

    def to_c(self) -> _lib.GemmConfigC:
        return _lib.make_config(**asdict(self))


def _stream_handle(stream) -> int:
    import torch

    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    handle = getattr(stream, "cuda_stream", None)
    if handle is None:
        raise TypeError("stream must be a torch.cuda.Stream, a raw cudaStream_t integer or None")
    return int(handle)


def _byte_view_ok(t, name: str) -> None:
    import torch

    if t.dtype not in (torch.uint8, torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.int8):
        raise TypeError(f"{name} must hold bytes (float8_e4m3fn / float8_e8m0fnu / uint8); got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def query(m: int, n: int, k: int, config: GemmConfig | None = None) -> dict[str, Any]:
    info = _lib.GemmInfoC()
    cfg = (config or GemmConfig()).to_c()
    _lib.check(_lib.load().cutex_mxfp8_query(ctypes.byref(cfg), m, n, k, ctypes.byref(info)), "cutex_mxfp8_query")
    return {name: getattr(info, name) for name, _ in _lib.GemmInfoC._fields_}


_WORKSPACES: dict[tuple[int, int], Any] = {}


def workspace_for(device, stream_handle: int, nbytes: int):
    """A zero-initialised device workspace of at least ``nbytes``, cached per (device, stream).

    The split-K skinny kernel leaves its arrival counters at zero when it
    finishes, so one workspace serves every later call on the same stream
    (calls on different streams get different workspaces: they may overlap).
    """

    import torch

    key = (int(device.index if device.index is not None else torch.cuda.current_device()), int(stream_handle))
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def dense_gemm(a, b, sfa, sfb, out, stream=None, config: GemmConfig | None = None, workspace=None):
    """D = dequant(A, SFA) @ dequant(B, SFB)^T in BF16 (FP32 accumulate); launches asynchronously.

    Shapes with M <= 128 run the split-K skinny kernel, which needs a device
    workspace (``query(...)["workspace_bytes"]``); when ``workspace`` is None a
    zero-initialised one is allocated once per (device, stream) and reused.
    """

    import torch

    for t, name in ((a, "a"), (b, "b"), (sfa, "sfa"), (sfb, "sfb")):
        _byte_view_ok(t, name)
    if a.dim() != 2 or b.dim() != 2 or out.dim() != 2:
        raise ValueError("a, b and out must be 2-D")
    m, k = a.shape
    n, kb = b.shape
    if kb != k:
        raise ValueError(f"a is [{m}, {k}] but b is [{n}, {kb}]: K must match")
    validate_mxfp8_gemm_shape(m, n, k)
    if not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("a and b must be contiguous K-major [rows, K]")
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or out.stride(1) != 1:
        raise ValueError(f"out must be a bf16 [{m}, {n}] tensor with unit column stride")
    if sfa.numel() * sfa.element_size() < scale_buffer_bytes(m, k):
        raise ValueError(f"sfa holds {sfa.numel()} bytes; {scale_buffer_bytes(m, k)} required")
    if sfb.numel() * sfb.element_size() < scale_buffer_bytes(n, k):
        raise ValueError(f"sfb holds {sfb.numel()} bytes; {scale_buffer_bytes(n, k)} required")
    cfg = (config or GemmConfig()).to_c()
    handle = _stream_handle(stream)
    if workspace is None and m <= 128:
        need = query(m, n, k, config)["workspace_bytes"]
        if need > 0:
            workspace = workspace_for(a.device, handle, need)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    status = _lib.load().cutex_mxfp8_gemm(
        a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(),
        m, n, k, out.stride(0), ctypes.byref(cfg), ws_ptr or None, ws_bytes, handle,
    )
    _lib.check(status, "cutex_mxfp8_gemm")
    return out


def dense_gemm_fused(a, b, sfa, sfb, out, *, alpha: float = 1.0, beta: float = 0.0, c=None, bias=None,
                     out_scales=None, stream=None, config: GemmConfig | None = None):
    """D = alpha * dequant(A) @ dequant(B)^T + beta * C + bias, fused into the GEMM's epilogue.

    ``out`` bf16 [M, N], or E4M3 [M, N] (``torch.float8_e4m3fn`` / ``uint8``) with
    ``out_scales`` (``scale_buffer_bytes(M, N)`` bytes): the next layer's MXFP8
    operand, 1x32 blocks along N, quantised with the same rule as
    ``quantize_mxfp8``. ``c`` bf16 [M, N] (may be ``out`` itself), ``bias`` bf16
    [N]. Runs the large-tile kernels only (any M).
    """

    import torch

    for t, name in ((a, "a"), (b, "b"), (sfa, "sfa"), (sfb, "sfb")):
        _byte_view_ok(t, name)
    m, k = a.shape
    n = b.shape[0]
    validate_mxfp8_gemm_shape(m, n, k)
    if b.shape[1] != k or not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("a [M, K] and b [N, K] must be contiguous with matching K")
    fp8_out = out.dtype in (torch.uint8, getattr(torch, "float8_e4m3fn", torch.uint8))
    if tuple(out.shape) != (m, n) or out.stride(1) != 1 or not (fp8_out or out.dtype == torch.bfloat16):
        raise ValueError(f"out must be a bf16 or e4m3 [{m}, {n}] tensor with unit column stride")
    epi = _lib.EpilogueC()
    epi.alpha = float(alpha)
    epi.beta = float(beta)
    if c is not None:
        if c.dtype != torch.bfloat16 or tuple(c.shape) != (m, n) or c.stride(1) != 1:
            raise ValueError(f"c must be a bf16 [{m}, {n}] tensor with unit column stride")
        epi.c = c.data_ptr()
        epi.ldc = c.stride(0)
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous():
            raise ValueError(f"bias must be a contiguous bf16 tensor of {n} elements")
        epi.bias = bias.data_ptr()
    if fp8_out:
        if out_scales is None or out_scales.numel() * out_scales.element_size() < scale_buffer_bytes(m, n):
            raise ValueError(f"e4m3 output needs out_scales of {scale_buffer_bytes(m, n)} bytes")
        epi.out_dtype = 1
        epi.d_scales = out_scales.data_ptr()
    cfg = (config or GemmConfig()).to_c()
    status = _lib.load().cutex_mxfp8_gemm_ex(
        a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(), m, n, k, out.stride(0),
        ctypes.byref(cfg), ctypes.byref(epi), None, 0, _stream_handle(stream))
    _lib.check(status, "cutex_mxfp8_gemm_ex")
    return out


class PreparedGemm:
    """A GEMM launch with every argument resolved once: calling it is a single C-ABI call.

    Validation, plan resolution and workspace selection happen at construction,
    so the call itself is cheap and safe to capture into a CUDA graph (the
    library encodes the TMA descriptors into the kernel's parameters).
    """

    def __init__(self, a, b, sfa, sfb, out, stream=None, config: GemmConfig | None = None, workspace=None):
        m, k = a.shape
        n = b.shape[0]
        # Full validation and a first launch-ready check through the public wrapper's rules.
        self.config = config or GemmConfig()
        self.handle = _stream_handle(stream)
        self.plan = query(m, n, k, self.config)
        if workspace is None and self.plan["workspace_bytes"] > 0:
            workspace = workspace_for(a.device, self.handle, self.plan["workspace_bytes"])
        self.workspace = workspace
        self._tensors = (a, b, sfa, sfb, out)
        self._cfg = self.config.to_c()
        ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
        self._args = (a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(), m, n, k,
                      out.stride(0), ctypes.byref(self._cfg), ws_ptr, ws_bytes, self.handle)
        self._fn = _lib.load().cutex_mxfp8_gemm
        dense_gemm(a, b, sfa, sfb, out, stream=self.handle, config=self.config, workspace=workspace)

    def __call__(self) -> None:
        status = self._fn(*self._args)
        if status != 0:
            _lib.check(status, "cutex_mxfp8_gemm")


class HostGemm:
    """GEMM from pinned host operands into a pinned host D through device staging buffers.

    Holds device buffers for one shape (A, B, their scales, D) and calls
    ``cutex_mxfp8_gemm_host``, which overlaps the host-to-device copies, the
    block GEMMs and the device-to-host copy of each finished block. The call is
    asynchronous on ``stream``: synchronise before reading ``d_host``.
    """

    def __init__(self, m: int, n: int, k: int, device=None, config: GemmConfig | None = None, blocks: int = 4):
        import torch

        validate_mxfp8_gemm_shape(m, n, k)
        if not 1 <= blocks <= 16:
            raise _lib.CutexArgumentError(_lib.CUTEX_ERR_INVALID_ARGUMENT, f"blocks must be in [1, 16], got {blocks}")
        self.m, self.n, self.k, self.blocks = m, n, k, blocks
        self.config = config or GemmConfig()
        self._cfg = self.config.to_c()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        u8 = torch.uint8
        self.a = torch.empty(m, k, dtype=u8, device=dev)
        self.b = torch.empty(n, k, dtype=u8, device=dev)
        self.sfa = torch.empty(scale_buffer_bytes(m, k), dtype=u8, device=dev)
        self.sfb = torch.empty(scale_buffer_bytes(n, k), dtype=u8, device=dev)
        self.d = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        self.device = dev
        plan = query(m, n, k, self.config)
        self.workspace = None
        if plan["workspace_bytes"] > 0:
            # Zeroed: the arrival counters must start at zero (every launch leaves them so).
            self.workspace = torch.zeros(plan["workspace_bytes"], dtype=u8, device=dev)

    @staticmethod
    def _host(t, shape_bytes: int, name: str) -> int:
        if t.device.type != "cpu" or not t.is_contiguous():
            raise _lib.CutexArgumentError(_lib.CUTEX_ERR_INVALID_ARGUMENT, f"{name} must be a contiguous host tensor")
        if t.numel() * t.element_size() < shape_bytes:
            raise _lib.CutexArgumentError(_lib.CUTEX_ERR_INVALID_ARGUMENT, f"{name} holds fewer than {shape_bytes} bytes")
        return t.data_ptr()

    def __call__(self, a_host, b_host, sfa_host, sfb_host, d_host, stream=None) -> None:
        m, n, k = self.m, self.n, self.k
        ptrs = (
            self._host(a_host, m * k, "a_host"),
            self._host(b_host, n * k, "b_host"),
            self._host(sfa_host, scale_buffer_bytes(m, k), "sfa_host"),
            self._host(sfb_host, scale_buffer_bytes(n, k), "sfb_host"),
            self._host(d_host, m * n * 2, "d_host"),
        )
        ws_ptr, ws_bytes = (None, 0) if self.workspace is None else (self.workspace.data_ptr(), self.workspace.numel())
        status = _lib.load().cutex_mxfp8_gemm_host(
            *ptrs, self.a.data_ptr(), self.b.data_ptr(), self.sfa.data_ptr(), self.sfb.data_ptr(),
            self.d.data_ptr(), m, n, k, ctypes.byref(self._cfg), self.blocks, ws_ptr, ws_bytes,
            _stream_handle(stream))
        _lib.check(status, "cutex_mxfp8_gemm_host")


def dense_gemm_host(a_host, b_host, sfa_host, sfb_host, d_host, stream=None, config: GemmConfig | None = None,
                    blocks: int = 4) -> None:
    """One-shot ``HostGemm`` (allocates the device staging buffers for this call)."""

    m, k = a_host.shape
    HostGemm(m, b_host.shape[0], k, config=config, blocks=blocks)(a_host, b_host, sfa_host, sfb_host, d_host,
                                                                 stream=stream)


def dense_gemm_v13(a_ptr: int, b_ptr: int, sfa_ptr: int, sfb_ptr: int, c_ptr: int,
                   max_active_clusters: int = 0, stream=None) -> None:
    """The reference's fixed M=N=K=16384 five-pointer launch, on the 2-CTA kernel."""

    status = _lib.load().cutex_dense_gemm_v13(
        a_ptr, b_ptr, sfa_ptr, sfb_ptr, c_ptr, int(max_active_clusters), _stream_handle(stream)
    )
    _lib.check(status, "cutex_dense_gemm_v13")


def device_target() -> str:
    """Autotune-cache key field: GPU name, compute capability, SM count and library build."""

    import torch

    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    return f"{props.name}|cc{props.major}.{props.minor}|sm{props.multi_processor_count}|{_lib.version()}"


# Search space: kernel family x tile x ring depth x raster order/group.
GEMM_CONFIGS = (
    [
        Config({"kernel": 2, "tile_n": 256, "stages": s, "epi_buffers": e, "raster_group": g, "raster_along_n": r},
               name=f"2cta_n256_s{s}_e{e}_g{g}_{'n' if r else 'm'}")
        for s, e in ((6, 1), (5, 2), (4, 2))
        for g in (4, 8, 16)
        for r in (0, 1)
    ]
    + [
        Config({"kernel": 1, "tile_n": 256, "stages": s, "epi_buffers": e, "raster_group": 8, "raster_along_n": 0},
               name=f"1cta_n256_s{s}_e{e}")
        for s, e in ((4, 1), (3, 2))
    ]
    + [
        Config({"kernel": 1, "tile_n": 128, "stages": s, "epi_buffers": e, "raster_group": 8, "raster_along_n": 0},
               name=f"1cta_n128_s{s}_e{e}")
        for s, e in ((6, 1), (5, 2))
    ]
    # M <= 128 only (larger M is rejected by the library and skipped by the search).
    + [Config({"kernel": 3, "split_k": s}, name=f"skinny_split{s}") for s in (1, 2, 3)]
)


@autotune(configs=GEMM_CONFIGS, key=["m", "n", "k", "target"], warmup=3, rep=10)
def mxfp8_gemm_launch(a, b, sfa, sfb, out, m, n, k, target, stream=None, *, kernel=0, tile_n=0,
                      stages=0, raster_group=0, raster_along_n=0, split_k=0, max_ctas=0, epi_buffers=0,
                      sf_buffers=0, scheduler=0):
    """Autotunable launcher: ``cutex_b200.compile(mxfp8_gemm_launch, a, b, sfa, sfb, out, m, n, k, target)``."""

    cfg = GemmConfig(kernel, tile_n, stages, raster_group, raster_along_n, split_k, max_ctas, epi_buffers,
                     sf_buffers, scheduler)
    return dense_gemm(a, b, sfa, sfb, out, stream=stream, config=cfg)


def _launch_device_status() -> int:
    """Health probe the autotuner runs after timing a candidate: the library's device status word.

    Synchronises the device first (candidates may have run on any stream); a
    non-zero value (an expired bounded wait, a device-side check) rejects the
    candidate and clears the word.
    """

    import torch

    torch.cuda.synchronize()
    return int(_lib.load().cutex_last_device_status(torch.cuda.current_stream().cuda_stream))


setattr(mxfp8_gemm_launch, DEVICE_STATUS_ATTRIBUTE, _launch_device_status)


__all__ = [
    "GEMM_CONFIGS",
    "GemmConfig",
    "HostGemm",
    "PreparedGemm",
    "dense_gemm",
    "dense_gemm_fused",
    "dense_gemm_host",
    "dense_gemm_v13",
    "device_target",
    "mxfp8_gemm_launch",
    "query",
    "workspace_for",
]
