"""MXFP8 quantiser (OCP MX E4M3 + E8M0, 128x4 swizzled scales) over the C ABI.

Replaces the Transformer Engine quantiser the reference runner calls
(``modal_dense_gemm.py:358-373``: ``MXFP8Quantizer(E4M3, rowwise=True)`` with
GEMM-swizzled scales), with the scale rule exponent = floor(log2 amax) - 8.
"""

from __future__ import annotations

from .. import _lib
from .dense_gemm import _stream_handle
from .dense_gemm_contract import SF_VECTOR_SIZE, scale_buffer_bytes


def quantize_mxfp8(x, q=None, sf=None, stream=None):
    """Quantise ``x`` [rows, K] (float32 or bfloat16, CUDA) -> (q uint8 [rows, K], sf uint8 flat).

    ``K`` must be a multiple of 128. Output tensors are allocated with torch
    when not given. Runs asynchronously on ``stream``.
    """

    import torch

    if not x.is_cuda or x.dim() != 2:
        raise ValueError("x must be a 2-D CUDA tensor")
    if x.dtype == torch.float32:
        dtype_code = 0
    elif x.dtype == torch.bfloat16:
        dtype_code = 1
    else:
        raise TypeError(f"x must be float32 or bfloat16; got {x.dtype}")
    if x.stride(1) != 1:
        raise ValueError("x must have unit column stride")
    rows, k = x.shape
    if k % 128:
        raise ValueError(f"K must be a multiple of 128; got {k}")
    if q is None:
        q = torch.empty((rows, k), dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = torch.empty(scale_buffer_bytes(rows, k), dtype=torch.uint8, device=x.device)
    if q.numel() * q.element_size() < rows * k or sf.numel() * sf.element_size() < scale_buffer_bytes(rows, k):
        raise ValueError("output buffers too small")
    status = _lib.load().cutex_mxfp8_quantize(
        x.data_ptr(), dtype_code, rows, k, x.stride(0), q.data_ptr(), sf.data_ptr(), _stream_handle(stream)
    )
    _lib.check(status, "cutex_mxfp8_quantize")
    return q, sf


def quantize_mxfp8_columnwise(x, qt=None, sft=None, stream=None):
    """Quantise ``x`` [rows, cols] along its columns -> (qt uint8 [cols, rows], sft uint8 flat).

    ``qt`` = quantise(x^T): the K-major operand (K = rows) of a GEMM that
    reduces over the rows of ``x`` (weight and input gradients), scales in the
    128x4 swizzled layout of a [cols, rows] operand. ``rows`` must be a
    multiple of 128. Runs asynchronously on ``stream``.
    """

    import torch

    if not x.is_cuda or x.dim() != 2:
        raise ValueError("x must be a 2-D CUDA tensor")
    if x.dtype == torch.float32:
        dtype_code = 0
    elif x.dtype == torch.bfloat16:
        dtype_code = 1
    else:
        raise TypeError(f"x must be float32 or bfloat16; got {x.dtype}")
    if x.stride(1) != 1:
        raise ValueError("x must have unit column stride")
    rows, cols = x.shape
    if rows % 128:
        raise ValueError(f"rows (the GEMM's K) must be a multiple of 128; got {rows}")
    if qt is None:
        qt = torch.empty((cols, rows), dtype=torch.uint8, device=x.device)
    if sft is None:
        sft = torch.empty(scale_buffer_bytes(cols, rows), dtype=torch.uint8, device=x.device)
    if qt.numel() * qt.element_size() < rows * cols or sft.numel() * sft.element_size() < scale_buffer_bytes(cols, rows):
        raise ValueError("output buffers too small")
    status = _lib.load().cutex_mxfp8_quantize_columnwise(
        x.data_ptr(), dtype_code, rows, cols, x.stride(0), qt.data_ptr(), sft.data_ptr(), _stream_handle(stream)
    )
    _lib.check(status, "cutex_mxfp8_quantize_columnwise")
    return qt, sft


__all__ = ["SF_VECTOR_SIZE", "quantize_mxfp8", "quantize_mxfp8_columnwise"]
