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


__all__ = ["SF_VECTOR_SIZE", "quantize_mxfp8"]
