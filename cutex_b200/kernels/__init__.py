"""B200 MXFP8 kernels behind the reference's kernel-module names."""

from . import dense_gemm_contract
from .dense_gemm import (GemmConfig, HostGemm, PreparedGemm, dense_gemm, dense_gemm_fused, dense_gemm_host,
                         dense_gemm_v13,
                         mxfp8_gemm_launch, query)
from .quantize import quantize_mxfp8, quantize_mxfp8_columnwise

__all__ = [
    "GemmConfig",
    "HostGemm",
    "PreparedGemm",
    "dense_gemm",
    "dense_gemm_contract",
    "dense_gemm_fused",
    "dense_gemm_host",
    "dense_gemm_v13",
    "mxfp8_gemm_launch",
    "quantize_mxfp8",
    "quantize_mxfp8_columnwise",
    "query",
]
