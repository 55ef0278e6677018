"""The MXFP8 Fprop contract, with the reference's names.

Same constants and functions as ``cutex/kernels/dense_gemm_contract.py:6-58``
(fixed M = N = K = 16384 benchmark shape, 128x256x128 CTA tile, 128x256x32 MMA,
one E8M0 scale per 32 K values). ``validate_dense_gemm_shape`` stays strict so
code written against the reference keeps its behaviour; the B200 kernels
accept general shapes through ``validate_mxfp8_gemm_shape``.
"""

from __future__ import annotations

M = N = K = 16384
PROBLEM_SHAPE = (M, N, K)

TILE_M, TILE_N, TILE_K = 128, 256, 128
MMA_SHAPE = (128, 256, 32)

SF_VECTOR_SIZE = 32
SCALE_FACTOR_ELEMENTS = M * K // SF_VECTOR_SIZE
SCALE_FACTOR_LOGICAL_SHAPE = (M, K // SF_VECTOR_SIZE)

OPERATION = "Y[M,N] = X[M,K] @ W[N,K].T"
INPUT_FORMAT = "MXFP8 E4M3FN"
SCALE_FORMAT = "E8M0FNU, one scale per 32 contiguous K values"
SCALE_LAYOUT = "tcgen05 Swizzle32x4x4"
MULTIPLY_FORMAT = "FP8 E4M3FN x E4M3FN"
ACCUMULATOR_FORMAT = "FP32"
OUTPUT_FORMAT = "BF16"

# General-shape rules of the B200 kernels (see include/cutex_mxfp8.h).
K_ALIGNMENT = 128
N_ALIGNMENT = 16
MAX_DIM = 2**31 - 1


def validate_dense_gemm_shape(m: int, n: int, k: int) -> tuple[int, int, int]:
    """Accept only the fixed benchmark shape (the reference's strict contract)."""

    shape = (int(m), int(n), int(k))
    if shape != PROBLEM_SHAPE:
        raise ValueError(
            f"dense_gemm is fixed to M=N=K=16384; got M={shape[0]}, N={shape[1]}, K={shape[2]}"
        )
    return shape


def validate_mxfp8_gemm_shape(m: int, n: int, k: int) -> tuple[int, int, int]:
    """Accept any shape the native kernels support: M >= 1, N % 16 == 0, K % 128 == 0."""

    m, n, k = int(m), int(n), int(k)
    if m < 1 or n < 1 or k < 1:
        raise ValueError(f"MXFP8 GEMM dimensions must be positive; got M={m}, N={n}, K={k}")
    if max(m, n, k) > MAX_DIM:
        raise ValueError(f"MXFP8 GEMM dimensions must be below 2^31; got M={m}, N={n}, K={k}")
    if k % K_ALIGNMENT:
        raise ValueError(f"K must be a multiple of {K_ALIGNMENT} (one 128x4 scale atom); got K={k}")
    if n % N_ALIGNMENT:
        raise ValueError(f"N must be a multiple of {N_ALIGNMENT}; got N={n}")
    return m, n, k


def scale_buffer_bytes(rows: int, k: int) -> int:
    """Bytes of a 128x4-swizzled E8M0 scale buffer for an operand of ``rows`` x ``k``."""

    return ((int(rows) + 127) // 128) * 128 * (int(k) // SF_VECTOR_SIZE)


def dense_gemm_flops(m: int = M, n: int = N, k: int = K) -> int:
    """Two FLOPs per multiply-add of the fixed contract shape."""

    m, n, k = validate_dense_gemm_shape(m, n, k)
    return 2 * m * n * k


def mxfp8_gemm_flops(m: int, n: int, k: int) -> int:
    m, n, k = validate_mxfp8_gemm_shape(m, n, k)
    return 2 * m * n * k


def mxfp8_gemm_bytes(m: int, n: int, k: int) -> int:
    """Compulsory HBM traffic: E4M3 A and B, E8M0 scales, BF16 D."""

    m, n, k = validate_mxfp8_gemm_shape(m, n, k)
    return m * k + n * k + (m + n) * (k // SF_VECTOR_SIZE) + 2 * m * n


def dense_gemm_contract() -> dict[str, object]:
    """Serializable precision and storage contract for runners (same keys as the reference)."""

    return {
        "operation": OPERATION,
        "shape": {"m": M, "n": N, "k": K},
        "inputs": INPUT_FORMAT,
        "scales": SCALE_FORMAT,
        "scale_layout": SCALE_LAYOUT,
        "multiply": MULTIPLY_FORMAT,
        "accumulator": ACCUMULATOR_FORMAT,
        "fast_accumulation": False,
        "output": OUTPUT_FORMAT,
        "quantization_in_timed_region": False,
    }


__all__ = [
    "ACCUMULATOR_FORMAT",
    "INPUT_FORMAT",
    "K",
    "K_ALIGNMENT",
    "M",
    "MMA_SHAPE",
    "MULTIPLY_FORMAT",
    "N",
    "N_ALIGNMENT",
    "OPERATION",
    "OUTPUT_FORMAT",
    "PROBLEM_SHAPE",
    "SCALE_FACTOR_ELEMENTS",
    "SCALE_FACTOR_LOGICAL_SHAPE",
    "SCALE_FORMAT",
    "SCALE_LAYOUT",
    "SF_VECTOR_SIZE",
    "TILE_K",
    "TILE_M",
    "TILE_N",
    "dense_gemm_contract",
    "dense_gemm_flops",
    "mxfp8_gemm_bytes",
    "mxfp8_gemm_flops",
    "scale_buffer_bytes",
    "validate_dense_gemm_shape",
    "validate_mxfp8_gemm_shape",
]
