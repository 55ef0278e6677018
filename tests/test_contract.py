"""Contract module: the reference's tests (tests/test_dense_gemm_contract.py) plus golden values."""

import json

import pytest

from cutex_b200.kernels import dense_gemm_contract as C
from cutex_b200.kernels.dense_gemm_contract import (
    K,
    M,
    N,
    SCALE_FACTOR_ELEMENTS,
    SF_VECTOR_SIZE,
    dense_gemm_contract,
    dense_gemm_flops,
    mxfp8_gemm_bytes,
    mxfp8_gemm_flops,
    scale_buffer_bytes,
    validate_dense_gemm_shape,
    validate_mxfp8_gemm_shape,
)
from tests.conftest import GOLDEN


def test_dense_gemm_contract_accepts_only_16384_cubed():
    assert validate_dense_gemm_shape(M, N, K) == (16384, 16384, 16384)
    assert dense_gemm_flops() == 2 * 16384**3
    assert SF_VECTOR_SIZE == 32
    assert SCALE_FACTOR_ELEMENTS == 16384 * 16384 // 32


def test_dense_gemm_precision_contract():
    contract = dense_gemm_contract()
    assert contract["inputs"] == "MXFP8 E4M3FN"
    assert contract["multiply"] == "FP8 E4M3FN x E4M3FN"
    assert contract["accumulator"] == "FP32"
    assert contract["fast_accumulation"] is False
    assert contract["output"] == "BF16"
    assert contract["quantization_in_timed_region"] is False


@pytest.mark.parametrize("shape", [(0, 16384, 16384), (128, 256, 128), (16384, 16384, 16383)])
def test_dense_gemm_contract_rejects_every_other_shape(shape):
    with pytest.raises(ValueError, match="fixed to M=N=K=16384"):
        validate_dense_gemm_shape(*shape)


def test_contract_matches_reference_golden():
    g = json.loads((GOLDEN / "contract.json").read_text())
    assert (C.M, C.N, C.K) == (g["M"], g["N"], g["K"])
    assert list(C.PROBLEM_SHAPE) == g["PROBLEM_SHAPE"]
    assert [C.TILE_M, C.TILE_N, C.TILE_K] == g["TILE"]
    assert list(C.MMA_SHAPE) == g["MMA_SHAPE"]
    assert C.SF_VECTOR_SIZE == g["SF_VECTOR_SIZE"]
    assert C.SCALE_FACTOR_ELEMENTS == g["SCALE_FACTOR_ELEMENTS"]
    assert list(C.SCALE_FACTOR_LOGICAL_SHAPE) == g["SCALE_FACTOR_LOGICAL_SHAPE"]
    for name in ("OPERATION", "INPUT_FORMAT", "SCALE_FORMAT", "SCALE_LAYOUT", "MULTIPLY_FORMAT",
                 "ACCUMULATOR_FORMAT", "OUTPUT_FORMAT"):
        assert getattr(C, name) == g[name]
    assert dense_gemm_flops() == g["dense_gemm_flops"]
    assert dense_gemm_contract() == g["dense_gemm_contract"]


@pytest.mark.parametrize("shape", [(1, 16, 128), (16, 28672, 8192), (8192, 28672, 8192), (300, 272, 384)])
def test_general_shapes_accepted(shape):
    assert validate_mxfp8_gemm_shape(*shape) == shape


@pytest.mark.parametrize("shape,match", [((0, 16, 128), "positive"), ((4, 16, 100), "multiple of 128"),
                                         ((4, 24, 128), "multiple of 16"), ((2**31, 16, 128), "below")])
def test_general_shapes_rejected(shape, match):
    with pytest.raises(ValueError, match=match):
        validate_mxfp8_gemm_shape(*shape)


def test_work_and_bytes():
    assert mxfp8_gemm_flops(16, 28672, 8192) == 2 * 16 * 28672 * 8192
    assert mxfp8_gemm_bytes(16384, 16384, 16384) == 1090519040
    assert scale_buffer_bytes(16, 8192) == 128 * 256
    assert scale_buffer_bytes(16384, 16384) == SCALE_FACTOR_ELEMENTS
