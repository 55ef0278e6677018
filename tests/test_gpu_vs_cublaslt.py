"""The tile kernels' BF16 output is bit-identical to NVIDIA cuBLASLt's MXFP8 GEMM.

cuBLASLt (reached through ``torch._scaled_mm`` with E4M3 operands and the same
128x4-swizzled E8M0 scales) is the comparator the reference benchmarks against
(Transformer Engine ``general_gemm``, ``modal_dense_gemm.py:532-540``). Both
accumulate each output element in FP32 in K order inside the tensor core and
round to BF16 once, so on shapes where cuBLASLt does not split K the two
outputs agree bit for bit; this pins the GEMM's numerics to an independent
implementation on the GPU, next to the CPU oracle. The oracle check runs too.
"""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import GemmConfig, check, make_operands, run_gemm

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512, 1024), (1024, 1024, 1024), (384, 2048, 2048), (2048, 2048, 2048)]
CONFIGS = [
    None,  # AUTO
    GemmConfig(kernel=2, tile_n=256),
    GemmConfig(kernel=1, tile_n=256, scheduler=1),
    GemmConfig(kernel=1, tile_n=128),
]


def _cublaslt(a, sfa, b, sfb):
    dev = torch.device("cuda")
    A = torch.from_numpy(a).to(dev).view(torch.float8_e4m3fn)
    B = torch.from_numpy(b).to(dev).view(torch.float8_e4m3fn)
    SA = torch.from_numpy(sfa).to(dev).view(torch.float8_e8m0fnu)
    SB = torch.from_numpy(sfb).to(dev).view(torch.float8_e8m0fnu)
    return torch._scaled_mm(A, B.t(), SA, SB, out_dtype=torch.bfloat16)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_bitwise_equal_to_cublaslt(shape):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=M + N + K)
    ref = _cublaslt(a, sfa, b, sfb)
    torch.cuda.synchronize()
    for cfg in CONFIGS:
        out = run_gemm(a, sfa, b, sfb, M, N, K, cfg)
        same = torch.equal(out.view(torch.int16), ref.view(torch.int16))
        if not same:
            diff = (out.float() - ref.float()).abs()
            pytest.fail(f"config {cfg}: {int((diff > 0).sum())} of {diff.numel()} elements differ, "
                        f"max |diff| {float(diff.max())}")
    report = check(out, a, sfa, b, sfb, M, N, K)
    assert report["ok"], report
