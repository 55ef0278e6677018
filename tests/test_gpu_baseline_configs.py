"""The CUDA GEMM against the CPU oracle on BASELINE's own configurations, at their full shapes.

* 4096^3, square generator, every output element checked;
* the square sweep generator with 1 % all-zero 1x32 blocks (E8M0
  minimum scale): 2048^3 in full, 8192^3 and 32768^3 on sampled 64 x 64 blocks;
* the LLM shape M = 8192, N = 28672, K = 8192 (activations with
  0.1 % of channels x50, weights N(0, 0.02)) on sampled blocks.

Sampled blocks sit at the corners, the first tile boundaries, the middle and
the N-shard boundaries of 2/4/8 GPUs. Where the operands are generated and
quantised on the GPU, the quantiser is first checked bit-exactly against the
oracle on source rows that the sampled blocks read. The reference's own
correctness gate for this GEMM is ``modal_dense_gemm.py:552-570``; the tolerance
is the contract's (``oracle/mxfp8_oracle.py``: relative Frobenius error <= 1e-3,
every element within 2 BF16 ulps plus 2^-16 * sum |a_k b_k|).
"""

import numpy as np
import pytest
import torch

from cutex_b200.kernels import dense_gemm
from tests.gpu_helpers import (O, boundary_starts, check, check_quantised_rows, check_sampled_blocks, device_ok,
                               device_operands, run_gemm)

pytestmark = pytest.mark.gpu


def _all_ok(reports):
    bad = [r for r in reports if not r["ok"]]
    assert not bad, bad[:3]


def test_config1_4096_cubed_in_full():
    n = 4096
    rng = np.random.default_rng(0)
    a, sfa = O.quantized_operands(O.make_square_source(n, n, rng))
    b, sfb = O.quantized_operands(O.make_square_source(n, n, rng))
    rep = check(run_gemm(a, sfa, b, sfb, n, n, n), a, sfa, b, sfb, n, n, n)
    assert rep["ok"], rep


def test_config3_sweep_2048_cubed_zero_blocks_in_full():
    n = 2048
    rng = np.random.default_rng(0)
    xa = O.make_square_source(n, n, rng, zero_block_frac=0.01)
    xb = O.make_square_source(n, n, rng, zero_block_frac=0.01)
    a, sfa = O.quantized_operands(xa)
    b, sfb = O.quantized_operands(xb)
    assert (O.unswizzle_scales(sfa, n, n) == 0).mean() > 0.005  # the minimum scale is exercised
    rep = check(run_gemm(a, sfa, b, sfb, n, n, n), a, sfa, b, sfb, n, n, n)
    assert rep["ok"], rep


def _device_gemm_sampled(M, N, K, kind, zero_block_frac=0.0, size=64):
    rows = boundary_starts(M, size)
    cols = boundary_starts(N, size)
    keep_a = [r for r in (rows[0], rows[-1])]
    keep_b = [c for c in (cols[0], cols[-1])]
    a, sfa, kept_a = device_operands(M, K, kind, seed=1, zero_block_frac=zero_block_frac, role="a", keep=keep_a)
    b, sfb, kept_b = device_operands(N, K, kind, seed=2, zero_block_frac=zero_block_frac, role="b", keep=keep_b)
    check_quantised_rows(a, sfa, kept_a, K)
    check_quantised_rows(b, sfb, kept_b, K)
    d = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dense_gemm(a, b, sfa, sfb, d)
    torch.cuda.synchronize()
    device_ok()
    assert not torch.isnan(d).any().item(), "some output element was not written"
    reports = check_sampled_blocks(d, a, sfa, b, sfb, K, rows, cols, size)
    return reports, (a, sfa, b, sfb)


@pytest.mark.parametrize("n", [8192, 32768])
def test_config3_sweep_zero_blocks_sampled(n):
    reports, (a, sfa, _, _) = _device_gemm_sampled(n, n, n, "square", zero_block_frac=0.01)
    _all_ok(reports)
    zero_frac = (sfa[: 1 << 20] == 0).float().mean().item()
    assert zero_frac > 0.005


def test_config4_llm_8192x28672x8192_sampled():
    reports, _ = _device_gemm_sampled(8192, 28672, 8192, "llm")
    _all_ok(reports)
