"""GPU quantiser vs the CPU oracle: bit-exact E4M3 codes and swizzled E8M0 scales."""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import O, device_ok

pytestmark = pytest.mark.gpu


def _run(x_np, dtype):
    from cutex_b200.kernels import quantize_mxfp8

    x = torch.from_numpy(x_np).to("cuda").to(dtype)
    q, sf = quantize_mxfp8(x)
    torch.cuda.synchronize()
    device_ok()
    # The oracle quantises exactly what the kernel saw (bf16 inputs widened to fp32).
    src = x.float().cpu().numpy()
    q_ref, sf_ref = O.quantize_mxfp8(src)
    return q.cpu().numpy(), sf.cpu().numpy(), q_ref, O.swizzle_scales(sf_ref, x_np.shape[1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
# K = 22528: whole 2048-group steps of 256 threads and a partial step in the same row.
@pytest.mark.parametrize("rows,K", [(1, 128), (130, 256), (256, 1024), (1000, 384), (40, 22528), (3, 16384)])
def test_quantize_bit_exact(dtype, rows, K):
    rng = np.random.default_rng(rows * 7 + K)
    x = O.make_square_source(rows, K, rng, zero_block_frac=0.05)
    q, sf, q_ref, sf_ref = _run(x, dtype)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(sf, sf_ref)  # includes 0x00 padding rows


def test_quantize_edge_values():
    K = 256
    x = np.zeros((8, K), dtype=np.float32)
    x[0] = 448.0 * 2.0**5  # exact power-of-two multiple of max
    x[1] = np.linspace(-1e-40, 1e-40, K)  # fp32 subnormals
    x[2] = 3e38  # near fp32 max
    x[3, :32] = np.inf  # non-finite block -> 0xFF scale, zero elements
    x[3, 32:] = 1.0
    x[4] = (np.arange(K) - 128) * 1.0001
    x[5, ::2] = 511.0  # saturation inside a block (amax in [256, 512) * 2^e)
    x[5, 1::2] = -300.0
    x[6, 5] = np.nan
    q, sf, q_ref, sf_ref = _run(x, torch.float32)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(sf, sf_ref)
    assert sf_ref[O.sf_offset(3, 0, K)] == 0xFF


def test_quantize_llm_outliers_and_large_rows():
    rng = np.random.default_rng(1)
    x = O.make_llm_activations(300, 2048, rng)
    q, sf, q_ref, sf_ref = _run(x, torch.bfloat16)
    assert np.array_equal(q, q_ref) and np.array_equal(sf, sf_ref)
