"""Columnwise MXFP8 quantiser (x -> quantise(x^T)) vs the CPU oracle, and the
weight/input-gradient GEMMs it enables, through the C ABI.

The columnwise result must equal the rowwise oracle applied to x^T bit for bit
(codes and swizzled scales, padding rows included). Wgrad and Dgrad are then
plain TN GEMMs of the existing kernel on columnwise/rowwise operands and are
checked with the GEMM tolerance against the oracle's dequantise-multiply.
"""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import O, check, device_ok

pytestmark = pytest.mark.gpu


def _col(x_np, dtype, ldx=None):
    from cutex_b200.kernels import quantize_mxfp8_columnwise

    rows, cols = x_np.shape
    if ldx is None and cols % 8:
        ldx = (cols + 7) // 8 * 8  # the row stride must be a multiple of 8 elements
    if ldx is None:
        x = torch.from_numpy(x_np).to("cuda").to(dtype)
    else:
        full = torch.zeros(rows, ldx, dtype=dtype, device="cuda")
        full[:, :cols] = torch.from_numpy(x_np).to("cuda").to(dtype)
        x = full[:, :cols]
    qt, sft = quantize_mxfp8_columnwise(x)
    torch.cuda.synchronize()
    device_ok()
    src_t = np.ascontiguousarray(x.float().cpu().numpy().T)  # what the kernel saw, transposed
    q_ref, sf_ref = O.quantize_mxfp8(src_t)
    return qt.cpu().numpy(), sft.cpu().numpy(), q_ref, O.swizzle_scales(sf_ref, rows)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
# (2176, 260): 17 row tiles, so the tile order's last group of row tiles is a partial one.
@pytest.mark.parametrize("rows,cols", [(128, 64), (128, 1), (256, 200), (384, 130), (1024, 512), (128, 4100),
                                       (2176, 260)])
def test_columnwise_bit_exact(dtype, rows, cols):
    rng = np.random.default_rng(rows * 11 + cols)
    x = O.make_square_source(rows, cols, rng, zero_block_frac=0.0)
    # Column-scale spread (the rows of x^T) plus some all-zero 32-row blocks.
    x *= np.exp2(rng.integers(-6, 7, size=(1, cols))).astype(np.float32)
    x[32:64, ::3] = 0.0
    qt, sft, q_ref, sf_ref = _col(x, dtype)
    assert np.array_equal(qt, q_ref)
    assert np.array_equal(sft, sf_ref)


def test_columnwise_row_stride_and_edge_values():
    rows, cols = 256, 72
    x = np.zeros((rows, cols), dtype=np.float32)
    x[:32, 0] = np.inf  # non-finite block -> 0xFF scale, zero codes
    x[32:64, 1] = 448.0 * 2.0**9
    x[:, 2] = np.linspace(-1e-40, 1e-40, rows)  # subnormals
    x[::2, 3] = 511.0
    x[1::2, 3] = -300.0
    x[:, 4] = 3e38
    qt, sft, q_ref, sf_ref = _col(x, torch.float32, ldx=80)
    assert np.array_equal(qt, q_ref)
    assert np.array_equal(sft, sf_ref)
    assert sf_ref[O.sf_offset(0, 0, rows)] == 0xFF


def test_wgrad_and_dgrad_through_columnwise_operands():
    from cutex_b200.kernels import dense_gemm, quantize_mxfp8, quantize_mxfp8_columnwise

    rng = np.random.default_rng(3)
    tokens, n_out, k_in = 512, 384, 256
    dy = (rng.standard_normal((tokens, n_out)) * 0.1).astype(np.float32)
    xin = rng.standard_normal((tokens, k_in)).astype(np.float32)
    w = (rng.standard_normal((n_out, k_in)) * 0.02).astype(np.float32)
    dev = "cuda"
    tdy, tx, tw = (torch.from_numpy(v).to(dev) for v in (dy, xin, w))

    # Wgrad: dW[n_out, k_in] = dY^T X, reduction over tokens: both operands columnwise.
    a_q, a_s = quantize_mxfp8_columnwise(tdy)  # [n_out, tokens]
    b_q, b_s = quantize_mxfp8_columnwise(tx)  # [k_in, tokens]
    dw = torch.empty(n_out, k_in, dtype=torch.bfloat16, device=dev)
    dense_gemm(a_q, b_q, a_s, b_s, dw)
    # Dgrad: dX[tokens, k_in] = dY W, reduction over n_out: dY rowwise, W columnwise.
    c_q, c_s = quantize_mxfp8(tdy)  # [tokens, n_out]
    d_q, d_s = quantize_mxfp8_columnwise(tw)  # [k_in, n_out]
    dx = torch.empty(tokens, k_in, dtype=torch.bfloat16, device=dev)
    dense_gemm(c_q, d_q, c_s, d_s, dx)
    torch.cuda.synchronize()
    device_ok()
    for out, (aq, asf, bq, bsf), (M, N, K) in (
        (dw, (a_q, a_s, b_q, b_s), (n_out, k_in, tokens)),
        (dx, (c_q, c_s, d_q, d_s), (tokens, k_in, n_out)),
    ):
        host = [t.cpu().numpy() for t in (aq, asf, bq, bsf)]
        r = check(out, host[0], host[1], host[2], host[3], M, N, K)
        assert r["ok"], r
