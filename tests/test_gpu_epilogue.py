"""Fused epilogue (cutex_mxfp8_gemm_ex / dense_gemm_fused) vs the CPU oracle.

D = alpha * (A . B^T) + beta * C + bias, in BF16, or in E4M3 with MX scales
along N (the next layer's operand). The exact reference is the oracle's
float64 product sum; the tolerance is the GEMM's (2 BF16 ulps + 2^-16 of
sum |a b|, scaled by |alpha|) plus the rounding of the BF16 C and bias terms.
For E4M3 output the oracle quantiser is applied to the reference and the
scales must agree except for blocks whose amax sits within the accumulation
slack of a power of two; decoded values must agree to one E4M3 step.
"""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import O, device_ok, make_operands

pytestmark = pytest.mark.gpu


def _bf16_to_f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _setup(M, N, K, seed):
    a, sfa, b, sfb = make_operands(M, N, K, seed=seed)
    dev = "cuda"
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    ref, absum = O.gemm_reference(a, sfa, b, sfb, M, N, K)
    return (ta, tb, tsa, tsb), ref, absum


def _check_bf16(out, expected, slack):
    got = _bf16_to_f64(out)
    tol = 2.0 * O.bf16_ulp(expected) + slack
    bad = np.abs(got - expected) > tol
    assert not bad.any(), (int(bad.sum()), float(np.abs(got - expected)[bad].max()))


@pytest.mark.parametrize("shape", [(512, 512, 512), (300, 784, 256), (64, 512, 384), (1024, 768, 1024)], ids=str)
@pytest.mark.parametrize("alpha,beta,use_bias", [(1.0, 0.0, True), (0.5, 1.0, False), (-2.0, 0.25, True)])
def test_affine_epilogue_bf16(shape, alpha, beta, use_bias):
    from cutex_b200.kernels import dense_gemm_fused

    M, N, K = shape
    ops, ref, absum = _setup(M, N, K, seed=M + N + int(alpha * 8))
    rng = np.random.default_rng(7)
    c = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to("cuda").to(torch.bfloat16)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to("cuda").to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dense_gemm_fused(*ops, out, alpha=alpha, beta=beta, c=c if beta != 0 else None, bias=bias if use_bias else None)
    torch.cuda.synchronize()
    device_ok()
    expected = alpha * ref + beta * _bf16_to_f64(c) + (_bf16_to_f64(bias)[None, :] if use_bias else 0.0)
    slack = abs(alpha) * O.ACC_SLACK * absum + 2.0**-20 * (np.abs(beta * _bf16_to_f64(c)) + 1.0)
    _check_bf16(out, expected, slack)


def test_in_place_accumulate_into_d():
    from cutex_b200.kernels import dense_gemm_fused

    M, N, K = 512, 1024, 512
    ops, ref, absum = _setup(M, N, K, seed=3)
    d0 = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    before = _bf16_to_f64(d0)
    dense_gemm_fused(*ops, d0, alpha=1.0, beta=1.0, c=d0)
    torch.cuda.synchronize()
    device_ok()
    _check_bf16(d0, ref + before, O.ACC_SLACK * absum + 2.0**-20 * (np.abs(before) + 1.0))


@pytest.mark.parametrize("shape", [(512, 512, 512), (200, 1024, 256), (1024, 256, 768)], ids=str)
def test_fp8_output_with_mx_scales(shape):
    from cutex_b200.kernels import dense_gemm_fused
    from cutex_b200.kernels.dense_gemm_contract import scale_buffer_bytes

    M, N, K = shape
    ops, ref, absum = _setup(M, N, K, seed=N + K)
    bias = torch.linspace(-1, 1, N, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, dtype=torch.uint8, device="cuda")
    sf = torch.full((scale_buffer_bytes(M, N),), 0x5A, dtype=torch.uint8, device="cuda")
    dense_gemm_fused(*ops, out, alpha=0.75, bias=bias, out_scales=sf)
    torch.cuda.synchronize()
    device_ok()
    expected = 0.75 * ref + _bf16_to_f64(bias)[None, :]
    q_ref, s_ref = O.quantize_mxfp8(expected.astype(np.float32))
    s_ref_sw = O.swizzle_scales(s_ref, N)
    s_got = sf.cpu().numpy()
    match = s_got == s_ref_sw  # includes the 0x00 padding rows of the scale layout
    assert match.mean() > 0.999, match.mean()
    s_got_logical = O.unswizzle_scales(s_got, M, N)
    deq_got = O.dequantize(out.cpu().numpy(), s_got_logical)
    deq_ref = O.dequantize(q_ref, s_ref)
    # One E4M3 step at the block's scale, plus the accumulation slack.
    step = np.exp2(np.floor(np.log2(np.maximum(np.abs(deq_ref), 1e-30))) - 3)
    step = np.maximum(step, np.exp2(s_got_logical.repeat(32, axis=1)[:, :N].astype(np.float64) - 127 - 9))
    tol = step + 0.75 * O.ACC_SLACK * absum
    same_scale = np.repeat(s_got_logical == s_ref, 32, axis=1)[:, :N]
    bad = (np.abs(deq_got - deq_ref) > tol) & same_scale
    assert not bad.any(), int(bad.sum())
    assert (out.cpu().numpy() == q_ref).mean() > 0.99


def test_fp8_output_feeds_the_next_gemm():
    # Layer 1 writes E4M3 + scales; layer 2 consumes them as its A operand unchanged.
    from cutex_b200.kernels import dense_gemm, dense_gemm_fused
    from cutex_b200.kernels.dense_gemm_contract import scale_buffer_bytes
    from tests.gpu_helpers import check

    M, N, K = 256, 512, 256
    ops, _, _ = _setup(M, N, K, seed=11)
    h = torch.empty(M, N, dtype=torch.uint8, device="cuda")
    hs = torch.empty(scale_buffer_bytes(M, N), dtype=torch.uint8, device="cuda")
    dense_gemm_fused(*ops, h, out_scales=hs)
    _, _, w2, sw2 = make_operands(M, 384, N, seed=12)
    out2 = torch.empty(M, 384, dtype=torch.bfloat16, device="cuda")
    dense_gemm(h, torch.from_numpy(w2).cuda(), hs, torch.from_numpy(sw2).cuda(), out2)
    torch.cuda.synchronize()
    device_ok()
    r = check(out2, h.cpu().numpy(), hs.cpu().numpy(), w2, sw2, M, 384, N)
    assert r["ok"], r
