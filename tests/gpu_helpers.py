"""Shared helpers for the GPU parity tests: build operands, run the CUDA path, check with the oracle."""

import numpy as np
import torch

from cutex_b200 import _lib
from cutex_b200.kernels import GemmConfig, dense_gemm
from oracle import mxfp8_oracle as O


def device_ok():
    assert _lib.load().cutex_last_device_status(torch.cuda.current_stream().cuda_stream) == 0


def make_operands(M, N, K, seed=0, zero_block_frac=0.0, kind="square"):
    rng = np.random.default_rng(seed)
    if kind == "square":
        xa = O.make_square_source(M, K, rng, zero_block_frac)
        xb = O.make_square_source(N, K, rng, zero_block_frac)
    elif kind == "llm":
        xa = O.make_llm_activations(M, K, rng)
        xb = O.make_llm_weights(N, K, rng)
    elif kind == "wide_exponent":
        xa = O.make_square_source(M, K, rng) * np.exp2(rng.integers(-40, 40, (M, 1))).astype(np.float32)
        xb = O.make_square_source(N, K, rng) * np.exp2(rng.integers(-40, 40, (N, 1))).astype(np.float32)
    else:
        raise ValueError(kind)
    a, sfa = O.quantized_operands(xa)
    b, sfb = O.quantized_operands(xb)
    return a, sfa, b, sfb


def run_gemm(a, sfa, b, sfb, M, N, K, config=None, ldd=None, out=None):
    dev = torch.device("cuda")
    ta = torch.from_numpy(a).to(dev)
    tb = torch.from_numpy(b).to(dev)
    tsa = torch.from_numpy(sfa).to(dev)
    tsb = torch.from_numpy(sfb).to(dev)
    ldd = ldd or N
    if out is None:
        full = torch.full((M, ldd), float("nan"), dtype=torch.bfloat16, device=dev)
        out = full[:, :N]
    dense_gemm(ta, tb, tsa, tsb, out, config=config)
    torch.cuda.synchronize()
    device_ok()
    return out


def check(out, a, sfa, b, sfb, M, N, K):
    ref, absum = O.gemm_reference(a, sfa, b, sfb, M, N, K)
    bits = out.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
    return O.check_gemm(bits, ref, absum)


__all__ = ["GemmConfig", "O", "check", "device_ok", "make_operands", "run_gemm"]
