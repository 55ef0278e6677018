"""The contract's PyTorch CPU path -- TEST/BASELINE INFRASTRUCTURE ONLY.

Decode E4M3 -> fp32, multiply by 2^(e8m0 - 127) per 1x32 block, fp32 matmul,
cast to BF16: the "dequantise, FP32 matmul, cast to BF16" reference of the
contract (``cutex/kernels/dense_gemm_v1.py:69-84``). ``bench.py`` times it on
the host cores as the CPU baseline (``cpu_baseline`` / ``--impl reference``);
it is never a fallback of the product path.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

from .mxfp8_oracle import sf_offset


def unswizzle_rows(sf_buffer: torch.Tensor, rows: np.ndarray, K: int) -> torch.Tensor:
    """Logical [len(rows), K/32] scales of the given rows from a 128x4-swizzled buffer (CPU tensor)."""

    r, c = np.meshgrid(np.asarray(rows, dtype=np.int64), np.arange(K // 32), indexing="ij")
    return sf_buffer[torch.from_numpy(sf_offset(r, c, K))]


def dequant(codes: torch.Tensor, sf_logical: torch.Tensor) -> torch.Tensor:
    rows, K = codes.shape
    vals = codes.view(torch.float8_e4m3fn).float().view(rows, K // 32, 32)
    scale = sf_logical.view(torch.float8_e8m0fnu).float()
    return (vals * scale.unsqueeze(-1)).view(rows, K)


def cpu_contract_gemm(a_codes, sfa_logical, b_codes, sfb_logical) -> torch.Tensor:
    """D = (dequant(A) @ dequant(B)^T) in fp32, cast to BF16 -- on the CPU."""

    a = dequant(a_codes, sfa_logical)
    b = dequant(b_codes, sfb_logical)
    return (a @ b.T).to(torch.bfloat16)


def time_cpu_contract(a_codes, sfa_logical, b_codes, sfb_logical, *, min_seconds=8.0, max_reps=5):
    """Median wall time (s) of the CPU contract path over repeated runs, using every host core."""

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu_contract_gemm(a_codes, sfa_logical, b_codes, sfb_logical)  # warm-up (allocator, thread pool)
    times = []
    t_start = time.perf_counter()
    while len(times) < max_reps and (len(times) < 2 or time.perf_counter() - t_start < min_seconds):
        t0 = time.perf_counter()
        cpu_contract_gemm(a_codes, sfa_logical, b_codes, sfb_logical)
        times.append(time.perf_counter() - t0)
    return float(np.median(times)), threads, len(times)


def cpu_sample_operands(rows_a: int, rows_b: int, K: int, dist: str = "square", seed: int = 0):
    """Seeded MXFP8 operands on the CPU for timing the contract path: (a, sfa, b, sfb), logical scales.

    Sources follow BASELINE's generators (``square``: N(0,1) x per-row
    2^U(-4,4); ``llm``: activations N(0,1) with 0.1 % of K-channels x50, weights
    N(0, 0.02)), drawn from a CPU ``torch.Generator``; quantisation is the OCP MX
    rule of the oracle (scale byte = exponent field of the block amax - 8,
    elements x * 2^(127 - byte) rounded to E4M3 with saturation), done with
    torch's float8 cast so that a 4096-row sample takes about a second. Both
    CPU timing legs of ``bench.py`` use this one function, so they time the same
    operands.
    """

    g = torch.Generator().manual_seed(seed)

    def source(rows, is_a):
        x = torch.randn(rows, K, generator=g)
        if dist == "llm":
            if is_a:
                x[:, torch.randperm(K, generator=g)[: max(1, K // 1000)]] *= 50.0
            else:
                x *= 0.02
            return x
        return x * torch.exp2(torch.empty(rows, 1).uniform_(-4.0, 4.0, generator=g))

    def quantise(x):
        rows = x.shape[0]
        blocks = x.view(rows, K // 32, 32)
        amax = blocks.abs().amax(dim=2)
        sbyte = ((amax.view(torch.int32) >> 23) - 8).clamp(min=0)
        mult = torch.ldexp(torch.ones(()), (127 - sbyte).float())
        y = (blocks * mult.unsqueeze(-1)).clamp(-448.0, 448.0)
        return y.to(torch.float8_e4m3fn).view(torch.uint8).view(rows, K), sbyte.to(torch.uint8)

    a, sfa = quantise(source(rows_a, True))
    b, sfb = quantise(source(rows_b, False))
    return a, sfa, b, sfb
