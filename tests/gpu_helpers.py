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




# --------------------------------------------------------------------------- full-size BASELINE operands


def device_source_rows(rows, K, kind, seed, zero_block_frac=0.0, role="a"):
    """Seeded fp32 source rows generated on the device with BASELINE's generators.

    ``square``: N(0,1) x per-row 2^U(-4,4), optionally with all-zero 1x32 blocks;
    ``llm``: activations (role "a") N(0,1) with 0.1 % of K-channels x50, weights
    (role "b") N(0, 0.02)."""

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(rows, K, device=dev, generator=g)
    if kind == "llm":
        if role == "a":
            cols = torch.randperm(K, device=dev, generator=g)[: max(1, K // 1000)]
            x[:, cols] *= 50.0
        else:
            x *= 0.02
        return x
    x *= torch.exp2(torch.empty(rows, 1, device=dev).uniform_(-4.0, 4.0, generator=g))
    if zero_block_frac > 0:
        mask = torch.rand(rows, K // 32, device=dev, generator=g) < zero_block_frac
        x.view(rows, K // 32, 32).masked_fill_(mask.unsqueeze(-1), 0.0)
    return x


def device_operands(rows, K, kind="square", seed=0, zero_block_frac=0.0, role="a", chunk=4096, keep=()):
    """Quantised operand [rows, K] + swizzled scales on the device, built in row chunks.

    Each chunk's source comes from ``device_source_rows`` (seed + chunk index) and is
    quantised by the library's quantiser. Returns (codes, scales, kept) where
    ``kept`` maps each row index in ``keep`` to its fp32 source row (numpy), so a
    test can check the quantiser against the oracle on those rows."""

    from cutex_b200.kernels import quantize_mxfp8

    dev = torch.device("cuda")
    q = torch.empty(rows, K, dtype=torch.uint8, device=dev)
    sf = torch.empty(O.sf_buffer_bytes(rows, K), dtype=torch.uint8, device=dev)
    per_row = K // 32
    kept = {}
    for i, r0 in enumerate(range(0, rows, chunk)):
        n = min(chunk, rows - r0)
        x = device_source_rows(n, K, kind, seed * 1000 + i, zero_block_frac, role)
        quantize_mxfp8(x, q=q[r0:r0 + n], sf=sf[r0 * per_row:])
        for r in keep:
            if r0 <= r < r0 + n:
                kept[r] = x[r - r0].cpu().numpy()
        del x
    torch.cuda.synchronize()
    device_ok()
    return q, sf, kept


def check_quantised_rows(q, sf, kept, K):
    """The device codes and scales of the kept rows equal the oracle's quantisation of their sources."""

    sf_c = sf.cpu().numpy()
    for r, src in kept.items():
        codes, scales = O.quantize_mxfp8(src[None, :])
        assert np.array_equal(q[r].cpu().numpy(), codes[0]), f"row {r}: codes differ from the oracle"
        got = sf_c[O.sf_offset(np.full(K // 32, r), np.arange(K // 32), K)]
        assert np.array_equal(got, scales[0]), f"row {r}: scales differ from the oracle"


def rows_scales(sf_buf, rows, K):
    """Logical [len(rows), K/32] scales of the given rows of a swizzled scale buffer (numpy)."""

    r, c = np.meshgrid(np.asarray(rows), np.arange(K // 32), indexing="ij")
    return sf_buf[O.sf_offset(r, c, K)]


def check_sampled_blocks(d, a, sfa, b, sfb, K, row_starts, col_starts, size=64):
    """Oracle check of size x size blocks of D at every (row start, column start); returns the reports."""

    sfa_c = sfa.cpu().numpy()
    sfb_c = sfb.cpu().numpy()
    reports = []
    for r0 in row_starts:
        rows = np.arange(r0, r0 + size)
        ra = a[r0:r0 + size].cpu().numpy()
        rsa = rows_scales(sfa_c, rows, K)
        for c0 in col_starts:
            cols = np.arange(c0, c0 + size)
            rb = b[c0:c0 + size].cpu().numpy()
            rsb = rows_scales(sfb_c, cols, K)
            ref, absum = O.gemm_reference_logical(ra, rsa, rb, rsb)
            got = d[r0:r0 + size, c0:c0 + size].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
            rep = O.check_gemm(got, ref, absum)
            rep["block"] = (int(r0), int(c0))
            reports.append(rep)
    return reports


def boundary_starts(extent, size=64, shard_ways=(2, 4, 8), tile=256):
    """Block starts at the corners, the first tile boundaries, the middle and N-shard boundaries."""

    starts = {0, tile - size // 2, 2 * tile - size // 2, extent // 2 - size // 2, extent - size}
    for g in shard_ways:
        if extent % (g * tile) == 0:
            starts.add(extent // g - size // 2)
    return sorted(s for s in starts if 0 <= s <= extent - size)


__all__ = ["GemmConfig", "O", "boundary_starts", "check", "check_quantised_rows", "check_sampled_blocks", "device_ok",
           "device_operands", "device_source_rows", "make_operands", "rows_scales", "run_gemm"]
