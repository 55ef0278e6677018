"""CPU oracle for the MXFP8 block-scaled GEMM contract -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker / CPU baseline.
The product path (``cutex_b200``) never imports it and has no CPU fallback.

It restates, in numpy, the arithmetic of the reference's fixed Fprop contract:

* contract constants and FLOP count: ``cutex/kernels/dense_gemm_contract.py:6-41``;
* scale-factor index of row ``r``, K element ``k`` in the 128x4 swizzled
  layout: ``cutex/kernels/dense_gemm_v1.py:24-30`` (``_scale_index``), byte map
  ``benchmarks/SM100_MXFP8_SF_LAYOUT_SMEM_TMEM.md:69-115``, SMEM/GMEM layout
  pinned in ``tests/test_dense_gemm_v2_scaffold.py:58-61,68-69``;
* dequantise ``a * sa`` / ``b * sb`` then FP32 multiply-accumulate:
  ``cutex/kernels/dense_gemm_v1.py:69-79`` (and ``dense_gemm_v2.py:190-195``);
* BF16 output by round-to-nearest-even: ``dense_gemm_v13.py:909`` (``acc.to(BF16)``);
* the OCP MX E4M3/E8M0 quantiser that the reference takes from Transformer
  Engine (``modal_dense_gemm.py:358-373``; TE 2.17 is not vendored), with the
  scale rule BASELINE fixes: exponent ``floor(log2(amax)) - 8``.

Parity pinning: the scale-factor index is checked against the reference's own
``_scale_index`` through committed golden vectors (``tests/golden``); the
contract constants against ``dense_gemm_contract``. The reference has no numeric
GEMM golden vectors (its tests are GPU-free and non-numeric), so GEMM parity is
pinned through the contract restated here plus two independent FP8 decoders.
"""

from __future__ import annotations

import math

import numpy as np

SF_VECTOR_SIZE = 32
E4M3_MAX = 448.0


# --------------------------------------------------------------------------- E4M3 / E8M0


def _build_e4m3_table() -> np.ndarray:
    """Decode table for all 256 E4M3FN codes (bias 7, 3 mantissa bits, NaN = S.1111.111)."""

    table = np.empty(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 0xF and man == 0x7:
            table[code] = np.nan
        elif exp == 0:
            table[code] = sign * man * 2.0**-9
        else:
            table[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return table


E4M3_TABLE = _build_e4m3_table()


def decode_e4m3(codes: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


def decode_e8m0(codes: np.ndarray) -> np.ndarray:
    """E8M0 (unsigned exponent, bias 127): byte b -> 2^(b-127); 0xFF -> NaN. Bit-exact in fp32."""

    b = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    with np.errstate(over="ignore"):
        out = np.ldexp(np.float64(1.0), np.minimum(b, 254) - 127).astype(np.float32)  # 2^-127: exact subnormal
    out[b == 255] = np.nan
    return out


def encode_e4m3_rne_sat(y: np.ndarray) -> np.ndarray:
    """fp32 -> E4M3FN code, round-to-nearest-even, saturating at +-448 (NaN -> 0x7F)."""

    y = np.asarray(y, dtype=np.float32)
    a = np.abs(y).astype(np.float64)
    sign = np.where(np.signbit(y), 0x80, 0x00).astype(np.int32)
    code = np.zeros(y.shape, dtype=np.int32)

    sub = a < 2.0**-6
    # Subnormals (and the rounding edge into the first normal): multiples of 2^-9;
    # code m = round_half_even(a / 2^-9) maps 8 onto the first normal code 0x08.
    code[sub] = np.rint(a[sub] * 2.0**9).astype(np.int32)

    # Non-finite inputs never reach the exponent arithmetic: infinities saturate
    # and NaN maps to 0x7F below.
    nrm = ~sub & np.isfinite(a)
    an = a[nrm]
    e = np.floor(np.log2(an)).astype(np.int32)
    # Guard log2 rounding at exact powers of two.
    e = np.where(np.ldexp(1.0, e) > an, e - 1, e)
    e = np.where(np.ldexp(1.0, e + 1) <= an, e + 1, e)
    q = np.rint((an / np.ldexp(1.0, e) - 1.0) * 8.0).astype(np.int32)
    carry = q == 8
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 0, q)
    code[nrm] = ((e + 7) << 3) | q

    code = np.where(a >= E4M3_MAX, 0x7E, code)  # satfinite
    code = np.where(np.isnan(y), 0x7F, code | sign)
    return code.astype(np.uint8)


# --------------------------------------------------------------------------- scale layout


def sf_offset(r, c, K: int):
    """Byte offset of the scale of row ``r``, K-block ``c`` (= k // 32) in the 128x4 layout."""

    r = np.asarray(r, dtype=np.int64)
    c = np.asarray(c, dtype=np.int64)
    return ((r // 128) * (K // 128) + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4


def sf_buffer_bytes(rows: int, K: int) -> int:
    return ((rows + 127) // 128) * 128 * (K // SF_VECTOR_SIZE)


def swizzle_scales(sf_logical: np.ndarray, K: int) -> np.ndarray:
    """[rows, K/32] logical E8M0 -> flat swizzled buffer; padding rows are 0x00."""

    rows, ncols = sf_logical.shape
    assert ncols == K // SF_VECTOR_SIZE and K % 128 == 0
    out = np.zeros(sf_buffer_bytes(rows, K), dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(ncols), indexing="ij")
    out[sf_offset(r, c, K)] = sf_logical
    return out


def unswizzle_scales(sf_buffer: np.ndarray, rows: int, K: int) -> np.ndarray:
    r, c = np.meshgrid(np.arange(rows), np.arange(K // SF_VECTOR_SIZE), indexing="ij")
    return np.asarray(sf_buffer, dtype=np.uint8)[sf_offset(r, c, K)]


# --------------------------------------------------------------------------- quantiser


def quantize_mxfp8(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """OCP MX E4M3 quantiser: returns (codes u8 [rows, K], logical scales u8 [rows, K/32]).

    Scale byte = exponent_field(amax) - 8 clamped at 0 (scale exponent
    floor(log2 amax) - 8, >= -127); a block with a non-finite value gets 0xFF and
    zero elements. Elements: x * 2^(127 - byte) in fp32 (exact), then E4M3 RNE
    with saturation.
    """

    x = np.asarray(x, dtype=np.float32)
    rows, K = x.shape
    assert K % SF_VECTOR_SIZE == 0
    blocks = x.reshape(rows, K // SF_VECTOR_SIZE, SF_VECTOR_SIZE)
    absb = np.abs(blocks)
    nonfinite = ~np.isfinite(blocks).all(axis=2)
    amax = np.where(nonfinite, 0.0, absb.max(axis=2)).astype(np.float32)
    exp_field = (amax.view(np.uint32) >> 23).astype(np.int32)
    sbyte = np.maximum(exp_field - 8, 0)
    sbyte = np.where(nonfinite, 255, sbyte).astype(np.uint8)
    mult = np.ldexp(np.float32(1.0), 127 - np.minimum(sbyte.astype(np.int32), 254)).astype(np.float32)
    y = blocks * mult[:, :, None]
    codes = encode_e4m3_rne_sat(y)
    codes = np.where(nonfinite[:, :, None], 0, codes).astype(np.uint8)
    return codes.reshape(rows, K), sbyte


def dequantize(codes: np.ndarray, sf_logical: np.ndarray) -> np.ndarray:
    """a * sa per 1x32 block, in fp32 (exact: E4M3 x 2^e)."""

    rows, K = codes.shape
    vals = decode_e4m3(codes).reshape(rows, K // SF_VECTOR_SIZE, SF_VECTOR_SIZE)
    scale = decode_e8m0(sf_logical)
    with np.errstate(invalid="ignore", over="ignore"):
        out = vals.astype(np.float64) * scale.astype(np.float64)[:, :, None]
    return out.reshape(rows, K)


# --------------------------------------------------------------------------- GEMM reference


def bf16_rne_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round-to-nearest-even; NaN stays NaN."""

    f = np.asarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(f)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemm_reference(a_codes, sfa_buffer, b_codes, sfb_buffer, M: int, N: int, K: int):
    """Contract reference: dequant A/B with their E8M0 scales, matmul, return (ref_f64, abs_f64).

    ``ref_f64`` is the exact product sum (float64 accumulation of exact fp32
    products); ``abs_f64`` = sum_k |a_k b_k| bounds the accumulation-order error
    of any FP32 summation order.
    """

    sfa = unswizzle_scales(sfa_buffer, M, K)
    sfb = unswizzle_scales(sfb_buffer, N, K)
    a = dequantize(np.asarray(a_codes).reshape(M, K), sfa)
    b = dequantize(np.asarray(b_codes).reshape(N, K), sfb)
    ref = a @ b.T
    absum = np.abs(a) @ np.abs(b).T
    return ref, absum


def contract_output_bf16(ref_f64: np.ndarray) -> np.ndarray:
    """FP32 matmul result cast to BF16 (RNE), as bit patterns."""

    return bf16_rne_bits(ref_f64.astype(np.float32))


# --------------------------------------------------------------------------- tolerance

REL_FRO_TOL = 1e-3  # max relative Frobenius error vs the BF16 contract output
ULP_TOL = 2.0  # per element: BF16 ulps of the FP32 reference ...
ACC_SLACK = 2.0**-16  # ... plus this fraction of sum_k |a_k b_k| (accumulation order)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    ax = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0**-126)))
    return np.ldexp(1.0, (e - 7).astype(np.int64))


def check_gemm(d_bits: np.ndarray, ref_f64: np.ndarray, absum: np.ndarray) -> dict:
    """Contract tolerance check; returns the measured errors and a pass flag."""

    d = bf16_bits_to_f32(d_bits).astype(np.float64)
    ref_bf16 = bf16_bits_to_f32(contract_output_bf16(ref_f64)).astype(np.float64)
    finite = np.isfinite(d).all()
    denom = np.linalg.norm(ref_bf16)
    rel_fro = float(np.linalg.norm(d - ref_bf16) / denom) if denom > 0 else float(np.linalg.norm(d))
    bound = ULP_TOL * bf16_ulp(ref_f64) + ACC_SLACK * absum
    err = np.abs(d - ref_f64)
    worst = float(np.max(err / np.maximum(bound, 1e-300))) if err.size else 0.0
    exact = float(np.mean(d_bits == contract_output_bf16(ref_f64))) if err.size else 1.0
    ok = bool(finite and rel_fro <= REL_FRO_TOL and worst <= 1.0)
    return {
        "ok": ok,
        "finite": bool(finite),
        "rel_fro": rel_fro,
        "worst_bound_ratio": worst,
        "bitexact_fraction": exact,
    }


# --------------------------------------------------------------------------- inputs


def make_square_source(rows: int, K: int, rng: np.random.Generator, zero_block_frac: float = 0.0):
    """N(0,1) x per-row 2^U(-4,4); optionally all-zero 1x32 blocks (E8M0 minimum scale)."""

    x = rng.standard_normal((rows, K), dtype=np.float32)
    x *= np.exp2(rng.uniform(-4.0, 4.0, size=(rows, 1))).astype(np.float32)
    if zero_block_frac > 0:
        mask = rng.random((rows, K // SF_VECTOR_SIZE)) < zero_block_frac
        x.reshape(rows, K // SF_VECTOR_SIZE, SF_VECTOR_SIZE)[mask] = 0.0
    return x


def make_llm_activations(rows: int, K: int, rng: np.random.Generator, outlier_frac=0.001, scale=50.0):
    x = rng.standard_normal((rows, K), dtype=np.float32)
    n_out = max(1, int(round(K * outlier_frac)))
    cols = rng.choice(K, size=n_out, replace=False)
    x[:, cols] *= scale
    return x


def make_llm_weights(rows: int, K: int, rng: np.random.Generator, std=0.02):
    return (rng.standard_normal((rows, K), dtype=np.float32) * np.float32(std)).astype(np.float32)


def quantized_operands(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Quantise and return (codes [rows, K], swizzled scale buffer)."""

    codes, sf = quantize_mxfp8(x)
    return codes, swizzle_scales(sf, x.shape[1])


def dense_gemm_flops(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def gemm_bytes(m: int, n: int, k: int) -> int:
    """Compulsory HBM bytes: E4M3 A and B, E8M0 scales, BF16 D."""

    return m * k + n * k + (m + n) * (k // SF_VECTOR_SIZE) + 2 * m * n


__all__ = [name for name in dir() if not name.startswith("_") and name not in {"annotations", "math", "np"}]


def gemm_reference_logical(a_codes, sfa_logical, b_codes, sfb_logical):
    """Same as gemm_reference for row subsets given logical [rows, K/32] scales."""

    a = dequantize(np.asarray(a_codes), np.asarray(sfa_logical))
    b = dequantize(np.asarray(b_codes), np.asarray(sfb_logical))
    return a @ b.T, np.abs(a) @ np.abs(b).T
