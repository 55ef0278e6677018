"""CPU oracle pinned against the reference's golden vectors and independent codecs."""

import json

import numpy as np
import pytest
import torch

from oracle import mxfp8_oracle as O
from tests.conftest import GOLDEN


def test_sf_offset_matches_reference_scale_index_golden():
    # Golden vectors produced by the reference's own _scale_index (dense_gemm_v1.py:24-30).
    data = json.loads((GOLDEN / "sf_index_k16384.json").read_text())
    K = data["K"]
    cases = np.array(data["cases"], dtype=np.int64)
    outer, k, expected = cases[:, 0], cases[:, 1], cases[:, 2]
    assert np.array_equal(O.sf_offset(outer, k // 32, K), expected)
    assert len(cases) > 4000


def test_sf_offset_reproduces_reference_cute_layout_strides():
    # tests/test_dense_gemm_v2_scaffold.py:58-61 pins the GMEM SF layout at 16384:
    #   shape  = (((32, 4), 128), ((32, 4), 128), 1)
    #   stride = (((16, 4), 65536), ((0, 1), 512), 8388608)
    K = 16384
    rng = np.random.default_rng(1)
    r = rng.integers(0, 16384, 5000)
    k = rng.integers(0, 16384, 5000)
    r0, r1, r2 = r % 32, (r // 32) % 4, r // 128
    k0, k1, k2 = k % 32, (k // 32) % 4, k // 128
    cute = r0 * 16 + r1 * 4 + r2 * 65536 + k0 * 0 + k1 * 1 + k2 * 512
    assert np.array_equal(O.sf_offset(r, k // 32, K), cute)
    # Total size = 8388608 bytes = SCALE_FACTOR_ELEMENTS.
    assert O.sf_buffer_bytes(16384, 16384) == 8388608


def test_sf_offset_is_a_bijection_for_padded_shapes():
    for rows, K in [(1, 128), (130, 256), (300, 512), (256, 1024)]:
        r, c = np.meshgrid(np.arange(((rows + 127) // 128) * 128), np.arange(K // 32), indexing="ij")
        offs = O.sf_offset(r, c, K).ravel()
        assert np.array_equal(np.sort(offs), np.arange(O.sf_buffer_bytes(rows, K)))


def test_e4m3_decode_table_matches_torch():
    codes = np.arange(256, dtype=np.uint8)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    ours = O.decode_e4m3(codes)
    assert np.array_equal(np.isnan(ours), np.isnan(theirs))
    assert np.array_equal(ours[~np.isnan(ours)], theirs[~np.isnan(theirs)])
    assert O.decode_e4m3(np.array([0x7E]))[0] == 448.0
    assert O.decode_e4m3(np.array([0x01]))[0] == 2.0**-9


def test_e8m0_decode_is_bit_exact():
    codes = np.arange(256, dtype=np.uint8)
    ours = O.decode_e8m0(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e8m0fnu).float().numpy()
    assert ours[127] == 1.0
    assert ours[0].view(np.uint32) == 0x00400000  # 2^-127, fp32 subnormal
    assert np.isnan(ours[255])
    finite = ~np.isnan(ours)
    assert np.array_equal(ours[finite].view(np.uint32), theirs[finite].view(np.uint32))
    for b in range(1, 255):
        assert ours[b].view(np.uint32) == (b << 23)


def test_e4m3_encoder_rne_saturating_matches_torch_cast():
    rng = np.random.default_rng(0)
    y = np.concatenate([rng.standard_normal(50000).astype(np.float32) * s for s in (1e-3, 0.05, 1, 30, 500)])
    mids = ((O.E4M3_TABLE[:126].astype(np.float64) + O.E4M3_TABLE[1:127]) / 2).astype(np.float32)
    y = np.concatenate([y, mids, -mids, np.float32([448, 449, 463.99, 464, 1e9, -1e9, 0.0, -0.0])])
    theirs = torch.from_numpy(np.clip(y, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.encode_e4m3_rne_sat(y), theirs)


def test_quantizer_scale_rule_and_range():
    rng = np.random.default_rng(3)
    x = O.make_square_source(64, 512, rng, zero_block_frac=0.1)
    codes, sf = O.quantize_mxfp8(x)
    blocks = x.reshape(64, 16, 32)
    amax = np.abs(blocks).max(axis=2)
    nz = amax > 0
    # scale exponent = floor(log2 amax) - 8
    assert np.array_equal(sf[nz].astype(np.int32) - 127, np.floor(np.log2(amax[nz])).astype(np.int32) - 8)
    assert np.all(sf[~nz] == 0)  # all-zero block -> E8M0 minimum
    deq = O.dequantize(codes, sf)
    scale = O.decode_e8m0(sf).astype(np.float64).repeat(32, axis=1)
    y = x / scale  # the value handed to the E4M3 cast
    sat = np.abs(y) >= 448
    # Saturated elements decode to +-448 * scale ...
    assert np.array_equal(deq[sat], np.sign(x[sat]) * 448 * scale[sat])
    # ... the rest are within half an E4M3 ulp: 2^-4 relative (normal) or 2^-10 (subnormal grid).
    err = np.abs(deq - x)[~sat]
    bound = np.maximum(np.abs(x[~sat]) * 2.0**-4, 2.0**-10 * scale[~sat])
    assert np.all(err <= bound * (1 + 1e-12))
    assert sat.any() and (~sat).any()


def test_quantizer_nonfinite_block():
    x = np.ones((1, 64), dtype=np.float32)
    x[0, 40] = np.inf
    codes, sf = O.quantize_mxfp8(x)
    assert sf[0, 1] == 255 and np.all(codes[0, 32:] == 0)
    assert sf[0, 0] == 127 - 8 and codes[0, 0] == O.encode_e4m3_rne_sat(np.float32([256.0]))[0]


def test_swizzle_roundtrip_and_padding():
    rng = np.random.default_rng(5)
    sf = rng.integers(0, 255, size=(200, 8), dtype=np.uint8)
    buf = O.swizzle_scales(sf, 256)
    assert buf.size == 256 * 8
    assert np.array_equal(O.unswizzle_scales(buf, 200, 256), sf)
    pad_r, pad_c = np.meshgrid(np.arange(200, 256), np.arange(8), indexing="ij")
    assert np.all(buf[O.sf_offset(pad_r, pad_c, 256)] == 0)


def test_gemm_reference_against_scalar_loop():
    rng = np.random.default_rng(7)
    M, N, K = 5, 3, 128
    a, sfa = O.quantized_operands(O.make_square_source(M, K, rng))
    b, sfb = O.quantized_operands(O.make_square_source(N, K, rng))
    ref, absum = O.gemm_reference(a, sfa, b, sfb, M, N, K)
    sa = O.unswizzle_scales(sfa, M, K)
    sb = O.unswizzle_scales(sfb, N, K)
    for i in range(M):
        for j in range(N):
            acc = 0.0
            for kk in range(K):
                acc += float(O.E4M3_TABLE[a[i, kk]]) * 2.0 ** (int(sa[i, kk // 32]) - 127) * float(
                    O.E4M3_TABLE[b[j, kk]]
                ) * 2.0 ** (int(sb[j, kk // 32]) - 127)
            assert ref[i, j] == pytest.approx(acc, rel=1e-12, abs=1e-30)


def test_bf16_rne_matches_torch():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(100000) * np.exp2(rng.uniform(-30, 30, 100000))).astype(np.float32)
    ours = O.bf16_rne_bits(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_tolerance_checker_accepts_contract_output_and_flags_planted_error():
    rng = np.random.default_rng(11)
    M, N, K = 64, 48, 256
    a, sfa = O.quantized_operands(O.make_square_source(M, K, rng))
    b, sfb = O.quantized_operands(O.make_square_source(N, K, rng))
    ref, absum = O.gemm_reference(a, sfa, b, sfb, M, N, K)
    good = O.contract_output_bf16(ref)
    assert O.check_gemm(good, ref, absum)["ok"]
    # Plant a mistake in the oracle's own output: double one scale block of row 3.
    sfa_bad = sfa.copy()
    sfa_bad[O.sf_offset(3, 2, K)] += 1
    ref_bad, _ = O.gemm_reference(a, sfa_bad, b, sfb, M, N, K)
    assert not O.check_gemm(O.contract_output_bf16(ref_bad), ref, absum)["ok"]
    # A single flipped low bit (1 bf16 ulp) is within tolerance.
    nudged = good.copy()
    nudged[0, 0] ^= 1
    assert O.check_gemm(nudged, ref, absum)["ok"]


def test_flops_and_bytes_per_baseline_table():
    assert O.dense_gemm_flops(16384, 16384, 16384) == 2 * 16384**3
    assert O.gemm_bytes(16384, 16384, 16384) == 1090519040  # 1090.5 MB
    assert O.gemm_bytes(16, 28672, 8192) == 243273728  # 243.3 MB


def test_cpu_sample_operands_match_the_oracle_quantiser():
    # The CPU timing legs' fast torch quantiser equals the oracle's on the same sources.
    import torch

    from oracle.cpu_contract import cpu_sample_operands

    for dist in ("square", "llm"):
        a, sfa, b, sfb = cpu_sample_operands(160, 96, 512, dist=dist, seed=3)
        g = torch.Generator().manual_seed(3)
        xa = torch.randn(160, 512, generator=g)
        if dist == "llm":
            xa[:, torch.randperm(512, generator=g)[:1]] *= 50.0
            xb = torch.randn(96, 512, generator=g) * 0.02
        else:
            xa = xa * torch.exp2(torch.empty(160, 1).uniform_(-4.0, 4.0, generator=g))
            xb = torch.randn(96, 512, generator=g)
            xb = xb * torch.exp2(torch.empty(96, 1).uniform_(-4.0, 4.0, generator=g))
        for (q, s), x in (((a, sfa), xa), ((b, sfb), xb)):
            q_ref, s_ref = O.quantize_mxfp8(x.numpy())
            assert np.array_equal(q.numpy(), q_ref) and np.array_equal(s.numpy(), s_ref)
