"""GPU MXFP8 GEMM vs the CPU oracle, through the C ABI, for every kernel variant.

Tolerance (the contract's): relative Frobenius error <= 1e-3 against the BF16
contract output, and every element within 2 BF16 ulps of the exact product sum
plus 2^-16 * sum_k |a_k b_k| of accumulation-order slack.
"""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import GemmConfig, O, check, device_ok, make_operands, run_gemm

pytestmark = pytest.mark.gpu

# Every instantiated kernel: dynamic (cluster launch control, scheduler=0) and static (scheduler=1).
VARIANTS = [
    GemmConfig(kernel=2, tile_n=256, stages=6, epi_buffers=1, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=2, tile_n=256, stages=5, epi_buffers=2, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=2, tile_n=256, stages=6, epi_buffers=1, sf_buffers=2, scheduler=0),
    GemmConfig(kernel=2, tile_n=256, stages=4, epi_buffers=2, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=1, tile_n=256, stages=4, epi_buffers=1, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=1, tile_n=256, stages=3, epi_buffers=2, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=1, tile_n=128, stages=6, epi_buffers=1, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=1, tile_n=128, stages=5, epi_buffers=2, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=1, tile_n=128, stages=6, epi_buffers=1, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=1, tile_n=128, stages=5, epi_buffers=2, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=1, tile_n=128, stages=4, epi_buffers=2, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=1, tile_n=128, stages=6, epi_buffers=1, sf_buffers=1, scheduler=1),
    GemmConfig(kernel=1, tile_n=256, stages=4, epi_buffers=1, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=1, tile_n=256, stages=3, epi_buffers=2, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=1, tile_n=256, stages=4, epi_buffers=1, sf_buffers=1, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=6, epi_buffers=1, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=5, epi_buffers=2, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=4, epi_buffers=2, sf_buffers=2, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=6, epi_buffers=1, sf_buffers=1, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=6, epi_buffers=1, sf_buffers=4, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=5, epi_buffers=2, sf_buffers=4, scheduler=1),
    GemmConfig(kernel=2, tile_n=256, stages=5, epi_buffers=2, sf_buffers=1, scheduler=1),
    GemmConfig(kernel=2, tile_n=128, stages=6, epi_buffers=2, sf_buffers=1, scheduler=0),
    GemmConfig(kernel=2, tile_n=128, stages=8, epi_buffers=1, sf_buffers=1, scheduler=0),
]
DYN_2CTA, DYN_1CTA_256, DYN_1CTA_128 = VARIANTS[0], VARIANTS[4], VARIANTS[6]
DYN_2CTA_128 = VARIANTS[23]
ST_1CTA_128, ST_1CTA_256, ST_2CTA = VARIANTS[11], VARIANTS[14], VARIANTS[18]


def _id(cfg):
    return f"k{cfg.kernel}_n{cfg.tile_n}_s{cfg.stages}_e{cfg.epi_buffers}_f{cfg.sf_buffers}_{'st' if cfg.scheduler else 'dyn'}"


def _assert_ok(report):
    assert report["ok"], report


@pytest.mark.parametrize("cfg", [DYN_2CTA, DYN_1CTA_256, DYN_1CTA_128, ST_1CTA_128, ST_2CTA, DYN_2CTA_128], ids=_id)
def test_single_tile(cfg):
    M, N, K = 128, 256, 128
    a, sfa, b, sfb = make_operands(M, N, K, seed=1)
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("cfg", VARIANTS, ids=_id)
@pytest.mark.parametrize("shape", [(256, 256, 256), (512, 512, 1024), (384, 768, 2048)], ids=str)
def test_variants_square(cfg, shape):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=sum(shape))
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("cfg", [DYN_2CTA, DYN_1CTA_128, ST_1CTA_256, ST_2CTA, DYN_2CTA_128], ids=_id)
@pytest.mark.parametrize("shape", [(200, 272, 384), (1, 16, 128), (129, 48, 256), (300, 528, 640), (777, 1040, 512)],
                         ids=str)
def test_ragged_shapes(cfg, shape):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=M + N)
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("cfg", [ST_1CTA_128, ST_1CTA_256, ST_2CTA], ids=_id)
def test_many_tiles_per_cta(cfg):
    # Few persistent CTAs walk many tiles: exercises ring wrap across tiles and
    # both TMEM accumulator buffers (and their overlap) many times over.
    M, N, K = 1024, 1024, 512
    a, sfa, b, sfb = make_operands(M, N, K, seed=3)
    cfg = GemmConfig(**{**cfg.__dict__, "max_ctas": 4})
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("cfg", [DYN_2CTA, ST_1CTA_128, ST_2CTA], ids=_id)
@pytest.mark.parametrize("raster", [(1, 0), (3, 1), (16, 0)], ids=str)
def test_rasterisation_orders(cfg, raster):
    M, N, K = 768, 1280, 256
    a, sfa, b, sfb = make_operands(M, N, K, seed=5)
    cfg = GemmConfig(**{**cfg.__dict__, "raster_group": raster[0], "raster_along_n": raster[1]})
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("cfg", [DYN_2CTA, DYN_1CTA_256, DYN_1CTA_128, DYN_2CTA_128], ids=_id)
def test_dynamic_scheduler_steals_pending_clusters(cfg):
    # Far more tiles than resident clusters: most tiles are taken over from
    # cancelled clusters through cluster launch control.
    M, N, K = 4096, 4096, 256
    a, sfa, b, sfb = make_operands(M, N, K, seed=29)
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("kind", ["wide_exponent", "llm"])
def test_value_distributions(kind):
    M, N, K = 256, 512, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=9, kind=kind)
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K))


def test_zero_blocks_and_minimum_scales():
    M, N, K = 256, 256, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=11, zero_block_frac=0.3)
    _assert_ok(check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K))


def test_output_row_stride_and_untouched_padding():
    M, N, K, ldd = 256, 256, 256, 384
    a, sfa, b, sfb = make_operands(M, N, K, seed=13)
    full = torch.full((M, ldd), 7.0, dtype=torch.bfloat16, device="cuda")
    out = run_gemm(a, sfa, b, sfb, M, N, K, out=full[:, :N])
    _assert_ok(check(out, a, sfa, b, sfb, M, N, K))
    assert torch.all(full[:, N:] == 7.0)


def test_repeated_calls_are_deterministic():
    M, N, K = 512, 512, 2048
    a, sfa, b, sfb = make_operands(M, N, K, seed=17)
    first = run_gemm(a, sfa, b, sfb, M, N, K).clone()
    for cfg in (GemmConfig(kernel=1, tile_n=128), GemmConfig(kernel=2), GemmConfig(kernel=2, scheduler=1),
                GemmConfig(kernel=1, tile_n=256, scheduler=1)):
        again = run_gemm(a, sfa, b, sfb, M, N, K, cfg)
        # Same K-order accumulation inside every MMA tile: bitwise identical across variants.
        assert torch.equal(first.view(torch.int16), again.view(torch.int16))


def test_fixed_contract_entry_16384_sampled():
    # The reference's fixed M=N=K=16384 launch, checked on sampled 64x64 blocks
    # (corners and tile boundaries) against the oracle on the same bytes.
    from cutex_b200.kernels import dense_gemm_v13, quantize_mxfp8

    n = 16384
    g = torch.Generator(device="cuda").manual_seed(0)
    xa = torch.randn(n, n, device="cuda", generator=g) * torch.exp2(torch.empty(n, 1, device="cuda").uniform_(-4, 4, generator=g))
    a, sfa = quantize_mxfp8(xa)
    del xa
    xb = torch.randn(n, n, device="cuda", generator=g) * torch.exp2(torch.empty(n, 1, device="cuda").uniform_(-4, 4, generator=g))
    b, sfb = quantize_mxfp8(xb)
    del xb
    d = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
    dense_gemm_v13(a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), d.data_ptr(), 0)
    torch.cuda.synchronize()
    device_ok()
    sfa_c = sfa.cpu().numpy()
    sfb_c = sfb.cpu().numpy()
    starts = [0, 128 - 32, 256 - 32, 8192 - 32, n - 64]
    for r0 in starts:
        rows = np.arange(r0, r0 + 64)
        ra = a[r0:r0 + 64].cpu().numpy()
        rsa = _rows_scales(sfa_c, rows, n)
        for c0 in starts:
            cols = np.arange(c0, c0 + 64)
            rb = b[c0:c0 + 64].cpu().numpy()
            rsb = _rows_scales(sfb_c, cols, n)
            ref, absum = O.gemm_reference_logical(ra, rsa, rb, rsb)
            got = d[r0:r0 + 64, c0:c0 + 64].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
            _assert_ok(O.check_gemm(got, ref, absum))


def _rows_scales(sf_buf, rows, K):
    r, c = np.meshgrid(rows, np.arange(K // 32), indexing="ij")
    return sf_buf[O.sf_offset(r, c, K)]
