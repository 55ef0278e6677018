"""Skinny (M <= 128) split-K kernel vs the CPU oracle, through the C ABI.

Same tolerance as tests/test_gpu_gemm.py. Covers every padded-M variant, ragged
N, the stream-K split with many contributors per tile (small grids), the
whole-tile mode, repeated calls reusing one workspace (arrival counters must be
left at zero), bitwise determinism, and the workspace contract.
"""

import ctypes

import numpy as np
import pytest
import torch

from cutex_b200 import _lib
from cutex_b200.kernels import GemmConfig, dense_gemm, query
from tests.gpu_helpers import check, device_ok, make_operands, run_gemm

pytestmark = pytest.mark.gpu

SKINNY = _lib.KERNEL_SKINNY


def _ok(r):
    assert r["ok"], r


@pytest.mark.parametrize("M", [1, 16, 17, 32, 50, 64, 100, 128])
def test_padded_m_variants(M):
    N, K = 512, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=M)
    _ok(check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("shape", [(16, 272, 384), (128, 2064, 640), (7, 16, 128), (128, 1024, 8192)], ids=str)
def test_ragged_and_long_k(shape):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=N)
    _ok(check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("grid", [1, 3, 7, 13, 64])
def test_stream_k_split_points(grid):
    # Few CTAs over 8 tiles x 16 K-stages: tiles cut into 1..many contributor segments.
    M, N, K = 48, 1024, 2048
    a, sfa, b, sfb = make_operands(M, N, K, seed=grid)
    cfg = GemmConfig(kernel=SKINNY, max_ctas=grid)
    _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("M,grid", [(128, 3), (128, 7), (64, 5), (16, 13), (100, 8), (128, 0)])
def test_data_parallel_waves_then_stream_k(M, grid):
    # split_k = 3: whole tiles for the full waves (tiles // grid * grid), stream-K over the rest;
    # 10 tiles x 8 K-stages, so every grid leaves a remainder cut between contributors.
    N, K = 1280, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=M * 7 + grid)
    cfg = GemmConfig(kernel=SKINNY, split_k=3, max_ctas=grid)
    _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


def test_split_modes_agree_bitwise():
    # Whole tiles, pure stream-K and waves + stream-K sum the same K products in the same
    # per-segment order only within a tile; across modes the results must all pass the oracle
    # and the deterministic modes must repeat exactly.
    M, N, K = 128, 28672 // 8, 8192 // 4
    a, sfa, b, sfb = make_operands(M, N, K, seed=11, kind="llm")
    outs = {}
    for split in (1, 2, 3):
        cfg = GemmConfig(kernel=SKINNY, split_k=split)
        o1 = run_gemm(a, sfa, b, sfb, M, N, K, cfg)
        o2 = run_gemm(a, sfa, b, sfb, M, N, K, cfg)
        _ok(check(o1, a, sfa, b, sfb, M, N, K))
        assert torch.equal(o1.contiguous().view(torch.int16), o2.contiguous().view(torch.int16))
        outs[split] = o1


@pytest.mark.parametrize("shape", [(128, 1280, 1024), (64, 1296, 512), (100, 2064, 768), (33, 512, 256),
                                   (128, 256, 4096), (128, 144, 384)], ids=str)
def test_double_b_tiles(shape):
    # tile_n = 256: two 128-row B tiles per CTA tile share each A stage (whole tiles);
    # ragged N leaves the second tile of the last pair partly or wholly past N.
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=M + N)
    for grid in (0, 2):
        cfg = GemmConfig(kernel=SKINNY, tile_n=256, split_k=1, max_ctas=grid)
        assert query(M, N, K, cfg)["tile_n"] == 256
        _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


@pytest.mark.parametrize("case", [(128, 2560, 2048, 7, 0), (100, 1280, 1024, 13, 3), (48, 4096, 1024, 0, 2),
                                  (16, 1552, 4096, 5, 0), (128, 1296, 768, 3, 2), (64, 512, 8192, 0, 0)], ids=str)
def test_double_b_tiles_stream_k(case):
    # tile_n = 256 with the split: a CTA tile (two 128-row B tiles) cut between contributors
    # goes through slots holding both tiles; ragged N leaves part of the second tile past N.
    M, N, K, grid, split = case
    a, sfa, b, sfb = make_operands(M, N, K, seed=M * 3 + N)
    cfg = GemmConfig(kernel=SKINNY, tile_n=256, split_k=split, max_ctas=grid)
    plan = query(M, N, K, cfg)
    assert plan["tile_n"] == 256 and plan["split_k"] == 0 and plan["workspace_bytes"] > 0
    for _ in range(2):  # the second call reuses the workspace the first left ready
        _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


def test_double_b_tiles_stream_k_llm_full_size():
    M, N, K = 128, 28672, 8192
    a, sfa, b, sfb = make_operands(M, N, K, seed=5, kind="llm")
    cfg = GemmConfig(kernel=SKINNY, tile_n=256)
    _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


def test_whole_tile_mode():
    M, N, K = 128, 1280, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=4)
    for grid in (0, 3):
        cfg = GemmConfig(kernel=SKINNY, split_k=1, max_ctas=grid)
        _ok(check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K))


def test_repeated_calls_reuse_workspace_and_are_deterministic():
    M, N, K = 16, 4096, 4096
    a, sfa, b, sfb = make_operands(M, N, K, seed=8, kind="llm")
    dev = "cuda"
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    need = query(M, N, K)["workspace_bytes"]
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    outs = []
    for cfg in (GemmConfig(), GemmConfig(max_ctas=37), GemmConfig()):
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            dense_gemm(ta, tb, tsa, tsb, out, config=cfg, workspace=ws)
        torch.cuda.synchronize()
        device_ok()
        _ok(check(out, a, sfa, b, sfb, M, N, K))
        outs.append(out)
    # Arrival counters (after the fixed 2 * SMs * 64 KiB partial region) are back at zero.
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    counters = ws[2 * sms * 128 * 128 * 4:][: (N // 128) * 4]
    assert int(counters.view(torch.int32).abs().sum()) == 0
    assert torch.equal(outs[0].view(torch.int16), outs[2].view(torch.int16))


def test_one_workspace_serves_every_shape():
    # Calls of different M, N, grids share one workspace: counters never alias partials.
    dev = "cuda"
    ws = torch.zeros(query(1, 8192, 128)["workspace_bytes"] * 2, dtype=torch.uint8, device=dev)
    for (M, N, K, grid) in [(128, 4096, 1024, 0), (16, 1024, 2048, 5), (64, 8192, 512, 0), (128, 512, 4096, 3),
                            (16, 4096, 1024, 0)]:
        a, sfa, b, sfb = make_operands(M, N, K, seed=M + N + K)
        ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
        tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        dense_gemm(ta, tb, tsa, tsb, out, config=GemmConfig(kernel=SKINNY, max_ctas=grid), workspace=ws)
        torch.cuda.synchronize()
        device_ok()
        _ok(check(out, a, sfa, b, sfb, M, N, K))


def test_llm_skinny_configs_full_size():
    # BASELINE LLM shapes: K = 8192, N = 28672, M in {16, 128}, outlier activations.
    for M in (16, 128):
        N, K = 28672, 8192
        a, sfa, b, sfb = make_operands(M, N, K, seed=M, kind="llm")
        _ok(check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K))


def test_workspace_contract():
    M, N, K = 16, 512, 512
    a, sfa, b, sfb = make_operands(M, N, K, seed=2)
    dev = "cuda"
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    cfg = _lib.make_config(kernel=SKINNY)
    args = (ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(), out.data_ptr(), M, N, K, N, ctypes.byref(cfg))
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.cutex_mxfp8_gemm(*args, None, 0, stream) == _lib.CUTEX_ERR_WORKSPACE
    ws = torch.zeros(query(M, N, K)["workspace_bytes"] + 512, dtype=torch.uint8, device=dev)
    assert lib.cutex_mxfp8_gemm(*args, ws.data_ptr() + 16, ws.numel() - 16, stream) == _lib.CUTEX_ERR_ALIGN
    assert lib.cutex_mxfp8_gemm(*args, ws.data_ptr(), ws.numel(), stream) == 0
    # AUTO without a workspace runs the whole-tile variant.
    auto = _lib.make_config()
    out2 = torch.empty_like(out)
    args2 = args[:4] + (out2.data_ptr(),) + args[5:9] + (ctypes.byref(auto),)
    assert lib.cutex_mxfp8_gemm(*args2, None, 0, stream) == 0
    torch.cuda.synchronize()
    device_ok()
    _ok(check(out, a, sfa, b, sfb, M, N, K))
    _ok(check(out2, a, sfa, b, sfb, M, N, K))
