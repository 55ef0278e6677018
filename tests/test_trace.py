"""Trace decoding/summary on a synthetic buffer (CPU) and one traced launch (GPU)."""

import json

import numpy as np
import pytest

from cutex_b200.trace import ROLES, GemmTrace, decode, disabled_trace_metadata


def _encode(regions, capacity):
    raw = np.zeros(6 * (capacity + 1) * 2, dtype=np.uint64)
    for (cta, role), recs in regions.items():
        base = (cta * 3 + ROLES.index(role)) * (capacity + 1) * 2
        raw[base] = len(recs)
        for i, (t, ev, tile, kb) in enumerate(recs, start=1):
            raw[base + 2 * i] = t
            raw[base + 2 * i + 1] = (ev << 56) | (tile << 24) | kb
    return raw


def test_decode_and_summary_from_synthetic_records():
    cap = 16
    mma = [(100, 1, 0, 0), (100, 5, 0, 0), (110, 6, 0, 0), (110, 7, 0, 0), (150, 8, 0, 0), (160, 9, 0, 0),
           (160, 7, 0, 1), (170, 8, 0, 1), (180, 9, 0, 1), (185, 10, 0, 0), (185, 5, 1, 0), (400, 6, 1, 0),
           (410, 2, 0, 0)]
    epi = [(100, 1, 0, 0), (100, 11, 0, 0), (300, 12, 0, 0), (380, 13, 0, 0), (600, 14, 0, 0)]
    raw = _encode({(0, "mma"): mma, (0, "epilogue"): epi, (1, "producer"): [(90, 1, 0, 0), (95, 3, 0, 0),
                                                                            (97, 4, 0, 0)]}, cap)
    events = decode(raw, cap)
    assert len(events) == len(mma) + len(epi) + 3
    tr = GemmTrace(events, cap, (256, 256, 256))
    s = tr.summary()
    m = s["ctas"][0]["mma"]
    assert m["spans"]["wait loaded stage"]["count"] == 2
    assert m["spans"]["wait loaded stage"]["total_us"] == pytest.approx((40 + 10) / 1e3)
    assert m["spans"]["wait accumulator"]["total_us"] == pytest.approx((10 + 215) / 1e3)
    assert m["tile_boundary_gap_ns"]["mean"] == pytest.approx(400 - 185)
    e = s["ctas"][0]["epilogue"]["spans"]
    assert e["wait accumulator full"]["total_us"] == pytest.approx(0.2)
    assert e["read overlap + release"]["mean_ns"] == 80
    chrome = tr.to_chrome_trace()
    assert any(ev.get("name") == "issue MMAs" for ev in chrome["traceEvents"])
    json.dumps(chrome)
    assert disabled_trace_metadata()["benchmark_instrumented"] is False


def test_tile_handover_and_launch_edges():
    # Two tiles on the traced pair: tile 0's MMAs issued at 1000, its accumulator seen full
    # at 1300, overlap chunk read at 1350, released at 1400, tile 1's MMAs start at 1500.
    cap = 32
    mma = [(500, 1, 0, 0), (500, 5, 0, 0), (520, 6, 0, 0), (600, 8, 0, 0), (700, 9, 0, 0), (1000, 10, 0, 0),
           (1000, 5, 1, 0), (1500, 6, 1, 0), (1600, 8, 1, 0), (1700, 9, 1, 0), (2000, 10, 1, 0), (2100, 2, 0, 0)]
    epi = [(500, 1, 0, 0), (500, 11, 0, 0), (1300, 12, 0, 0), (1350, 15, 0, 0), (1400, 13, 0, 0), (1900, 14, 0, 0),
           (1900, 11, 1, 0), (2300, 12, 1, 0), (2350, 15, 1, 0), (2400, 13, 1, 0), (2900, 14, 1, 0)]
    tr = GemmTrace(decode(_encode({(0, "mma"): mma, (0, "epilogue"): epi}, cap), cap), cap, (256, 512, 256),
                   cta_times=[(400, 3000), (450, 2950)], cta_cycles=[(0, 1), (0, 1)])
    h = tr.tile_handover()
    assert h == {"issued_to_full": 300.0, "full_to_loaded": 50.0, "loaded_to_released": 50.0,
                 "released_to_next_issue": 100.0, "boundaries": 1}
    edges = tr.launch_edges()
    assert edges["cta_start_spread_us"] == pytest.approx(0.05)
    assert edges["start_to_first_loaded_stage_us"] == pytest.approx(0.2)
    assert edges["start_to_first_mmas_issued_us"] == pytest.approx(0.3)
    assert edges["last_mmas_to_last_tile_stored_us"] == pytest.approx(0.9)
    assert tr.summary()["tile_handover_ns"]["boundaries"] == 1


def test_sm_clock_from_cycle_counters():
    tr = GemmTrace([], 1, (1, 1, 1), cta_times=[(1000, 2000), (1000, 3000), (0, 0)],
                   cta_cycles=[(10, 1910), (5, 3805), (0, 0)])
    clk = tr.sm_clock_mhz()
    assert clk["ctas"] == 2 and clk["min"] == pytest.approx(1900.0) and clk["max"] == pytest.approx(1900.0)
    assert GemmTrace([], 1, (1, 1, 1)).sm_clock_mhz() == {}


def test_truncated_region_is_capped():
    cap = 2
    raw = _encode({(0, "mma"): [(1, 1, 0, 0), (2, 7, 0, 0)]}, cap)
    raw[0 + 3 * (cap + 1) * 2 * 0 + (cap + 1) * 2] = 99  # count claims more than capacity
    assert len([e for e in decode(raw, cap) if e.role == "mma"]) == cap


@pytest.mark.gpu
def test_traced_launch_matches_and_records_every_stage():
    import torch

    from cutex_b200.kernels import GemmConfig
    from cutex_b200.trace import run_gemm_trace
    from tests.gpu_helpers import check, make_operands

    M, N, K = 1024, 1024, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=21)
    dev = "cuda"
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    for cfg in (GemmConfig(kernel=2, stages=6, epi_buffers=1, sf_buffers=1, max_ctas=4, scheduler=1),
                GemmConfig(kernel=1, tile_n=256, stages=4, epi_buffers=1, sf_buffers=1, max_ctas=2, scheduler=1),
                GemmConfig(kernel=2, stages=6, epi_buffers=1, sf_buffers=1, scheduler=0)):
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        tr = run_gemm_trace(ta, tb, tsa, tsb, out, cfg)
        assert check(out, a, sfa, b, sfb, M, N, K)["ok"]
        tiles = len({e.tile for e in tr.events if e.role == "mma" and e.name == "mma_tile_done"})
        issued = [e for e in tr.events if e.role == "mma" and e.name == "mma_issued"]
        assert len(issued) == tiles * (K // 128) and tiles >= (2 if cfg.scheduler else 1)
        s = tr.summary()["ctas"][0]
        assert s["mma"]["elapsed_us"] > 0 and "wait loaded stage" in s["mma"]["spans"]
        clk = tr.sm_clock_mhz()
        assert clk["ctas"] >= 2 and 300.0 < clk["median"] < 2500.0
