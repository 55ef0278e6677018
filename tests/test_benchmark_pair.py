"""Benchmark statistics: the reference's tests (tests/test_benchmark_pair.py) plus its golden outputs."""

import json

import pytest

from cutex_b200.benchmark import paired_comparison, stats_from_samples, tflops
from tests.conftest import GOLDEN


def test_paired_comparison_preserves_pairing_and_direction() -> None:
    custom = stats_from_samples([9.0, 12.0, 10.0])
    reference = stats_from_samples([10.0, 10.0, 11.0])
    paired = paired_comparison(custom, reference)
    assert paired["sample_pairs"] == 3
    assert paired["delta_us"]["samples"] == [-1.0, 2.0, -1.0]
    assert paired["delta_us"]["median"] == -1.0
    assert paired["efficiency_pct"]["median"] == pytest.approx(110.0)
    assert paired["first_faster_samples"] == 2
    assert paired["first_faster_pct"] == pytest.approx(200.0 / 3.0)


def test_paired_comparison_rejects_mismatched_counts() -> None:
    with pytest.raises(ValueError, match="counts"):
        paired_comparison(stats_from_samples([1.0]), stats_from_samples([1.0, 2.0]))


def test_stats_and_pairs_match_reference_golden() -> None:
    g = json.loads((GOLDEN / "benchmark_stats.json").read_text())
    a = stats_from_samples(g["samples_a"])
    b = stats_from_samples(g["samples_b"])
    assert a.to_dict(include_samples=True) == g["stats_a"]
    assert b.to_dict() == g["stats_b"]
    assert paired_comparison(a, b) == g["paired"]


def test_stats_reject_empty_and_tflops():
    with pytest.raises(ValueError):
        stats_from_samples([])
    assert tflops(2 * 16384**3, 3244.848) == pytest.approx(2710.787, rel=1e-6)
