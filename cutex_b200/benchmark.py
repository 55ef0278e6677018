"""CUDA-event timing and sample statistics.

Same functions and semantics as the reference's ``cutex/benchmark.py``:
``stats_from_samples`` (p95 = sample at index ceil(0.95 n) - 1 of the sorted
samples, ``:29-41``), ``cuda_benchmark`` (one event pair per launch, all events
queued before one final synchronisation, ``:44-83``), ``cuda_benchmark_pair``
(order alternates every pair, ``:86-139``) and ``paired_comparison``
(delta = first - second, efficiency = 100 * second / first, ``:142-186``).

Additions for B200 measurement: an optional L2 flush between samples
(``flush_l2=True`` writes a buffer larger than the 126 MB L2 before every timed
launch, outside the timed interval) and an explicit stream argument that is
used for every event.
"""

from __future__ import annotations

import math
import statistics
from dataclasses import asdict, dataclass
from typing import Any, Callable

L2_FLUSH_BYTES = 256 * 1024 * 1024  # 2x the B200 L2


@dataclass(frozen=True)
class BenchmarkStats:
    samples_us: tuple[float, ...]
    mean_us: float
    median_us: float
    min_us: float
    max_us: float
    p95_us: float

    def to_dict(self, *, include_samples: bool = False) -> dict[str, Any]:
        out = asdict(self)
        if include_samples:
            out["samples_us"] = list(self.samples_us)
        else:
            del out["samples_us"]
        return out


def stats_from_samples(samples_us) -> BenchmarkStats:
    values = [float(x) for x in samples_us]
    if not values:
        raise ValueError("at least one timing sample is required")
    ordered = sorted(values)
    p95 = ordered[max(0, math.ceil(0.95 * len(ordered)) - 1)]
    return BenchmarkStats(
        samples_us=tuple(values),
        mean_us=statistics.fmean(ordered),
        median_us=statistics.median(ordered),
        min_us=ordered[0],
        max_us=ordered[-1],
        p95_us=p95,
    )


class _L2Flusher:
    def __init__(self, device=None):
        import torch

        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device or "cuda")

    def __call__(self):
        self.buf.zero_()


def _event_pair(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def cuda_benchmark(
    fn: Callable[..., Any],
    *args: Any,
    warmup: int = 5,
    rep: int = 30,
    stream=None,
    flush_l2: bool = False,
    **kwargs: Any,
) -> BenchmarkStats:
    """Time ``rep`` launches of ``fn`` with one CUDA-event pair each (microseconds)."""

    if warmup < 0 or rep < 1:
        raise ValueError("warmup must be >= 0 and rep must be >= 1")
    import torch

    flusher = _L2Flusher() if flush_l2 else None
    for _ in range(warmup):
        fn(*args, **kwargs)
    torch.cuda.synchronize()
    events = []
    for _ in range(rep):
        if flusher is not None:
            flusher()
        start, end = _event_pair(torch)
        if stream is None:
            start.record()
            fn(*args, **kwargs)
            end.record()
        else:
            start.record(stream)
            fn(*args, **kwargs)
            end.record(stream)
        events.append((start, end))
    events[-1][1].synchronize()
    return stats_from_samples([s.elapsed_time(e) * 1000.0 for s, e in events])


def cuda_benchmark_pair(
    first_fn: Callable[[], Any],
    second_fn: Callable[[], Any],
    *,
    warmup: int = 5,
    rep: int = 30,
    stream=None,
    flush_l2: bool = False,
) -> tuple[BenchmarkStats, BenchmarkStats]:
    """Time two launches per sample, alternating their order, one event pair per launch."""

    if warmup < 0 or rep < 1:
        raise ValueError("warmup must be >= 0 and rep must be >= 1")
    import torch

    fns = (first_fn, second_fn)
    for i in range(warmup):
        order = (0, 1) if i % 2 == 0 else (1, 0)
        for j in order:
            fns[j]()
    torch.cuda.synchronize()
    flusher = _L2Flusher() if flush_l2 else None
    events: list[list[tuple[Any, Any]]] = [[], []]
    last = None
    for i in range(rep):
        order = (0, 1) if i % 2 == 0 else (1, 0)
        for j in order:
            if flusher is not None:
                flusher()
            start, end = _event_pair(torch)
            if stream is None:
                start.record()
                fns[j]()
                end.record()
            else:
                start.record(stream)
                fns[j]()
                end.record(stream)
            events[j].append((start, end))
            last = end
    last.synchronize()
    first = stats_from_samples([s.elapsed_time(e) * 1000.0 for s, e in events[0]])
    second = stats_from_samples([s.elapsed_time(e) * 1000.0 for s, e in events[1]])
    return first, second


def paired_comparison(first: BenchmarkStats, second: BenchmarkStats) -> dict[str, Any]:
    """Per-pair latency deltas (first - second) and efficiencies (100 * second / first)."""

    a, b = first.samples_us, second.samples_us
    if len(a) != len(b):
        raise ValueError("paired sample counts must match")
    if not a:
        raise ValueError("at least one sample pair is required")
    if any(x <= 0 for x in a):
        raise ValueError("first samples must be positive")
    deltas = [x - y for x, y in zip(a, b)]
    effs = [100.0 * y / x for x, y in zip(a, b)]

    def summary(values):
        s = stats_from_samples(values)
        return {
            "samples": list(s.samples_us),
            "mean": s.mean_us,
            "median": s.median_us,
            "min": s.min_us,
            "max": s.max_us,
            "p95": s.p95_us,
        }

    faster = sum(1 for d in deltas if d < 0)
    return {
        "sample_pairs": len(deltas),
        "delta_us": summary(deltas),
        "efficiency_pct": summary(effs),
        "first_faster_samples": faster,
        "first_faster_pct": 100.0 * faster / len(deltas),
    }


def tflops(flops: float, microseconds: float) -> float:
    """Throughput in TFLOP/s from a FLOP count and a duration in microseconds."""

    return flops / microseconds / 1e6
