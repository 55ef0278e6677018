"""In-kernel event tracing of the MXFP8 GEMM (replaces the reference's IKET tracing).

The reference collects in-kernel ranges with the external ``run-iket`` profiler
(``cutex/trace.py:96-175``) from one cluster selected by a predicate
(``dense_gemm_v9.py:116-122``). Here the kernel itself has an instrumented
twin (``cutex_mxfp8_gemm_trace``) that records ``%globaltimer`` events of the
first CTA pair per warp role: TMA producer, MMA issuer, epilogue warp 0. This
module runs it, decodes the records, summarises where each role waited, and
writes a Chrome/Perfetto trace (``chrome://tracing`` / ui.perfetto.dev).
Benchmark builds carry no instrumentation (``disabled_trace_metadata``).
"""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from . import _lib

ROLES = ("producer", "mma", "epilogue")
EVENTS = {
    1: "start", 2: "end", 3: "prod_wait", 4: "prod_go", 5: "mma_acc_wait", 6: "mma_acc_go",
    7: "mma_full_wait", 8: "mma_full_go", 9: "mma_issued", 10: "mma_tile_done",
    11: "epi_wait", 12: "epi_go", 13: "epi_release", 14: "epi_tile_done", 15: "epi_loaded",
}
# (begin event, end event) -> span name
SPANS = {
    ("prod_wait", "prod_go"): "wait empty stage",
    ("mma_acc_wait", "mma_acc_go"): "wait accumulator",
    ("mma_full_wait", "mma_full_go"): "wait loaded stage",
    ("mma_full_go", "mma_issued"): "issue MMAs",
    ("epi_wait", "epi_go"): "wait accumulator full",
    ("epi_go", "epi_release"): "read overlap + release",
    ("epi_go", "epi_loaded"): "read overlap chunk",
    ("epi_go", "epi_tile_done"): "drain tile",
}


class TraceError(RuntimeError):
    """The traced launch failed or produced no events."""


@dataclass
class Event:
    cta: int
    role: str
    t_ns: int
    name: str
    tile: int
    k_block: int


@dataclass
class GemmTrace:
    events: list[Event]
    capacity: int
    shape: tuple[int, int, int]
    config: dict[str, Any] = field(default_factory=dict)
    cta_times: list[tuple[int, int]] = field(default_factory=list)  # (start_ns, end_ns) per CTA
    cta_cycles: list[tuple[int, int]] = field(default_factory=list)  # (start, end) SM cycle counter per CTA

    def sm_clock_mhz(self) -> dict[str, float]:
        """SM clock each CTA actually ran at: cycle-counter delta over timer delta."""

        rates = sorted((ce - cs) / (te - ts) * 1e3 for (ts, te), (cs, ce) in zip(self.cta_times, self.cta_cycles)
                       if ts and te > ts and ce > cs)
        if not rates:
            return {}
        return {"ctas": len(rates), "min": rates[0], "median": rates[len(rates) // 2], "max": rates[-1]}

    def cta_spread(self) -> dict[str, float]:
        """How unevenly the persistent CTAs finish: end-time spread relative to the kernel span."""

        times = [(s, e) for s, e in self.cta_times if s and e]
        if not times:
            return {}
        t0 = min(s for s, _ in times)
        ends = sorted(e - t0 for _, e in times)
        span = ends[-1]
        return {"ctas": len(times), "span_us": span / 1e3, "first_end_us": ends[0] / 1e3,
                "median_end_us": ends[len(ends) // 2] / 1e3,
                "idle_fraction": sum(span - e for e in ends) / (span * len(ends)) if span else 0.0}

    def role_events(self, cta: int, role: str) -> list[Event]:
        return [e for e in self.events if e.cta == cta and e.role == role]

    def spans(self, cta: int, role: str):
        """(name, begin_ns, end_ns, tile, k_block) for every matched begin/end pair of a role."""

        evs = self.role_events(cta, role)
        out = []
        for (b, e), name in SPANS.items():
            pending = {}
            for ev in evs:
                if ev.name == b:
                    pending[(ev.tile, ev.k_block)] = ev.t_ns
                elif ev.name == e:
                    key = (ev.tile, ev.k_block if b != "epi_go" else 0)
                    if key in pending:
                        out.append((name, pending.pop(key), ev.t_ns, ev.tile, ev.k_block))
        return sorted(out, key=lambda s: s[1])

    def summary(self) -> dict[str, Any]:
        """Per CTA and role: elapsed time and the total/mean of each wait span."""

        result: dict[str, Any] = {"shape": list(self.shape), "config": self.config, "ctas": {},
                                  "cta_finish": self.cta_spread(), "sm_clock_mhz": self.sm_clock_mhz()}
        for cta in sorted({e.cta for e in self.events}):
            per_role = {}
            for role in ROLES:
                evs = self.role_events(cta, role)
                if not evs:
                    continue
                t0 = min(e.t_ns for e in evs)
                t1 = max(e.t_ns for e in evs)
                totals: dict[str, list[int]] = {}
                for name, b, e, _, _ in self.spans(cta, role):
                    totals.setdefault(name, []).append(e - b)
                per_role[role] = {
                    "elapsed_us": (t1 - t0) / 1e3,
                    "events": len(evs),
                    "spans": {
                        name: {"count": len(v), "total_us": sum(v) / 1e3, "mean_ns": sum(v) / len(v),
                               "share_of_elapsed": (sum(v) / (t1 - t0)) if t1 > t0 else 0.0}
                        for name, v in totals.items()
                    },
                }
                if role == "mma":
                    done = [e.t_ns for e in evs if e.name == "mma_tile_done"]
                    go = [e.t_ns for e in evs if e.name == "mma_acc_go"]
                    gaps = [g - d for d, g in zip(done, go[1:])]
                    if gaps:
                        per_role[role]["tile_boundary_gap_ns"] = {"mean": sum(gaps) / len(gaps), "max": max(gaps),
                                                                  "count": len(gaps)}
            result["ctas"][cta] = per_role
        result["tile_handover_ns"] = self.tile_handover()
        result["launch_edges_us"] = self.launch_edges()
        return result

    def tile_handover(self) -> dict[str, float]:
        """Medians over the traced pair's tile boundaries of the accumulator hand-over steps (ns).

        last MMAs of tile i issued -> its accumulator seen full by the epilogue ->
        the overlapping chunk read -> accumulator released -> first MMAs of tile
        i + 1 issued."""

        def by_tile(role, name):
            return {e.tile: e.t_ns for e in self.events if e.cta == 0 and e.role == role and e.name == name}

        done, go = by_tile("mma", "mma_tile_done"), by_tile("epilogue", "epi_go")
        loaded, rel = by_tile("epilogue", "epi_loaded"), by_tile("epilogue", "epi_release")
        acc_go = [(e.t_ns, e.tile) for e in self.events if e.cta == 0 and e.role == "mma" and e.name == "mma_acc_go"]
        acc_go.sort()
        nxt = {acc_go[i][1]: acc_go[i + 1][0] for i in range(len(acc_go) - 1)}  # tile -> next tile's start
        steps = {"issued_to_full": [], "full_to_loaded": [], "loaded_to_released": [], "released_to_next_issue": []}
        for t in done:
            if t in go and t in loaded and t in rel and t in nxt:
                steps["issued_to_full"].append(go[t] - done[t])
                steps["full_to_loaded"].append(loaded[t] - go[t])
                steps["loaded_to_released"].append(rel[t] - loaded[t])
                steps["released_to_next_issue"].append(nxt[t] - rel[t])
        out = {k: float(sorted(v)[len(v) // 2]) for k, v in steps.items() if v}
        if out:
            out["boundaries"] = len(steps["issued_to_full"])
        return out

    def launch_edges(self) -> dict[str, float]:
        """Fill and drain of the launch (us): first CTA start to the traced pair's first loaded
        stage and first issued MMAs, its last MMAs to its last stored tile, and the spread of
        CTA starts."""

        times = [(s, e) for s, e in self.cta_times if s and e]
        ev = [e for e in self.events if e.cta == 0]
        if not times or not ev:
            return {}
        t0 = min(s for s, _ in times)
        first = lambda role, name: min((e.t_ns for e in ev if e.role == role and e.name == name), default=None)  # noqa: E731
        last = lambda role, name: max((e.t_ns for e in ev if e.role == role and e.name == name), default=None)  # noqa: E731
        out = {"cta_start_spread_us": (max(s for s, _ in times) - t0) / 1e3}
        if first("mma", "mma_full_go") is not None:
            out["start_to_first_loaded_stage_us"] = (first("mma", "mma_full_go") - self.cta_times[0][0]) / 1e3
        if first("mma", "mma_issued") is not None:
            out["start_to_first_mmas_issued_us"] = (first("mma", "mma_issued") - self.cta_times[0][0]) / 1e3
        if last("mma", "mma_tile_done") is not None and last("epilogue", "epi_tile_done") is not None:
            out["last_mmas_to_last_tile_stored_us"] = (last("epilogue", "epi_tile_done") -
                                                      last("mma", "mma_tile_done")) / 1e3
        return out

    def to_chrome_trace(self) -> dict[str, Any]:
        t0 = min((e.t_ns for e in self.events), default=0)
        trace_events = []
        for cta in sorted({e.cta for e in self.events}):
            for tid, role in enumerate(ROLES):
                trace_events.append({"name": "thread_name", "ph": "M", "pid": cta, "tid": tid,
                                     "args": {"name": role}})
                for name, b, e, tile, kb in self.spans(cta, role):
                    trace_events.append({"name": name, "ph": "X", "pid": cta, "tid": tid, "ts": (b - t0) / 1e3,
                                         "dur": max(e - b, 1) / 1e3, "args": {"tile": tile, "k_block": kb}})
        return {"traceEvents": trace_events, "displayTimeUnit": "ns",
                "metadata": {"shape": list(self.shape), "config": self.config}}

    def write(self, directory: str | Path, stem: str = "gemm_trace") -> dict[str, Path]:
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        paths = {"trace_json": directory / f"{stem}.trace.json", "summary": directory / f"{stem}.summary.json"}
        paths["trace_json"].write_text(json.dumps(self.to_chrome_trace()))
        paths["summary"].write_text(json.dumps(self.summary(), indent=1))
        return paths


def decode(raw, capacity: int, ctas: int = 2) -> list[Event]:
    """Decode the flat uint64 trace buffer written by cutex_mxfp8_gemm_trace."""

    events = []
    stride = (capacity + 1) * 2
    for cta in range(ctas):
        for r, role in enumerate(ROLES):
            base = (cta * 3 + r) * stride
            count = int(raw[base])
            for i in range(1, min(count, capacity) + 1):
                t = int(raw[base + 2 * i])
                info = int(raw[base + 2 * i + 1])
                ev = EVENTS.get(info >> 56, f"event{info >> 56}")
                events.append(Event(cta, role, t, ev, (info >> 24) & 0xFFFFFFF, info & 0xFFFFFF))
    return events


def run_gemm_trace(a, b, sfa, sfb, out, config=None, capacity: int = 1 << 16) -> GemmTrace:
    """Run one instrumented GEMM launch (torch CUDA tensors) and return its decoded trace."""

    import torch

    from .kernels.dense_gemm import GemmConfig, _stream_handle, query

    cfg = config or GemmConfig(kernel=2, stages=6, epi_buffers=1, sf_buffers=1)
    m, k = a.shape
    n = b.shape[0]
    grid = query(m, n, k, cfg)["grid_ctas"]
    buf = torch.zeros(6 * (capacity + 1) * 2 + 4 * grid, dtype=torch.int64, device=out.device)
    status = _lib.load().cutex_mxfp8_gemm_trace(
        a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(), m, n, k, out.stride(0),
        ctypes.byref(cfg.to_c()), buf.data_ptr(), capacity, _stream_handle(None))
    _lib.check(status, "cutex_mxfp8_gemm_trace")
    torch.cuda.synchronize()
    raw = buf.cpu().numpy().view("uint64")
    events = decode(raw, capacity)
    if not events:
        raise TraceError("the traced launch recorded no events")
    base = 6 * (capacity + 1) * 2
    cta_times = [(int(raw[base + 2 * c]), int(raw[base + 2 * c + 1])) for c in range(grid)]
    base += 2 * grid
    cta_cycles = [(int(raw[base + 2 * c]), int(raw[base + 2 * c + 1])) for c in range(grid)]
    return GemmTrace(events, capacity, (m, n, k), dict(cfg.__dict__), cta_times, cta_cycles)


def main(argv=None) -> int:
    """``python -m cutex_b200.trace --m M --n N --k K [--out DIR] [--config JSON]``: one traced launch.

    Seeded N(0,1) operands quantised on the GPU by the library's quantiser; the
    traced launch runs after one untimed traced warm-up launch; prints the
    summary (per-CTA SM clock, end-of-launch spread, tile hand-over, launch
    edges, per-role wait spans) as JSON and, with --out, writes the Chrome trace.
    """

    import argparse

    import torch

    from .kernels import GemmConfig, quantize_mxfp8

    ap = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=16384)
    ap.add_argument("--k", type=int, default=16384)
    ap.add_argument("--config", default='{"kernel": 2, "stages": 6, "epi_buffers": 1, "sf_buffers": 1}')
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    g = torch.Generator(device="cuda").manual_seed(0)
    a, sfa = quantize_mxfp8(torch.randn(args.m, args.k, device="cuda", generator=g))
    b, sfb = quantize_mxfp8(torch.randn(args.n, args.k, device="cuda", generator=g))
    d = torch.empty(args.m, args.n, dtype=torch.bfloat16, device="cuda")
    cfg = GemmConfig(**json.loads(args.config))
    run_gemm_trace(a, b, sfa, sfb, d, config=cfg)
    tr = run_gemm_trace(a, b, sfa, sfb, d, config=cfg)
    summary = tr.summary()
    if args.out:
        tr.write(args.out, stem=f"gemm_trace_m{args.m}_n{args.n}_k{args.k}")
    print(json.dumps(summary, default=str))
    return 0


def disabled_trace_metadata() -> dict[str, Any]:
    """Result-metadata stanza for runs without tracing (same role as ``disabled_iket_metadata``)."""

    return {"enabled": False, "benchmark_instrumented": False, "tool": "cutex_mxfp8_gemm_trace"}


__all__ = ["Event", "GemmTrace", "TraceError", "decode", "disabled_trace_metadata", "main", "run_gemm_trace"]


if __name__ == "__main__":
    raise SystemExit(main())
