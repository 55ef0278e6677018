"""Benchmark: MXFP8 block-scaled GEMM TFLOPS on 1..8 B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cutex|reference]
                    [--m M --n N --k K] [--dist square|llm] [--config JSON]
                    [--no-allgather] [--no-configs] [--vs-cublaslt ROUNDS]
    python bench.py --quantize rowwise|columnwise [--qdtype f32|bf16]
    python bench.py --host-ceiling        (under torchrun for N > 1)

Workload (default): the reference's fixed contract M = N = K = 16384
(BASELINE configs[2]); at N > 1 GPUs the GEMM is N-sharded (rank r computes
D[:, r*N/g:(r+1)*N/g] from all of A and its slice of B), total work fixed.
A step is one GEMM launch over resident inputs. Operands (256 MiB + 256 MiB
E4M3 + scales at 1 GPU) exceed the 126 MB L2, so no L2 flush is done between
steps. ``value`` = 2*M*N*K*steps / (max over ranks of the device time of the
timed region). ``e2e`` repeats the measurement from pinned host buffers, inside the
CUDA-event timed interval: on 1 GPU through the library's host-buffer entry
(``cutex_mxfp8_gemm_host``: A, B, SFA, SFB in, D out, copies and block GEMMs
overlapped; independent steps alternate over ``--e2e-streams`` streams so one
step's D2H overlaps the next step's H2D); on N GPUs through ``ShardedHostGemm``
(each rank copies 1/N of A and its B slice in, A is all-gathered over NVLink,
D slices come back in row blocks; steps alternate over ``--e2e-sharded-streams``
streams, each with its own process group). At N > 1 the line also times gathering
D on every rank, NCCL after the GEMM against the all-gather fused into the
GEMM's epilogue (``allgather``); at N = 1 it carries cuBLASLt on the same
operands (``vs_cublaslt``) and BASELINE's other configurations (``configs``).

``--impl reference`` times the contract's CPU path (dequantise, fp32 matmul,
cast to BF16: the oracle port) on the host cores, on bounded row/column
samples of the same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PROFILES = ROOT / "profiles"
METRIC = "MXFP8 GEMM TFLOPS (device-timed) and % of FP8 TC peak / HBM roofline at 1/2/4/8 B200"
RIDGE_FLOP_PER_BYTE = 500.0  # ~4.5 PFLOP/s FP8 / ~8 TB/s HBM: below it a GEMM is HBM-bound
SEED = 0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("cutex", "reference"), default="cutex")
    p.add_argument("--m", type=int, default=16384)
    p.add_argument("--n", type=int, default=16384)
    p.add_argument("--k", type=int, default=16384)
    p.add_argument("--e2e-steps", type=int, default=12,
                   help="end-to-end steps in the timed region (a stream of independent requests: more steps "
                        "amortise the first step's uncovered H2D and the last step's uncovered D2H)")
    p.add_argument("--e2e-streams", type=int, default=2,
                   help="N = 1: independent steps alternate over this many streams, each with its own HostGemm "
                        "(device buffers) and pinned result, so one step's D2H overlaps the next step's H2D")
    p.add_argument("--e2e-sharded-streams", type=int, default=2,
                   help="N > 1: the same alternation over this many streams, each ShardedHostGemm with its own "
                        "process group (NCCL communicator) so that their all-gathers never share one")
    p.add_argument("--e2e-blocks", type=int, default=4,
                   help="host pipeline: output cut into up to BxB blocks (copies and GEMMs overlapped)")
    p.add_argument("--no-allgather", dest="allgather", action="store_false",
                   help="N > 1: skip timing the gather of D on every rank (NCCL after the GEMM vs fused into it)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--config", type=str, default="", help="native config as JSON, e.g. '{\"kernel\": 2}'")
    p.add_argument("--no-graph", action="store_true", help="plain launches instead of one CUDA graph")
    p.add_argument("--sustained-s", type=float, default=2.0,
                   help="also run the launches back to back for this many seconds (0: skip)")
    p.add_argument("--vs-cublaslt", type=int, default=3, metavar="ROUNDS",
                   help="N = 1: also time cuBLASLt MXFP8 (torch._scaled_mm) on the same operands, alternating "
                        "ROUNDS graph replays of each with this kernel's, and compare the outputs bitwise (0: skip)")
    p.add_argument("--cublaslt-sustained", action="store_true",
                   help="with --vs-cublaslt: also run cuBLASLt back to back for --sustained-s seconds")
    p.add_argument("--no-configs", action="store_true",
                   help="N = 1: skip the other BASELINE configurations timed beside the headline (`configs`)")
    p.add_argument("--quantize", choices=("rowwise", "columnwise"), default=None,
                   help="N = 1: time the MXFP8 quantiser on an [M, K] input instead of the GEMM (GB/s vs HBM)")
    p.add_argument("--qdtype", choices=("f32", "bf16"), default="f32", help="quantiser input type")
    p.add_argument("--measure-fp8-peak", action="store_true",
                   help="measure cuBLASLt MXFP8 (torch._scaled_mm) 8192^3: best-of-10 burst and 4 s sustained")
    p.add_argument("--host-ceiling", action="store_true",
                   help="measure the host-link ceiling of all ranks (concurrent pinned copies) and the phases of one "
                        "end-to-end step (ShardedHostGemm at N > 1, HostGemm's copies at N = 1) instead of the GEMM")
    p.add_argument("--dist", choices=("square", "llm"), default="square",
                   help="input distribution: BASELINE square-sweep generator or LLM activations/weights")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_name(m, n, k):
    return f"mxfp8_fprop_m{m}_n{n}_k{k}"


def workload_config(m, n, k, world, dist):
    """The ``config`` object, identical in both arms (this library and ``--impl reference``)."""

    return {
        "workload": workload_name(m, n, k),
        "m": m, "n": n, "k": k,
        "parallelism": f"n-shard{world}" if world > 1 else "single",
        "l2": "no flush: operands (E4M3 A + B slice + scales) exceed the 126 MB L2",
        "inputs": ("N(0,1) x per-row 2^U(-4,4)" if dist == "square" else
                   "activations N(0,1) with 0.1% of channels x50, weights N(0,0.02)") + ", OCP MX quantised, seed 0",
    }


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except ValueError:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def fp8_peak(peaks, source, sustained):
    """Dense FP8 tensor-core denominator: 2 x the driver-measured dense BF16 rate (B200 FP8 = 2 x BF16).

    ``sustained`` selects the power-capped figure (a kernel timed inside a long
    run) instead of the burst one. A vendor library's FP8 rate is a comparator,
    reported as ``vs_cublaslt``, never a denominator."""

    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    return 2.0 * float(peaks[key]), f"2 x {source} dense BF16 ({key}) of MEASURED_PEAKS.json"


def recorded_traffic(workload, n_gpus):
    """DRAM bytes per launch from a committed ncu capture summary (or None)."""

    path = PROFILES / "traffic.json"
    if not path.exists():
        return None
    try:
        rec = json.loads(path.read_text()).get(f"{workload}@{n_gpus}")
    except ValueError:
        return None
    return None if rec is None else float(rec["bytes_per_launch"])


class ClockSampler:
    """Read-only NVML samples of SM clock, power and clock-event reasons every ``period_s``.

    ``mark()`` opens and ``close()`` ends the window that ``stop()`` summarises
    (host ``perf_counter`` times bracketing the device-timed region: the host
    enqueues the region's work after ``mark()`` and returns from the final
    synchronisation before ``close()``), so a region of a few ms (20 steps of a
    rank's slice at 8 GPUs: ~7 ms) gets its own samples.
    Without ``nvidia_ml_py`` it falls back to ``nvidia-smi -lms 200``. Nothing is
    ever set through NVML.
    """

    REASONS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu_index = gpu_index
        self.period_s = period_s
        self.samples: list[tuple[float, float, float, float, int]] = []  # (t, sm MHz, max MHz, W, reasons)
        self.window = None
        self._stop = threading.Event()
        self._thread = None
        self._smi = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)
        except Exception:  # no NVML binding or no driver: the nvidia-smi fallback
            self._start_smi()
            return self
        reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        smax = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

        def run():
            while not self._stop.is_set():
                t = time.perf_counter()
                try:
                    sm = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                    watts = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                    reasons = int(reasons_fn(handle))
                except Exception:
                    break
                self.samples.append((t, sm, smax, watts, reasons))
                self._stop.wait(self.period_s)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.sw_power_cap,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown")
        try:
            self._smi = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu_index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._smi = None
            return

        def read():
            for line in self._smi.stdout:
                parts = [x.strip() for x in line.split(",")]
                try:
                    bits = sum(bit for (_, bit), v in zip(self.REASONS[:4], parts[3:7]) if v.lower() == "active")
                    self.samples.append((time.perf_counter(), float(parts[0]), float(parts[1]), float(parts[2]), bits))
                except (ValueError, IndexError):
                    continue

        self._thread = threading.Thread(target=read, daemon=True)
        self._thread.start()
        self.period_s = 0.2

    def mark(self):
        self.window = [time.perf_counter(), None]

    def close(self):
        if self.window is not None:
            self.window[1] = time.perf_counter()

    def stop(self):
        self._stop.set()
        if self._smi is not None:
            self._smi.terminate()
            try:
                self._smi.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._smi.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)
        picked = self.samples
        if self.window is not None and self.window[1] is not None:
            t0, t1 = self.window
            picked = [x for x in self.samples if t0 <= x[0] <= t1]
        if not picked:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"], "samples": 0,
                    "source": "nvml" if self._smi is None else "nvidia-smi"}
        reasons = sorted({name for _, _, _, _, bits in picked for name, bit in self.REASONS if bits & bit})
        return {
            "sm_mhz": statistics.median(x[1] for x in picked),
            "sm_mhz_min": min(x[1] for x in picked),
            "sm_max_mhz": max(x[2] for x in picked),
            "power_w_median": statistics.median(x[3] for x in picked),
            "power_w_max": max(x[3] for x in picked),
            "reasons": reasons,
            "samples": len(picked),
            "period_ms": 1000.0 * self.period_s,
            "window_ms": None if self.window is None or self.window[1] is None
            else 1000.0 * (self.window[1] - self.window[0]),
            "source": "nvml" if self._smi is None else "nvidia-smi",
        }


def physical_gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def make_operands_on_device(m, n_local, k, n0, device, dist="square"):
    """Seeded synthetic sources, quantised on the GPU by our kernel (BASELINE distributions).

    ``square``: A and B ~ N(0,1) x per-row 2^U(-4,4). ``llm``: activations A ~ N(0,1)
    with 0.1 % of K-channels x50, weights B ~ N(0, 0.02). A is identical on every
    rank; rows of B are generated per global row block so a slice equals the same
    rows of the unsharded B."""

    import torch

    from cutex_b200.kernels import quantize_mxfp8

    def source(rows, seed, is_a=False):
        g = torch.Generator(device=device).manual_seed(seed)
        x = torch.randn(rows, k, device=device, generator=g)
        if dist == "llm":
            if is_a:
                cols = torch.randperm(k, device=device, generator=g)[: max(1, k // 1000)]
                x[:, cols] *= 50.0
            else:
                x *= 0.02
            return x
        x *= torch.exp2(torch.empty(rows, 1, device=device).uniform_(-4.0, 4.0, generator=g))
        return x

    xa = source(m, SEED, is_a=True)
    a, sfa = quantize_mxfp8(xa)
    del xa
    b = torch.empty(n_local, k, dtype=torch.uint8, device=device)
    sfb = torch.empty(((n_local + 127) // 128) * 128 * (k // 32), dtype=torch.uint8, device=device)
    chunk = 2048
    for r0 in range(0, n_local, chunk):
        rows = min(chunk, n_local - r0)
        xb = source(rows, SEED + 1 + (n0 + r0) // chunk)
        per_row = k // 32
        quantize_mxfp8(xb, q=b[r0:r0 + rows], sf=sfb[r0 * per_row:])
        del xb
    torch.cuda.synchronize()
    return a, sfa, b, sfb


CPU_SAMPLE_ROWS = 4096  # rows of A and of B in the CPU legs' sub-GEMM (K as the workload)


def cpu_sample(m, n, k, dist):
    """The CPU legs' operands: a seeded CPU_SAMPLE_ROWS x CPU_SAMPLE_ROWS x K sample of the workload."""

    from oracle.cpu_contract import cpu_sample_operands

    ms, ns = min(CPU_SAMPLE_ROWS, m), min(CPU_SAMPLE_ROWS, n)
    return (ms, ns) + tuple(cpu_sample_operands(ms, ns, k, dist=dist, seed=SEED))


def cpu_sample_text(ms, ns, m, n, k, dist, how):
    return (f"{ms}x{ns}x{k} sub-GEMM of the {m}x{n}x{k} workload ({dist} generator, seed {SEED}, OCP MX "
            f"quantised on the CPU): torch CPU dequant + fp32 matmul + bf16 cast, {how}")


def run_cpu_baseline(m, n, k, dist):
    """Time the contract's CPU path on the same seeded sample ``--impl reference`` times."""

    from oracle.cpu_contract import time_cpu_contract

    ms, ns, a_s, sfa_s, b_s, sfb_s = cpu_sample(m, n, k, dist)
    secs, threads, reps = time_cpu_contract(a_s, sfa_s, b_s, sfb_s)
    flops = 2.0 * ms * ns * k
    return {
        "value": flops / secs / 1e12,
        "unit": "TFLOP/s",
        "cores": threads,
        "kind": "port",
        "sample": cpu_sample_text(ms, ns, m, n, k, dist, f"median of {reps} runs of {secs:.3f} s"),
    }


def bench_reference(args):
    """--impl reference: the contract's CPU path on the host cores (rank 0 only), same sample as cpu_baseline."""

    world, rank, _ = dist_env()
    if rank != 0:
        return
    import torch

    from oracle.cpu_contract import cpu_contract_gemm

    m, n, k = args.m, args.n, args.k
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ms, ns, a, sfa, b, sfb = cpu_sample(m, n, k, args.dist)
    for _ in range(max(1, args.warmup)):
        cpu_contract_gemm(a, sfa, b, sfb)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_contract_gemm(a, sfa, b, sfb)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    flops = 2.0 * ms * ns * k
    value = flops * len(times) / total / 1e12
    sample = cpu_sample_text(ms, ns, m, n, k, args.dist, f"{len(times)} timed steps, {threads} threads")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / len(times),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3xe4m3->f32->bf16",
        "data": "synthetic",
        "config": workload_config(m, n, k, world, args.dist),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def bench_cutex(args):
    import torch
    import torch.distributed as dist

    from cutex_b200 import _lib
    from cutex_b200.kernels import GemmConfig, PreparedGemm, query
    from cutex_b200.sharding import shard_bounds

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    m, n, k = args.m, args.n, args.k
    shard = shard_bounds(n, world, rank, align=256 if world > 1 else 16)
    n_local = shard.n
    cfg = GemmConfig(**json.loads(args.config)) if args.config else GemmConfig()
    plan = query(m, n_local, k, cfg)

    a, sfa, b, sfb = make_operands_on_device(m, n_local, k, shard.n0, device, args.dist)
    d = torch.empty(m, n_local, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    torch.cuda.synchronize()

    # One prepared C-ABI launch per step; the timed loop is a CUDA graph of `steps`
    # launches (host launch overhead would otherwise show up as idle GPU time for
    # the ~50 us skinny shapes), or plain launches with --no-graph.
    with torch.cuda.stream(stream):
        step = PreparedGemm(a, b, sfa, sfb, d, stream=stream, config=cfg)
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.synchronize()
    if _lib.load().cutex_last_device_status(stream.cuda_stream) != 0:
        raise RuntimeError("device-side timeout during warm-up")
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(args.steps):
                step()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            graph.replay()  # first replay outside the timed region
        torch.cuda.synchronize()

    # The timed region starts after a 0.5 s pause (the bench's burst protocol); the 2 s
    # back-to-back `sustained` entry below is the power-capped rate.
    sampler = ClockSampler(physical_gpu_index(local)).start()
    time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sampler.mark()
    with torch.cuda.stream(stream):
        start.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.steps):
                step()
        end.record(stream)
    torch.cuda.synchronize()
    sampler.close()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    if _lib.load().cutex_last_device_status(stream.cuda_stream) != 0:
        raise RuntimeError("device-side timeout in the timed region")
    elapsed_ms = start.elapsed_time(end)

    # Sustained rate: the same launches back to back for ~args.sustained_s seconds
    # (power-capped steady state on a 1 kW part), reported beside the timed value.
    sustained = None
    if args.sustained_s > 0:
        sampler2 = ClockSampler(physical_gpu_index(local), period_s=0.05).start()
        s4, e4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 0
        sampler2.mark()
        t_wall = time.time()
        with torch.cuda.stream(stream):
            s4.record(stream)
            while time.time() - t_wall < args.sustained_s:
                if graph is not None:
                    graph.replay()
                else:
                    for _ in range(args.steps):
                        step()
                launches += args.steps
                stream.synchronize()
            e4.record(stream)
        torch.cuda.synchronize()
        sampler2.close()
        clocks2 = sampler2.stop()
        ts = torch.tensor([s4.elapsed_time(e4)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        sustained_value = 2.0 * m * n * k * launches / (float(ts[0]) / 1e3) / 1e12
        peak_s, peak_s_src = fp8_peak(*load_peaks(), True)
        sustained = {"value": sustained_value, "unit": "TFLOP/s", "launches": launches,
                     "seconds": float(ts[0]) / 1e3, "clocks": clocks2,
                     "frac": sustained_value / world / peak_s, "peak": peak_s, "peak_source": peak_s_src}
        if clocks2.get("power_w_median"):
            # Energy per GEMM at the power cap: median board power x time per launch (per GPU).
            sustained["joules_per_gemm"] = clocks2["power_w_median"] * (float(ts[0]) / 1e3) / launches
    # Back-to-back launches in one graph: the average launch duration is the
    # timed interval over the launch count (inter-kernel gaps included).
    t = torch.tensor([elapsed_ms, elapsed_ms / args.steps], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, launch_avg_ms = float(t[0]), float(t[1])

    total_flops = 2.0 * m * n * k
    value = total_flops * args.steps / (elapsed_ms / 1e3) / 1e12
    flops_launch = 2.0 * m * n_local * k
    bytes_launch = float(m * k + n_local * k + (m + n_local) * (k // 32) + 2 * m * n_local)
    peaks, source = load_peaks()
    long_timed = elapsed_ms > 2000.0
    workload = workload_name(m, n, k)
    hbm_bound = flops_launch / bytes_launch < RIDGE_FLOP_PER_BYTE
    if hbm_bound:
        achieved = bytes_launch / (launch_avg_ms / 1e3) / 1e9
        peak, peak_src = float(peaks["hbm_gbs"]), f"{source} HBM copy (hbm_gbs)"
    else:
        achieved = flops_launch / (launch_avg_ms / 1e3) / 1e12
        peak, peak_src = fp8_peak(peaks, source, long_timed)

    # ---- end to end through the library with pinned host buffers
    e2e = None
    if args.e2e_steps > 0:
        hb = b.cpu().pin_memory()
        hsb = sfb.cpu().pin_memory()
        hd = torch.empty(d.shape, dtype=d.dtype).pin_memory()
        if world == 1:
            from cutex_b200.kernels import HostGemm

            # The library's host-buffer entry: H2D copies, block GEMMs and D2H
            # copies overlapped on its own streams, joined back into `stream`.
            ha = a.cpu().pin_memory()
            hsa = sfa.cpu().pin_memory()
            # Steps are independent requests: step i runs on stream i % S with its
            # own HostGemm (device buffers) and its own pinned result, in stream
            # order on that stream; the library's copy/compute streams are shared,
            # so one step's D2H tail overlaps the next step's H2D.
            n_streams = max(1, args.e2e_streams)
            e2e_streams = [stream] + [torch.cuda.Stream(device) for _ in range(n_streams - 1)]
            host_gemms = [HostGemm(m, n_local, k, device=device, config=cfg, blocks=args.e2e_blocks)
                          for _ in range(n_streams)]
            hds = [hd] + [torch.empty(d.shape, dtype=d.dtype).pin_memory() for _ in range(n_streams - 1)]
            step_no = [0]

            def e2e_step():
                j = step_no[0] % n_streams
                step_no[0] += 1
                host_gemms[j](ha, hb, hsa, hsb, hds[j], stream=e2e_streams[j])

            h2d = ha.numel() + hb.numel() + hsa.numel() + hsb.numel()
            d2h = hd.numel() * hd.element_size()
            path = (f"cutex_mxfp8_gemm_host C ABI (HostGemm, {args.e2e_blocks}x{args.e2e_blocks} blocks), "
                    f"pinned host A/B/SFA/SFB in, D out; steps alternate over {n_streams} stream(s)")
        else:
            from cutex_b200.sharding import ShardedHostGemm

            # Each rank copies 1/world of A (A is the same on every rank) plus its
            # B slice in, NCCL gathers A over NVLink, D[:, n0:n1] comes back in row
            # blocks while the next block computes.
            # Steps alternate over S streams as on one GPU; each stream's
            # ShardedHostGemm has its own process group, so two all-gathers in
            # flight never share an NCCL communicator (every rank creates the
            # groups and runs the steps in the same order).
            n_streams = max(1, args.e2e_sharded_streams)
            groups = [None] + [dist.new_group(backend="nccl") for _ in range(n_streams - 1)]
            host_gemms = [ShardedHostGemm(m, n, k, group=g, config=cfg, device=device) for g in groups]
            host_gemm = host_gemms[0]
            r0, r1 = host_gemm.rows.n0, host_gemm.rows.n1
            sf_row = k // 32
            ha = a[r0:r1].cpu().pin_memory()
            hsa = sfa[r0 * sf_row:r1 * sf_row].cpu().pin_memory()
            e2e_streams = [stream] + [torch.cuda.Stream(device) for _ in range(n_streams - 1)]
            hds = [hd] + [torch.empty(d.shape, dtype=d.dtype).pin_memory() for _ in range(n_streams - 1)]
            step_no = [0]

            def e2e_step():
                j = step_no[0] % n_streams
                step_no[0] += 1
                host_gemms[j](ha, hsa, hb, hsb, hds[j], stream=e2e_streams[j])

            h_in, h_out = host_gemm.host_bytes()
            h2d, d2h = h_in * world, h_out * world
            path = ("ShardedHostGemm: pinned host rows of A (1/world per rank) + B slice in, "
                    f"NCCL all-gather of A, D slice out in row blocks; steps alternate over {n_streams} stream(s)")

        with torch.cuda.stream(stream):
            for _ in range(len(e2e_streams)):
                e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s2.record(stream)
            for other in e2e_streams[1:]:
                other.wait_event(s2)
            for _ in range(args.e2e_steps):
                e2e_step()
            for other in e2e_streams[1:]:
                stream.wait_stream(other)
            e2.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s2.elapsed_time(e2)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {
            "value": total_flops * args.e2e_steps / (float(te[0]) / 1e3) / 1e12,
            "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "steps": args.e2e_steps,
            "path": path,
        }
        del ha, hb, hsa, hsb, hd, host_gemms, hds

    allgather = None
    if args.allgather and world > 1:
        from cutex_b200.sharding import allgather_columns

        with torch.cuda.stream(stream):
            allgather_columns(d, world)
        torch.cuda.synchronize()
        dist.barrier()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s3.record(stream)
            full = allgather_columns(d, world)
            e3.record(stream)
        torch.cuda.synchronize()
        tg = torch.tensor([s3.elapsed_time(e3)], dtype=torch.float64, device=device)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        allgather = {"nccl_ms": float(tg[0]), "gemm_ms": launch_avg_ms,
                     "gemm_then_nccl_ms": launch_avg_ms + float(tg[0]),
                     "bytes_per_rank_received": int(full.numel() * 2 * (world - 1) / world)}
        # The same result with the gather fused into the GEMM's epilogue (peer TMA
        # stores over NVLink) and a one-element all-reduce as the closing barrier.
        from cutex_b200.sharding import FusedAllGatherGemm

        fused = FusedAllGatherGemm(m, n, k, config=cfg)
        with torch.cuda.stream(stream):
            for _ in range(2):
                fused(a, b, sfa, sfb, stream=stream)
        torch.cuda.synchronize()
        # Every rank's gathered D from the fused path equals the NCCL-gathered one, bit for bit.
        same = torch.tensor([1.0 if torch.equal(fused.d_full.view(torch.int16), full.view(torch.int16)) else 0.0],
                            dtype=torch.float64, device=device)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        allgather["bitwise_ok"] = bool(same[0] == 1.0)
        del full
        dist.barrier()
        s5, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        with torch.cuda.stream(stream):
            s5.record(stream)
            for _ in range(reps):
                fused(a, b, sfa, sfb, stream=stream)
            e5.record(stream)
        torch.cuda.synchronize()
        tf = torch.tensor([s5.elapsed_time(e5) / reps], dtype=torch.float64, device=device)
        dist.all_reduce(tf, op=dist.ReduceOp.MAX)
        allgather["fused_ms"] = float(tf[0])
        allgather["fused_path"] = "cutex_mxfp8_gemm_allgather + one-element NCCL all-reduce"
        dist.barrier()
        fused.close()
        del fused

    # ---- the vendor library on the same operands (comparator only, never the product path)
    cublaslt = None
    if args.vs_cublaslt > 0 and world == 1:
        cublaslt = compare_cublaslt(args, a, sfa, b, sfb, d, graph, step, stream, m, n, k)

    side = None
    if world == 1 and not args.no_configs:
        del graph
        graph = None
        side = bench_configs(args, device, stream)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_baseline = run_cpu_baseline(m, n, k, args.dist)

    if rank == 0:
        traffic = recorded_traffic(workload, world)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3xe4m3->f32->bf16",
            "data": "synthetic",
            "config": workload_config(m, n, k, world, args.dist),
            "kernel_plan": dict(plan, n_per_gpu=n_local),
            "roofline": {
                "bound": "hbm" if hbm_bound else "tensor",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s" if hbm_bound else "TFLOP/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "peak_source": peak_src,
                "algorithmic_flops_per_launch": flops_launch,
                "algorithmic_bytes_per_launch": bytes_launch,
                "launch_avg_ms": launch_avg_ms,
                "frac_of_nominal": achieved / (8000.0 if hbm_bound else 4500.0),
            },
            "cpu_baseline": cpu_baseline,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "clocks": clocks,
            "sustained": sustained,
        }
        if allgather is not None:
            line["allgather"] = allgather
        if cublaslt is not None:
            line["cublaslt"] = cublaslt
            if "value" in cublaslt:
                # This kernel over cuBLASLt's MXFP8 GEMM on the same operands, alternating graph
                # replays in the same run (a comparator, not a roofline).
                line["vs_cublaslt"] = {"ratio": cublaslt["cutex_value_same_rounds"] / cublaslt["value"],
                                       "cublaslt_tflops": cublaslt["value"],
                                       "bitwise_equal": cublaslt["bitwise_equal"]}
        if side is not None:
            line["configs"] = side
        print(json.dumps(line), flush=True)

    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def compare_cublaslt(args, a, sfa, b, sfb, d, graph, step, stream, m, n, k):
    """cuBLASLt's MXFP8 GEMM (torch._scaled_mm) on the same device operands.

    Each round replays one CUDA graph of `steps` launches of this kernel, then one
    of cuBLASLt, after 0.3 s idle each; the medians over the rounds are reported
    with the outputs' bitwise agreement."""
    import torch

    A, B = a.view(torch.float8_e4m3fn), b.view(torch.float8_e4m3fn)
    SA, SB = sfa.view(torch.float8_e8m0fnu), sfb.view(torch.float8_e8m0fnu)
    try:
        with torch.cuda.stream(stream):
            ref = torch._scaled_mm(A, B.t(), SA, SB, out_dtype=torch.bfloat16)
            for _ in range(max(args.warmup, 3)):
                torch._scaled_mm(A, B.t(), SA, SB, out_dtype=torch.bfloat16)
            step()
        torch.cuda.synchronize()
    except RuntimeError as exc:  # e.g. a scale shape cuBLASLt does not take
        return {"unavailable": str(exc).splitlines()[0][:200]}
    equal = bool(torch.equal(ref.view(torch.int16), d.view(torch.int16)))
    lt_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(lt_graph, stream=stream):
        for _ in range(args.steps):
            torch._scaled_mm(A, B.t(), SA, SB, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()

    def timed(replay):
        time.sleep(0.3)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s0.record(stream)
            replay()
            s1.record(stream)
        torch.cuda.synchronize()
        return s0.elapsed_time(s1) / args.steps

    def ours():
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.steps):
                step()

    mine, theirs = [], []
    for _ in range(args.vs_cublaslt):
        mine.append(timed(ours))
        theirs.append(timed(lt_graph.replay))
    sustained = None
    if args.sustained_s > 0 and args.cublaslt_sustained:
        # The same back-to-back protocol as this kernel's `sustained` entry.
        time.sleep(1.0)
        sampler = ClockSampler(physical_gpu_index(0), period_s=0.05).start()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 0
        sampler.mark()
        t_wall = time.time()
        with torch.cuda.stream(stream):
            s2.record(stream)
            while time.time() - t_wall < args.sustained_s:
                lt_graph.replay()
                launches += args.steps
                stream.synchronize()
            e2.record(stream)
        torch.cuda.synchronize()
        sampler.close()
        secs = s2.elapsed_time(e2) / 1e3
        sustained = {"value": 2.0 * m * n * k * launches / secs / 1e12, "unit": "TFLOP/s", "launches": launches,
                     "seconds": secs, "clocks": sampler.stop()}
    del lt_graph
    flops = 2.0 * m * n * k
    med = lambda xs: sorted(xs)[len(xs) // 2]  # noqa: E731
    return {"value": flops / (med(theirs) / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_launch": med(theirs),
            "cutex_value_same_rounds": flops / (med(mine) / 1e3) / 1e12, "cutex_ms_per_launch": med(mine),
            "rounds": args.vs_cublaslt, "bitwise_equal": equal, "sustained": sustained,
            "path": "torch._scaled_mm (cuBLASLt MXFP8, E4M3 x E4M3, E8M0 1x32 scales -> BF16), CUDA graph"}


def time_quantizer(kind, qdtype, m, k, steps, warmup, dev, stream):
    """Device time per launch of one MXFP8 quantiser on a seeded [m, k] input (one CUDA graph of ``steps``).

    Returns (ms per launch, algorithmic bytes per launch, clocks of the timed window)."""
    import torch

    from cutex_b200.kernels import quantize_mxfp8, quantize_mxfp8_columnwise
    from cutex_b200.kernels.dense_gemm import scale_buffer_bytes

    g = torch.Generator(device=dev).manual_seed(SEED)
    x = torch.randn(m, k, device=dev, generator=g)
    x *= torch.exp2(torch.empty(m, 1, device=dev).uniform_(-4.0, 4.0, generator=g))
    if qdtype == "bf16":
        x = x.to(torch.bfloat16)
    stream.wait_stream(torch.cuda.current_stream(dev))
    if kind == "rowwise":
        q = torch.empty(m, k, dtype=torch.uint8, device=dev)
        sf = torch.empty(scale_buffer_bytes(m, k), dtype=torch.uint8, device=dev)
        step = lambda: quantize_mxfp8(x, q=q, sf=sf, stream=stream)  # noqa: E731
    else:
        q = torch.empty(k, m, dtype=torch.uint8, device=dev)
        sf = torch.empty(scale_buffer_bytes(k, m), dtype=torch.uint8, device=dev)
        step = lambda: quantize_mxfp8_columnwise(x, qt=q, sft=sf, stream=stream)  # noqa: E731
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            step()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu_index(dev.index or 0)).start()
    time.sleep(0.5)  # the same pause before the timed region as the GEMM's burst protocol
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.mark()
    with torch.cuda.stream(stream):
        s0.record(stream)
        graph.replay()
        s1.record(stream)
    torch.cuda.synchronize()
    sampler.close()
    clocks = sampler.stop()
    ms = s0.elapsed_time(s1) / steps
    in_bytes = 4 if qdtype == "f32" else 2
    nbytes = float(m * k * (in_bytes + 1) + m * k // 32)
    del graph
    return ms, nbytes, clocks


def bench_quantize(args):
    """The MXFP8 quantisers (the step before the GEMM) on an [M, K] input, device-timed.

    Rowwise: x [M, K] -> E4M3 [M, K] + 1x32 E8M0 scales along K (128x4 layout).
    Columnwise: x [M, K] -> E4M3 [K, M] = quantise(x^T) + scales of a [K, M]
    operand. Algorithmic bytes per launch: M*K*(input bytes + 1) + M*K/32; one CUDA
    graph of `steps` launches; the 1 GB (f32) or 512 MB (bf16) input exceeds the L2."""
    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    m, k = args.m, args.k
    stream = torch.cuda.Stream(dev)
    ms, nbytes, clocks = time_quantizer(args.quantize, args.qdtype, m, k, args.steps, args.warmup, dev, stream)
    peaks, source = load_peaks()
    achieved = nbytes / (ms / 1e3) / 1e9
    peak = float(peaks["hbm_gbs"])
    print(json.dumps({
        "metric": f"MXFP8 {args.quantize} quantiser GB/s (device-timed)",
        "value": achieved, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": f"{args.qdtype}->e4m3+e8m0", "data": "synthetic",
        "config": {"workload": f"mxfp8_quantize_{args.quantize}_{args.qdtype}_m{m}_k{k}", "m": m, "k": k,
                   "l2": "no flush: the input exceeds the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": f"{source} HBM copy (hbm_gbs)",
                     "algorithmic_bytes_per_launch": nbytes, "launch_avg_ms": ms},
        "gpu_launches": args.steps, "clocks": clocks,
    }), flush=True)


# Other BASELINE configurations timed beside the headline in the default N = 1 run:
# (name, M, N, K, input distribution, launches per timed region, L2 policy).
SIDE_GEMMS = (
    ("mxfp8_fprop_m4096_n4096_k4096", 4096, 4096, 4096, "square", 64, "rotate"),
    ("mxfp8_fprop_m8192_n28672_k8192", 8192, 28672, 8192, "llm", 20, "graph"),
    ("mxfp8_fprop_m128_n28672_k8192", 128, 28672, 8192, "llm", 200, "graph"),
    ("mxfp8_fprop_m16_n28672_k8192", 16, 28672, 8192, "llm", 200, "graph"),
)
SIDE_QUANTIZERS = (("rowwise", "f32"), ("rowwise", "bf16"), ("columnwise", "bf16"))


def roofline_entry(flops, nbytes, ms, peaks, source):
    """Both rates of one launch and the fraction of the roofline that bounds its shape."""

    hbm_bound = flops / nbytes < RIDGE_FLOP_PER_BYTE
    tflops = flops / (ms / 1e3) / 1e12
    gbs = nbytes / (ms / 1e3) / 1e9
    if hbm_bound:
        peak, unit, achieved, src = float(peaks["hbm_gbs"]), "GB/s", gbs, f"{source} HBM copy (hbm_gbs)"
    else:
        peak, src = fp8_peak(peaks, source, False)
        unit, achieved = "TFLOP/s", tflops
    return {"tflops": tflops, "gbs": gbs,
            "roofline": {"bound": "hbm" if hbm_bound else "tensor", "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak, "peak_source": src}}


def bench_configs(args, dev, stream):
    """BASELINE's other configurations, each timed on the device in this run (N = 1).

    Each is timed as one CUDA graph of back-to-back launches. GEMMs whose B
    exceeds the 126 MB L2 run on one operand set; 4096^3 (operands and D fit in
    the L2) cycles over enough operand sets to exceed twice the L2. Each entry
    carries its clocks, kernel plan and roofline fraction."""
    import torch

    from cutex_b200 import _lib
    from cutex_b200.benchmark import L2_FLUSH_BYTES
    from cutex_b200.kernels import PreparedGemm, query

    peaks, source = load_peaks()
    out = {}
    for name, m, n, k, dist, reps, policy in SIDE_GEMMS:
        # "rotate": operands and D fit in the L2, so the launches cycle over `sets` operand
        # sets whose bytes together exceed twice the 126 MB L2: every launch reads A and B
        # that the launches in between have evicted. (A 256 MB write between launches
        # leaves the whole L2 dirty, and the next GEMM pays for writing it back.)
        per_set = m * k + n * k + (m + n) * (k // 32) + 2 * m * n
        sets = max(1, -(-(2 * L2_FLUSH_BYTES) // per_set)) if policy == "rotate" else 1
        stream.wait_stream(torch.cuda.current_stream(dev))
        steps, keep = [], []
        for i in range(sets):
            a, sfa, b, sfb = make_operands_on_device(m, n, k, 0, dev, dist)
            d = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(stream):
                steps.append(PreparedGemm(a, b, sfa, sfb, d, stream=stream))
            keep.append((a, sfa, b, sfb, d))
        with torch.cuda.stream(stream):
            for _ in range(5):
                for st in steps:
                    st()
        torch.cuda.synchronize()
        sampler = ClockSampler(physical_gpu_index(dev.index or 0)).start()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(reps):
                steps[i % sets]()
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        time.sleep(0.5)  # the headline's burst protocol: a 0.5 s pause before each timed region
        sampler.mark()
        with torch.cuda.stream(stream):
            s0.record(stream)
            graph.replay()
            s1.record(stream)
        torch.cuda.synchronize()
        sampler.close()
        ms = s0.elapsed_time(s1) / reps
        if sets > 1:
            l2 = (f"inputs rotate over {sets} operand sets ({sets * per_set / 1e6:.0f} MB, over twice the 126 MB "
                  "L2): every launch reads operands the launches in between evicted; one CUDA graph")
        else:
            l2 = "no flush: B exceeds the 126 MB L2; one CUDA graph of back-to-back launches"
        del graph
        if _lib.load().cutex_last_device_status(stream.cuda_stream) != 0:
            raise RuntimeError(f"device-side timeout in {name}")
        flops = 2.0 * m * n * k
        nbytes = float(m * k + n * k + (m + n) * (k // 32) + 2 * m * n)
        plan = query(m, n, k)
        entry = {"m": m, "n": n, "k": k, "inputs": dist, "launches": reps, "ms_per_launch": ms,
                 "kernel": {key: plan[key] for key in ("kernel", "tile_m", "tile_n", "stages", "grid_ctas",
                                                       "split_k", "scheduler")},
                 "l2": l2, "clocks": sampler.stop()}
        entry.update(roofline_entry(flops, nbytes, ms, peaks, source))
        out[name] = entry
        del keep, steps
        torch.cuda.empty_cache()
    for kind, qdtype in SIDE_QUANTIZERS:
        m = k = 16384
        ms, nbytes, clocks = time_quantizer(kind, qdtype, m, k, 20, 3, dev, stream)
        gbs = nbytes / (ms / 1e3) / 1e9
        out[f"mxfp8_quantize_{kind}_{qdtype}_m{m}_k{k}"] = {
            "m": m, "k": k, "launches": 20, "ms_per_launch": ms, "gbs": gbs, "clocks": clocks,
            "l2": "no flush: the input exceeds the 126 MB L2; one CUDA graph of back-to-back launches",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                         "frac": gbs / float(peaks["hbm_gbs"]), "peak_source": f"{source} HBM copy (hbm_gbs)"}}
        torch.cuda.empty_cache()
    return out


def bench_host_ceiling(args):
    """What bounds the end-to-end rate: the host links of all ranks, and the phases of one step.

    Every rank times, at the same time as the others (barrier, max over ranks):
    512 MiB pinned host -> device, device -> host, and both directions at once
    (two streams); then one rank alone. Then one end-to-end step at M, N, K and
    each of its phases alone: at N > 1 ShardedHostGemm (this rank's rows of A in,
    the NCCL all-gather of A, the B slice in, the GEMM, the D slice out); at
    N = 1 the same copies and GEMM without the gather. Rank 0 prints one JSON line."""
    import torch
    import torch.distributed as dist

    from cutex_b200.kernels import dense_gemm
    from cutex_b200.kernels.dense_gemm_contract import scale_buffer_bytes

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def tmax(ms):
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    def timed(fn, reps=3):
        fn()  # untimed first call: module loading, attributes, allocator
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return tmax(e0.elapsed_time(e1) / reps)

    nb = 512 << 20
    h_in = torch.empty(nb, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nb, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nb, dtype=torch.uint8, device=dev)
    d_out = torch.zeros(nb, dtype=torch.uint8, device=dev)
    side = torch.cuda.Stream(dev)

    def both():
        side.wait_stream(torch.cuda.current_stream())
        d_in.copy_(h_in, non_blocking=True)
        with torch.cuda.stream(side):
            h_out.copy_(d_out, non_blocking=True)
        torch.cuda.current_stream().wait_stream(side)

    links = {
        "h2d_GBs_all_ranks": world * nb / timed(lambda: d_in.copy_(h_in, non_blocking=True)) / 1e6,
        "d2h_GBs_all_ranks": world * nb / timed(lambda: h_out.copy_(d_out, non_blocking=True)) / 1e6,
        "both_directions_GBs_all_ranks": 2 * world * nb / timed(both) / 1e6,
    }
    one = timed(lambda: d_in.copy_(h_in, non_blocking=True) if rank == 0 else None)
    links["h2d_GBs_one_rank_alone"] = nb / one / 1e6
    # The host pipeline copies each finished D block (rows x cols of a row-major [M, N] D) back
    # as a pitched 2-D copy: the same bytes as a 512 MiB contiguous copy, in 4096 x 4096 bf16
    # blocks with the 16384-element row pitch of D.
    try:
        from cuda.bindings import runtime as cudart

        pitch = 16384 * 2
        rows_blk, cols_blk = 4096, 4096
        nblk = nb // (rows_blk * cols_blk * 2)
        kind = cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost

        def pitched():
            hs = torch.cuda.current_stream().cuda_stream
            for i in range(nblk):
                off = (i // 4) * rows_blk * pitch + (i % 4) * cols_blk * 2
                err = cudart.cudaMemcpy2DAsync(h_out.data_ptr() + off, pitch, d_out.data_ptr() + off, pitch,
                                               cols_blk * 2, rows_blk, kind, hs)[0]
                if err != cudart.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaMemcpy2DAsync: {err}")

        links["d2h_pitched_blocks_GBs_all_ranks"] = world * nb / timed(pitched) / 1e6
    except ImportError:
        links["d2h_pitched_blocks_GBs_all_ranks"] = None
    del h_in, h_out, d_in, d_out

    m, n, k = args.m, args.n, args.k
    sfr = k // 32
    phases = {}
    if world > 1:
        from cutex_b200.sharding import ShardedHostGemm

        g = ShardedHostGemm(m, n, k)
        r0, r1 = g.rows.n0, g.rows.n1
        ha = torch.randint(0, 120, (r1 - r0, k), dtype=torch.uint8).pin_memory()
        hsa = torch.full(((r1 - r0) * sfr,), 120, dtype=torch.uint8).pin_memory()
        hb = torch.randint(0, 120, (g.cols.n, k), dtype=torch.uint8).pin_memory()
        hsb = torch.full((g.sfb.numel(),), 120, dtype=torch.uint8).pin_memory()
        hd = torch.empty(m, g.cols.n, dtype=torch.bfloat16).pin_memory()
        g(ha, hsa, hb, hsb, hd)
        phases["step_ms"] = timed(lambda: g(ha, hsa, hb, hsb, hd))
        phases["a_rows_h2d_ms"] = timed(lambda: (g.a_part.copy_(ha.reshape(-1), non_blocking=True),
                                                 g.sfa_part.copy_(hsa, non_blocking=True)))
        phases["a_allgather_ms"] = timed(lambda: (dist.all_gather_into_tensor(g.a, g.a_part),
                                                  dist.all_gather_into_tensor(g.sfa[: m * sfr], g.sfa_part)))
        phases["b_h2d_ms"] = timed(lambda: (g.b.copy_(hb, non_blocking=True), g.sfb.copy_(hsb, non_blocking=True)))
        phases["gemm_ms"] = timed(lambda: dense_gemm(g.a.view(m, k), g.b, g.sfa, g.sfb, g.d))
        phases["d_d2h_ms"] = timed(lambda: hd.copy_(g.d, non_blocking=True))
        host_bytes = world * sum(g.host_bytes())
    else:
        ha = torch.randint(0, 120, (m, k), dtype=torch.uint8).pin_memory()
        hb = torch.randint(0, 120, (n, k), dtype=torch.uint8).pin_memory()
        hsa = torch.full((scale_buffer_bytes(m, k),), 120, dtype=torch.uint8).pin_memory()
        hsb = torch.full((scale_buffer_bytes(n, k),), 120, dtype=torch.uint8).pin_memory()
        hd = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
        a, b = torch.empty_like(ha, device=dev), torch.empty_like(hb, device=dev)
        sfa, sfb = torch.empty_like(hsa, device=dev), torch.empty_like(hsb, device=dev)
        d = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        phases["a_h2d_ms"] = timed(lambda: (a.copy_(ha, non_blocking=True), sfa.copy_(hsa, non_blocking=True)))
        phases["b_h2d_ms"] = timed(lambda: (b.copy_(hb, non_blocking=True), sfb.copy_(hsb, non_blocking=True)))
        phases["gemm_ms"] = timed(lambda: dense_gemm(a, b, sfa, sfb, d))
        phases["d_d2h_ms"] = timed(lambda: hd.copy_(d, non_blocking=True))
        host_bytes = ha.numel() + hb.numel() + hsa.numel() + hsb.numel() + hd.numel() * 2
    flops = 2.0 * m * n * k
    ceiling_ms = host_bytes / links["both_directions_GBs_all_ranks"] / 1e6
    line = {"metric": "host-link ceiling and end-to-end step phases", "n_gpus": world,
            "config": workload_config(m, n, k, world, args.dist), "links": links, "phases": phases,
            "host_bytes_per_step": int(host_bytes),
            "step_floor_ms_at_both_directions_rate": ceiling_ms,
            "e2e_ceiling_tflops": flops / (ceiling_ms / 1e3) / 1e12}
    if "step_ms" in phases:
        line["e2e_one_stream_tflops"] = flops / (phases["step_ms"] / 1e3) / 1e12
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measure_fp8_peak(args):
    """Dense FP8 denominator measured like the driver's BF16 peak: the vendor library on 8192^3.

    cuBLASLt's MXFP8 GEMM through torch._scaled_mm (never part of the product
    path): best of 10 single launches (burst) and back-to-back launches for 4 s
    (sustained, power-capped)."""

    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    n = 8192
    a, sfa, b, sfb = make_operands_on_device(n, n, n, 0, dev)
    A, B = a.view(torch.float8_e4m3fn), b.view(torch.float8_e4m3fn)
    SA, SB = sfa.view(torch.float8_e8m0fnu), sfb.view(torch.float8_e8m0fnu)
    fn = lambda: torch._scaled_mm(A, B.t(), SA, SB, out_dtype=torch.bfloat16)  # noqa: E731
    flops = 2.0 * n ** 3
    for _ in range(10):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    sampler = ClockSampler(physical_gpu_index(0), period_s=0.05).start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    count = 0
    sampler.mark()
    t0 = time.time()
    s.record()
    while time.time() - t0 < 4.0:
        for _ in range(20):
            fn()
        count += 20
        torch.cuda.synchronize()
    e.record()
    e.synchronize()
    sampler.close()
    clocks = sampler.stop()
    out = {
        "tflops": flops / best / 1e9,
        "tflops_sustained": flops * count / s.elapsed_time(e) / 1e9,
        "how": "cuBLASLt MXFP8 via torch._scaled_mm, 8192^3, E4M3 x E4M3 with E8M0 1x32 scales -> BF16: "
               "best of 10 (burst) and back to back for 4 s (sustained)",
        "clocks_sustained": clocks,
        "gpu": torch.cuda.get_device_name(0),
    }
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    if args.measure_fp8_peak:
        measure_fp8_peak(args)
        return
    if args.quantize is not None:
        bench_quantize(args)
        return
    if args.host_ceiling:
        bench_host_ceiling(args)
        return
    if args.impl == "reference":
        bench_reference(args)
    else:
        bench_cutex(args)


if __name__ == "__main__":
    main()
