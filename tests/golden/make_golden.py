"""Generate golden fixtures by running the reference's own pure-Python code.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/reference

It imports, from the reference:

* ``cutex.kernels.dense_gemm_v1._scale_index`` (``dense_gemm_v1.py:24-30``):
  the 128x4 scale-factor byte index at the fixed K = 16384;
* ``cutex.kernels.dense_gemm_contract`` (``dense_gemm_contract.py:6-58``):
  constants, FLOP count, the serialised contract dict;
* ``cutex.benchmark.stats_from_samples`` / ``paired_comparison``
  (``benchmark.py:29-41,142-186``) on fixed literal samples;
* ``cutex.compiler.compile`` with a fake compiler and benchmark
  (the injection points its own tests use, ``tests/test_compiler.py:30-44``)
  to capture the on-disk autotune cache format (``compiler.py:135-140,167-186``).

The fixtures are small JSON files committed next to this script; the GPU box
and the test suite read only the fixtures, never the reference.
"""

from __future__ import annotations

import json
import random
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from cutex import Config, autotune  # noqa: E402
    from cutex.benchmark import paired_comparison, stats_from_samples  # noqa: E402
    from cutex.compiler import compile as ref_compile  # noqa: E402
    from cutex.kernels import dense_gemm_contract as contract  # noqa: E402
    from cutex.kernels.dense_gemm_v1 import _scale_index  # noqa: E402

    # ---- scale-factor index at K = 16384 (outer = row of A or B, k = element column)
    rng = random.Random(20260822)
    pairs = []
    for outer in list(range(0, 260)) + [16383, 16256, 8191, 4097]:
        for k in (0, 31, 32, 95, 96, 127, 128, 159, 4095, 8192, 16383):
            pairs.append((outer, k))
    for _ in range(4000):
        pairs.append((rng.randrange(16384), rng.randrange(16384)))
    sf_cases = [[o, k, int(_scale_index(o, k))] for o, k in pairs]
    (HERE / "sf_index_k16384.json").write_text(
        json.dumps({"K": 16384, "source": "cutex/kernels/dense_gemm_v1.py:24-30", "cases": sf_cases})
    )

    # ---- contract
    payload = {
        "source": "cutex/kernels/dense_gemm_contract.py",
        "M": contract.M,
        "N": contract.N,
        "K": contract.K,
        "PROBLEM_SHAPE": list(contract.PROBLEM_SHAPE),
        "TILE": [contract.TILE_M, contract.TILE_N, contract.TILE_K],
        "MMA_SHAPE": list(contract.MMA_SHAPE),
        "SF_VECTOR_SIZE": contract.SF_VECTOR_SIZE,
        "SCALE_FACTOR_ELEMENTS": contract.SCALE_FACTOR_ELEMENTS,
        "SCALE_FACTOR_LOGICAL_SHAPE": list(contract.SCALE_FACTOR_LOGICAL_SHAPE),
        "OPERATION": contract.OPERATION,
        "INPUT_FORMAT": contract.INPUT_FORMAT,
        "SCALE_FORMAT": contract.SCALE_FORMAT,
        "SCALE_LAYOUT": contract.SCALE_LAYOUT,
        "MULTIPLY_FORMAT": contract.MULTIPLY_FORMAT,
        "ACCUMULATOR_FORMAT": contract.ACCUMULATOR_FORMAT,
        "OUTPUT_FORMAT": contract.OUTPUT_FORMAT,
        "dense_gemm_flops": contract.dense_gemm_flops(),
        "dense_gemm_contract": contract.dense_gemm_contract(),
    }
    (HERE / "contract.json").write_text(json.dumps(payload, indent=1, sort_keys=True))

    # ---- benchmark statistics
    samples_a = [9.0, 12.0, 10.0, 11.5, 10.25, 9.75, 30.0, 10.0, 10.5, 9.5, 10.0]
    samples_b = [10.0, 10.0, 11.0, 11.0, 10.0, 10.0, 12.0, 9.0, 10.5, 10.5, 10.0]
    sa = stats_from_samples(samples_a)
    sb = stats_from_samples(samples_b)
    bench = {
        "source": "cutex/benchmark.py",
        "samples_a": samples_a,
        "samples_b": samples_b,
        "stats_a": sa.to_dict(include_samples=True),
        "stats_b": sb.to_dict(),
        "paired": paired_comparison(sa, sb),
    }
    (HERE / "benchmark_stats.json").write_text(json.dumps(bench, indent=1, sort_keys=True))

    # ---- autotune cache format written by the reference's compile()
    @autotune(
        configs=[Config({"tile": 64}, name="tile64"), Config({"tile": 128}, name="tile128")],
        key=["m", "n"],
        warmup=1,
        rep=2,
    )
    def kernel(m, n, tile=64):
        return m + n + tile

    class Fake:
        def __init__(self, tile):
            self.tile = tile

        def __call__(self, *args, **kwargs):
            return self.tile

    with tempfile.TemporaryDirectory() as tmp:
        cache = Path(tmp) / "autotune.json"
        ref_compile(
            kernel,
            4096,
            8192,
            cache_path=cache,
            do_bench=lambda c, *a, **k: {64: 7.5, 128: 3.25}[c.tile],
            _compile_fn=lambda _k, *a, **kw: Fake(kw["tile"]),
        )
        text = cache.read_text()
    (HERE / "autotune_cache_v1.json").write_text(text)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
