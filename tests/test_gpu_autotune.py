"""cutex_b200.compile on a B200: the GEMM launcher's search space timed, cached, recalled.

The reference's ``cutex.compile`` times every candidate on first use and keeps
the fastest in a JSON cache (``cutex/compiler.py:189-306``). Here the search
runs over the native configurations of ``mxfp8_gemm_launch`` on a compute-bound
square shape and on an HBM-bound M = 128 LLM shape; the second request must be
a cache hit that times nothing, and the winner's output must pass the oracle.
"""

import json

import numpy as np
import pytest
import torch

from cutex_b200 import compile
from cutex_b200.kernels.dense_gemm import GEMM_CONFIGS, device_target, mxfp8_gemm_launch
from tests.gpu_helpers import O, boundary_starts, check_sampled_blocks, device_ok, device_operands

pytestmark = pytest.mark.gpu


def _no_bench(*_a, **_k):
    raise AssertionError("a cache hit must not time anything")


@pytest.mark.parametrize("shape,kind", [((2048, 2048, 2048), "square"), ((128, 28672, 8192), "llm")], ids=str)
def test_search_caches_and_recalls_a_correct_winner(tmp_path, shape, kind):
    M, N, K = shape
    a, sfa, _ = device_operands(M, K, kind, seed=4, role="a")
    b, sfb, _ = device_operands(N, K, kind, seed=5, role="b")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    target = device_target()
    cache = tmp_path / "tune.json"

    first = compile(mxfp8_gemm_launch, a, b, sfa, sfb, out, M, N, K, target, cache_path=cache)
    device_ok()
    assert first.cache_hit is None
    timed = set(first.timings_us)
    skinny = {c.name for c in GEMM_CONFIGS if c.name.startswith("skinny")}
    if M <= 128:
        assert skinny <= timed  # the M <= 128 kernel competes
    else:
        assert not (skinny & timed)  # rejected by the library for M > 128, skipped by the search
    assert len(timed - skinny) == len(GEMM_CONFIGS) - len(skinny)
    entry = json.loads(cache.read_text())["entries"][0]
    assert entry["key"] == {"m": M, "n": N, "k": K, "target": target}
    assert entry["best_config"]["name"] == first.best_config.name

    second = compile(mxfp8_gemm_launch, a, b, sfa, sfb, out, M, N, K, target, cache_path=cache, do_bench=_no_bench)
    assert second.cache_hit == "disk"
    assert second.best_config == first.best_config

    out.fill_(float("nan"))
    second(a, b, sfa, sfb, out, M, N, K, target)
    torch.cuda.synchronize()
    device_ok()
    rows = [0, M - 64] if M >= 128 else [0]
    cols = boundary_starts(N, 64)
    reports = check_sampled_blocks(out, a, sfa, b, sfb, K, rows, cols, 64)
    bad = [r for r in reports if not r["ok"]]
    assert not bad, (first.best_config.name, bad[:2])
    assert not torch.isnan(out).any().item()
    assert np.isfinite(first.timings_us[first.best_config.label])
    assert O.REL_FRO_TOL == 1e-3
