"""compile(): the reference's tests (tests/test_compiler.py) plus cache-format interop."""

import json
import shutil
from dataclasses import dataclass

import pytest

from cutex_b200 import AutotuneError, Config, autotune
from cutex_b200.compiler import CompiledKernel, bind_config, compile
from tests.conftest import GOLDEN


@dataclass
class FakeCompiled:
    tile: int

    def __call__(self, *_args, **_kwargs):
        return self.tile


def test_compile_selects_and_persists_best_config(tmp_path):
    @autotune(configs=[Config({"tile": 32}, name="tile32"), Config({"tile": 128}, name="tile128")],
              key=["m"], warmup=1, rep=3)
    def kernel(m, tile=32):
        return m + tile

    compile_calls = []

    def fake_compile(_kernel, *_args, **kwargs):
        compile_calls.append(kwargs["tile"])
        return FakeCompiled(kwargs["tile"])

    def fake_benchmark(compiled, *_args, **_kwargs):
        return {32: 8.0, 128: 3.0}[compiled.tile]

    cache_path = tmp_path / "autotune.json"
    first = compile(kernel, 1024, cache_path=cache_path, do_bench=fake_benchmark, _compile_fn=fake_compile)
    assert isinstance(first, CompiledKernel)
    assert first.best_config.name == "tile128"
    assert first.cache_hit is None
    assert first(1024) == 128
    assert cache_path.exists()
    assert compile_calls == [32, 128]

    compile_calls.clear()
    second = compile(
        kernel, 1024, cache_path=cache_path,
        do_bench=lambda *_a, **_k: (_ for _ in ()).throw(AssertionError("disk cache should skip benchmarking")),
        _compile_fn=fake_compile,
    )
    assert second.best_config.name == "tile128"
    assert second.cache_hit == "disk"
    assert compile_calls == [128]


def test_force_retune_ignores_persistent_choice(tmp_path):
    @autotune(configs=[Config({"tile": 1}, name="one"), Config({"tile": 2}, name="two")], key=["m"], rep=1)
    def kernel(m, tile=1):
        return m + tile

    def fake_compile(_kernel, *_args, **kwargs):
        return FakeCompiled(kwargs["tile"])

    cache_path = tmp_path / "autotune.json"
    compile(kernel, 8, cache_path=cache_path, do_bench=lambda c, *_a, **_k: float(c.tile), _compile_fn=fake_compile)
    retuned = compile(kernel, 8, cache_path=cache_path, force_retune=True,
                      do_bench=lambda c, *_a, **_k: float(3 - c.tile), _compile_fn=fake_compile)
    assert retuned.best_config.name == "two"
    assert retuned.cache_hit is None


def test_reads_cache_written_by_the_reference(tmp_path):
    # autotune_cache_v1.json was written by the reference's own compile() (tests/golden/make_golden.py).
    cache = tmp_path / "autotune.json"
    shutil.copy(GOLDEN / "autotune_cache_v1.json", cache)
    entry = json.loads(cache.read_text())["entries"][0]

    @autotune(configs=[Config({"tile": 64}, name="tile64"), Config({"tile": 128}, name="tile128")], key=["m", "n"])
    def kernel(m, n, tile=64):
        return tile

    kernel.__qualname__ = entry["kernel"].split(".", 1)[1]
    kernel.__module__ = entry["kernel"].split(".", 1)[0]
    hit = compile(kernel, 4096, 8192, cache_path=cache, _compile_fn=lambda _k, *a, **kw: FakeCompiled(kw["tile"]),
                  do_bench=lambda *a, **k: (_ for _ in ()).throw(AssertionError("should hit the cache")))
    assert hit.cache_hit == "disk"
    assert hit.best_config.name == "tile128"
    assert hit.timings_us == entry["candidate_timings_us"]


def test_written_cache_has_reference_schema(tmp_path):
    @autotune(configs=[Config({"tile": 64}, name="tile64"), Config({"tile": 128}, name="tile128")], key=["m", "n"])
    def kernel(m, n, tile=64):
        return tile

    cache = tmp_path / "c.json"
    compile(kernel, 4096, 8192, cache_path=cache, _compile_fn=lambda _k, *a, **kw: FakeCompiled(kw["tile"]),
            do_bench=lambda c, *a, **k: {64: 7.5, 128: 3.25}[c.tile])
    ours = json.loads(cache.read_text())
    ref = json.loads((GOLDEN / "autotune_cache_v1.json").read_text())
    assert ours["version"] == ref["version"] == 1
    for e_ours, e_ref in zip(ours["entries"], ref["entries"]):
        assert set(e_ours) == set(e_ref)
        assert e_ours["key"] == e_ref["key"]
        assert e_ours["best_config"] == e_ref["best_config"]
        assert e_ours["candidate_timings_us"] == e_ref["candidate_timings_us"]


def test_corrupt_or_versioned_cache_is_ignored(tmp_path):
    @autotune(configs=[Config({"tile": 1}, name="one")], key=["m"])
    def kernel(m, tile=1):
        return tile

    cache = tmp_path / "c.json"
    for text in ("{not json", json.dumps({"version": 99, "entries": []})):
        cache.write_text(text)
        out = compile(kernel, 1, cache_path=cache, _compile_fn=lambda _k, *a, **kw: FakeCompiled(kw["tile"]),
                      do_bench=lambda *a, **k: 1.0)
        assert out.cache_hit is None
    assert json.loads(cache.read_text())["version"] == 1


def test_all_candidates_failing_raises(tmp_path):
    @autotune(configs=[Config({"tile": 1}, name="one"), Config({"tile": 2}, name="two")], key=["m"])
    def kernel(m, tile=1):
        return tile

    def broken(*_a, **_k):
        raise RuntimeError("candidate failed to launch")

    with pytest.raises(AutotuneError, match="all autotune candidates failed"):
        compile(kernel, 1, cache_path=tmp_path / "c.json", _compile_fn=broken)


def test_missing_key_field_raises():
    @autotune(configs=[Config({"tile": 1})], key=["m", "zz"])
    def kernel(m, tile=1):
        return tile

    with pytest.raises(AutotuneError, match="missing autotune key field 'zz'"):
        compile(kernel, 1, _compile_fn=lambda *a, **k: None, do_bench=lambda *a, **k: 1.0)


def test_default_binding_fixes_config_kwargs():
    def launcher(x, y, *, tile=0, stages=0):
        return (x, y, tile, stages)

    bound = bind_config(launcher, 1, 2, tile=128, stages=6, unrelated=5)
    assert bound(1, 2) == (1, 2, 128, 6)


def test_candidate_leaving_a_device_error_is_rejected(tmp_path):
    # The launcher's health probe reports a non-zero device status (e.g. an
    # expired bounded wait) after the first candidate: that candidate is out
    # even though it timed fastest.
    from cutex_b200.compiler import DEVICE_STATUS_ATTRIBUTE

    @autotune(configs=[Config({"tile": 1}, name="one"), Config({"tile": 2}, name="two")], key=["m"])
    def kernel(m, tile=1):
        return tile

    statuses = iter([6, 0])
    setattr(kernel, DEVICE_STATUS_ATTRIBUTE, lambda: next(statuses))
    out = compile(kernel, 1, cache_path=tmp_path / "c.json", _compile_fn=lambda _k, *a, **kw: FakeCompiled(kw["tile"]),
                  do_bench=lambda c, *a, **k: float(c.tile))
    assert out.best_config.name == "two"
    assert set(out.timings_us) == {"two"}
    assert json.loads((tmp_path / "c.json").read_text())["entries"][0]["best_config"]["name"] == "two"


def test_stale_cached_choice_outside_the_search_space_is_retuned(tmp_path):
    @autotune(configs=[Config({"tile": 1}, name="one")], key=["m"])
    def kernel(m, tile=1):
        return tile

    cache = tmp_path / "c.json"
    from cutex_b200.compiler import launcher_id

    cache.write_text(json.dumps({"version": 1, "entries": [{
        "kernel": launcher_id(kernel), "key": {"m": 1}, "best_config": {"name": "gone", "kwargs": {"tile": 9}},
        "candidate_timings_us": {"gone": 1.0}}]}))
    out = compile(kernel, 1, cache_path=cache, _compile_fn=lambda _k, *a, **kw: FakeCompiled(kw["tile"]),
                  do_bench=lambda *a, **k: 2.0)
    assert out.cache_hit is None and out.best_config.name == "one"
    assert [e["best_config"]["name"] for e in json.loads(cache.read_text())["entries"]] == ["one"]


def test_gemm_launcher_carries_the_device_health_probe():
    from cutex_b200.compiler import DEVICE_STATUS_ATTRIBUTE
    from cutex_b200.kernels.dense_gemm import mxfp8_gemm_launch

    assert callable(getattr(mxfp8_gemm_launch, DEVICE_STATUS_ATTRIBUTE))


def test_launcher_config_field_named_kernel_binds():
    # The GEMM launcher's config has a field called `kernel`; binding and compiling must pass it through.
    def launcher(x, *, kernel=0, tile_n=0):
        return (x, kernel, tile_n)

    assert bind_config(launcher, 1, kernel=3, tile_n=128)(1) == (1, 3, 128)

    @autotune(configs=[Config({"kernel": 1}, name="one"), Config({"kernel": 2}, name="two")], key=["x"])
    def tuned(x, *, kernel=0):
        return kernel

    out = compile(tuned, 5, cache_path=None,
                  do_bench=lambda bound, *a, warmup=0, rep=0, **k: float(bound(*a, **k)))
    assert out.best_config.name == "one" and out(5) == 1
