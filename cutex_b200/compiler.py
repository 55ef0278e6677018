"""Configuration binding plus persistent first-use autotuning.

Same contract as the reference's ``cutex.compile`` (``cutex/compiler.py:189-306``):

* a launcher without an ``@autotune`` spec is bound once and returned;
* with a spec, the key fields are read from the call's arguments, the JSON
  cache (format version 1: ``{"version": 1, "entries": [{"kernel", "key",
  "best_config": {"name", "kwargs"}, "candidate_timings_us"}]}``) is consulted
  and, on a miss or ``force_retune``, every candidate is bound and timed
  (median of CUDA-event samples); failing candidates are skipped, the fastest
  is persisted atomically (temp file + ``os.replace``);
* ``do_bench(compiled, *runtime_args, warmup=, rep=, **runtime_kwargs)``
  returns microseconds; ``_compile_fn`` is the injection point tests use.

The kernels are compiled ahead of time (``libcutex_mxfp8.so``), so "compile"
here binds the candidate's native config fields to the launcher; nothing is
JIT-compiled at run time.
"""

from __future__ import annotations

import functools
import inspect
import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

from .autotune import AutotuneError, AutotuneSpec, Config, read_autotune_spec
from .benchmark import cuda_benchmark

CACHE_FORMAT_VERSION = 1


@dataclass
class CompiledKernel:
    """The selected configuration bound to its launcher; calling it launches."""

    compiled: Callable[..., Any]
    best_config: Config
    timings_us: dict[str, float]
    cache_hit: str | None = None
    cache_path: Path | None = None

    def __call__(self, *args: Any, **kwargs: Any):
        return self.compiled(*args, **kwargs)

    @property
    def metadata(self) -> dict[str, Any]:
        return {
            "best_config": {"name": self.best_config.name, "kwargs": dict(self.best_config.kwargs)},
            "candidate_timings_us": dict(self.timings_us),
            "cache_hit": self.cache_hit,
            "cache_path": None if self.cache_path is None else str(self.cache_path),
        }


def bind_config(kernel: Callable[..., Any], *args: Any, **kwargs: Any) -> Callable[..., Any]:
    """Default "compile": fix the configuration keyword arguments of a launcher.

    Positional ``args`` are only used for key resolution; the returned callable
    takes the runtime arguments again, like a compiled CuTe function does.
    """

    sig = _signature(kernel)
    config_kwargs = {k: v for k, v in kwargs.items() if k in sig.parameters}
    return functools.partial(kernel, **config_kwargs)


def _signature(kernel) -> inspect.Signature:
    try:
        return inspect.signature(kernel)
    except (TypeError, ValueError):
        return inspect.signature(kernel.__call__)


def _json_value(value: Any) -> Any:
    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    if isinstance(value, (list, tuple)):
        return [_json_value(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _json_value(v) for k, v in value.items()}
    inner = getattr(value, "value", None)
    if inner is not None and inner is not value:
        return _json_value(inner)
    return str(value)


def _resolve_key_values(kernel, spec: AutotuneSpec, args, kwargs) -> dict[str, Any]:
    sig = _signature(kernel)
    try:
        values = dict(sig.bind_partial(*args, **kwargs).arguments)
    except TypeError:
        values = dict(zip(sig.parameters, args))
        values.update(kwargs)
    for name in spec.key:
        if name not in values:
            available = ", ".join(sorted(values)) or "none"
            raise AutotuneError(f"missing autotune key field {name!r}; available fields: {available}")
    return {name: _json_value(values[name]) for name in spec.key}


def _is_constexpr(annotation: Any) -> bool:
    text = str(annotation)
    return getattr(annotation, "__name__", None) == "Constexpr" or text.endswith(".Constexpr") or text.endswith(
        "Constexpr'>"
    )


def _runtime_arguments(kernel, args, kwargs):
    """Drop parameters annotated as compile-time constants from a launch."""

    params = list(_signature(kernel).parameters.values())
    rt_args = tuple(v for i, v in enumerate(args) if i >= len(params) or not _is_constexpr(params[i].annotation))
    by_name = {p.name: p for p in params}
    rt_kwargs = {k: v for k, v in kwargs.items() if k not in by_name or not _is_constexpr(by_name[k].annotation)}
    return rt_args, rt_kwargs


def _kernel_identifier(kernel) -> str:
    for target in (kernel, getattr(kernel, "__wrapped__", None), getattr(kernel, "fn", None)):
        if target is None:
            continue
        module = getattr(target, "__module__", None)
        qualname = getattr(target, "__qualname__", None) or getattr(target, "__name__", None)
        if module and qualname:
            return f"{module}.{qualname}"
    cls = type(kernel)
    return f"{cls.__module__}.{cls.__qualname__}"


def _read_cache(path: Path) -> list[dict[str, Any]]:
    try:
        payload = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, ValueError):
        return []
    if not isinstance(payload, dict) or payload.get("version") != CACHE_FORMAT_VERSION:
        return []
    entries = payload.get("entries")
    return [e for e in entries if isinstance(e, dict)] if isinstance(entries, list) else []


def _write_cache(path: Path, entries: list[dict[str, Any]]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + f".{os.getpid()}.tmp")
    tmp.write_text(
        json.dumps({"version": CACHE_FORMAT_VERSION, "entries": entries}, indent=2, sort_keys=True),
        encoding="utf-8",
    )
    os.replace(tmp, path)


def _matches(entry: dict[str, Any], kernel_id: str, key_values: dict[str, Any]) -> bool:
    return entry.get("kernel") == kernel_id and entry.get("key") == key_values


def _cached_choice(entries, kernel_id, key_values, configs):
    for entry in entries:
        if not _matches(entry, kernel_id, key_values):
            continue
        best = entry.get("best_config") or {}
        for config in configs:
            if best.get("name") == config.name and best.get("kwargs") == dict(config.kwargs):
                timings = {str(k): float(v) for k, v in (entry.get("candidate_timings_us") or {}).items()}
                return config, timings
    return None


def _persist(path, entries, kernel_id, key_values, config, timings_us) -> None:
    kept = [e for e in entries if not _matches(e, kernel_id, key_values)]
    kept.append(
        {
            "kernel": kernel_id,
            "key": key_values,
            "best_config": {"name": config.name, "kwargs": dict(config.kwargs)},
            "candidate_timings_us": timings_us,
        }
    )
    _write_cache(path, kept)


def compile(
    kernel,
    *args: Any,
    verbose: bool = False,
    force_retune: bool | None = None,
    cache_path: str | os.PathLike[str] | None = None,
    do_bench: Callable[..., float] | None = None,
    _compile_fn: Callable[..., Any] | None = None,
    **kwargs: Any,
):
    """Bind ``kernel`` and, when it carries an autotune spec, pick and cache the fastest config."""

    compile_fn = bind_config if _compile_fn is None else _compile_fn
    spec = read_autotune_spec(kernel)
    if spec is None:
        return compile_fn(kernel, *args, **kwargs)

    force = spec.force_retune if force_retune is None else force_retune
    path = Path(cache_path) if cache_path is not None else spec.cache_path
    key_values = _resolve_key_values(kernel, spec, args, kwargs)
    kernel_id = _kernel_identifier(kernel)
    entries = _read_cache(path) if path is not None else []

    hit = _cached_choice(entries, kernel_id, key_values, spec.configs) if spec.cache_results and not force else None
    if hit is not None:
        config, timings = hit
        if verbose:
            print(f"[cutex.autotune] disk cache hit: {config.label}")
        if config.pre_hook is not None:
            config.pre_hook(kernel, *args, **kwargs)
        bound = compile_fn(kernel, *args, **{**kwargs, **dict(config.kwargs)})
        return CompiledKernel(bound, config, timings, cache_hit="disk", cache_path=path)

    rt_args, rt_kwargs = _runtime_arguments(kernel, args, kwargs)
    bench = do_bench or spec.do_bench
    failures: list[tuple[str, BaseException]] = []
    measured: list[tuple[float, int, Config, Callable[..., Any]]] = []
    timings_us: dict[str, float] = {}
    for index, config in enumerate(spec.configs):
        try:
            if config.pre_hook is not None:
                config.pre_hook(kernel, *args, **kwargs)
            bound = compile_fn(kernel, *args, **{**kwargs, **dict(config.kwargs)})
            if bench is None:
                t = cuda_benchmark(bound, *rt_args, warmup=spec.warmup, rep=spec.rep, **rt_kwargs).median_us
            else:
                t = float(bench(bound, *rt_args, warmup=spec.warmup, rep=spec.rep, **rt_kwargs))
            if t < 0:
                raise ValueError("benchmark returned a negative duration")
            timings_us[config.label] = t
            measured.append((t, index, config, bound))
            if verbose:
                print(f"[cutex.autotune] {config.label}: {t:.3f} us")
        except Exception as exc:  # a failing candidate is recorded and skipped
            failures.append((config.label, exc))
            if verbose:
                print(f"[cutex.autotune] rejected {config.label}: {type(exc).__name__}: {exc}")

    if not measured:
        details = "\n".join(f"- {label}: {type(exc).__name__}: {exc}" for label, exc in failures)
        raise AutotuneError(f"all autotune candidates failed\n{details}")

    _, _, best, bound = min(measured, key=lambda item: (item[0], item[1]))
    if verbose:
        print(f"[cutex.autotune] selected: {best.label}")
    if spec.cache_results and path is not None:
        _persist(path, entries, kernel_id, key_values, best, timings_us)
    return CompiledKernel(bound, best, timings_us, cache_path=path)
