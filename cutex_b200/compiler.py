"""``cutex_b200.compile``: pick a native GEMM configuration on first use and remember it.

Public surface (kept so code written against the reference's ``cutex.compile``,
``cutex/compiler.py:189-306``, keeps working): ``compile(kernel, *args,
verbose=, force_retune=, cache_path=, do_bench=, **kwargs)`` returning a
``CompiledKernel``, ``AutotuneError`` when no candidate survives, and the cache
file format version 1::

    {"version": 1, "entries": [{"kernel": "<module>.<qualname>",
                                "key": {<key field>: <value>, ...},
                                "best_config": {"name": ..., "kwargs": {...}},
                                "candidate_timings_us": {<label>: <us>, ...}}]}

so a cache written by either implementation is read by the other.

How it works here. The kernels are compiled ahead of time into
``libcutex_mxfp8.so``; a candidate is a set of ``cutex_gemm_config`` fields, and
"compiling" it means binding those fields to the launcher (``bind_config``).
A request goes through three steps:

1. ``_request_key``: the autotune key fields are looked up by name among the
   call's arguments (``mxfp8_gemm_launch`` keys on M, N, K and a device target
   string that carries the GPU name, compute capability, SM count and
   ``cutex_version()``, so a cache never crosses devices or library builds);
2. ``TuneCache.lookup``: a stored choice for (launcher, key) is used only if it
   is still one of the launcher's candidates;
3. ``_Search.run``: otherwise every candidate is bound, timed with CUDA events
   (``cutex_b200.benchmark.cuda_benchmark``, median) and then checked with the
   launcher's device health probe, if it has one (attribute
   ``__cutex_device_status__``: a callable returning the library's
   ``cutex_last_device_status`` for the stream). A candidate that raised or left
   a non-zero device status (a bounded wait that expired, a device-side check)
   is rejected; the fastest remaining one is stored and returned.
"""

from __future__ import annotations

import inspect
import json
import os
import tempfile
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Mapping

from .autotune import AutotuneError, AutotuneSpec, Config, read_autotune_spec
from .benchmark import cuda_benchmark

CACHE_FORMAT_VERSION = 1
DEVICE_STATUS_ATTRIBUTE = "__cutex_device_status__"


@dataclass
class CompiledKernel:
    """A launcher with its chosen configuration bound; calling it launches."""

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


def bind_config(kernel: Callable[..., Any], /, *args: Any, **kwargs: Any) -> Callable[..., Any]:
    """Bind the configuration keywords ``kernel`` accepts; the result takes the call's arguments.

    ``args`` only serve key resolution and are not bound. Keywords the launcher
    does not declare are dropped (a candidate may carry fields another launcher
    of the same search space uses). ``kernel`` is positional-only, so a launcher
    may itself take a ``kernel`` keyword (the GEMM's kernel-family field).
    """

    accepted = _parameters(kernel)
    fixed = {name: value for name, value in kwargs.items() if name in accepted}

    def launch(*call_args: Any, **call_kwargs: Any):
        return kernel(*call_args, **{**fixed, **call_kwargs})

    launch.bound_config = dict(fixed)  # type: ignore[attr-defined]
    return launch


def _parameters(kernel) -> Mapping[str, inspect.Parameter]:
    target = kernel if callable(kernel) and not isinstance(kernel, type) else kernel.__call__
    try:
        return inspect.signature(target).parameters
    except (TypeError, ValueError):
        return inspect.signature(target.__call__).parameters


def launcher_id(kernel) -> str:
    """``module.qualname`` of the launcher: the cache's ``kernel`` field."""

    for obj in (kernel, getattr(kernel, "__wrapped__", None), getattr(kernel, "fn", None)):
        module = getattr(obj, "__module__", None)
        name = getattr(obj, "__qualname__", None) or getattr(obj, "__name__", None)
        if obj is not None and module and name:
            return f"{module}.{name}"
    return f"{type(kernel).__module__}.{type(kernel).__qualname__}"


def _plain(value: Any) -> Any:
    """A JSON-representable form of a key value (numbers, strings, lists, dicts; else its str)."""

    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    if isinstance(value, Mapping):
        return {str(k): _plain(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_plain(v) for v in value]
    item = getattr(value, "item", None)  # numpy / torch scalars
    if callable(item) and getattr(value, "ndim", 1) == 0:
        return _plain(item())
    return str(value)


def _request_key(kernel, spec: AutotuneSpec, args: tuple, kwargs: dict) -> dict[str, Any]:
    """Values of the spec's key fields, found by parameter name among the call's arguments."""

    named: dict[str, Any] = {}
    positional = [p.name for p in _parameters(kernel).values()
                  if p.kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD)]
    named.update(zip(positional, args))
    named.update(kwargs)
    missing = [name for name in spec.key if name not in named]
    if missing:
        have = ", ".join(sorted(named)) or "none"
        raise AutotuneError(f"missing autotune key field {missing[0]!r}; available fields: {have}")
    return {name: _plain(named[name]) for name in spec.key}


class TuneCache:
    """The JSON cache file: one choice per (launcher id, key values).

    A missing, unreadable or other-version file reads as empty and is replaced
    on the next store; stores rewrite the whole file through a temporary file
    in the same directory and an atomic rename, so a reader never sees half a
    file.
    """

    def __init__(self, path: str | os.PathLike[str] | None):
        self.path = None if path is None else Path(path)
        self.entries: list[dict[str, Any]] = self._load()

    def _load(self) -> list[dict[str, Any]]:
        if self.path is None or not self.path.exists():
            return []
        try:
            doc = json.loads(self.path.read_text(encoding="utf-8"))
        except (OSError, UnicodeDecodeError, ValueError):
            return []
        if not isinstance(doc, dict) or doc.get("version") != CACHE_FORMAT_VERSION:
            return []
        found = doc.get("entries")
        return [e for e in found if isinstance(e, dict)] if isinstance(found, list) else []

    @staticmethod
    def _is(entry: dict[str, Any], kernel_id: str, key: dict[str, Any]) -> bool:
        return entry.get("kernel") == kernel_id and entry.get("key") == key

    def lookup(self, kernel_id: str, key: dict[str, Any], candidates) -> tuple[Config, dict[str, float]] | None:
        for entry in self.entries:
            if not self._is(entry, kernel_id, key):
                continue
            chosen = entry.get("best_config") or {}
            for cand in candidates:
                if chosen.get("name") == cand.name and chosen.get("kwargs") == dict(cand.kwargs):
                    raw = entry.get("candidate_timings_us") or {}
                    return cand, {str(label): float(us) for label, us in raw.items()}
        return None

    def store(self, kernel_id: str, key: dict[str, Any], chosen: Config, timings_us: dict[str, float]) -> None:
        if self.path is None:
            return
        self.entries = [e for e in self.entries if not self._is(e, kernel_id, key)]
        self.entries.append({"kernel": kernel_id, "key": key,
                             "best_config": {"name": chosen.name, "kwargs": dict(chosen.kwargs)},
                             "candidate_timings_us": dict(timings_us)})
        self.path.parent.mkdir(parents=True, exist_ok=True)
        fd, tmp = tempfile.mkstemp(prefix=f".{self.path.name}.", dir=self.path.parent)
        try:
            with os.fdopen(fd, "w", encoding="utf-8") as fh:
                json.dump({"version": CACHE_FORMAT_VERSION, "entries": self.entries}, fh, indent=2, sort_keys=True)
            os.replace(tmp, self.path)
        except BaseException:
            Path(tmp).unlink(missing_ok=True)
            raise


@dataclass
class _Search:
    """Time every candidate of one request; keep the survivors."""

    kernel: Any
    spec: AutotuneSpec
    bind: Callable[..., Any]
    bench: Callable[..., float] | None
    verbose: bool
    timings_us: dict[str, float] = field(default_factory=dict)
    rejected: dict[str, str] = field(default_factory=dict)

    def _log(self, text: str) -> None:
        if self.verbose:
            print(f"[cutex_b200.compile] {text}")

    def _time(self, bound, args, kwargs) -> float:
        if self.bench is not None:
            return float(self.bench(bound, *args, warmup=self.spec.warmup, rep=self.spec.rep, **kwargs))
        return cuda_benchmark(bound, *args, warmup=self.spec.warmup, rep=self.spec.rep, **kwargs).median_us

    def run(self, args: tuple, kwargs: dict) -> tuple[Config, Callable[..., Any]]:
        health = getattr(self.kernel, DEVICE_STATUS_ATTRIBUTE, None)
        best: tuple[float, Config, Callable[..., Any]] | None = None
        for cand in self.spec.configs:
            try:
                if cand.pre_hook is not None:
                    cand.pre_hook(self.kernel, *args, **kwargs)
                bound = self.bind(self.kernel, *args, **{**kwargs, **dict(cand.kwargs)})
                us = self._time(bound, args, kwargs)
                if not us >= 0.0:
                    raise ValueError(f"benchmark returned {us!r}")
                status = health() if health is not None else 0
                if status:
                    raise RuntimeError(f"device status {status} after the candidate ran")
            except Exception as exc:  # the candidate is out; the search goes on
                self.rejected[cand.label] = f"{type(exc).__name__}: {exc}"
                self._log(f"rejected {cand.label}: {self.rejected[cand.label]}")
                continue
            self.timings_us[cand.label] = us
            self._log(f"{cand.label}: {us:.3f} us")
            if best is None or us < best[0]:  # ties keep the earlier candidate
                best = (us, cand, bound)
        if best is None:
            lines = "\n".join(f"- {label}: {why}" for label, why in self.rejected.items())
            raise AutotuneError(f"all autotune candidates failed\n{lines}")
        self._log(f"selected {best[1].label}")
        return best[1], best[2]


def compile(kernel, /, *args: Any, verbose: bool = False, force_retune: bool | None = None,
            cache_path: str | os.PathLike[str] | None = None, do_bench: Callable[..., float] | None = None,
            _compile_fn: Callable[..., Any] | None = None, **kwargs: Any):
    """Bind ``kernel``; if it carries an ``@autotune`` spec, choose (or recall) its fastest configuration.

    ``args``/``kwargs`` are the launch's arguments: they supply the key fields and
    are what each candidate is timed on. ``do_bench(bound, *args, warmup=, rep=,
    **kwargs)`` replaces the CUDA-event timing (microseconds); ``_compile_fn``
    replaces ``bind_config`` (tests inject fakes through both).
    """

    bind = _compile_fn or bind_config
    spec = read_autotune_spec(kernel)
    if spec is None:
        return bind(kernel, *args, **kwargs)

    key = _request_key(kernel, spec, args, kwargs)
    kid = launcher_id(kernel)
    cache = TuneCache(cache_path if cache_path is not None else spec.cache_path)
    retune = spec.force_retune if force_retune is None else force_retune

    if spec.cache_results and not retune:
        hit = cache.lookup(kid, key, spec.configs)
        if hit is not None:
            chosen, timings = hit
            if verbose:
                print(f"[cutex_b200.compile] cache hit {cache.path}: {chosen.label}")
            if chosen.pre_hook is not None:
                chosen.pre_hook(kernel, *args, **kwargs)
            bound = bind(kernel, *args, **{**kwargs, **dict(chosen.kwargs)})
            return CompiledKernel(bound, chosen, timings, cache_hit="disk", cache_path=cache.path)

    search = _Search(kernel, spec, bind, do_bench or spec.do_bench, verbose)
    chosen, bound = search.run(args, kwargs)
    if spec.cache_results:
        cache.store(kid, key, chosen, search.timings_us)
    return CompiledKernel(bound, chosen, dict(search.timings_us), cache_path=cache.path)


__all__ = ["CACHE_FORMAT_VERSION", "CompiledKernel", "DEVICE_STATUS_ATTRIBUTE", "TuneCache", "bind_config",
           "compile", "launcher_id"]
