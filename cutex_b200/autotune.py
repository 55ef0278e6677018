"""Declarative autotune search spaces (no CUDA imports).

Mirrors the reference API ``cutex.autotune`` (``cutex/autotune.py:19-103``):
``Config`` is one point of the search space, ``@autotune(configs=..., key=...)``
attaches an ``AutotuneSpec`` to a launcher, and ``cutex_b200.compile`` does the
measuring and the persistent, shape-keyed caching. In this framework a config's
kwargs are fields of the native ``cutex_gemm_config`` (kernel family, tile_n,
stages, raster group/order, epilogue buffers, CTA cap) rather than CuTeDSL
compile-time arguments.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from os import PathLike
from pathlib import Path
from typing import Any, Callable, Mapping, Sequence

SPEC_ATTRIBUTE = "__cutex_autotune__"


class AutotuneError(RuntimeError):
    """No candidate configuration could be bound and measured."""


@dataclass(frozen=True)
class Config:
    """One configuration of a search space: keyword arguments plus an optional name/pre-hook."""

    kwargs: Mapping[str, Any] = field(default_factory=dict)
    name: str | None = None
    pre_hook: Callable[..., Any] | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "kwargs", {str(k): v for k, v in dict(self.kwargs).items()})
        if self.name is not None and not self.name.strip():
            raise ValueError("Config.name cannot be blank")

    @property
    def label(self) -> str:
        return self.name if self.name is not None else repr(dict(self.kwargs))


@dataclass(frozen=True)
class AutotuneSpec:
    configs: tuple[Config, ...]
    key: tuple[str, ...]
    warmup: int = 5
    rep: int = 30
    cache_results: bool = True
    force_retune: bool = False
    cache_path: Path | None = None
    do_bench: Callable[..., float] | None = None


def autotune(
    *,
    configs: Sequence[Config],
    key: Sequence[str],
    warmup: int = 5,
    rep: int = 30,
    cache_results: bool = True,
    force_retune: bool = False,
    cache_path: str | PathLike[str] | None = None,
    do_bench: Callable[..., float] | None = None,
):
    """Attach a validated search space to a launcher; measuring happens in ``compile``."""

    configs = tuple(configs)
    key = tuple(str(k) for k in key)
    if len(configs) == 0:
        raise ValueError("autotune requires at least one Config")
    if any(k == "" for k in key):
        raise ValueError("autotune key names cannot be blank")
    if len(key) != len(set(key)):
        raise ValueError("autotune key names must be unique")
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    if rep < 1:
        raise ValueError("rep must be at least one")
    spec = AutotuneSpec(
        configs=configs,
        key=key,
        warmup=warmup,
        rep=rep,
        cache_results=cache_results,
        force_retune=force_retune,
        cache_path=None if cache_path is None else Path(cache_path),
        do_bench=do_bench,
    )

    def attach(kernel):
        setattr(kernel, SPEC_ATTRIBUTE, spec)
        return kernel

    return attach


def read_autotune_spec(kernel) -> AutotuneSpec | None:
    spec = getattr(kernel, SPEC_ATTRIBUTE, None)
    if spec is None:
        spec = getattr(getattr(kernel, "__call__", None), SPEC_ATTRIBUTE, None)
    return spec
