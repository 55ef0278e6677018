"""Ahead-of-time build of libcutex_mxfp8.so for sm_100a (in-tree, no JIT cache).

``python -m cutex_b200.build`` compiles ``cutex_b200/csrc/cutex_abi.cu`` (which
includes every kernel of the library) with nvcc into ``cutex_b200/_lib``;
``--checked`` also builds ``libcutex_mxfp8_checked.so`` (``-DCUTEX_CHECKED``:
device-side index checks in every kernel; selected at load time by
``CUTEX_B200_CHECKED=1``).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_NAME = "libcutex_mxfp8.so"
LIB_PATH = LIB_DIR / LIB_NAME
CHECKED_LIB_NAME = "libcutex_mxfp8_checked.so"
CHECKED_LIB_PATH = LIB_DIR / CHECKED_LIB_NAME
CHECKED_FLAGS = ["-DCUTEX_CHECKED"]
INCLUDE_DIR = PACKAGE_DIR.parent / "include"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build cutex_b200")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


STAMP_PATH = LIB_DIR / (LIB_NAME + ".sha256")


def _paths(checked: bool) -> tuple[Path, Path]:
    lib = CHECKED_LIB_PATH if checked else LIB_PATH
    return lib, lib.with_name(lib.name + ".sha256")


def source_digest(extra_flags: list[str] | None = None) -> str:
    """SHA-256 over every source file's name and bytes and the compiler flags.

    The library is rebuilt when this differs from the digest recorded beside it
    at its last build, so a copied or checked-out tree whose file times say
    nothing (the built library travels with the sources) still rebuilds exactly
    when a source or a flag changed."""

    h = hashlib.sha256()
    for flag in [*NVCC_FLAGS, *(extra_flags or [])]:
        h.update(flag.encode() + b"\0")
    for src in sources():
        h.update(src.name.encode() + b"\0")
        h.update(src.read_bytes())
        h.update(b"\0")
    return h.hexdigest()


def _flags(extra_flags: list[str] | None, checked: bool) -> list[str]:
    return [*(CHECKED_FLAGS if checked else []), *(extra_flags or [])]


def is_stale(extra_flags: list[str] | None = None, checked: bool = False) -> bool:
    lib, stamp = _paths(checked)
    if not lib.exists() or not stamp.exists():
        return True
    return stamp.read_text().strip() != source_digest(_flags(extra_flags, checked))


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          checked: bool = False) -> Path:
    """Compile the shared library if it is missing or its sources or flags changed since it was built.

    ``checked=True`` builds the checked library (``-DCUTEX_CHECKED``) beside the
    product one instead."""

    lib, stamp = _paths(checked)
    if not force and not is_stale(extra_flags, checked):
        return lib
    flags = _flags(extra_flags, checked)
    digest = source_digest(flags)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_DIR / f".{lib.name}.{os.getpid()}.tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, *flags, "-o", str(tmp), str(CSRC / "cutex_abi.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-8000:]}")
    os.replace(tmp, lib)
    stamp.write_text(digest + "\n")
    return lib


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
    if "--checked" in sys.argv:
        print(build(force="--force" in sys.argv, verbose=True, checked=True))
