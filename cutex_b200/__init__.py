"""cutex-b200: B200-native MXFP8 block-scaled GEMM behind the cutex API.

Public names mirror the reference package ``cutex`` (``cutex/__init__.py``):
``Config``, ``autotune``, ``compile``, ``CompiledKernel``, ``AutotuneError``,
``AutotuneSpec``. Kernels live in ``cutex_b200.kernels``; timing helpers in
``cutex_b200.benchmark``; N-sharding across GPUs in ``cutex_b200.sharding``.
"""

from .autotune import AutotuneError, AutotuneSpec, Config, autotune
from .compiler import CompiledKernel, compile

__all__ = [
    "AutotuneError",
    "AutotuneSpec",
    "CompiledKernel",
    "Config",
    "autotune",
    "compile",
]

__version__ = "0.1.0"
