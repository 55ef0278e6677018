"""The checked build (-DCUTEX_CHECKED): device-side index checks in every kernel.

* In the checked library the check mechanism itself works: a kernel whose lane
  fails a check leaves the site and the value in the record and
  CUTEX_ERR_DEVICE_CHECK in the status word, and the device stays usable.
* The GPU parity suites (every GEMM variant, ragged shapes, many tiles per CTA,
  rasterisation orders, cluster-launch-control stealing, the skinny kernel's
  stream-K, the fused epilogues, both quantisers, the all-gather peer stores, the
  host pipeline, the no-allocation entry) run again in a child process with the
  checked library loaded; tests/conftest.py then asserts after every GPU test
  that no check failed, and the suites themselves compare every result with the
  oracle.
* The product library has no checks: its self-test entry launches nothing.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from cutex_b200 import _lib

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CHECKED = os.environ.get(_lib.CHECKED_ENV) == "1"

SUITES = [
    "tests/test_gpu_device_checks.py",
    "tests/test_gpu_gemm.py",
    "tests/test_gpu_skinny.py",
    "tests/test_gpu_epilogue.py",
    "tests/test_gpu_quantize.py",
    "tests/test_gpu_columnwise.py",
    "tests/test_gpu_allgather.py",
    "tests/test_gpu_host.py",
    "tests/test_zz_no_alloc.py",
]


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.skipif(CHECKED, reason="the product library is not loaded in this process")
def test_product_build_has_no_checks():
    lib = _lib.load()
    assert lib.cutex_build_checked() == 0
    assert lib.cutex_selftest_device_check(_stream()) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert _lib.check_record(_stream()) == (0, 0)
    assert lib.cutex_last_device_status(_stream()) == _lib.CUTEX_OK


@pytest.mark.skipif(not CHECKED, reason="needs the checked library (CUTEX_B200_CHECKED=1)")
def test_failed_check_is_recorded_and_the_device_stays_usable():
    from tests.gpu_helpers import check, make_operands, run_gemm

    lib = _lib.load()
    assert lib.cutex_build_checked() == 1 and _lib.version().endswith("checked")
    assert lib.cutex_selftest_device_check(_stream()) == _lib.CUTEX_OK
    assert _lib.check_record(_stream()) == (0x21F, 0x5EED07)
    assert _lib.check_record(_stream()) == (0, 0)  # read and cleared
    assert lib.cutex_last_device_status(_stream()) == _lib.CUTEX_ERR_DEVICE_CHECK
    assert lib.cutex_last_device_status(_stream()) == _lib.CUTEX_OK
    M, N, K = 256, 512, 512
    a, sfa, b, sfb = make_operands(M, N, K, seed=41)
    assert check(run_gemm(a, sfa, b, sfb, M, N, K), a, sfa, b, sfb, M, N, K)["ok"]


@pytest.mark.skipif(CHECKED, reason="this is the child run")
def test_gpu_suites_pass_on_the_checked_build():
    from cutex_b200.build import CHECKED_LIB_PATH

    assert CHECKED_LIB_PATH.exists(), "build it with `python -m cutex_b200.build --checked`"
    env = {**os.environ, _lib.CHECKED_ENV: "1"}
    proc = subprocess.run([sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider", *SUITES],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=1500)
    tail = "\n".join((proc.stdout + proc.stderr).strip().splitlines()[-30:])
    assert proc.returncode == 0, tail
    assert " passed" in tail and "failed" not in tail, tail
