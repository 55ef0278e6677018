"""The device error path, driven to the end without a fault: bounded waits that expire.

``cutex_mxfp8_selftest_wait_timeout`` runs a GEMM on the self-test build of the
single-CTA kernel: waits give up after 1 ms and the TMA producer withholds one
K-stage, so no copy is in flight for it and nothing faults. Every role must time
out in turn, settle, free TMEM and exit; the host reads CUTEX_ERR_TIMEOUT from
the status word, the word is cleared by the read, the output is untouched, and
ordinary GEMMs on the same device still pass the oracle afterwards.
"""

import time

import pytest
import torch

from cutex_b200 import _lib
from tests.gpu_helpers import GemmConfig, check, make_operands, run_gemm

pytestmark = pytest.mark.gpu


def _launch(ta, tb, tsa, tsb, d, M, N, K, withhold, stream):
    return _lib.load().cutex_mxfp8_selftest_wait_timeout(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(),
                                                          tsb.data_ptr(), d.data_ptr(), M, N, K, withhold, stream)


@pytest.mark.parametrize("withhold", [0, 2, 7])
def test_expired_waits_report_timeout_and_leave_the_device_usable(withhold):
    M, N, K = 512, 512, 1024  # 16 CTAs of one 128 x 128 tile each, 8 K-stages per tile
    a, sfa, b, sfb = make_operands(M, N, K, seed=21)
    dev = torch.device("cuda")
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    d = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    lib = _lib.load()
    assert lib.cutex_last_device_status(stream) == _lib.CUTEX_OK  # nothing left over from earlier tests
    t0 = time.perf_counter()
    assert _launch(ta, tb, tsa, tsb, d, M, N, K, withhold, stream) == _lib.CUTEX_OK
    assert lib.cutex_last_device_status(stream) == _lib.CUTEX_ERR_TIMEOUT
    elapsed = time.perf_counter() - t0
    assert elapsed < 5.0, f"the self-test launch took {elapsed:.2f} s (limits are 1 ms per wait)"
    assert lib.cutex_last_device_status(stream) == _lib.CUTEX_OK  # the read cleared the word
    torch.cuda.synchronize()  # no sticky CUDA error in the context
    assert torch.isnan(d).all().item(), "no tile may be stored when its accumulation never finished"
    # The same device and stream, ordinary launches: correct results.
    for cfg in (GemmConfig(kernel=1, tile_n=128, scheduler=1), GemmConfig()):
        rep = check(run_gemm(a, sfa, b, sfb, M, N, K, cfg), a, sfa, b, sfb, M, N, K)
        assert rep["ok"], rep


def test_self_test_rejects_a_stage_outside_the_first_tile():
    M, N, K = 128, 128, 256
    dev = torch.device("cuda")
    t = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)  # real, large enough buffers for every operand
    d = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for bad in (-1, K // 128):
        assert _launch(t, t, t, t, d, M, N, K, bad, stream) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert _lib.load().cutex_last_device_status(stream) == _lib.CUTEX_OK
    assert not d.any().item()  # nothing was launched
