"""The no-allocation skinny entry point (cutex_mxfp8_gemm_skinny_static) vs the regular one.

For callers that cannot allocate device memory when they launch a GEMM (a
memory-capped pool, an allocator that forbids out-of-band cudaMalloc, a plugin
that is only handed its operands and output), the library runs the split-K
skinny kernel with scratch in a fixed device array it owns. This test calls it
through the C ABI twice in a row per shape and checks each result against the
regular entry point (cutex_mxfp8_gemm with a caller-provided workspace) and the
CPU oracle, within the contract tolerance of tests/test_gpu_gemm.py. It builds
its own operands so it also passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from cutex_b200 import _lib
from cutex_b200.kernels import GemmConfig, query
from tests.gpu_helpers import O, check, device_ok, make_operands

pytestmark = pytest.mark.gpu


def _regular(ta, tb, tsa, tsb, M, N, K):
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(query(M, N, K, GemmConfig(kernel=_lib.KERNEL_SKINNY))["workspace_bytes"], dtype=torch.uint8,
                     device="cuda")
    cfg = _lib.make_config(kernel=_lib.KERNEL_SKINNY)
    rc = _lib.load().cutex_mxfp8_gemm(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(), out.data_ptr(),
                                      M, N, K, N, ctypes.byref(cfg), ws.data_ptr(), ws.numel(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.status_string(rc)
    return out


def _static(ta, tb, tsa, tsb, M, N, K):
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = _lib.load().cutex_mxfp8_gemm_skinny_static(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(),
                                                    out.data_ptr(), M, N, K, N,
                                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.status_string(rc)
    return out


@pytest.mark.parametrize("shape", [(16, 4096, 2048), (128, 2048, 1024), (50, 1280, 4096)], ids=str)
def test_static_scratch_entry_matches_regular_entry_twice(shape):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=sum(shape), kind="llm")
    dev = "cuda"
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tsa, tsb = torch.from_numpy(sfa).to(dev), torch.from_numpy(sfb).to(dev)
    ref_out = _regular(ta, tb, tsa, tsb, M, N, K)
    for _ in range(2):  # two calls in a row share (and must re-clear) the scratch counters
        out = _static(ta, tb, tsa, tsb, M, N, K)
        torch.cuda.synchronize()
        device_ok()
        assert check(out, a, sfa, b, sfb, M, N, K)["ok"]
        # Same kernel, same split, same reduction order: identical to the regular entry.
        got = out.float().cpu().numpy()
        want = ref_out.float().cpu().numpy()
        assert np.array_equal(got, want)


def _buffers(M, N, K):
    """Real, full-size device buffers for an (M, N, K) call: a rejected call touches
    nothing, and a call that were accepted by mistake would still read valid memory."""

    dev = "cuda"
    a = torch.zeros(M, K, dtype=torch.uint8, device=dev)
    b = torch.zeros(N, K, dtype=torch.uint8, device=dev)
    sfa = torch.zeros(((M + 127) // 128) * 128 * (K // 32), dtype=torch.uint8, device=dev)
    sfb = torch.zeros(((N + 127) // 128) * 128 * (K // 32), dtype=torch.uint8, device=dev)
    d = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    return a, b, sfa, sfb, d


def test_static_scratch_entry_rejects_what_it_cannot_hold():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # M above the skinny range.
    a, b, sfa, sfb, d = _buffers(129, 256, 256)
    assert lib.cutex_mxfp8_gemm_skinny_static(a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(),
                                              d.data_ptr(), 129, 256, 256, 256, stream) == _lib.CUTEX_ERR_SHAPE
    # N one 128-row tile beyond the 16384 arrival counters the fixed array holds.
    n = 2097152 + 128
    a, b, sfa, sfb, d = _buffers(16, n, 128)
    assert lib.cutex_mxfp8_gemm_skinny_static(a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(),
                                              d.data_ptr(), 16, n, 128, n, stream) == _lib.CUTEX_ERR_WORKSPACE
    del a, b, sfa, sfb, d
    # A missing operand.
    a, b, sfa, sfb, d = _buffers(16, 256, 256)
    assert lib.cutex_mxfp8_gemm_skinny_static(None, b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), d.data_ptr(),
                                              16, 256, 256, 256, stream) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
    device_ok()
