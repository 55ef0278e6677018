"""Host-buffer pipeline (cutex_mxfp8_gemm_host): pinned host operands in, pinned host D out.

Every block GEMM is the device kernel on a sub-rectangle with the full K
reduction, so the host pipeline's D must equal the device path's D bit for
bit; one case is also checked against the CPU oracle. Covers blocks = 1..16,
ragged last blocks in both dimensions, M <= 128 (skinny kernel per block),
M x N grids that are not square, and repeated calls on one HostGemm (the
library reuses its streams and events).
"""

import numpy as np
import pytest
import torch

from cutex_b200 import _lib
from cutex_b200.kernels import HostGemm, dense_gemm, dense_gemm_host
from tests.gpu_helpers import check, make_operands

pytestmark = pytest.mark.gpu


def _pinned(x):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.pin_memory()


def _device_result(a, sfa, b, sfb, M, N):
    dev = "cuda"
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    dense_gemm(torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), torch.from_numpy(sfa).to(dev),
               torch.from_numpy(sfb).to(dev), out)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize(
    "shape,blocks",
    [((1024, 1024, 512), 1), ((1024, 1024, 512), 2), ((1024, 1024, 512), 8), ((1000, 784, 256), 4),
     ((2304, 512, 384), 3), ((512, 2560, 256), 16), ((130, 2048, 512), 8), ((64, 1024, 1024), 4)],
    ids=str)
def test_host_pipeline_equals_device_path(shape, blocks):
    M, N, K = shape
    a, sfa, b, sfb = make_operands(M, N, K, seed=M + N + blocks)
    ha, hb, hsa, hsb = _pinned(a), _pinned(b), _pinned(sfa), _pinned(sfb)
    hd = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    hg = HostGemm(M, N, K, blocks=blocks)
    hg(ha, hb, hsa, hsb, hd)
    torch.cuda.synchronize()
    ref = _device_result(a, sfa, b, sfb, M, N)
    assert torch.equal(hd.view(torch.int16), ref.view(torch.int16))
    # A second call on the same object (streams and events reused) with new data.
    a2, sfa2, b2, sfb2 = make_operands(M, N, K, seed=M + N + blocks + 1)
    hd2 = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    host2 = (_pinned(a2), _pinned(b2), _pinned(sfa2), _pinned(sfb2))  # alive until the copies have run
    hg(*host2, hd2)
    torch.cuda.synchronize()
    ref2 = _device_result(a2, sfa2, b2, sfb2, M, N)
    assert torch.equal(hd2.view(torch.int16), ref2.view(torch.int16))


def test_host_pipeline_against_oracle():
    M, N, K = 768, 640, 1024
    a, sfa, b, sfb = make_operands(M, N, K, seed=5)
    hd = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    host = (_pinned(a), _pinned(b), _pinned(sfa), _pinned(sfb))  # alive until the copies have run
    dense_gemm_host(*host, hd, blocks=3)
    torch.cuda.synchronize()
    r = check(hd, a, sfa, b, sfb, M, N, K)
    assert r["ok"], r


def test_host_pipeline_orders_after_and_before_the_callers_stream():
    M, N, K = 512, 512, 256
    a, sfa, b, sfb = make_operands(M, N, K, seed=9)
    ha, hb, hsa, hsb = _pinned(a), _pinned(b), _pinned(sfa), _pinned(sfb)
    hd = torch.zeros(M, N, dtype=torch.bfloat16).pin_memory()
    hg = HostGemm(M, N, K, blocks=2)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        hg(ha, hb, hsa, hsb, hd, stream=s)
        marker = torch.ones(1, device="cuda")
        copy = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        copy.copy_(hd, non_blocking=True)  # enqueued after the call: must see the finished D
    s.synchronize()
    ref = _device_result(a, sfa, b, sfb, M, N)
    assert torch.equal(copy.cpu().view(torch.int16), ref.view(torch.int16))
    assert marker.item() == 1.0


def test_host_pipeline_rejects_bad_arguments():
    hg = HostGemm(256, 256, 128, blocks=2)
    small = torch.empty(10, dtype=torch.uint8)
    good_a = torch.empty(256, 128, dtype=torch.uint8)
    with pytest.raises(_lib.CutexArgumentError):
        hg(small, good_a, good_a, good_a, torch.empty(256, 256, dtype=torch.bfloat16))
    with pytest.raises(_lib.CutexArgumentError):
        hg(good_a.cuda(), good_a, good_a, good_a, torch.empty(256, 256, dtype=torch.bfloat16))


def test_independent_requests_on_two_streams():
    # Two HostGemm objects (own device buffers) on two streams share the
    # library's copy/compute streams: alternating calls overlap, and every
    # result must still equal the device path bit for bit.
    M, N, K = 1024, 1536, 512
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    gemms = [HostGemm(M, N, K, blocks=4), HostGemm(M, N, K, blocks=4)]
    cases, outs, keep = [], [], []
    for i in range(6):
        a, sfa, b, sfb = make_operands(M, N, K, seed=100 + i)
        cases.append((a, sfa, b, sfb))
        host = (_pinned(a), _pinned(b), _pinned(sfa), _pinned(sfb))
        keep.append(host)  # pinned inputs stay alive until the copies have run
        hd = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        gemms[i % 2](*host, hd, stream=streams[i % 2])
        outs.append(hd)
    torch.cuda.synchronize()
    for (a, sfa, b, sfb), hd in zip(cases, outs):
        ref = _device_result(a, sfa, b, sfb, M, N)
        assert torch.equal(hd.view(torch.int16), ref.view(torch.int16))
