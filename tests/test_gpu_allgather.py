"""Fused GEMM + all-gather (cutex_mxfp8_gemm_allgather).

* On 2 GPUs of one node: tests/allgather_worker.py under torch.distributed.run (one process
  per GPU, NVLS off, short process-group timeout, an outer `timeout` as the last bound);
  skipped with fewer than two visible GPUs.
* On one GPU: the same kernel with every peer copy of D a local buffer, 2/4/8 ranks
  emulated by one launch each.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_fused_allgather_matches_unsharded_gemm():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "allgather_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=420)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("fused all-gather OK") == 2, r.stdout[-3000:]


def test_fused_allgather_peer_stores_emulated_on_one_gpu():
    # The fused epilogue's peer stores with every "peer" copy of D a buffer on this
    # GPU: `world` ranks emulated by one launch per rank (the launches do not wait on
    # one another, so running them one after the other on one GPU is safe). Each
    # copy must equal the unsharded GEMM bit for bit and pass the oracle.
    import ctypes

    from cutex_b200 import _lib
    from cutex_b200.kernels import GemmConfig, dense_gemm
    from cutex_b200.sharding import scale_rows_slice, shard_bounds
    from tests.gpu_helpers import O, device_ok, make_operands

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for world, (M, N, K) in ((4, (512, 2048, 512)), (8, (300, 4096, 256)), (2, (1024, 1536, 1024))):
        a, sfa, b, sfb = make_operands(M, N, K, seed=world)
        ta, tsa = torch.from_numpy(a).cuda(), torch.from_numpy(sfa).cuda()
        tb, tsb = torch.from_numpy(b).cuda(), torch.from_numpy(sfb).cuda()
        ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        dense_gemm(ta, tb, tsa, tsb, ref)
        copies = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        cfg = GemmConfig().to_c()
        keep = []
        for r in range(world):
            shard = shard_bounds(N, world, r)
            s0, s1 = scale_rows_slice(shard, K)
            b_loc, sfb_loc = tb[shard.n0:shard.n1].contiguous(), tsb[s0:s1].contiguous()
            peers = [copies[p].data_ptr() + shard.n0 * 2 for p in range(world) if p != r]
            maps = torch.empty(128 * len(peers), dtype=torch.uint8, device="cuda")
            _lib.check(lib.cutex_mxfp8_allgather_maps((ctypes.c_void_p * len(peers))(*peers), len(peers), M, shard.n,
                                                      N, maps.data_ptr(), maps.numel(), stream),
                       "cutex_mxfp8_allgather_maps")
            _lib.check(lib.cutex_mxfp8_gemm_allgather(ta.data_ptr(), b_loc.data_ptr(), tsa.data_ptr(),
                                                      sfb_loc.data_ptr(), copies[r].data_ptr() + shard.n0 * 2, M,
                                                      shard.n, K, N, maps.data_ptr(), len(peers), ctypes.byref(cfg),
                                                      stream),
                       "cutex_mxfp8_gemm_allgather")
            keep.append((b_loc, sfb_loc, maps))  # alive until the launches have run
        torch.cuda.synchronize()
        device_ok()
        for r in range(world):
            assert torch.equal(copies[r].view(torch.int16), ref.view(torch.int16)), (world, r)
        o_ref, o_abs = O.gemm_reference(a, sfa, b, sfb, M, N, K)
        rep = O.check_gemm(copies[-1].cpu().view(torch.int16).numpy().view(np.uint16), o_ref, o_abs)
        assert rep["ok"], rep
