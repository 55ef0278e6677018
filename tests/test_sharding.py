"""N-sharding partition math and the all-gather re-layout, on CPU ranks (gloo, world size 2 and 4)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cutex_b200.sharding import SHARD_ALIGN, allgather_columns, scale_rows_slice, shard_bounds
from oracle import mxfp8_oracle as O


@pytest.mark.parametrize("n,world", [(16384, 1), (16384, 2), (16384, 8), (28672, 8), (28672, 3), (512, 2)])
def test_shards_cover_n_contiguously_and_aligned(n, world):
    shards = [shard_bounds(n, world, r) for r in range(world)]
    assert shards[0].n0 == 0 and shards[-1].n1 == n
    for a, b in zip(shards, shards[1:]):
        assert a.n1 == b.n0
    assert all(s.n0 % SHARD_ALIGN == 0 and s.n > 0 for s in shards)
    assert max(s.n for s in shards) - min(s.n for s in shards) <= SHARD_ALIGN


def test_shard_sizes_match_baseline_configs():
    assert shard_bounds(16384, 8, 3).n == 2048
    assert shard_bounds(28672, 8, 7).n == 3584


@pytest.mark.parametrize("bad", [(1000, 2, 0), (256, 2, 0), (512, 2, 2), (512, 0, 0)])
def test_shard_rejects_bad_splits(bad):
    with pytest.raises(ValueError):
        shard_bounds(*bad)


def test_scale_slice_equals_unsharded_rows():
    rng = np.random.default_rng(0)
    n, k, world = 1024, 256, 4
    codes, sf = O.quantized_operands(O.make_square_source(n, k, rng))
    for r in range(world):
        s = shard_bounds(n, world, r)
        lo, hi = scale_rows_slice(s, k)
        # The slice of the swizzled buffer is exactly the buffer of the sliced rows.
        local = O.swizzle_scales(O.unswizzle_scales(sf, n, k)[s.n0:s.n1], k)
        assert np.array_equal(sf[lo:hi], local)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ok = False
    try:
        rng = np.random.default_rng(1)
        a, sfa = O.quantized_operands(O.make_square_source(m, k, rng))
        b, sfb = O.quantized_operands(O.make_square_source(n, k, rng))
        s = shard_bounds(n, world, rank)
        lo, hi = scale_rows_slice(s, k)
        # Each rank computes its column slice with the CPU contract path from its shard only.
        ref_local, _ = O.gemm_reference(a, sfa, b[s.n0:s.n1], sfb[lo:hi], m, s.n, k)
        d_local = torch.from_numpy(O.bf16_bits_to_f32(O.contract_output_bf16(ref_local)))
        full = allgather_columns(d_local, world)
        ref_full, _ = O.gemm_reference(a, sfa, b, sfb, m, n, k)
        want = O.bf16_bits_to_f32(O.contract_output_bf16(ref_full))
        ok = bool(np.array_equal(full.numpy(), want))
    finally:
        q.put((rank, ok))
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_gemm_allgather_equals_unsharded_on_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 64, 256 * world, 256, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=90) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in results), results
