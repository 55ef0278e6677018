"""Worker for tests/test_gpu_allgather.py (run under torch.distributed.run, one process per GPU).

Per shape, each rank:
* computes its N-slice with the fused-all-gather GEMM and checks its full copy of D bit for
  bit against the unsharded GEMM computed locally (every output element is the same MMA
  sequence in both), and against the CPU oracle (contract tolerance) on every element;
* makes back-to-back calls with two different operand sets and no host barrier between
  them, copying each call's result on the stream before the next call is made, and checks
  every copy: a rank that runs ahead must never overwrite a result a peer is still reading;
* runs the same slice through ShardedHostGemm (pinned host rows of A in, A gathered over
  NVLink, D slice out).
Exits non-zero on a mismatch.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cutex_b200.kernels import GemmConfig, dense_gemm  # noqa: E402
from cutex_b200.sharding import FusedAllGatherGemm, ShardedHostGemm, scale_rows_slice, shard_bounds  # noqa: E402
from tests.gpu_helpers import O, make_operands  # noqa: E402


def _bits(t):
    return t.contiguous().view(torch.int16)


def fused_family(M, n_local):
    """The kernel cutex_mxfp8_gemm_allgather chooses for an [M, n_local] slice (its AUTO rule)."""

    if M > 128 and n_local % 256 == 0:
        return GemmConfig(kernel=2)
    return GemmConfig(kernel=1, tile_n=128)


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()
    failures = 0
    for M, N, K, seed in ((512, 512 * world, 512, 1), (100, 256 * world, 256, 2), (1024, 768 * world, 1024, 3)):
        shard = shard_bounds(N, world, rank)
        s0, s1 = scale_rows_slice(shard, K)
        sets = []
        for sd in (seed, seed + 100):
            a, sfa, b, sfb = make_operands(M, N, K, seed=sd)  # identical on every rank
            ta, tsa = torch.from_numpy(a).to(dev), torch.from_numpy(sfa).to(dev)
            tb, tsb = torch.from_numpy(b).to(dev), torch.from_numpy(sfb).to(dev)
            ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            # The bitwise reference runs the tile kernel the fused path picks for this rank's
            # slice: every output element is then the same MMA sequence in one accumulator.
            # (AUTO would take the split-K kernel for M <= 128, whose split tiles round
            # differently.)
            dense_gemm(ta, tb, tsa, tsb, ref, config=fused_family(M, shard.n))
            sets.append({"np": (a, sfa, b, sfb), "dev": (ta, tsa, tsb), "b_loc": tb[shard.n0:shard.n1].contiguous(),
                         "sfb_loc": tsb[s0:s1].contiguous(), "ref": ref})
        torch.cuda.synchronize()
        # The oracle on this rank's first operand set: every element of the gathered D.
        a, sfa, b, sfb = sets[0]["np"]
        o_ref, o_abs = O.gemm_reference(a, sfa, b, sfb, M, N, K)
        g = FusedAllGatherGemm(M, N, K)
        for rep in range(2):
            for buf in g._buffers:
                buf.fill_(float("nan"))
            dist.barrier()
            st = sets[0]
            full = g(st["dev"][0], st["b_loc"], st["dev"][1], st["sfb_loc"])
            torch.cuda.synchronize()
            if not torch.equal(_bits(full), _bits(st["ref"])):
                bad = (_bits(full) != _bits(st["ref"])).sum().item()
                print(f"rank {rank}: M={M} N={N} K={K} rep={rep}: {bad} elements differ from the unsharded GEMM",
                      flush=True)
                failures += 1
            report = O.check_gemm(_bits(full).cpu().numpy().view(np.uint16), o_ref, o_abs)
            if not report["ok"]:
                print(f"rank {rank}: M={M} N={N} K={K} rep={rep}: outside the oracle tolerance {report}", flush=True)
                failures += 1
        # Back to back, alternating operand sets, no host barrier: each result is copied on
        # the stream before the next call; peers may run ahead by a call.
        dist.barrier()
        copies = []
        for i in range(6):
            st = sets[i % 2]
            out = g(st["dev"][0], st["b_loc"], st["dev"][1], st["sfb_loc"])
            copies.append(out.clone())
        torch.cuda.synchronize()
        for i, got in enumerate(copies):
            if not torch.equal(_bits(got), _bits(sets[i % 2]["ref"])):
                print(f"rank {rank}: M={M} N={N} K={K} back-to-back call {i} read an overwritten result", flush=True)
                failures += 1
        torch.cuda.synchronize()
        dist.barrier()
        g.close()
        # Host-buffer path: this rank's rows of A in, A gathered over NVLink, D[:, n0:n1] out.
        if M % (128 * world) == 0:
            h = ShardedHostGemm(M, N, K)
            r0, r1 = h.rows.n0, h.rows.n1
            sfr = K // 32
            ha = torch.from_numpy(a[r0:r1]).contiguous().pin_memory()
            hsa = torch.from_numpy(sfa[r0 * sfr:r1 * sfr]).contiguous().pin_memory()
            hb = sets[0]["b_loc"].cpu().pin_memory()
            hsb = sets[0]["sfb_loc"].cpu().pin_memory()
            hd = torch.empty(M, shard.n, dtype=torch.bfloat16).pin_memory()
            for rep in range(2):
                hd.fill_(float("nan"))
                h(ha, hsa, hb, hsb, hd)
                torch.cuda.synchronize()
                want = sets[0]["ref"][:, shard.n0:shard.n1].cpu()
                if not torch.equal(_bits(hd), _bits(want)):
                    print(f"rank {rank}: ShardedHostGemm M={M} N={N} K={K} rep={rep} differs", flush=True)
                    failures += 1
            dist.barrier()
    dist.barrier()
    dist.destroy_process_group()
    if failures == 0:
        print(f"rank {rank}: fused all-gather OK", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
