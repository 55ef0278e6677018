"""Worker for tests/test_gpu_allgather.py (run under torch.distributed.run, one process per GPU).

Each rank computes its N-slice with the fused-all-gather GEMM and checks that its full copy of D
equals the unsharded GEMM computed locally, bit for bit (every output element is the same MMA
sequence in both); then the same slice through ShardedHostGemm (pinned host rows of A in, A
gathered over NVLink, D slice out). Exits non-zero on a mismatch.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cutex_b200.kernels import dense_gemm  # noqa: E402
from cutex_b200.sharding import FusedAllGatherGemm, ShardedHostGemm, scale_rows_slice, shard_bounds  # noqa: E402
from tests.gpu_helpers import make_operands  # noqa: E402


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()
    failures = 0
    for M, N, K, seed in ((512, 512 * world, 512, 1), (100, 256 * world, 256, 2), (1024, 768 * world, 1024, 3)):
        a, sfa, b, sfb = make_operands(M, N, K, seed=seed)  # identical on every rank
        shard = shard_bounds(N, world, rank)
        s0, s1 = scale_rows_slice(shard, K)
        ta, tsa = torch.from_numpy(a).to(dev), torch.from_numpy(sfa).to(dev)
        tb, tsb = torch.from_numpy(b).to(dev), torch.from_numpy(sfb).to(dev)
        b_loc, sfb_loc = tb[shard.n0:shard.n1].contiguous(), tsb[s0:s1].contiguous()
        g = FusedAllGatherGemm(M, N, K)
        for rep in range(2):
            g.d_full.fill_(float("nan"))
            dist.barrier()
            full = g(ta, b_loc, tsa, sfb_loc)
            ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            dense_gemm(ta, tb, tsa, tsb, ref)
            torch.cuda.synchronize()
            if not torch.equal(full.view(torch.int16), ref.view(torch.int16)):
                bad = (full.view(torch.int16) != ref.view(torch.int16)).sum().item()
                print(f"rank {rank}: M={M} N={N} K={K} rep={rep}: {bad} mismatching elements", flush=True)
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
            hb = b_loc.cpu().pin_memory()
            hsb = sfb_loc.cpu().pin_memory()
            hd = torch.empty(M, shard.n, dtype=torch.bfloat16).pin_memory()
            for rep in range(2):
                hd.fill_(float("nan"))
                h(ha, hsa, hb, hsb, hd)
                torch.cuda.synchronize()
                want = ref[:, shard.n0:shard.n1].cpu()
                if not torch.equal(hd.view(torch.int16), want.contiguous().view(torch.int16)):
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
