"""One process per GPU: rank plumbing for the row-sharded path (no collective on the data path).

Ranks reads RANK / LOCAL_RANK / WORLD_SIZE (torchrun) and, for more than one rank, joins a process group
used only to line ranks up before and after a timed region and to take the max of per-rank times.  The
data path itself never communicates: rank r owns rows `shard_span(M, world, r)` of A and C.
"""
from __future__ import annotations

import datetime
import os


def shard_span(M: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """(row0, rows) of the M-row problem owned by `rank` (pf_shard_rows of the C ABI)."""
    from . import shard_rows
    return shard_rows(M, world, rank, align)


class Ranks:
    def __init__(self, backend: str = "nccl", timeout_s: int = 180):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist
            kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl":
                import torch
                torch.cuda.set_device(self.local_rank)
                kw["device_id"] = torch.device("cuda", self.local_rank)
            dist.init_process_group(backend, **kw)
            self.pg = dist

    def barrier(self):
        if not self.pg:
            return
        if self.backend == "nccl":
            import torch
            self.pg.barrier(device_ids=[self.local_rank])
            torch.cuda.synchronize()
        else:
            self.pg.barrier()

    def max(self, x: float) -> float:
        """Max of a per-rank scalar over all ranks (timings, error flags)."""
        if not self.pg:
            return x
        import torch
        dev = "cuda" if self.backend == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.barrier()
            self.pg.destroy_process_group()
            self.pg = None
