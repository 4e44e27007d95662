"""Row-sharded fused GEMM + bias + GELU over one process per GPU, fed from host buffers.

Every rank owns rows `shard_span(M, world, rank)` of A and C; B and bias are needed whole on every GPU.
Instead of every rank copying all of B from host memory over its PCIe link, rank r copies only rows
[r*Kp/world, (r+1)*Kp/world) of B (Kp = K rounded up to a multiple of world) and the slices are
all-gathered over NVLink (NCCL, in place), so each input byte crosses PCIe once per step in total.
Then the kernel runs on the local rows (no collective on the compute path) and the rank's rows of C go
back to host memory.

    ranks = Ranks("nccl")
    run = ShardedHostGemm(ranks, "bf16", None, M, N, K)
    run(hA_rows, hB, hbias, hC_rows)                    # pinned host numpy/torch buffers
"""
from __future__ import annotations

import numpy as np

from . import Context, DEFAULT_TILES, ELEM_BYTES, OUT_BYTES
from .dist import Ranks, shard_span


class ShardedHostGemm:
    def __init__(self, ranks: Ranks, dtype: str, tile, M: int, N: int, K: int, scale_a: float = 1.0,
                 scale_b: float = 1.0):
        import torch

        self.torch = torch
        self.ranks = ranks
        self.dtype = dtype
        self.M, self.N, self.K = M, N, K
        self.scale_a, self.scale_b = scale_a, scale_b
        tile = tuple(tile) if tile else DEFAULT_TILES[dtype]
        self.r0, self.rows = shard_span(M, ranks.world, ranks.rank, tile[0])
        e, o = ELEM_BYTES[dtype], OUT_BYTES[dtype]
        self.kslice = -(-K // ranks.world)                      # rows of B each rank brings in
        dev = torch.device("cuda", ranks.local_rank)
        u8 = torch.uint8
        self.A = torch.empty(max(1, self.rows) * K * e, dtype=u8, device=dev)
        self.Bp = torch.empty(self.kslice * ranks.world * N * e, dtype=u8, device=dev)  # padded K rows
        self.bias = torch.empty(N, dtype=torch.float32, device=dev)
        self.C = torch.empty(max(1, self.rows) * N * o, dtype=u8, device=dev)
        self.ctx = Context(ranks.local_rank)
        if self.rows:
            self.ctx.prepare(dtype, tile, self.rows, N, K)
            self.ctx.bind(self.A, self.Bp, self.bias, self.C, scale_a, scale_b)
        self.e, self.o = e, o

    @staticmethod
    def _bytes(x):
        """A uint8 torch view of a host buffer (numpy array or torch tensor)."""
        import torch
        if isinstance(x, np.ndarray):
            x = torch.from_numpy(np.ascontiguousarray(x))
        return x.reshape(-1).view(torch.uint8)

    def __call__(self, hA_rows, hB, hbias, hC_rows):
        """One step: H2D of this rank's A rows and B slice, NCCL all-gather of B, kernel, D2H of C rows."""
        torch = self.torch
        dist = self.ranks.pg
        stream = torch.cuda.current_stream()
        N, K, e = self.N, self.K, self.e
        rank, world = self.ranks.rank, self.ranks.world
        k0 = min(K, rank * self.kslice)
        k1 = min(K, k0 + self.kslice)
        hb = self._bytes(hB)
        slice_bytes = self.kslice * N * e
        mine = self.Bp[rank * slice_bytes:(rank + 1) * slice_bytes]
        if k1 > k0:
            mine[:(k1 - k0) * N * e].copy_(hb[k0 * N * e:k1 * N * e], non_blocking=True)
        if self.rows:
            self.A.copy_(self._bytes(hA_rows), non_blocking=True)
        self.bias.copy_(self._bytes(hbias).view(torch.float32), non_blocking=True)
        if dist is not None and world > 1:
            dist.all_gather_into_tensor(self.Bp, mine)
        if self.rows:
            self.ctx.launch(stream)
            self._bytes(hC_rows).copy_(self.C[:self.rows * N * self.o], non_blocking=True)
        stream.synchronize()

    def h2d_bytes(self) -> int:
        k0 = min(self.K, self.ranks.rank * self.kslice)
        k1 = min(self.K, k0 + self.kslice)
        return self.rows * self.K * self.e + (k1 - k0) * self.N * self.e + self.N * 4

    def d2h_bytes(self) -> int:
        return self.rows * self.N * self.o

    def close(self):
        self.ctx.close()
