"""Row-sharded fused GEMM + bias + GELU over one process per GPU, fed from host buffers.

Every rank owns rows `shard_span(M, world, rank)` of A and C; B and bias are needed whole on every GPU.
Instead of every rank copying all of B from host memory over its PCIe link, rank r copies only rows
[r*Kp/world, (r+1)*Kp/world) of B (Kp = K rounded up to a multiple of world) and the slices are
all-gathered over NVLink (NCCL, in place), so each input byte crosses PCIe once per step in total.
Then the rank's rows of A go in, the kernel runs on them and its rows of C come back in overlapping row
chunks (pf_run_host_rows: H2D of A, kernels and D2H of C pipelined; no collective on the compute path).
RowGather is the optional, separately timed all-gather of C's row shards for consumers that need the whole
result on every GPU.

    ranks = Ranks("nccl")
    run = ShardedHostGemm(ranks, "bf16", None, M, N, K)
    run(hA_rows, hB, hbias, hC_rows)                    # pinned host numpy/torch buffers
    whole_c = RowGather(ranks, M, N, 2, 256)(c_rows_on_device).full()
"""
from __future__ import annotations

import numpy as np

from . import Context, DEFAULT_TILES, ELEM_BYTES, OUT_BYTES, default_tile
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
        self.r0, self.rows = shard_span(M, ranks.world, ranks.rank, tuple(tile or DEFAULT_TILES[dtype])[0])
        tile = tuple(tile) if tile else default_tile(dtype, self.rows, N, K)
        e, o = ELEM_BYTES[dtype], OUT_BYTES[dtype]
        self.kslice = -(-K // ranks.world)                      # rows of B each rank brings in
        dev = torch.device("cuda", ranks.local_rank)
        u8 = torch.uint8
        self.A = torch.empty(max(1, self.rows) * K * e, dtype=u8, device=dev)
        self.Bp = torch.empty(self.kslice * ranks.world * N * e, dtype=u8, device=dev)  # padded K rows
        self.bias = torch.empty(N, dtype=torch.float32, device=dev)
        self.C = torch.empty(max(1, self.rows) * N * o, dtype=u8, device=dev)
        self.copy_stream = torch.cuda.Stream(device=dev)          # host -> device copy of B's slice
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
        """One step: H2D of this rank's B slice, NCCL all-gather of B, then its A rows in / kernel / C rows
        out, pipelined in row chunks.  The host link carries B's slice first and A's rows right after it,
        while the all-gather runs over NVLink; the kernels wait for the gather."""
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
        self.copy_stream.wait_stream(stream)
        with torch.cuda.stream(self.copy_stream):
            if k1 > k0:
                mine[:(k1 - k0) * N * e].copy_(hb[k0 * N * e:k1 * N * e], non_blocking=True)
            self.bias.copy_(self._bytes(hbias).view(torch.float32), non_blocking=True)
        stream.wait_stream(self.copy_stream)
        if dist is not None and world > 1:
            dist.all_gather_into_tensor(self.Bp, mine)
        if self.rows:
            self.ctx.run_host_rows(self._bytes(hA_rows), self._bytes(hC_rows), after_stream=stream,
                                   copies_after_stream=self.copy_stream)
        stream.synchronize()

    def h2d_bytes(self) -> int:
        k0 = min(self.K, self.ranks.rank * self.kslice)
        k1 = min(self.K, k0 + self.kslice)
        return self.rows * self.K * self.e + (k1 - k0) * self.N * self.e + self.N * 4

    def d2h_bytes(self) -> int:
        return self.rows * self.N * self.o

    def close(self):
        self.ctx.close()


class RowGather:
    """Optional all-gather of C's row shards, so that every rank holds the whole M x N result.

    The compute path has no collective; a consumer that needs all of C on one GPU calls this after the
    kernel, as a separate, separately timed step.  Every rank contributes the `rows` x N block it owns
    (`shard_span(M, world, rank, align)`).  When all shards have the same height the gathered buffer
    already is C, row-major; otherwise each rank's block sits in a slot of the tallest shard's height and
    `full()` packs the blocks together.  NCCL (`all_gather_into_tensor`, over NVLink on one box) for GPU
    tensors; the list form of all_gather for gloo ranks on the CPU.
    """

    def __init__(self, ranks: Ranks, M: int, N: int, out_bytes: int, align: int, device=None):
        import torch

        self.torch = torch
        self.ranks = ranks
        self.N, self.o = N, out_bytes
        self.spans = [shard_span(M, ranks.world, r, align) for r in range(ranks.world)]
        self.slot_rows = max(1, max(n for _, n in self.spans))
        self.equal = all(n == self.slot_rows for _, n in self.spans)
        self.slot_bytes = self.slot_rows * N * out_bytes
        dev = device if device is not None else torch.device("cuda", ranks.local_rank)
        self.buf = torch.empty(ranks.world * self.slot_bytes, dtype=torch.uint8, device=dev)
        self.send = None if self.equal else torch.zeros(self.slot_bytes, dtype=torch.uint8, device=dev)

    def bytes_per_rank(self) -> int:
        """Bytes of C each rank receives from the others in one gather."""
        me = self.ranks.rank
        return sum(n for r, (_, n) in enumerate(self.spans) if r != me) * self.N * self.o

    def __call__(self, c_rows):
        """Gather: `c_rows` is this rank's rows x N block of C (any dtype, contiguous, on the device)."""
        torch = self.torch
        mine = c_rows.reshape(-1).view(torch.uint8)
        rows = self.spans[self.ranks.rank][1]
        if mine.numel() < rows * self.N * self.o:
            raise ValueError("c_rows holds fewer bytes than this rank's shard of C")
        src = mine[:self.slot_bytes] if self.equal else self.send
        if not self.equal:
            src[:rows * self.N * self.o].copy_(mine[:rows * self.N * self.o])
        pg = self.ranks.pg
        if pg is None or self.ranks.world == 1:
            self.buf.copy_(src)
        elif self.ranks.backend == "nccl":
            pg.all_gather_into_tensor(self.buf, src)
        else:
            pg.all_gather(list(self.buf.split(self.slot_bytes)), src)
        return self

    def full(self):
        """The gathered C as M x N * out_bytes uint8 rows (a view when all shards have the same height)."""
        torch = self.torch
        row = self.N * self.o
        if self.equal:
            return self.buf.view(-1, row)
        parts = [self.buf[r * self.slot_bytes:r * self.slot_bytes + n * row].view(-1, row)
                 for r, (_, n) in enumerate(self.spans) if n]
        return torch.cat(parts)
