"""The N>1 host path on the CPU: world-size-2 gloo ranks (no GPU).

Each rank takes its rows with ptxforge_b200.dist.shard_span (pf_shard_rows of the C ABI), computes them --
here with the oracle, standing in for the GPU kernel on a machine without one -- and the ranks check that
the shards tile the problem exactly once and that the max-over-ranks reduction used for timing returns
the slowest rank's value.  The data path has no collective; only the test gathers the shards to compare.
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, M, N, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    try:
        import torch.distributed as dist

        import oracle
        from ptxforge_b200 import workloads as wl
        from ptxforge_b200.dist import Ranks, shard_span

        r = Ranks("gloo", timeout_s=60)
        w = wl.scaled(wl.CONFIGS["cfg1_f32_512"], M, N, K)
        inp = wl.make_inputs(w, seed=4)
        r0, rows = shard_span(M, r.world, r.rank, 64)
        C = np.full((M, N), np.nan, dtype=np.float32)
        if rows:
            oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=r0, rows=rows, threads=1, out=C)
        r.barrier()
        slowest = r.max(float(10 + r.rank))
        spans = [None] * r.world
        dist.all_gather_object(spans, (r0, rows, C[r0:r0 + rows].copy()))
        r.close()
        if rank == 0:
            full = oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, threads=1)
            pos, parts = 0, []
            for s0, n, part in spans:
                assert s0 == pos
                pos += n
                parts.append(part)
            assert pos == M
            assert np.array_equal(np.concatenate(parts), full)
            assert slowest == 10.0 + world - 1
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.parametrize("M", [256, 200])
def test_two_gloo_ranks_tile_the_rows(M):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, M, 96, 80, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def _gather_main(rank, world, port, M, N, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    try:
        import torch

        import oracle
        from ptxforge_b200 import workloads as wl
        from ptxforge_b200.dist import Ranks, shard_span
        from ptxforge_b200.sharded import RowGather

        r = Ranks("gloo", timeout_s=60)
        w = wl.scaled(wl.CONFIGS["cfg1_f32_512"], M, N, K)
        inp = wl.make_inputs(w, seed=5)
        r0, rows = shard_span(M, r.world, r.rank, 64)
        C = np.full((M, N), np.nan, dtype=np.float32)
        if rows:
            oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=r0, rows=rows, threads=1, out=C)
        g = RowGather(r, M, N, 4, 64, device="cpu")
        block = torch.from_numpy(np.ascontiguousarray(C[r0:r0 + max(rows, 1)]))
        full = g(block).full().view(torch.float32).numpy()
        expect_bytes = (M - rows) * N * 4
        r.close()
        ref = oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, threads=1)
        assert full.shape == (M, N), full.shape
        assert np.array_equal(full, ref)
        assert g.bytes_per_rank() == expect_bytes
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,M", [(2, 256), (2, 200), (3, 200)])
def test_row_gather_assembles_c_on_every_rank(world, M):
    """The optional C all-gather (RowGather): every rank ends with the whole result, equal or ragged shards."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_main, args=(r, world, port, M, 96, 80, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}, results
