#!/usr/bin/env python3
"""Benchmark of the fused C = GELU_tanh(A.B + bias) hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3_bf16_8192] [--impl ours|reference]

Metric: TFLOP/s of fused GEMM+bias+GELU, bf16 8192^3, at 1/2/4/8 GPUs.  One step is one
launch of the fused kernel over the whole problem; with N GPUs (one process each, launched by torchrun)
rows of M are split across the ranks (B and bias replicated, no collective on the data path) and the
step time is the max over ranks of each rank's CUDA-event time (strong scaling: the 8192^3 problem is
fixed).  FLOPs are 2*M*N*K (the epilogue is not counted, as in the reference, space.hpp:55).
`--shard-of G` times, on one GPU, the row shard that rank 0 of a G-GPU run gets (value = that GPU's
TFLOP/s): the per-GPU half of a scaling measurement at 1/G of its GPU time.

Besides the device-timed `value`, the line carries
  e2e           the same metric end to end from pinned host buffers, every step: at N=1 the C ABI's
                pf_run_host (H2D of A, B, bias, the kernel, D2H of C, overlapped in row chunks); at N>1
                ptxforge_b200.sharded.ShardedHostGemm (each rank copies 1/N of B, B is all-gathered over
                NVLink, then its A rows in / kernel / C rows out overlap in row chunks, pf_run_host_rows)
  roofline      achieved TFLOP/s of the kernel over the measured dense bf16 peak
  comparators   cuBLAS GEMM alone and cuBLAS + a separate bias+GELU pass (pf_time_cublas), same inputs
  cpu_baseline  the CPU-lowered schedule (oracle port) on the host cores, on a bounded sample (N=1)
  clocks        SM clock and throttle reasons sampled (NVML) during the timed region
  energy        this GPU's energy per step over the timed region (NVML total-energy counter): under the
                ~1 kW power cap the clock, and so the throughput, follows energy per launch
`--impl reference` times the reference's CPU implementation of the path (the port of its CPU-lowered
schedule, all host threads) on the same workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "TFLOP/s fused GEMM+bias+GELU bf16 8192³, % B200 dense peak, at 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
PEAK_NOTE = {"bf16": "bf16_tflops", "e4m3": "bf16_tflops x 2, the fp8 rate",
             "f32_3xtf32": "bf16_tflops / 2 (the tf32 rate) / 3 (tf32 products per fp32 product)",
             "f32": "SIMT FFMA nominal, 148 SMs x 128 lanes x 2 x 1.965 GHz"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--config", default="cfg3_bf16_8192")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tile", default=None,
                    help="BM,BN,BK,TM,TN,PAD (default: ptxforge_b200.default_tile, the best measured for the shape)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparators", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU-baseline sample budget")
    ap.add_argument("--shard-of", type=int, default=0, metavar="G",
                    help="on one GPU, time rank 0's row shard of a G-GPU run instead of the whole problem "
                         "(a development measurement: value is then that one GPU's TFLOP/s)")
    return ap.parse_args()


def l2_note(w) -> str:
    """How the timed steps stand to the 126 MB L2 (no flush between steps either way)."""
    mb = w.algorithmic_bytes() / 1e6
    if mb > 126:
        return f"no flush: A+B+C ({mb:.0f} MB) exceed the 126 MB L2"
    return (f"no flush: A+B+C ({mb:.1f} MB) fit in the 126 MB L2, so steps re-read cached operands, as back-to-back "
            "launches of the reference protocol (median_ms) do")


def host_threads() -> int:
    """Every host core this process may run on (torchrun sets OMP_NUM_THREADS=1; the CPU legs ignore it)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------------------------------------
# clocks during the timed region (NVML, read only)
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device: int, interval: float = 0.002):
        self.samples = []
        self.reasons = set()
        self.power = []
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = None
            try:  # match the CUDA device to its NVML handle by UUID
                import torch
                uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
                if uuid is not None:
                    self.h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(uuid))
            except Exception:
                self.h = None
            if self.h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[device]) if vis else device
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report null clocks
            self.err = str(e)
        self.interval = interval
        self._stop = threading.Event()

    def _run(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = get_reasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
                self.power.append(nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0)
            except Exception:
                pass
            time.sleep(self.interval)

    def _energy(self):
        try:
            return self.nv.nvmlDeviceGetTotalEnergyConsumption(self.h)  # mJ since the driver loaded
        except Exception:
            return None

    def __enter__(self):
        self.e0 = self.e1 = None
        self.t0 = self.t1 = time.perf_counter()
        if self.ok:
            self.e0 = self._energy()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self.t1 = time.perf_counter()
        if self.ok:
            self._stop.set()
            self.t.join()
            self.e1 = self._energy()

    def energy(self, steps: int):
        """Energy of this GPU per step over the timed region (NVML's total-energy counter), or null with the
        reason: the counter advances in coarse steps (tens of milliseconds), so over a region shorter than half
        a second it reads zero or one step's worth -- neither is the region's energy."""
        src = "nvml total energy counter, this rank's GPU, over the timed region"
        if self.e0 is None or self.e1 is None or steps <= 0:
            return {"mj_per_step": None, "source": src, "reason": "counter unavailable"}
        if self.t1 - self.t0 < 0.5:
            return {"mj_per_step": None, "source": src,
                    "reason": f"timed region of {1e3 * (self.t1 - self.t0):.1f} ms is shorter than the counter's "
                              "resolution allows (>= 500 ms)"}
        if self.e1 <= self.e0:
            return {"mj_per_step": None, "source": src, "reason": "the counter did not advance during the timed region"}
        return {"mj_per_step": round((self.e1 - self.e0) / steps, 1), "source": src}

    def summary(self):
        if not self.ok or not self.samples:
            why = "NVML unavailable" if not self.ok else "no sample fell inside the timed region"
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0,
                    "source": "nvml", "reason": why}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples),
                "power_w_max": round(max(self.power), 1) if self.power else None, "source": "nvml",
                "note": "NVML reports the SM clock the driver targets; under heavy tensor load the effective "
                        "clock (ncu: sm__cycles_elapsed / duration) can be lower without a throttle reason"}


# ------------------------------------------------------------------------------------------------
# distributed plumbing (one process per GPU; no collective on the data path): ptxforge_b200.dist
# ------------------------------------------------------------------------------------------------
def Dist(n_gpus: int):
    from ptxforge_b200.dist import Ranks
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    return Ranks("nccl")


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def device_operands(torch, w, inp, r0, rows):
    dt = {"f32": torch.float32, "f32_3xtf32": torch.float32, "bf16": torch.bfloat16,
          "e4m3": torch.float8_e4m3fn}[w.dtype]
    out_dt = torch.float32 if w.dtype in ("f32", "f32_3xtf32") else torch.bfloat16

    def dev(x):
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        if w.dtype == "bf16":
            t = t.view(torch.int16).view(torch.bfloat16)
        elif w.dtype == "e4m3":
            t = t.view(torch.float8_e4m3fn)
        return t

    A = dev(inp.A_raw[r0:r0 + rows])
    B = dev(inp.B_raw)
    bias = torch.from_numpy(inp.bias).cuda()
    C = torch.empty((rows, w.N), dtype=out_dt, device="cuda")
    assert A.dtype == dt
    return A, B, bias, C


def gate_sampled(torch, A, B, bias, C, scale, tol, n=256, seed=1234):
    """Correctness before speed (the reference gates every trial before timing it,
    core/src/cuda_runner.cpp:185-203): fp64 on the GPU at n random outputs."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    rows = torch.randint(0, A.shape[0], (n,), generator=g).cuda()
    cols = torch.randint(0, B.shape[1], (n,), generator=g).cuda()
    def pick(t, dim, idx):  # index_select has no fp8 kernel: gather the byte codes
        if t.dtype == torch.float8_e4m3fn:
            return t.view(torch.uint8).index_select(dim, idx).view(t.dtype).float().double()
        return t.index_select(dim, idx).double()

    a = pick(A, 0, rows)
    b = pick(B, 1, cols).t()
    x = (a * b).sum(1) * scale + bias.index_select(0, cols).double()
    ref = 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))
    got = C[rows, cols].double()
    err = float(((ref - got).abs() / (1.0 + ref.abs())).max())
    return err, err <= tol


def schedule_rows(w, inp, threads: int, seconds: float, out, row0: int = 0):
    """Time the oracle port of the CPU-lowered schedule on as many rows as fit `seconds` (calibrated on a few
    rows first); returns (rows, seconds taken)."""
    import oracle
    cal = min(w.M, 8 if threads > 1 else 2)
    t0 = time.perf_counter()
    oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=0, rows=cal, threads=threads, out=out)
    per_row = max(time.perf_counter() - t0, 1e-5) / cal
    rows = int(max(1, min(w.M - row0, seconds / per_row)))
    t0 = time.perf_counter()
    oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=row0, rows=rows, threads=threads, out=out)
    return rows, time.perf_counter() - t0


def cpu_baseline_sample(w, inp, seconds: float):
    """Time the oracle port of the CPU-lowered schedule on a bounded row sample: every host thread (the
    headline figure) and one thread (the reference's own lowering runs serially, scf.for,
    tests/check_lowering_cpu.py:94)."""
    threads = host_threads()
    out = np.empty((w.M, w.N), dtype=np.float32)
    rows, dt = schedule_rows(w, inp, threads, seconds, out)
    flops = 2.0 * rows * w.N * w.K
    rows1, dt1 = schedule_rows(w, inp, 1, max(2.0, seconds / 3), out)
    flops1 = 2.0 * rows1 * w.N * w.K
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"rows 0..{rows} of the {w.M}x{w.N}x{w.K} problem ({flops / 1e9:.1f} GFLOP, {dt:.1f} s): "
                      f"oracle port of the reference's CPU-lowered schedule (fp32, 64x64x16 tiles) on the "
                      f"dequantised {w.dtype} inputs, gcc -O3, OpenMP {threads} threads",
            "single_thread": {"value": flops1 / dt1 / 1e12, "unit": "TFLOP/s", "cores": 1,
                              "sample": f"rows 0..{rows1} ({flops1 / 1e9:.1f} GFLOP, {dt1:.1f} s), one thread: the "
                                        "reference's lowering runs serially"}}


def run_ours(args, dist):
    import torch

    import ptxforge_b200 as pf
    from ptxforge_b200 import workloads as wl

    w = wl.CONFIGS[args.config]
    torch.cuda.set_device(dist.local_rank)
    inp = wl.make_inputs(w)
    if args.shard_of and dist.world != 1:
        raise SystemExit("--shard-of times one shard on one GPU: run it without torchrun")
    shards = args.shard_of if args.shard_of else dist.world
    r0, rows = pf.shard_rows(w.M, shards, dist.rank, 128)
    A, B, bias, C = device_operands(torch, w, inp, r0, rows)
    scale = inp.scale_a * inp.scale_b
    tile = tuple(int(x) for x in args.tile.split(",")) if args.tile else pf.default_tile(w.dtype, rows, w.N, w.K)
    ctx = pf.Context(dist.local_rank)
    ctx.prepare(w.dtype, tile, rows, w.N, w.K)
    ctx.bind(A, B, bias, C, inp.scale_a, inp.scale_b)
    stream = torch.cuda.current_stream()

    # correctness gate first
    ctx.launch(stream)
    torch.cuda.synchronize()
    if ctx.status() != 0:
        raise SystemExit("device status nonzero after the gate launch")
    gate_err, gate_ok = gate_sampled(torch, A, B, bias, C, scale, w.tolerance)
    if not dist.max(0.0 if gate_ok else 1.0) == 0.0:
        raise SystemExit(f"correctness gate failed on some rank (rank {dist.rank}: max err {gate_err:.3e})")

    for _ in range(args.warmup):
        ctx.launch(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dist.local_rank) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            ctx.launch(stream)
        ev1.record(stream)
        while not ev1.query():  # poll with the GIL released so the clock sampler keeps sampling
            time.sleep(0.0005)
        torch.cuda.synchronize()
    dist.barrier()
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = dist.max(ms_local)
    status = ctx.status()
    if dist.max(float(status)) != 0.0:
        raise SystemExit(f"device status 0x{status:x} after the timed region")

    # end to end through the C ABI with host buffers (pinned), copies inside the timed region
    pin = {}
    for name, arr in (("A", inp.A_raw[r0:r0 + rows]), ("B", inp.B_raw), ("bias", inp.bias)):
        t = torch.empty(arr.shape, dtype={1: torch.uint8, 2: torch.int16, 4: torch.float32}[arr.itemsize],
                        pin_memory=True)
        t.numpy().view(arr.dtype)[...] = arr
        pin[name] = t
    out_bytes = 4 if w.dtype in ("f32", "f32_3xtf32") else 2
    hC = torch.empty((rows, w.N), dtype=torch.float32 if out_bytes == 4 else torch.int16, pin_memory=True)
    if dist.world == 1:
        # one GPU: pf_run_host (C ABI), row chunks whose copies and kernels overlap
        ctx_e2e = pf.Context(dist.local_rank)
        ctx_e2e.prepare(w.dtype, tile, rows, w.N, w.K)
        step = lambda: ctx_e2e.run_host(pin["A"], pin["B"], pin["bias"], hC, inp.scale_a, inp.scale_b)  # noqa: E731
        e2e_api = "pf_run_host (C ABI): pinned host buffers, row-chunked H2D / kernel / D2H overlap"
        h2d = pin["A"].numel() * pin["A"].element_size() + pin["B"].numel() * pin["B"].element_size() + \
            pin["bias"].numel() * 4
        d2h = hC.numel() * hC.element_size()
    else:
        # N GPUs: each rank brings in its rows of A and 1/N of B over its own PCIe link; B is all-gathered
        # over NVLink (NCCL); kernel on the local rows; C rows back (ptxforge_b200.sharded)
        from ptxforge_b200.sharded import ShardedHostGemm
        ctx_e2e = ShardedHostGemm(dist, w.dtype, tile, w.M, w.N, w.K, inp.scale_a, inp.scale_b)
        step = lambda: ctx_e2e(pin["A"], pin["B"], pin["bias"], hC)  # noqa: E731
        e2e_api = ("ShardedHostGemm: pinned host buffers, per-rank H2D of 1/N of B, NCCL all-gather of B over "
                   "NVLink, then its A rows in / kernel / C rows out in overlapping row chunks (pf_run_host_rows)")
        h2d, d2h = ctx_e2e.h2d_bytes(), ctx_e2e.d2h_bytes()
    step()  # warm: allocations, first-use set-up
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        step()
    e2e_ms = dist.max((time.perf_counter() - t0) * 1e3 / args.e2e_steps)
    e2e_same = dist.max(0.0 if np.array_equal(hC.numpy().view(np.uint8), C.view(torch.uint8).cpu().numpy().reshape(
        hC.numpy().view(np.uint8).shape)) else 1.0) == 0.0
    # Bitwise equality holds whenever the device launch sums every tile whole; a launch with a stream-K tail
    # splits its last tiles' k range, so the (chunked, whole-tile) host path then differs in rounding only.
    got = (hC.view(C.dtype) if C.dtype != torch.float32 else hC).to(C.device).float()
    ref = C.float()
    e2e_diff = dist.max(float(((got - ref).abs() / (1.0 + ref.abs())).max()) if ref.numel() else 0.0)
    del got, ref
    ctx_e2e.close()

    # optional all-gather of C's row shards (every rank ends with all of C), timed on its own and kept out
    # of `value`: NCCL all_gather_into_tensor over NVLink
    c_gather = None
    if dist.world > 1:
        from ptxforge_b200.sharded import RowGather
        gat = RowGather(dist, w.M, w.N, out_bytes, tile[0])
        gat(C)
        torch.cuda.synchronize()

        def checksum(block):
            b = block.reshape(-1).view(torch.uint8).to(torch.int64)
            return float((b * (torch.arange(b.numel(), device=b.device) % 65521 + 1)).sum().item())

        row_bytes = w.N * out_bytes
        full = gat.full()
        mine = checksum(C.reshape(-1).view(torch.uint8)[:rows * row_bytes])
        sums = torch.zeros(dist.world, dtype=torch.float64, device=C.device)
        sums[dist.rank] = mine
        dist.pg.all_reduce(sums)  # each rank's checksum of its own rows, everywhere
        got = [checksum(full[s0:s0 + n]) for s0, n in gat.spans]
        gather_ok = dist.max(0.0 if got == sums.tolist() else 1.0) == 0.0
        n_g = 20
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        g0.record()
        for _ in range(n_g):
            gat(C)
        g1.record()
        g1.synchronize()
        g_ms = dist.max(g0.elapsed_time(g1) / n_g)
        c_bytes = w.M * w.N * out_bytes
        c_gather = {"ms": round(g_ms, 4), "bytes_total": c_bytes, "bytes_received_per_rank": gat.bytes_per_rank(),
                    "algbw_GBps": round(c_bytes / (g_ms * 1e-3) / 1e9, 1),
                    "busbw_GBps": round(c_bytes * (dist.world - 1) / dist.world / (g_ms * 1e-3) / 1e9, 1),
                    "op": "NCCL all_gather_into_tensor of each rank's C rows (ptxforge_b200.sharded.RowGather), "
                          "after the kernel, outside the timed region of `value`",
                    "matches_shards": gather_ok}
        del gat, full

    attrs = ctx.attrs()
    comp = None
    if not args.no_comparators and dist.world == 1:
        # the library's cuBLAS comparator (pf_time_cublas) with as many launches as the timed region
        g_ms, u_ms = ctx.time_cublas(warmup=5, iters=max(20, args.steps // 5), reps=5)
        comp = {"cublas_gemm_only": g_ms, "cublas_plus_separate_bias_gelu": u_ms}

    res = None
    if dist.rank == 0:
        pk, pk_kind = peaks()
        total_flops = w.flops if not args.shard_of else 2.0 * rows * w.N * w.K
        value = total_flops / (ms * 1e-3) / 1e12
        per_gpu_flops = 2.0 * rows * w.N * w.K
        achieved = per_gpu_flops / (ms_local * 1e-3) / 1e12
        peak_key = {"bf16": "bf16_tflops", "e4m3": "bf16_tflops", "f32_3xtf32": "bf16_tflops", "f32": None}[w.dtype]
        peak = pk.get(peak_key) if peak_key else None
        if w.dtype == "e4m3" and peak:
            peak = 2.0 * peak  # fp8 dense rate is twice bf16 on the same tensor cores
        if w.dtype == "f32_3xtf32" and peak:
            peak = peak / 2.0 / 3.0  # tf32 runs at half the bf16 rate; three tf32 products per fp32 product
        if w.dtype == "f32":
            peak = 148 * 128 * 2 * 1.965e9 / 1e12  # SIMT FFMA peak at max SM clock
        # the same scaled from the sustained (seconds-long, power-capped) cuBLAS figure: the regime of a long
        # timed loop that ran under sw_power_cap
        peak_sus = pk.get("bf16_tflops_sustained") if peak_key else None
        if peak_sus and w.dtype == "e4m3":
            peak_sus *= 2.0
        if peak_sus and w.dtype == "f32_3xtf32":
            peak_sus /= 6.0
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get(f"{w.name}@{shards}")
        res = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic (seeded, BASELINE "
            "distributions)",
            "config": {"workload": w.name, "M": w.M, "N": w.N, "K": w.K, "rows_per_gpu": rows,
                       **({"shard_of": args.shard_of} if args.shard_of else {}),
                       "tile": list(tile), "parallelism": f"M-rows x{dist.world}, B+bias replicated, no "
                       "collective", "l2": l2_note(w),
                       "global_batch": w.M, "seq_len": None},
            "pct_of_peak": round(100.0 * value / (peak * dist.world), 2) if peak else None,
            "roofline": {"bound": "tensor" if w.dtype != "f32" else "fp32-simt", "achieved": round(achieved, 2),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4) if peak else None,
                         "peak_source": f"{pk_kind} ({PEAK_NOTE[w.dtype]}; burst, kernel timed alone)",
                         "peak_sustained": round(peak_sus, 1) if peak_sus else None,
                         "frac_sustained": round(achieved / peak_sus, 4) if peak_sus else None,
                         "traffic": traffic,
                         "algorithmic_bytes": w.algorithmic_bytes()},
            "e2e": {"value": round(total_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "api": e2e_api,
                    "matches_device_result": e2e_same, "max_rel_diff_vs_device": e2e_diff,
                    "within_tolerance_of_device": e2e_diff <= w.tolerance},
            "gpu_launches": args.steps,
            "gate": {"max_rel_err": gate_err, "tolerance": w.tolerance, "samples": 256},
            "clocks": clk.summary(),
            "energy": clk.energy(args.steps),
            "kernel": {"attrs": attrs},
        }
        if c_gather:
            res["c_allgather"] = c_gather
        if comp:
            res["comparators"] ={k: {"ms": round(v, 4), "tflops": round(total_flops / (v * 1e-3) / 1e12, 2)}
                                  for k, v in comp.items()}
        if dist.world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_sample(w, inp, args.cpu_seconds)
    ctx.close()
    return res


# ------------------------------------------------------------------------------------------------
# reference arm: the reference's CPU implementation of the path (port of its CPU-lowered schedule)
# ------------------------------------------------------------------------------------------------
def run_reference(args, dist):
    """Each step runs the schedule port on every host thread over a bounded sample of rows (the same rows'
    share of the whole problem's work), sized so warm-up plus timed steps take about two minutes; `value` is
    that sample's TFLOP/s and `ms_per_step` its measured time, so steps x ms_per_step is the timed region.
    A one-thread figure of the same schedule (the reference runs its lowering serially) is measured once,
    outside the steps."""
    if dist.rank != 0:
        return None
    import oracle
    from ptxforge_b200 import workloads as wl

    w = wl.CONFIGS[args.config]
    inp = wl.make_inputs(w)
    threads = host_threads()
    out = np.empty((w.M, w.N), dtype=np.float32)
    cal = min(w.M, 8)
    t0 = time.perf_counter()
    oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=0, rows=cal, threads=threads, out=out)
    per_row = max(time.perf_counter() - t0, 1e-5) / cal
    budget = 120.0
    rows = int(max(1, min(w.M, budget / (args.steps + args.warmup) / per_row)))
    for i in range(args.warmup):
        oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=0, rows=rows, threads=threads, out=out)
    times = []
    for i in range(args.steps):
        r0 = (i * rows) % max(1, w.M - rows + 1)
        t0 = time.perf_counter()
        oracle.cpu_schedule(inp.A, inp.B, inp.bias, 64, 64, 16, row0=r0, rows=rows, threads=threads, out=out)
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    flops_step = 2.0 * rows * w.N * w.K
    value = flops_step / dt / 1e12
    rows1, dt1 = schedule_rows(w, inp, 1, 8.0, out)
    value1 = 2.0 * rows1 * w.N * w.K / dt1 / 1e12
    sample = (f"{rows} rows of the {w.M}x{w.N}x{w.K} problem per step ({flops_step / 1e9:.2f} GFLOP, "
              f"{rows / w.M:.4f} of the whole problem's work): port of the reference's CPU-lowered schedule (fp32 FMA, "
              "k ascending, 64x64x16 tiles; MLIR/LLVM 19 absent so its own lowering cannot be built) on dequantised "
              f"inputs, OpenMP {threads} threads")
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": w.name, "M": w.M, "N": w.N, "K": w.K, "rows_sampled": rows,
                   "sampled": f"each step computes {rows} of the {w.M} rows of C (all {w.N} columns, full K); "
                              "value = that sample's FLOPs / its time; the CPU cost is linear in rows",
                   "parallelism": f"host cores (OpenMP, {threads} threads)"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample,
                         "single_thread": {"value": round(value1, 6), "unit": "TFLOP/s", "cores": 1,
                                           "sample": f"rows 0..{rows1} ({2.0 * rows1 * w.N * w.K / 1e9:.2f} GFLOP, "
                                                     f"{dt1:.1f} s), one thread, measured once after the steps: the "
                                                     "reference's lowering runs serially"}},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def main():
    args = parse_args()
    dist = Dist(args.gpus) if args.impl == "ours" else None
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))

        class _D:
            pass
        dist = _D()
        dist.world, dist.rank = world, rank
        res = run_reference(args, dist)
        if res:
            print(json.dumps(res), flush=True)
        return 0
    try:
        res = run_ours(args, dist)
    finally:
        dist.close()
    if res:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
