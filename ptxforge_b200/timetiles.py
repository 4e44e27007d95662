"""Time tiles (and library builds) of one fused GEMM+bias+GELU shape side by side on one GPU.

    python -m ptxforge_b200.timetiles bf16 8192 8192 8192 --tiles default 256,512,32,3,16,0 [--cublas]
    python -m ptxforge_b200.timetiles f32 2048 2048 2048 --tiles 64,32,16,8,4,0 --libs old/libpf_b200.so new/libpf_b200.so

Every candidate (tile x library) gets the same seeded operands.  The candidates are timed in bursts of `--iters`
back-to-back launches (CUDA events through pf_time, 2 warm-up launches), one burst per candidate in turn with a
short pause between bursts, the order reversed every other round, and the median burst reported: under the
B200's 1 kW cap a long loop settles at a clock set by power, and interleaved bursts keep candidates comparable.
The first launch of each candidate writes its own C; the line reports whether every C is bit-identical to the
first candidate's.  `--cublas` adds cuBLAS's GEMM alone (pf_time_cublas) on the same operands.  `--libs` loads
each library build into this process (each keeps its own context), for comparing builds of the same source
tree at two commits.  Output: one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import ptxforge_b200 as pf


def _operands(dtype: str, M: int, N: int, K: int, seed: int):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    if dtype in ("f32", "f32_3xtf32"):
        A = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1) / K ** 0.5
        B = (torch.rand(K, N, device="cuda", generator=g) * 2 - 1) / K ** 0.5
        out = torch.float32
        scales = (1.0, 1.0)
    elif dtype == "bf16":
        A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
        B = torch.randn(K, N, device="cuda", generator=g).to(torch.bfloat16)
        out = torch.bfloat16
        scales = (1.0, 1.0)
    elif dtype == "e4m3":
        A = torch.randn(M, K, device="cuda", generator=g).to(torch.float8_e4m3fn)
        B = torch.randn(K, N, device="cuda", generator=g).to(torch.float8_e4m3fn)
        out = torch.bfloat16
        scales = (1.0 / 128, 1.0 / 128)
    else:
        raise ValueError(f"unknown dtype {dtype!r}")
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    return A, B, bias, out, scales


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("dtype", choices=["f32", "f32_3xtf32", "bf16", "e4m3"])
    ap.add_argument("M", type=int)
    ap.add_argument("N", type=int)
    ap.add_argument("K", type=int)
    ap.add_argument("--tiles", nargs="+", default=["default"], help="'default' or BM,BN,BK,TM,TN,PAD")
    ap.add_argument("--libs", nargs="+", default=[None], help="libpf_b200.so builds (default: the package's)")
    ap.add_argument("--bursts", type=int, default=12)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--pause", type=float, default=0.08, help="seconds between bursts")
    ap.add_argument("--cublas", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)

    import torch
    M, N, K = args.M, args.N, args.K
    A, B, bias, out, scales = _operands(args.dtype, M, N, K, args.seed)
    cands = []  # (name, ctx, C)
    for lib_path in args.libs:
        lib = pf.load_library(os.path.abspath(lib_path)) if lib_path else pf.load_library()
        for t in args.tiles:
            tile = None if t == "default" else tuple(int(x) for x in t.split(","))
            ctx = pf.Context(0, lib=lib)
            C = torch.empty(M, N, device="cuda", dtype=out)
            ctx.prepare(args.dtype, tile, M, N, K)
            ctx.bind(A, B, bias, C, *scales)
            ctx.launch()
            name = str(ctx.tile.astuple()) + (f" {lib_path}" if lib_path else "")
            cands.append((name, ctx, C))
    torch.cuda.synchronize()
    same = [torch.equal(cands[0][2], c[2]) for c in cands[1:]]
    times = {name: [] for name, _, _ in cands}
    if args.cublas:
        times["cublas_gemm"] = []
    for b in range(args.bursts):
        order = cands if b % 2 == 0 else cands[::-1]
        for name, ctx, _ in order:
            times[name].append(ctx.time(2, args.iters, 1))
            time.sleep(args.pause)
        if args.cublas:
            times["cublas_gemm"].append(cands[0][1].time_cublas(2, args.iters, 1)[0])
            time.sleep(args.pause)
    status = [ctx.status() for _, ctx, _ in cands]
    for _, ctx, _ in cands:
        ctx.close()
    flops = 2.0 * M * N * K
    med = {k: sorted(v)[len(v) // 2] for k, v in times.items()}
    line = {"shape": f"{args.dtype} {M}x{N}x{K}", "bursts": args.bursts, "iters": args.iters,
            "same_bits_as_first": same, "status": status,
            "us_median": {k: round(v * 1e3, 2) for k, v in med.items()},
            "us_min": {k: round(min(v) * 1e3, 2) for k, v in times.items()},
            "tflops_median": {k: round(flops / (v * 1e-3) / 1e12, 1) for k, v in med.items()}}
    print(json.dumps(line), flush=True)
    return line


if __name__ == "__main__":
    main()
