"""Hardware counters for a tuner trace, read with Nsight Compute: counters only, never IR, PTX or SASS.

PTXForge plans CUPTI counters validated against `ncu --metrics ... --csv`, with the tuner parsing the CSV
where counters cannot be read in-process (runtime/cupti_hook.md:12-24).  This module does that for the
sm_100a backend: it takes a trace written by `ptxforge-tune-b200 tune`, re-runs the best trial through the
tuner's own `measure` subcommand (gate launch plus one timed launch), captures the first launch of the
fused kernel with `ncu` and attaches the values to the trace:

    python -m ptxforge_b200.counters --trace runs/trace_b200.json [--exe build/ptxforge-tune-b200]

The metric list is the reference's (occupancy, shared-memory bank conflicts, DRAM bytes, L2 hit rate,
FFMA count) plus the tensor-pipe utilisation and the launch's duration.  From them the trace also gets the
measured arithmetic intensity (FLOPs / DRAM bytes) next to the cost model's, and the DRAM bytes against
the algorithmic A + B + bias + C bytes.

Capture rules kept here: the same command must exit 0 without ncu first; ncu always runs with
`--clock-control none` (the GPU's clocks are never locked); one kernel (`-k`) and one launch (`-c 1`).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import shlex
import subprocess
import sys

METRICS = [
    "gpu__time_duration.sum",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "l1tex__data_bank_conflicts_pipe_lsu_mem_shared_op_ld.sum",
    "l1tex__data_bank_conflicts_pipe_lsu_mem_shared_op_st.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "lts__t_sector_hit_rate.pct",
    "smsp__sass_thread_inst_executed_op_ffma_pred_on.sum",
]

ELEM_BYTES = {"f32": 4, "f32_3xtf32": 4, "bf16": 2, "e4m3": 1}
OUT_BYTES = {"f32": 4, "f32_3xtf32": 4, "bf16": 2, "e4m3": 2}
DTYPE_OF_PEAK = {4.5e6: "e4m3", 2.25e6: "bf16", 375000.0: "f32_3xtf32"}  # b200_gpu()'s peak_gflops


def best_trial(trace: dict) -> dict:
    i = trace.get("best_index")
    if i is None:
        raise ValueError("trace has no passing trial to profile")
    return trace["trials"][i]


def measure_command(exe: str, trace: dict, dtype: str, gpus: int = 1, root: str = ".") -> list[str]:
    """The tuner's `measure` of the trace's best config: gate launch, then one timed launch, no cuBLAS."""
    cfg = best_trial(trace)["cfg"]
    p = trace["problem"]
    cmd = [exe, "measure", "--dtype", dtype, "--gpus", str(gpus), "--root", root,
           "--M", str(p["M"]), "--N", str(p["N"]), "--K", str(p["K"]),
           "--warmup", "0", "--iters", "1", "--reps", "1", "--cublas", "0"]
    for k in ("BM", "BN", "BK", "TM", "TN", "PAD"):
        cmd += [f"--{k}", str(cfg[k])]
    return cmd


def ncu_command(cmd: list[str], csv_path: str, kernel_regex: str = "gemm_bias_gelu", ncu: str = "ncu",
                metrics: list[str] | None = None) -> list[str]:
    """One launch of the fused kernel, the listed metrics, clocks left alone."""
    return [ncu, "--metrics", ",".join(metrics or METRICS), "--clock-control", "none",
            "-k", f"regex:{kernel_regex}", "-c", "1", "--csv", "--log-file", csv_path, *cmd]


def _number(s: str):
    s = s.strip().replace(",", "")
    if s in ("", "n/a", "N/A"):
        return None
    try:
        v = float(s)
    except ValueError:
        return None
    return int(v) if v.is_integer() and "." not in s else v


def parse_csv(text: str) -> dict:
    """ncu's `--csv` output (one row per metric) -> {metric: {"value", "unit"}} of the first launch."""
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    if not lines:
        return {}
    rows = list(csv.DictReader(io.StringIO("\n".join(lines))))
    if not rows:
        return {}
    first = rows[0].get("ID")
    out = {"kernel": rows[0].get("Kernel Name")}
    metrics = {}
    for r in rows:
        if r.get("ID") != first:
            break
        metrics[r["Metric Name"]] = {"value": _number(r.get("Metric Value", "")), "unit": r.get("Metric Unit", "")}
    out["metrics"] = metrics
    return out


def attach(trace: dict, parsed: dict, dtype: str, command: list[str]) -> dict:
    """Put the counters into the trace: top-level `counters` and the best trial's `counters`."""
    p = trace["problem"]
    m = parsed.get("metrics", {})
    val = lambda k: (m.get(k) or {}).get("value")  # noqa: E731
    rd, wr = val("dram__bytes_read.sum"), val("dram__bytes_write.sum")
    flops = float(p["flops"])
    algo = (p["M"] * p["K"] + p["K"] * p["N"]) * ELEM_BYTES[dtype] + p["N"] * 4 + p["M"] * p["N"] * OUT_BYTES[dtype]
    derived = {"algorithmic_bytes": algo}
    if rd is not None and wr is not None and rd + wr > 0:
        derived["dram_bytes"] = rd + wr
        derived["dram_over_algorithmic"] = round((rd + wr) / algo, 3)
        derived["measured_ai"] = round(flops / (rd + wr), 2)
    best = best_trial(trace)
    modeled = best.get("modeled", {}).get("ai")
    if modeled is not None:
        derived["modeled_ai"] = modeled
    block = {"source": "ncu", "kernel": parsed.get("kernel"), "cfg": best["cfg"],
             "command": " ".join(shlex.quote(c) for c in command),
             "metrics": {k: v["value"] for k, v in m.items()},
             "units": {k: v["unit"] for k, v in m.items()}, "derived": derived}
    trace["counters"] = block
    best["counters"] = block["metrics"]
    return trace


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--trace", required=True)
    ap.add_argument("--out", help="where to write the trace with counters (default: in place)")
    ap.add_argument("--exe", default=os.path.join("build", "ptxforge-tune-b200"))
    ap.add_argument("--dtype", help="dtype the trace was tuned for (default: from the trace's GPU peak)")
    ap.add_argument("--root", default=".")
    ap.add_argument("--ncu", default="ncu")
    ap.add_argument("--csv", default=None, help="ncu CSV log path (default: beside --out)")
    a = ap.parse_args(argv)
    with open(a.trace) as f:
        trace = json.load(f)
    dtype = a.dtype or DTYPE_OF_PEAK.get(trace["gpu"].get("peak_gflops"), "f32")
    out = a.out or a.trace
    csv_path = a.csv or os.path.splitext(out)[0] + ".ncu.csv"
    cmd = measure_command(a.exe, trace, dtype, root=a.root)
    plain = subprocess.run(cmd, capture_output=True, text=True)
    if plain.returncode != 0:
        print(f"the measure command failed without ncu (rc {plain.returncode}); not profiling:\n"
              f"{plain.stdout[-2000:]}{plain.stderr[-2000:]}", file=sys.stderr)
        return 2
    prof = subprocess.run(ncu_command(cmd, csv_path, ncu=a.ncu), capture_output=True, text=True)
    if prof.returncode != 0:
        print(f"ncu failed (rc {prof.returncode}):\n{prof.stdout[-2000:]}{prof.stderr[-2000:]}", file=sys.stderr)
        return 3
    with open(csv_path) as f:
        parsed = parse_csv(f.read())
    if not parsed.get("metrics"):
        print(f"no counters in {csv_path}", file=sys.stderr)
        return 4
    attach(trace, parsed, dtype, cmd)
    with open(out, "w") as f:
        json.dump(trace, f, indent=1)
    print(json.dumps(trace["counters"]["derived"]))
    return 0


if __name__ == "__main__":
    sys.exit(main())
