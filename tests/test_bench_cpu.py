"""bench.py's parts that run without a GPU.

* The reference arm (`--impl reference`): the driver runs it every round, on rank 0 only, and the line it
  prints must carry the contract's keys (impl, metric, value, unit, cpu_baseline, e2e with zero copies,
  gpu_launches 0).  On config 1 (512^3) one step is the whole problem, so the run takes seconds.
* Ranks other than 0 of a torchrun reference arm print nothing and exit 0.
* The L2 note names whether the operands fit in the 126 MB L2.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _bench(args, **env):
    e = dict(os.environ, **env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, cwd=ROOT, env=e)


def test_reference_arm_prints_the_contract_line():
    r = _bench(["--impl", "reference", "--config", "cfg1_f32_512", "--steps", "2", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1 and d["gpu_launches"] == 0
    assert d["config"]["workload"] == "cfg1_f32_512"
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "port" and "rows" in d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # ms_per_step is the measured time of one step's row sample (steps x ms_per_step is the timed region), and
    # the sample is named in config
    rows = d["config"]["rows_sampled"]
    assert 1 <= rows <= 512 and d["ms_per_step"] > 0
    assert abs(d["value"] - 2.0 * rows * 512 * 512 / (d["ms_per_step"] * 1e-3) / 1e12) <= 0.02 * d["value"]
    one = d["cpu_baseline"]["single_thread"]
    assert one["cores"] == 1 and one["value"] > 0 and one["unit"] == "TFLOP/s"


def test_reference_arm_other_ranks_print_nothing():
    r = _bench(["--impl", "reference", "--config", "cfg1_f32_512", "--steps", "1", "--warmup", "0"],
               RANK="1", WORLD_SIZE="2")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [line for line in r.stdout.splitlines() if line.strip().startswith("{")]


def test_l2_note():
    import bench
    from ptxforge_b200 import workloads as wl
    assert "exceed the 126 MB L2" in bench.l2_note(wl.CONFIGS["cfg3_bf16_8192"])
    assert "fit in the 126 MB L2" in bench.l2_note(wl.CONFIGS["cfg1_f32_512"])


def test_energy_and_clocks_print_null_with_a_reason():
    import bench
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.ok, c.samples, c.reasons, c.power, c.max_mhz = True, [], set(), [], 1965
    c.e0 = c.e1 = 1000
    c.t0, c.t1 = 0.0, 2.0
    e = c.energy(20)
    assert e["mj_per_step"] is None and "did not advance" in e["reason"]
    s = c.summary()
    assert s["sm_mhz"] is None and s["samples"] == 0 and "no sample" in s["reason"]
    c.e1 = 3000
    assert c.energy(20)["mj_per_step"] == 100.0
    c.t1 = 0.002  # a 20-step burst of 0.1 ms steps: one counter step would read as kilowatts
    assert c.energy(20)["mj_per_step"] is None and "shorter" in c.energy(20)["reason"]
