"""B200Runner and PTXForge's tuner, on a fake libpf_b200 (CPU only).

The C++ runner (include/ptxforge_b200/b200_runner.hpp) and the tuner CLI (ptxforge_b200/host/tune_b200.cpp)
are compiled against PTXForge's own headers and linked to tests/fake_pf/fake_pf.c, a CPU implementation of
the C ABI -- the reference's fake-driver pattern (tests/fake_cuda/run.sh) moved to this backend's boundary.
Checked: the correctness gate, M-row sharding over several devices, the trace contract of tune(), and
failure handling (refused tiles, wrong results, launch failure, out of memory, a device-side timeout on one
shard, a device that does not open) -- every failure is a failed trial with a message, never a crash.
Needs the PTXForge headers at build time (skipped where they are absent).
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from ptxforge_b200 import build as pbuild  # noqa: E402

HAVE_REF = os.path.isdir(os.path.join(pbuild.REF_ROOT, "core", "include", "ptxforge"))
pytestmark = pytest.mark.skipif(not HAVE_REF, reason="PTXForge headers not available")


@pytest.fixture(scope="module")
def tune_fake(tmp_path_factory):
    d = tmp_path_factory.mktemp("fake_pf")
    lib = d / "libpf_b200.so"
    subprocess.run(["gcc", "-std=c11", "-O1", "-fPIC", "-shared", "-Wall", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "fake_pf", "fake_pf.c"), "-o", str(lib), "-lm"], check=True)
    exe = d / "ptxforge-tune-b200"
    r = subprocess.run(pbuild.tune_command(str(exe), str(d), str(d)), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return str(exe), d


def run(tune_fake, args, **env):
    exe, d = tune_fake
    e = dict(os.environ)
    e.update({k: str(v) for k, v in env.items()})
    return subprocess.run([exe, *args], capture_output=True, text=True, env=e, cwd=str(d), timeout=120)


SMALL = ["--M", "256", "--N", "256", "--K", "128"]
GOOD = ["--BM", "128", "--BN", "256", "--BK", "32", "--TM", "4", "--TN", "16", "--PAD", "0"]


def measure(tune_fake, extra, **env):
    r = run(tune_fake, ["measure", "--dtype", "bf16", *SMALL, *extra], **env)
    line = r.stdout.strip().splitlines()[-1] if r.stdout.strip() else "{}"
    return r.returncode, json.loads(line), r


def test_measure_ok_and_gated(tune_fake):
    rc, j, _ = measure(tune_fake, GOOD)
    assert rc == 0 and j["ok"] and j["gflops"] > 0
    assert j["profile"]["max_err"] < 2e-2
    assert j["profile"]["regs"] == 149
    # the fake's cuBLAS comparator reports 0.9 ms (GEMM alone) and 1.4 ms (GEMM + separate bias/GELU)
    flops = 2.0 * 256 * 256 * 128
    assert abs(j["cublas_gflops"] - flops / 0.9e6) < 1e-6 and abs(j["cublas_unfused_gflops"] - flops / 1.4e6) < 1e-6


@pytest.mark.parametrize("gpus", [2, 3, 8])
def test_measure_sharded_over_gpus(tune_fake, tmp_path, gpus):
    log = tmp_path / "calls.log"
    rc, j, _ = measure(tune_fake, GOOD + ["--gpus", str(gpus), "--M", "1000"], FAKE_PF_LOG=log)
    assert rc == 0 and j["ok"], j
    lines = log.read_text().split()
    devices = {int(d) for what, d in zip(lines[::2], lines[1::2]) if what == "launch"}
    # 1000 rows = 8 units of up to 128 rows: every device got a shard and launched
    assert devices == set(range(gpus))
    # the trial's time is the slowest shard's (the fake reports 0.01 ms more per device index)
    slowest = max(devices)
    assert abs(j["ms"] - (1.0 + 0.001 * (256 + 8 + 16) + 0.01 * slowest)) < 1e-9


def test_fp32_path(tune_fake):
    r = run(tune_fake, ["measure", "--dtype", "f32", "--M", "128", "--N", "128", "--K", "64", "--BM", "128", "--BN",
                        "128", "--BK", "8", "--TM", "8", "--TN", "8", "--PAD", "4"])
    j = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and j["ok"] and j["profile"]["max_err"] < 1e-5


def test_e4m3_path(tune_fake):
    r = run(tune_fake, ["measure", "--dtype", "e4m3", *SMALL, *GOOD])
    j = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and j["ok"] and j["profile"]["max_err"] < 5e-2


def test_unmappable_config_is_a_failed_trial(tune_fake):
    rc, j, _ = measure(tune_fake, ["--BM", "64", "--BN", "64", "--BK", "8", "--TM", "4", "--TN", "4", "--PAD", "0"])
    assert rc == 4 and not j["ok"] and "BM must be" in j["error"]


@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_512_column_pair_tiles(tune_fake, dtype):
    # 256 x 512 pair tiles: one k-atom per stage (PAD 0), at least 3 stages; PAD >= 1 asks for two k-atoms,
    # which no 512-wide kernel has: a failed trial, never a crash
    wide = ["--BM", "256", "--BN", "512", "--BK", "32", "--TM", "3", "--TN", "16"]
    rc, j, _ = measure(tune_fake, ["--dtype", dtype, *wide, "--PAD", "0"])
    assert rc == 0 and j["ok"], j
    rc, j, _ = measure(tune_fake, ["--dtype", dtype, *wide, "--PAD", "1"])
    assert rc == 4 and not j["ok"] and "k-atom" in j["error"]


@pytest.mark.parametrize("pad,wide", [(0, False), (1, False), (2, True), (4, True), (8, False)])
def test_search_configs_reach_the_512_column_tiles_through_pad(tune_fake, tmp_path, pad, wide):
    # the search domain's BN stops at 256: BM=256, BN=256 with PAD=2 or 4 are the 256 x 512 pair tiles
    log = tmp_path / "calls.log"
    rc, j, _ = measure(tune_fake, ["--BM", "256", "--BN", "256", "--BK", "32", "--TM", "4", "--TN", "16", "--PAD", str(pad)],
                       FAKE_PF_LOG=log)
    assert rc == 0 and j["ok"], j
    events = log.read_text().split()[::2]
    assert ("prepare_bn512" in events) == wide and ("prepare" in events) == (not wide)


def test_bk_and_pad_are_canonical_on_the_tensor_path(tune_fake):
    rc, j, _ = measure(tune_fake, ["--BM", "128", "--BN", "128", "--BK", "8", "--TM", "4", "--TN", "8", "--PAD", "2"])
    assert rc == 0 and j["ok"]


@pytest.mark.parametrize("env,needle", [({"FAKE_PF_WRONG": 1}, "incorrect result"),
                                        ({"FAKE_PF_FAIL_LAUNCH": 1}, "fake launch failure"),
                                        ({"FAKE_PF_NOMEM": 1}, "cudaMalloc")])
def test_injected_failures(tune_fake, env, needle):
    rc, j, _ = measure(tune_fake, GOOD, **env)
    assert rc == 4 and not j["ok"] and needle in j["error"], j


def test_timeout_on_one_shard_names_the_gpu(tune_fake):
    rc, j, _ = measure(tune_fake, GOOD + ["--gpus", "2"], FAKE_PF_TIMEOUT_DEV=1)
    assert rc == 4 and j["error"].startswith("gpu 1:") and "bounded device wait" in j["error"]


def test_device_that_does_not_open(tune_fake):
    rc, _, r = measure(tune_fake, GOOD + ["--gpus", "2"], FAKE_PF_FAIL_OPEN=1)
    assert rc == 1 and "pf_open(device 1)" in r.stderr


def test_tune_trace_contract(tune_fake, tmp_path):
    out = tmp_path / "trace.json"
    r = run(tune_fake, ["tune", "--dtype", "bf16", *SMALL, "--budget", "10", "--advisor", "rules", "--gpus", "2",
                        "--out", str(out)])
    assert r.returncode == 0, r.stderr
    t = json.loads(out.read_text())
    assert t["schema"] == 1 and t["source"] == "harness" and t["warning"] is None
    assert t["gpu"]["arch"] == "sm_100a" and t["gpu"]["sms"] == 148
    assert len(t["trials"]) == 10
    cfgs = [json.dumps(x["cfg"], sort_keys=True) for x in t["trials"]]
    assert len(set(cfgs)) == len(cfgs)  # no duplicate trials
    for tr in t["trials"]:
        assert tr["ok"] or tr["error"]
    assert any(tr["ok"] for tr in t["trials"])
    assert t["best_gflops"] is not None
    names = [s["name"] for s in t["stages"]]
    assert names == ["CUDA C++ source", "LLVM IR", "PTX"]
    assert ".entry" not in t["stages"][2]["text"]  # no compiler-written PTX embedded


def tune_trace(tune_fake, tmp_path, name, *extra, **env):
    out = tmp_path / name
    r = run(tune_fake, ["tune", "--dtype", "bf16", *SMALL, "--budget", "12", "--advisor", "rules", "--out", str(out),
                        *extra], **env)
    assert r.returncode == 0, r.stderr
    return json.loads(out.read_text())


def test_tune_fanout_one_is_the_reference_tune(tune_fake, tmp_path):
    # --fanout 1 (the default) calls ptxforge::tune itself: the trace carries no fan-out record
    a = tune_trace(tune_fake, tmp_path, "a.json")
    b = tune_trace(tune_fake, tmp_path, "b.json", "--fanout", "1")
    assert "fanout" not in a
    for t in (a, b):
        del t["created"]
    assert a == b


@pytest.mark.parametrize("width,gpus", [(4, 1), (3, 2)])
def test_tune_fanout_spreads_trials_over_gpus(tune_fake, tmp_path, width, gpus):
    log = tmp_path / "calls.log"
    seq = tune_trace(tune_fake, tmp_path, "seq.json", "--gpus", str(gpus))
    fan = tune_trace(tune_fake, tmp_path, "fan.json", "--fanout", str(width), "--gpus", str(gpus), FAKE_PF_LOG=log)
    # same schema-1 document, plus the fan-out record
    assert set(fan) == set(seq) | {"fanout"}
    assert fan["fanout"]["width"] == width and fan["fanout"]["rounds"] >= 12 // width
    assert [set(t) for t in fan["trials"]] == [set(t) for t in seq["trials"]]
    assert len(fan["trials"]) == 12
    cfgs = [json.dumps(t["cfg"], sort_keys=True) for t in fan["trials"]]
    assert len(set(cfgs)) == len(cfgs)
    assert [t["i"] for t in fan["trials"]] == list(range(12))
    # the seeding phase proposes tune()'s sequence: baseline, then the cost model's top picks (budget/4 = 3)
    for s, f in zip(seq["trials"][:3], fan["trials"][:3]):
        assert (s["cfg"], s["origin"]) == (f["cfg"], f["origin"])
    assert fan["trials"][0]["origin"] == "baseline"
    assert all(t["origin"] in ("baseline", "cost-model", "neighbor") or t["origin"].startswith("advisor:")
               for t in fan["trials"])
    # every trial slot's GPUs launched: slot s owns devices [s*gpus, (s+1)*gpus)
    lines = log.read_text().split()
    launched = {int(d) for what, d in zip(lines[::2], lines[1::2]) if what == "launch"}
    assert launched == set(range(width * gpus))
    # the cuBLAS comparator is measured once per problem and reported on every passing trial
    assert fan["cublas_gflops"] is not None
    assert all(t["cublas_gflops"] == fan["cublas_gflops"] for t in fan["trials"] if t["ok"])
    assert sum(1 for what in lines[::2] if what == "cublas") == gpus


def test_fp32_tile_outside_the_library_is_jit_compiled(tune_fake, tmp_path):
    # (64,32,8,4,4,0) is not precompiled: the runner nvcc's ptxforge_b200/csrc/simt_image.cu for it (as
    # CudaRunner compiles every config, cuda_runner.cpp:219-237) and loads it through pf_prepare_image.
    log = tmp_path / "calls.log"
    work = tmp_path / "kernels"
    args = ["measure", "--dtype", "f32", "--M", "128", "--N", "64", "--K", "64", "--BM", "64", "--BN", "32", "--BK", "8",
            "--TM", "4", "--TN", "4", "--PAD", "0", "--root", ROOT, "--workdir", str(work)]
    r = run(tune_fake, args, FAKE_PF_LOG=log)
    j = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and j["ok"], j
    assert (work / "simt_64_32_8_4_4_0.cubin").exists()
    assert "prepare_image" in log.read_text()


def test_fp32_tile_that_does_not_compile_is_a_failed_trial(tune_fake, tmp_path):
    # one stage alone is 4 x (32*(256+0) + 32*256) = 64 KB of static shared memory (above 48 KB): nvcc refuses,
    # the trial fails with its log
    args = ["measure", "--dtype", "f32", "--M", "256", "--N", "256", "--K", "64", "--BM", "256", "--BN", "256", "--BK",
            "32", "--TM", "16", "--TN", "16", "--PAD", "0", "--root", ROOT, "--workdir", str(tmp_path / "k")]
    r = run(tune_fake, args)
    j = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 4 and not j["ok"] and j["error"].startswith("nvcc failed")


FAKE_NCU = """#!/bin/bash
# stands in for ncu: checks the flags the capture must carry, runs the profiled command, writes a CSV
args=("$@"); log=""; cmd=()
for ((i=0; i<${#args[@]}; i++)); do
  case "${args[$i]}" in
    --log-file) log="${args[$((i+1))]}"; i=$((i+1));;
    --metrics|-k|-c|--clock-control) i=$((i+1));;
    --csv) ;;
    *) cmd=("${args[@]:$i}"); break;;
  esac
done
echo "$*" > "$log.args"
"${cmd[@]}" > /dev/null || exit 9
cat > "$log" <<CSV
==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","tune","h","void pf::gemm_bias_gelu_tc<x>(p)","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","byte","1,048,576"
"0","1","tune","h","void pf::gemm_bias_gelu_tc<x>(p)","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_write.sum","byte","131072"
"0","1","tune","h","void pf::gemm_bias_gelu_tc<x>(p)","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed","%","61.5"
"1","1","tune","h","void pf::gemm_bias_gelu_tc<x>(p)","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","byte","7"
CSV
"""


def test_ncu_counters_attached_to_the_trace(tune_fake, tmp_path):
    """ptxforge_b200.counters: plain run first, ncu with clocks left alone on one launch, counters in the trace."""
    from ptxforge_b200 import counters

    exe, _ = tune_fake
    trace_path = tmp_path / "t.json"
    r = run(tune_fake, ["tune", "--dtype", "bf16", *SMALL, "--budget", "4", "--out", str(trace_path)])
    assert r.returncode == 0, r.stderr
    ncu = tmp_path / "ncu"
    ncu.write_text(FAKE_NCU)
    ncu.chmod(0o755)
    out = tmp_path / "t_counters.json"
    rc = counters.main(["--trace", str(trace_path), "--out", str(out), "--exe", exe, "--ncu", str(ncu),
                        "--root", ROOT])
    assert rc == 0
    t = json.loads(out.read_text())
    c = t["counters"]
    assert c["metrics"]["dram__bytes_read.sum"] == 1048576  # first launch only, thousands separators read
    assert c["metrics"]["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"] == 61.5
    assert c["derived"]["dram_bytes"] == 1048576 + 131072
    algo = (256 * 128 + 128 * 256) * 2 + 256 * 4 + 256 * 256 * 2
    assert c["derived"]["algorithmic_bytes"] == algo
    assert c["derived"]["measured_ai"] == round(2.0 * 256 * 256 * 128 / (1048576 + 131072), 2)
    assert t["trials"][t["best_index"]]["counters"] == c["metrics"]
    assert c["cfg"] == t["trials"][t["best_index"]]["cfg"]
    args = (tmp_path / "t_counters.ncu.csv.args").read_text()
    assert "--clock-control none" in args and "-c 1" in args and "-k regex:gemm_bias_gelu" in args
    assert "measure" in args and "--cublas 0" in args


def test_ncu_counters_refuse_when_the_plain_run_fails(tune_fake, tmp_path):
    from ptxforge_b200 import counters

    exe, _ = tune_fake
    trace_path = tmp_path / "t.json"
    r = run(tune_fake, ["tune", "--dtype", "bf16", *SMALL, "--budget", "3", "--out", str(trace_path)])
    assert r.returncode == 0, r.stderr
    ncu = tmp_path / "ncu"
    ncu.write_text("#!/bin/bash\ntouch " + str(tmp_path / "ncu_ran") + "\n")
    ncu.chmod(0o755)
    os.environ["FAKE_PF_FAIL_LAUNCH"] = "1"
    try:
        rc = counters.main(["--trace", str(trace_path), "--exe", exe, "--ncu", str(ncu)])
    finally:
        del os.environ["FAKE_PF_FAIL_LAUNCH"]
    assert rc == 2 and not (tmp_path / "ncu_ran").exists()


def test_fp32_3xtf32_path(tune_fake):
    r = run(tune_fake, ["measure", "--dtype", "f32_3xtf32", "--M", "256", "--N", "256", "--K", "64", "--BM", "256",
                        "--BN", "256", "--BK", "8", "--TM", "3", "--TN", "8", "--PAD", "4"])
    j = json.loads(r.stdout.strip().splitlines()[-1])
    # BK and PAD are canonicalised (32, 0) as on the tensor path; the gate is the fp32 one
    assert r.returncode == 0 and j["ok"] and j["profile"]["max_err"] < 1e-5, j
    r = run(tune_fake, ["measure", "--dtype", "f32_3xtf32", "--M", "256", "--N", "256", "--K", "64", *GOOD])
    j = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 4 and "3xTF32" in j["error"]
    g = json.loads(run(tune_fake, ["gpus", "--dtype", "f32_3xtf32"]).stdout)
    assert g["peak_gflops"] == 375000.0
