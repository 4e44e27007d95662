"""The 256 x 512 pair kernel's tail split changes when MMAs run, not what they sum (needs a B200: -m gpu).

In a pair's last tile the second half's MMAs of the last L k steps run after all of the first half's
(TcParams::tail_split, PF_TAIL_SPLIT in the environment, read once per process).  Every output still sums its
k blocks in the same order, so C must be bit-identical for every L: each case is run in child processes with
L = 0 (off), 1, 3 and the default, and the outputs compared byte for byte, and the default's against fp64.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# dtype, M, N, K, tile, stream-K mode: ragged edges; one k step (no split possible) and three (L <= 1); a launch
# with several tiles per pair (only the last one splits); the 4-stage variant; e4m3; row bands (never split).
CASES = [
    ("bf16", 1000, 8000, 1000, (256, 512, 32, 3, 16, 0), -1),
    ("bf16", 512, 1024, 64, (256, 512, 32, 4, 16, 0), -1),
    ("bf16", 512, 1024, 192, (256, 512, 32, 4, 16, 0), -1),
    ("bf16", 2048, 8192, 1024, (256, 512, 32, 3, 16, 0), -1),
    ("bf16", 1024, 8192, 2048, (256, 512, 32, 4, 16, 0), -1),
    ("e4m3", 768, 2560, 2304, (256, 512, 32, 3, 16, 0), -1),
    ("bf16", 1024, 8192, 1024, (256, 512, 32, 3, 16, 0), 2),
]

CHILD = r"""
import json, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
import ptxforge_b200 as pf
dtype, M, N, K, tile, sk = json.loads(sys.argv[2])
g = torch.Generator(device="cuda").manual_seed(7)
A = torch.rand(M, K, device="cuda", generator=g) - 0.5
B = torch.rand(K, N, device="cuda", generator=g) - 0.5
bias = torch.rand(N, device="cuda", generator=g) - 0.5
tdt = torch.bfloat16 if dtype == "bf16" else torch.float8_e4m3fn
A, B = A.to(tdt), B.to(tdt)
C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
ctx = pf.Context(0)
ctx.prepare(dtype, tuple(tile), M, N, K)
ctx.set_stream_k(sk)
ctx.bind(A, B, bias, C, 1.0, 1.0)
ctx.launch(); torch.cuda.synchronize()
assert ctx.status() == 0, ctx.status()
np.save(sys.argv[3], C.view(torch.int16).cpu().numpy())
if sys.argv[4] == "ref":
    ref = torch.nn.functional.gelu(A.double() @ B.double() + bias.double(), approximate="tanh")
    err = ((ref - C.double()).abs() / (1 + ref.abs())).max().item()
    print(json.dumps({"err": err}))
ctx.close()
"""


def _run(case, split, out, ref=False):
    env = dict(os.environ)
    if split is None:
        env.pop("PF_TAIL_SPLIT", None)
    else:
        env["PF_TAIL_SPLIT"] = str(split)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, json.dumps(case), out, "ref" if ref else "-"],
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1]) if ref else None


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}x{c[3]}-st{c[4][3]}-sk{c[5]}")
def test_tail_split_is_bit_identical(case, tmp_path):
    tol = {"bf16": 2e-2, "e4m3": 5e-2}[case[0]]
    info = _run(case, None, str(tmp_path / "default.npy"), ref=True)
    assert info["err"] <= tol, info
    base = np.load(tmp_path / "default.npy")
    for split in (0, 1, 3):
        _run(case, split, str(tmp_path / f"s{split}.npy"))
        other = np.load(tmp_path / f"s{split}.npy")
        assert np.array_equal(base, other), f"tail split {split} changed {np.count_nonzero(base != other)} outputs"
