"""The fp32 SIMT kernel as a JIT image (ptxforge_b200/csrc/simt_image.cu) compiles for the tiles of the
reference's search space that take its fallbacks (no GPU needed: nvcc cross-compiles for sm_100a).

* BM + PAD not a multiple of 4: the transposed A tile's rows are not 16-byte multiples, so A is read with
  scalar loads (float4 reads there would be misaligned).
* the ring depth: up to 4 stages within the shared memory a CTA gets at its register-limited occupancy
  (at most 48 KB of static shared memory); where two stages do not fit, one stage with two barriers per k step.
The GPU side (bit-for-bit equality with a precompiled tile) is tests/test_gpu_image_runner.py.
"""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FALLBACK_TILES = [(32, 64, 32, 8, 4, 1), (64, 64, 8, 8, 4, 2), (64, 64, 16, 4, 8, 3), (128, 128, 32, 4, 4, 1)]


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not on PATH")
@pytest.mark.parametrize("tile", FALLBACK_TILES)
def test_fallback_tiles_compile_without_spills(tile, tmp_path):
    BM, BN, BK, TM, TN, PAD = tile
    defs = [f"-D{k}={v}" for k, v in zip(("BM", "BN", "BK", "TM", "TN", "PAD"), tile)]
    r = subprocess.run(["nvcc", "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-Xptxas", "-v", *defs,
                        "-I", os.path.join(ROOT, "ptxforge_b200", "csrc"),
                        os.path.join(ROOT, "ptxforge_b200", "csrc", "simt_image.cu"), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "0 bytes spill stores" in r.stderr
    smem = int(re.search(r"(\d+) bytes smem", r.stderr).group(1))
    stage = 4 * (BK * (BM + PAD) + BK * BN)
    threads = (BM // TM) * (BN // TN)
    min_blocks = 512 // threads if TM * TN <= 64 and threads <= 512 else 1
    budget = min(227 * 1024 // min_blocks - 1024, 48 * 1024)
    fit = budget // stage
    assert smem == stage * (4 if fit >= 4 else (fit if fit >= 2 else 1))
