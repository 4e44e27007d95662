"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run where the reference tree is mounted (its root in $PTXFORGE_REFERENCE, default as in oracle/build.py):

    python tests/golden/make_golden.py

Writes
  fakecuda_cases.npz   small seeded problems and the C that the reference's fake CUDA driver computes for
                       them (tests/fake_cuda/fake_cuda.cpp:45-50: fp64 accumulate over k ascending, fp64
                       gelu_tanh, stored as float).  Built by oracle/build.py into oracle/_ref/ from the
                       reference's source with the reference's own flags (tests/fake_cuda/run.sh:14).
  mt19937.npz          the first 2048 outputs of std::mt19937(99) (the generator of the reference gate's
                       sample positions, core/src/cuda_runner.cpp:190) and of std::mt19937(1234) (its
                       input generator, cuda_runner.cpp:98), from a libstdc++ program compiled here, and the
                       first 2048 floats of std::uniform_real_distribution<float>(-0.5f, 0.5f) drawn from
                       std::mt19937(1234) (the runner's input values, cuda_runner.cpp:98-102).

The GPU box has no reference tree: tests read these files instead.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle import build as obuild  # noqa: E402

# (M, N, K, seed): square, ragged and K-heavy shapes; small enough to keep the file a few hundred KB.
CASES = [(64, 48, 40, 1), (96, 80, 72, 2), (128, 128, 128, 3), (33, 65, 129, 4)]

MT_PROGRAM = r"""
#include <cstdio>
#include <cstring>
#include <random>
int main() {
  for (unsigned seed : {99u, 1234u}) {
    std::mt19937 g(seed);
    for (int i = 0; i < 2048; ++i) std::printf("%u\n", static_cast<unsigned>(g()));
  }
  std::mt19937 g(1234);
  std::uniform_real_distribution<float> U(-0.5f, 0.5f);
  for (int i = 0; i < 2048; ++i) {
    const float v = U(g);
    unsigned bits;
    std::memcpy(&bits, &v, sizeof bits);
    std::printf("%u\n", bits);
  }
}
"""


def make_cases():
    out = {}
    for i, (M, N, K, seed) in enumerate(CASES):
        rng = np.random.default_rng(seed)
        A = (rng.uniform(-1, 1, (M, K)) / np.sqrt(K)).astype(np.float32)
        B = (rng.uniform(-1, 1, (K, N)) / np.sqrt(K)).astype(np.float32)
        bias = rng.normal(0, 0.1, N).astype(np.float32)
        C = oracle.fakecuda_launch(A, B, bias)
        out[f"A{i}"], out[f"B{i}"], out[f"bias{i}"], out[f"C{i}"] = A, B, bias, C
    out["shapes"] = np.array([c[:3] for c in CASES], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "fakecuda_cases.npz"), **out)


def make_mt():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "mt.cpp"), os.path.join(d, "mt")
        open(src, "w").write(MT_PROGRAM)
        subprocess.run(["g++", "-std=c++20", "-O1", src, "-o", exe], check=True)
        vals = np.array([int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                                         check=True).stdout.split()], dtype=np.uint32)
    np.savez_compressed(os.path.join(HERE, "mt19937.npz"), seed99=vals[:2048], seed1234=vals[2048:4096],
                        uniform1234=vals[4096:6144].view(np.float32))


if __name__ == "__main__":
    obuild.build()
    if not oracle.have_fakecuda():
        sys.exit("the reference tree is not available: cannot build oracle/_ref/libfakecuda_ref.so")
    make_cases()
    make_mt()
    print("wrote", os.listdir(HERE))
