"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY -- see oracle/oracle.c).

    python -m oracle.build          # liboracle.so, plus oracle/_ref/* when the reference tree exists

Outputs
  oracle/liboracle.so                   the C restatement of the reference's algorithm
  oracle/_ref/libfakecuda_ref.so        the reference's fake CUDA driver (tests/fake_cuda/fake_cuda.cpp),
                                        compiled from its own source with the reference's own flags
                                        (tests/fake_cuda/run.sh:14); its cuLaunchKernel is the fp64 result
                                        the reference's tests accept as correct
  oracle/_ref/gemm_bias_gelu_ref_<cfg>.cubin  the same kernel as an image, compiled as CudaRunner does
                                        (cuda_runner.cpp:228-230), for the image path (pf_prepare_image)
  oracle/_ref/libref_kernel_<cfg>.so    the reference's fp32 kernel (kernels/gemm_bias_gelu.cu) compiled
                                        for sm_100a at a tile config, behind oracle/ref_kernel_launch.cu

The _ref outputs are built here (where the reference is mounted) and travel to the GPU box as
files; nothing at run time reads the reference tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# The reference source tree: $PTXFORGE_REFERENCE, else a `reference` directory beside the repository; where
# neither exists the reference builds are skipped (the prebuilt files in _ref/, if any, stay in use).
REF_ROOT = os.environ.get("PTXFORGE_REFERENCE") or os.path.normpath(os.path.join(ROOT, os.pardir, "reference"))
REF_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(HERE, "liboracle.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

# Tile configs of the reference kernel built for the GPU comparison: the reference's untuned default
# (core/include/ptxforge/space.hpp:115) and the best config of its recorded RTX 5050 run
# (runs/rtx5050_2048.json, trial 13: 128x64x32 t8x4 p2).
REF_KERNEL_CONFIGS = {
    "default": dict(BM=64, BN=64, BK=8, TM=4, TN=4, PAD=0),
    "best5050": dict(BM=128, BN=64, BK=32, TM=8, TN=4, PAD=2),
}


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    if force or _stale(LIB, [src, os.path.abspath(__file__)]):
        _run(["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
              "-std=c11", "-Wall", src, "-o", LIB + ".tmp", "-lm"])
        os.replace(LIB + ".tmp", LIB)
    return LIB


def ref_kernel_lib(name: str) -> str:
    return os.path.join(REF_DIR, f"libref_kernel_{name}.so")


FAKECUDA = os.path.join(REF_DIR, "libfakecuda_ref.so")


def ref_kernel_cubin(name: str) -> str:
    return os.path.join(REF_DIR, f"gemm_bias_gelu_ref_{name}.cubin")


def build_ref(force: bool = False) -> list[str]:
    """Compile the reference's own code (when the reference tree is present) into oracle/_ref/."""
    if not os.path.isdir(REF_ROOT):
        return []
    os.makedirs(REF_DIR, exist_ok=True)
    out = []
    fake_src = os.path.join(REF_ROOT, "tests", "fake_cuda", "fake_cuda.cpp")
    if os.path.exists(fake_src):
        if force or _stale(FAKECUDA, [fake_src]):
            _run(["g++", "-std=c++20", "-O1", "-fPIC", "-shared", f"-I{CUDA_HOME}/include", fake_src,
                  "-o", FAKECUDA])
        out.append(FAKECUDA)
    kern_src = os.path.join(REF_ROOT, "kernels", "gemm_bias_gelu.cu")
    launcher = os.path.join(HERE, "ref_kernel_launch.cu")
    if os.path.exists(kern_src):
        # the reference kernel as an image, compiled the way CudaRunner compiles it
        # (cuda_runner.cpp:228-230: nvcc -cubin -arch=<arch> -O3 -lineinfo -D<tile>)
        for name, cfg in REF_KERNEL_CONFIGS.items():
            cub = ref_kernel_cubin(name)
            if force or _stale(cub, [kern_src]):
                defs = [f"-D{k}={v}" for k, v in cfg.items()]
                _run([os.path.join(CUDA_HOME, "bin", "nvcc"), "-cubin", "-arch=sm_100a", "-O3", "-lineinfo", *defs,
                      kern_src, "-o", cub])
            out.append(cub)
        for name, cfg in REF_KERNEL_CONFIGS.items():
            lib = ref_kernel_lib(name)
            if force or _stale(lib, [kern_src, launcher]):
                defs = [f"-D{k}={v}" for k, v in cfg.items()]
                _run([os.path.join(CUDA_HOME, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
                      "-O3", "-lineinfo", *defs, "-include", kern_src, "-Xcompiler", "-fPIC", "-shared",
                      "-cudart", "static", launcher, "-o", lib])
            out.append(lib)
    return out


def build(force: bool = False) -> list[str]:
    return [build_oracle(force)] + build_ref(force)


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv):
        print(p)
