"""Build recipe for the sm_100a shared library ``libpf_b200.so`` (the C ABI of include/pf_b200.h).

    python -m ptxforge_b200.build            # builds in place, next to this file

nvcc cross-compiles for sm_100a on a machine without a GPU.  The CUDA runtime is linked
statically and the driver is reached through cudaGetDriverEntryPoint, so the library loads (and
reports PF_ENODEV) where no GPU driver is installed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libpf_b200.so")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME")
    return found


def _sources() -> list[str]:
    out = []
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h", ".hpp")):
                out.append(os.path.join(d, name))
    return out


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libpf_b200.so if any source is newer than it; return its path."""
    if not force and not _stale(LIB, _sources() + [os.path.abspath(__file__)]):
        return LIB
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-Wall", "-shared", "-cudart", "static",
        "-I", INCLUDE, "-I", CSRC, "-Xptxas", "-v",
        os.path.join(CSRC, "pf_b200.cu"), "-o", LIB + ".tmp",
    ]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = r.stdout + r.stderr
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + log[-6000:])
    os.replace(LIB + ".tmp", LIB)
    with open(os.path.join(HERE, "libpf_b200.ptxas.txt"), "w") as f:
        f.write(log)
    if verbose:
        print(log)
    return LIB


# The PTXForge source tree the runner plugs into: $PTXFORGE_REFERENCE, else a `reference` directory beside the
# repository.  Where neither exists the tuner CLI is not built (build_tune returns None).
REF_ROOT = os.environ.get("PTXFORGE_REFERENCE") or os.path.normpath(os.path.join(ROOT, os.pardir, "reference"))
TUNE_SRC = os.path.join(HERE, "host", "tune_b200.cpp")
TUNE_BIN = os.path.join(ROOT, "build", "ptxforge-tune-b200")


def tune_command(out: str, lib_dir: str, rpath: str, ref_root: str = REF_ROOT) -> list[str]:
    """g++ line for PTXForge's tuner CLI with the B200 runner, against the libpf_b200.so in lib_dir."""
    return ["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-I", INCLUDE,
            "-I", os.path.join(ref_root, "core", "include"), "-I", os.path.join(ref_root, "compiler", "include"),
            TUNE_SRC, "-L", lib_dir, "-lpf_b200", f"-Wl,-rpath,{rpath}", "-lpthread", "-o", out]


def build_tune(force: bool = False, ref_root: str = REF_ROOT) -> str | None:
    """Build build/ptxforge-tune-b200 when the PTXForge headers are available (they are not shipped here:
    the runner is compiled inside the PTXForge tree it plugs into)."""
    if not os.path.isdir(os.path.join(ref_root, "core", "include", "ptxforge")):
        return None
    deps = [TUNE_SRC, LIB, os.path.join(INCLUDE, "ptxforge_b200", "b200_runner.hpp"), os.path.join(INCLUDE, "pf_b200.h")]
    if force or _stale(TUNE_BIN, deps):
        os.makedirs(os.path.dirname(TUNE_BIN), exist_ok=True)
        # $ORIGIN-relative rpath: the binary finds the library wherever the repository is copied
        cmd = tune_command(TUNE_BIN + ".tmp", HERE, "$ORIGIN/../ptxforge_b200", ref_root)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("g++ failed:\n" + (r.stdout + r.stderr)[-6000:])
        os.replace(TUNE_BIN + ".tmp", TUNE_BIN)
    return TUNE_BIN


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_tune(force="--force" in sys.argv))
