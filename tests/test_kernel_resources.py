"""Resource budget of every kernel compiled into libpf_b200.so, from ptxas's own report (no GPU needed).

The build keeps ptxas's -v output beside the library.  Every entry function must compile without register
spills and with at most a 16-byte stack frame; each persistent tensor-core kernel runs one CTA per SM, so its
registers x threads must fit the SM's 65,536 registers (a launch above that fails, and a register split
that asked for more would wait forever).
"""
import os
import re

import pytest

from ptxforge_b200 import build as pbuild

LOG = os.path.join(os.path.dirname(pbuild.LIB), "libpf_b200.ptxas.txt")


def _kernels():
    pbuild.build()
    if not os.path.exists(LOG):
        pytest.skip("no ptxas report beside the library")
    text = open(LOG).read()
    out = {}
    for m in re.finditer(r"Function properties for (\S+)\n\s+(\d+) bytes stack frame, (\d+) bytes spill stores, "
                         r"(\d+) bytes spill loads\n.*?Used (\d+) registers", text):
        name, stack, st, ld, regs = m.group(1), *map(int, m.groups()[1:])
        out[name] = dict(stack=stack, spill_stores=st, spill_loads=ld, regs=regs)
    return out


def _threads(name):
    """Threads per CTA of a persistent tensor-core kernel, from its template arguments (None: not one)."""
    m = re.search(r"Tc2wConfigILi\d+ELi\d+ELi(\d+)E", name)
    if m:
        return 32 * (2 + int(m.group(1)))  # producer, MMA and the epilogue warps
    if "gemm_bias_gelu_tf32x3" in name:
        return 448
    if "gemm_bias_gelu_tc2" in name or "gemm_bias_gelu_tcINS" in name:
        return 192
    return None


def test_every_kernel_compiles_without_spills():
    k = _kernels()
    assert len(k) >= 40, f"only {len(k)} kernels in the ptxas report"
    bad = {n: r for n, r in k.items() if r["spill_stores"] or r["spill_loads"] or r["stack"] > 16}
    assert not bad, bad


def test_persistent_kernels_fit_one_cta_per_sm():
    k = _kernels()
    seen = set()
    for name, r in k.items():
        t = _threads(name)
        if t is None:
            continue
        seen.add(t)
        # the register file hands a warp its registers in blocks of 512 (16 per thread): 200 registers x 10 warps
        # was refused at launch ("too many resources requested") though 200 x 320 < 65,536
        per_warp = -(-r["regs"] * 32 // 512) * 512
        assert per_warp * (t // 32) <= 65536, (name, r["regs"], t)
    assert {192, 320, 448} <= seen  # the 1-CTA / pair kernels, the 8-warp 256x512 kernel, 3xTF32
