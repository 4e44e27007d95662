"""Seeded synthetic inputs for the five benchmark configurations of the fused GEMM + bias + GELU path.

Plays the role of CudaRunner::Impl::ensure (core/src/cuda_runner.cpp:91-108), which fills A, B and bias
from mt19937(1234) U(-0.5, 0.5); here each configuration has its own value distributions, seed 0 and
one independent stream per tensor (numpy SeedSequence(0).spawn(3) -> A, B, bias).  The reference
measures on no public dataset; these synthetic inputs stand in for the configurations only.

Quantisation (setup, never timed): bf16 by round-to-nearest-even; e4m3 with a per-tensor fp32 scale
s = amax/448, codes = RNE(clamp(x/s, -448, 448)), dequantised value = code * s.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

E4M3_MAX = 448.0


@dataclass(frozen=True)
class Workload:
    name: str
    dtype: str          # "f32" | "f32_3xtf32" | "bf16" | "e4m3"
    M: int
    N: int
    K: int
    a_dist: tuple       # ("uniform_sqrtk",) | ("normal", std) | ("normal_sqrtk",)
    b_dist: tuple
    bias_std: float
    tolerance: float    # max |ref - C| / (1 + |ref|) against fp64 of the (dequantised) inputs

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K

    def algorithmic_bytes(self) -> int:
        e = {"f32": 4, "f32_3xtf32": 4, "bf16": 2, "e4m3": 1}[self.dtype]
        o = 4 if self.dtype in ("f32", "f32_3xtf32") else 2
        return self.M * self.K * e + self.K * self.N * e + self.N * 4 + self.M * self.N * o


# BASELINE configs (BASELINE.json "configs", in order).
CONFIGS = {
    "cfg1_f32_512": Workload("cfg1_f32_512", "f32", 512, 512, 512, ("uniform_sqrtk",), ("uniform_sqrtk",), 0.1, 1e-5),
    "cfg2_f32_2048": Workload("cfg2_f32_2048", "f32", 2048, 2048, 2048, ("uniform_sqrtk",), ("uniform_sqrtk",), 0.1,
                              1e-5),
    # configs 1 and 2 again on the 3xTF32 tensor-core path (same inputs and tolerance)
    "cfg1_f32_512_3xtf32": Workload("cfg1_f32_512_3xtf32", "f32_3xtf32", 512, 512, 512, ("uniform_sqrtk",),
                                    ("uniform_sqrtk",), 0.1, 1e-5),
    "cfg2_f32_2048_3xtf32": Workload("cfg2_f32_2048_3xtf32", "f32_3xtf32", 2048, 2048, 2048, ("uniform_sqrtk",),
                                     ("uniform_sqrtk",), 0.1, 1e-5),
    "cfg3_bf16_8192": Workload("cfg3_bf16_8192", "bf16", 8192, 8192, 8192, ("normal_sqrtk",), ("normal_sqrtk",), 0.1,
                               2e-2),
    "cfg4_bf16_mlp": Workload("cfg4_bf16_mlp", "bf16", 16384, 14336, 4096, ("normal", 1.0), ("normal", 0.02), 0.02,
                              2e-2),
    "cfg5_e4m3_16384": Workload("cfg5_e4m3_16384", "e4m3", 16384, 16384, 16384, ("normal", 1.0), ("normal", 1.0),
                                0.1, 5e-2),
}


def scaled(w: Workload, M: int | None = None, N: int | None = None, K: int | None = None) -> Workload:
    """The same distributions and tolerance at another shape (parity tests at small sizes)."""
    return Workload(w.name + "_scaled", w.dtype, M or w.M, N or w.N, K or w.K, w.a_dist, w.b_dist, w.bias_std,
                    w.tolerance)


def _draw(rng: np.random.Generator, dist: tuple, shape, K: int) -> np.ndarray:
    kind = dist[0]
    if kind == "uniform_sqrtk":
        return (rng.uniform(-1.0, 1.0, size=shape).astype(np.float32) * np.float32(1.0 / np.sqrt(K)))
    if kind == "normal_sqrtk":
        return rng.standard_normal(size=shape, dtype=np.float32) * np.float32(1.0 / np.sqrt(K))
    if kind == "normal":
        return rng.standard_normal(size=shape, dtype=np.float32) * np.float32(dist[1])
    raise ValueError(dist)


@dataclass
class Inputs:
    """Host operands.  A/B hold the values the kernel sees, as float32 (exact for bf16 and e4m3), plus
    the raw encodings the kernel reads (bf16 bit patterns or e4m3 codes) for the tensor path."""
    A: np.ndarray           # float32 [M, K] (dequantised codes for e4m3: codes only, scale separate)
    B: np.ndarray           # float32 [K, N]
    bias: np.ndarray        # float32 [N]
    A_raw: np.ndarray       # float32 / uint16 (bf16 bits) / uint8 (e4m3 codes)
    B_raw: np.ndarray
    scale_a: float = 1.0
    scale_b: float = 1.0


def _to_bf16_bits(x: np.ndarray) -> np.ndarray:
    import torch
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _e4m3_quantize(x: np.ndarray) -> tuple[np.ndarray, float]:
    import torch
    amax = float(np.abs(x).max())
    s = amax / E4M3_MAX if amax > 0 else 1.0
    t = torch.from_numpy(x).div(s).clamp_(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy(), float(np.float32(s))


def e4m3_codes_to_f32(codes: np.ndarray) -> np.ndarray:
    import torch
    return torch.from_numpy(np.ascontiguousarray(codes)).view(torch.float8_e4m3fn).to(torch.float32).numpy()


def make_inputs(w: Workload, seed: int = 0) -> Inputs:
    ra, rb, rbias = (np.random.default_rng(s) for s in np.random.SeedSequence(seed).spawn(3))
    A = _draw(ra, w.a_dist, (w.M, w.K), w.K)
    B = _draw(rb, w.b_dist, (w.K, w.N), w.K)
    bias = (rbias.standard_normal(size=w.N, dtype=np.float32) * np.float32(w.bias_std)).astype(np.float32)
    if w.dtype in ("f32", "f32_3xtf32"):
        return Inputs(A, B, bias, A, B)
    if w.dtype == "bf16":
        Ab, Bb = _to_bf16_bits(A), _to_bf16_bits(B)
        return Inputs(_bf16_bits_to_f32(Ab), _bf16_bits_to_f32(Bb), bias, Ab, Bb)
    if w.dtype == "e4m3":
        Aq, sa = _e4m3_quantize(A)
        Bq, sb = _e4m3_quantize(B)
        return Inputs(e4m3_codes_to_f32(Aq), e4m3_codes_to_f32(Bq), bias, Aq, Bq, sa, sb)
    raise ValueError(w.dtype)
