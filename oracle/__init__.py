"""Oracle for the fused GEMM + bias + GELU path -- TEST INFRASTRUCTURE ONLY.

Python view of oracle/liboracle.so (the C restatement in oracle/oracle.c) and of the reference's own
code compiled into oracle/_ref/ by oracle/build.py.  Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py may use this package, and only as the checker or the timed CPU baseline;
the product (ptxforge_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build_oracle()
        L = ctypes.CDLL(path)
        vp, i, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
        L.oracle_mt_stream.argtypes = [ctypes.c_uint32, vp, i]
        L.oracle_gelu_f64.argtypes = [d]
        L.oracle_gelu_f64.restype = d
        L.oracle_gelu_f32_mlir.argtypes = [ctypes.c_float]
        L.oracle_gelu_f32_mlir.restype = ctypes.c_float
        L.oracle_full_f64.argtypes = [vp, vp, vp, i, i, i, d, vp]
        L.oracle_sampled_gate.argtypes = [vp, vp, vp, vp, i, i, i, d, i, ctypes.c_uint32, vp, vp]
        L.oracle_sampled_gate.restype = d
        L.oracle_ref_at.argtypes = [vp, vp, vp, i, i, d, vp, vp, i, vp]
        L.oracle_cpu_schedule.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, i, i]
        L.oracle_bf16_rne.argtypes = [ctypes.c_float]
        L.oracle_bf16_rne.restype = ctypes.c_uint16
        L.oracle_bf16_to_f32_array.argtypes = [vp, vp, ctypes.c_size_t]
        L.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.oracle_e4m3_to_f32.restype = ctypes.c_float
        L.oracle_e4m3_to_f32_array.argtypes = [vp, vp, ctypes.c_size_t]
        L.oracle_e4m3_rne_sat.argtypes = [ctypes.c_float]
        L.oracle_e4m3_rne_sat.restype = ctypes.c_uint8
        L.oracle_e4m3_quantize_array.argtypes = [vp, ctypes.c_float, vp, ctypes.c_size_t]
        L.oracle_max_rel_err.argtypes = [vp, vp, ctypes.c_size_t]
        L.oracle_max_rel_err.restype = d
        L.oracle_num_threads.restype = i
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def num_threads() -> int:
    return lib().oracle_num_threads()


def mt_stream(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    lib().oracle_mt_stream(seed, _p(out), n)
    return out


def uniform_f32(seed: int, n: int, a: float = -0.5, b: float = 0.5) -> np.ndarray:
    """n draws of std::uniform_real_distribution<float>(a, b) from std::mt19937(seed), as libstdc++ makes
    them: generate_canonical<float, 24> takes one 32-bit output w and forms u = float(w) / 2^32 in float
    arithmetic (a quotient of 1 becomes the largest float below 1); the value is u * (b - a) + a."""
    u = mt_stream(seed, n).astype(np.float32) / np.float32(4294967296.0)
    u = np.where(u >= np.float32(1), np.nextafter(np.float32(1), np.float32(0)), u)
    return (u * (np.float32(b) - np.float32(a)) + np.float32(a)).astype(np.float32)


def runner_inputs(M: int, N: int, K: int):
    """The reference runner's own inputs (CudaRunner::Impl::ensure, core/src/cuda_runner.cpp:97-102): one
    std::mt19937(1234) stream through U(-0.5, 0.5), filling A (M x K), then B (K x N), then bias (N)."""
    v = uniform_f32(1234, M * K + K * N + N)
    A = v[:M * K].reshape(M, K)
    B = v[M * K:M * K + K * N].reshape(K, N)
    return A, B, v[M * K + K * N:]


def gelu_f64(x: float) -> float:
    return lib().oracle_gelu_f64(x)


def gelu_f32_mlir(x: float) -> float:
    return lib().oracle_gelu_f32_mlir(x)


def full_f64(A, B, bias, scale: float = 1.0) -> np.ndarray:
    A, B, bias = _f32(A), _f32(B), _f32(bias)
    M, K = A.shape
    N = B.shape[1]
    out = np.empty((M, N), dtype=np.float64)
    lib().oracle_full_f64(_p(A), _p(B), _p(bias), M, N, K, float(scale), _p(out))
    return out


def sampled_gate(A, B, bias, C, scale: float = 1.0, samples: int = 512, seed: int = 99):
    """The reference's gate (core/src/cuda_runner.cpp:189-197): (max_err, rows, cols)."""
    A, B, bias, C = _f32(A), _f32(B), _f32(bias), _f32(C)
    M, K = A.shape
    N = B.shape[1]
    rows = np.empty(samples, dtype=np.int32)
    cols = np.empty(samples, dtype=np.int32)
    err = lib().oracle_sampled_gate(_p(A), _p(B), _p(bias), _p(C), M, N, K, float(scale), samples, seed,
                                    _p(rows), _p(cols))
    return err, rows, cols


def ref_at(A, B, bias, rows, cols, scale: float = 1.0) -> np.ndarray:
    A, B, bias = _f32(A), _f32(B), _f32(bias)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    cols = np.ascontiguousarray(cols, dtype=np.int32)
    N = B.shape[1]
    K = A.shape[1]
    out = np.empty(len(rows), dtype=np.float64)
    lib().oracle_ref_at(_p(A), _p(B), _p(bias), N, K, float(scale), _p(rows), _p(cols), len(rows), _p(out))
    return out


def cpu_schedule(A, B, bias, BM=64, BN=64, BK=16, row0: int = 0, rows: int | None = None, threads: int = 0,
                 out: np.ndarray | None = None) -> np.ndarray:
    """The CPU-lowered schedule (fp32 accumulation, k ascending, MLIR GELU with tanhf)."""
    A, B, bias = _f32(A), _f32(B), _f32(bias)
    M, K = A.shape
    N = B.shape[1]
    if rows is None:
        rows = M - row0
    C = out if out is not None else np.full((M, N), np.nan, dtype=np.float32)
    lib().oracle_cpu_schedule(_p(A), _p(B), _p(bias), _p(C), M, N, K, BM, BN, BK, row0, rows, threads)
    return C


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    lib().oracle_bf16_to_f32_array(_p(bits), _p(out), bits.size)
    return out


def bf16_rne(x: float) -> int:
    return int(lib().oracle_bf16_rne(x))


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(codes.shape, dtype=np.float32)
    lib().oracle_e4m3_to_f32_array(_p(codes), _p(out), codes.size)
    return out


def e4m3_quantize(x: np.ndarray, scale: float) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().oracle_e4m3_quantize_array(_p(x), 1.0 / scale, _p(out), x.size)
    return out


def max_rel_err(ref: np.ndarray, C: np.ndarray) -> float:
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    C = _f32(C)
    return lib().oracle_max_rel_err(_p(ref), _p(C), ref.size)


# ---------------------------------------------------------------------------------------------
# The reference's own code, compiled from its sources into oracle/_ref/ (see oracle/build.py)
# ---------------------------------------------------------------------------------------------
def have_fakecuda() -> bool:
    return os.path.exists(_build.FAKECUDA)


def fakecuda_launch(A, B, bias) -> np.ndarray:
    """C from the reference's fake driver cuLaunchKernel (tests/fake_cuda/fake_cuda.cpp:45-50):
    fp64 accumulate + fp64 GELU, stored as float.  Its parameter block is {&A,&B,&bias,&C,&M,&N,&K}
    (core/src/cuda_runner.cpp:182)."""
    A, B, bias = _f32(A), _f32(B), _f32(bias)
    M, K = A.shape
    N = B.shape[1]
    C = np.full((M, N), np.nan, dtype=np.float32)
    L = ctypes.CDLL(_build.FAKECUDA)
    L.cuLaunchKernel.restype = ctypes.c_int
    ptrs = [ctypes.c_void_p(_p(x)) for x in (A, B, bias, C)]
    ints = [ctypes.c_int(v) for v in (M, N, K)]
    params = (ctypes.c_void_p * 7)(*[ctypes.cast(ctypes.byref(x), ctypes.c_void_p) for x in ptrs + ints])
    rc = L.cuLaunchKernel(None, 1, 1, 1, 1, 1, 1, 0, None, params, None)
    assert rc == 0, rc
    return C


def ref_kernel_path(name: str) -> str:
    return _build.ref_kernel_lib(name)


def ref_kernel_cubin(name: str) -> str:
    """The reference's fp32 kernel compiled to an sm_100a cubin (what CudaRunner would load)."""
    return _build.ref_kernel_cubin(name)


def ref_kernel(name: str):
    """ctypes handle of the reference's fp32 kernel built for sm_100a (GPU only)."""
    L = ctypes.CDLL(ref_kernel_path(name))
    L.ref_launch.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    L.ref_launch.restype = ctypes.c_int
    L.ref_tile.argtypes = [ctypes.POINTER(ctypes.c_int)] * 6
    return L
