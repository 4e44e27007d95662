"""ptxforge_b200 -- sm_100a backend for PTXForge's fused GEMM + bias + GELU hot path.

Python view of the C ABI in include/pf_b200.h (libpf_b200.so, built by ``ptxforge_b200.build``).
It mirrors what PTXForge's CudaRunner does per trial (core/src/cuda_runner.cpp:152-217): pick a
kernel for a tile config, bind operands, launch, time with the reference protocol, read kernel
attributes.  There is no CPU fallback: without the library or an sm_100 GPU every call raises.

    import torch, ptxforge_b200 as pf
    C = pf.gemm_bias_gelu(A, B, bias, dtype="bf16")          # A, B, bias CUDA tensors
"""
from __future__ import annotations

import ctypes
import os
import threading
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpf_b200.so")

PF_OK, PF_EINVAL, PF_ENODEV, PF_ECUDA, PF_ETILE, PF_ESHAPE, PF_ESTATE, PF_ETIMEOUT, PF_ENOMEM = range(9)
ERROR_NAMES = {0: "PF_OK", 1: "PF_EINVAL", 2: "PF_ENODEV", 3: "PF_ECUDA", 4: "PF_ETILE", 5: "PF_ESHAPE",
               6: "PF_ESTATE", 7: "PF_ETIMEOUT", 8: "PF_ENOMEM"}

DTYPES = {"f32": 0, "f32_3xtf32": 1, "bf16": 2, "e4m3": 3}
ELEM_BYTES = {"f32": 4, "f32_3xtf32": 4, "bf16": 2, "e4m3": 1}
OUT_BYTES = {"f32": 4, "f32_3xtf32": 4, "bf16": 2, "e4m3": 2}

# Exported symbols (every entry point of include/pf_b200.h).
SYMBOLS = ("pf_open", "pf_close", "pf_prepare", "pf_bind", "pf_launch", "pf_time", "pf_attrs",
           "pf_device_status", "pf_set_wait_timeout", "pf_last_error", "pf_run_host", "pf_shard_rows",
           "pf_elem_bytes", "pf_out_bytes", "pf_version", "pf_selftest_wait_timeout", "pf_upload", "pf_download",
           "pf_gemm_bias_gelu_noalloc", "pf_prepare_image", "pf_time_cublas",
           "pf_set_stream_k", "pf_run_host_rows", "pf_set_host_chunks")


class Tile(ctypes.Structure):
    """ptxforge::Config (core/include/ptxforge/space.hpp:58): BM, BN, BK, TM, TN, PAD."""
    _fields_ = [(n, ctypes.c_int) for n in ("BM", "BN", "BK", "TM", "TN", "PAD")]

    def astuple(self):
        return (self.BM, self.BN, self.BK, self.TM, self.TN, self.PAD)

    def __repr__(self):
        return "Tile(%d, %d, %d, %d, %d, %d)" % self.astuple()


class Attr(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("regs", "local_bytes", "smem_bytes", "blocks_per_sm", "threads",
                                            "grid", "num_sms")]

    def asdict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


# Base tiles per dtype (default_tile() picks by shape from these and WIDE_TILE).  Tensor path: CTA pair (BM=256) x BN=256, two 128-byte k-atoms per
# stage (PAD=1) and as many stages as fit (TM=8 -> 3), raster group 16 M-blocks (TN=16; with the pair kernel's
# alternating k direction the least DRAM traffic: 0.95 GB per bf16 8192^3 launch vs 1.20 GB at TN=8) -- the lowest energy
# per launch under the 1 kW cap; fp32: 128x64x16 block tile, 8x8 micro-tile, fed by TMA (large problems); 3xTF32: CTA pair,
# 2 raw + 2 split slots (depth 4), raster group 8.
DEFAULT_TILES = {
    "f32": (128, 64, 16, 8, 8, 0),
    "f32_3xtf32": (256, 256, 32, 4, 8, 0),
    "bf16": (256, 256, 32, 8, 16, 1),
    "e4m3": (256, 256, 32, 8, 16, 1),
}
# 256 x 512 CTA-pair tiles, 8 epilogue warps (gemm_tc2w.cuh); default_tile picks them for long tiles: for bf16, 4 stages
# with one staging box per epilogue warp (bursts of 20, us per launch, 3 -> 4 stages: 8192^3 681.8 -> 678.5, 688.5 ->
# 684.8, 706.9 -> 703.5 on three boxes; 2,048 x 8192 x 8192 189.2 -> 187.3; 1,024 x 8192 x 8192 96.0 -> 93.5); for
# e4m3, 3 stages with two staging boxes (16384^3: 2,978 vs 3,032 us), except launches of at most one tile per pair.
WIDE_TILE = (256, 512, 32, 3, 16, 0)
WIDE_TILE_DEEP = (256, 512, 32, 4, 16, 0)


def default_tile(dtype: str, rows: int, N: int, K: int | None = None, pairs: int = 74) -> tuple:
    """The best-measured tile for a rows x N x K problem on one GPU (what prepare() uses when given no tile).

    bf16 / e4m3: CTA-pair tiles 256 rows high.  256 x 512 tiles with 8 epilogue warps (WIDE_TILE) move a quarter
    fewer operand bytes through L2 per output and, under the power cap, ran faster with long tiles: sustained
    8192^3 bf16 +1 %, 16384^3 e4m3 +4.9 %, both with less energy per launch; with 64 k steps per tile (the
    4096-deep MLP) they lost 3 %.  On row shards of 8192^3 (rows x 8192 x 8192) they won at 1,024 and 2,048 rows
    (+3 %, +0.9 %: there both widths leave the same share of the last wave idle, and idle SMs free power for
    the busy ones) and lost at 4,096 rows (-3.8 %: 256 x 512 tiles fill 86.5 % of their waves, 256 x 256 ones
    98.8 %).  So: 512-wide from 128 k steps per tile when their wave fill is within 2 points of the 256-wide
    kernel's.  Otherwise 256 columns, or 224 where the 256-wide schedule's last
    wave is nearly empty and 224-wide tiles add no wave: MLP shards of 2048 x 14336 (448 tiles, 4 in the last
    wave of 74 pairs) ran 6 % faster with 224; 8192-column shards of 1024 / 2048 rows and MLP shards of 4096
    rows ran 1.6-3.7 % slower.
    f32: every SIMT tile gives the same bits (the reference kernel's fmaf chain); small problems get small tiles,
    larger ones the TMA-fed kernel's 8-row micro-tiles.  Measured TFLOP/s at n^3 (CUDA events, bursts of 20, B200,
    packed fp32 FMA): 512: 16.1 on 32 x 32 x 32; 1024: 35.0 on 64 x 32 x 16 (t8x4, TMA); 2048: 48.5 on 64 x 32 x 16
    (TMA) vs 48.3 on 32 x 64 x 16 (t4x8) and 45.5 on 64 x 64 x 16 (t8x8); 4096: 56.0 on 128 x 64 x 16 (t8x8, TMA)
    vs 52.5 on 64 x 32 x 16.
    """
    base = DEFAULT_TILES[dtype]
    if dtype == "f32":
        t128 = -(-rows // 128) * -(-N // 128)
        if t128 < 48:
            return (32, 32, 32, 4, 2, 2)
        if t128 < 512:
            return (64, 32, 16, 8, 4, 0)
        return (128, 64, 16, 8, 8, 0)
    if dtype not in ("bf16", "e4m3") or base[0] != 256:
        return base
    t256 = -(-rows // 256) * -(-N // 256)
    if K is not None:
        k_steps = -(-K // (64 if dtype == "bf16" else 128))
        t512 = -(-rows // 256) * -(-N // 512)
        fill512 = t512 / (-(-t512 // pairs) * pairs)
        fill256 = t256 / (-(-t256 // pairs) * pairs)
        if k_steps >= 128 and fill512 >= fill256 - 0.02:
            return WIDE_TILE_DEEP if (dtype == "bf16" or t512 <= pairs) else WIDE_TILE
    t224 = -(-rows // 256) * -(-N // 224)
    tail = t256 % pairs
    if 0 < tail <= pairs // 10 and -(-t224 // pairs) <= -(-t256 // pairs):
        return base[:1] + (224,) + base[2:]
    return base


class PFError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load libpf_b200.so (raises if it is missing: the CUDA path has no fallback)."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(f"{p} is missing: build it with `python -m ptxforge_b200.build` "
                               "(there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        vp, ip, i = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int
        lib.pf_open.argtypes = [i, ctypes.POINTER(vp)]
        lib.pf_close.argtypes = [vp]
        lib.pf_prepare.argtypes = [vp, i, ctypes.POINTER(Tile), i, i, i]
        lib.pf_bind.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, ctypes.c_float]
        lib.pf_launch.argtypes = [vp, vp]
        lib.pf_time.argtypes = [vp, i, i, i, ctypes.POINTER(ctypes.c_double)]
        lib.pf_attrs.argtypes = [vp, ctypes.POINTER(Attr)]
        lib.pf_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint)]
        lib.pf_set_wait_timeout.argtypes = [vp, ctypes.c_ulonglong]
        lib.pf_last_error.argtypes = [vp]
        lib.pf_last_error.restype = ctypes.c_char_p
        lib.pf_run_host.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, ctypes.c_float]
        lib.pf_run_host_rows.argtypes = [vp, vp, vp, vp, vp]
        lib.pf_shard_rows.argtypes = [i, i, i, i, ip, ip]
        lib.pf_upload.argtypes = [vp, vp, vp, vp, ctypes.c_float, ctypes.c_float]
        lib.pf_download.argtypes = [vp, vp]
        lib.pf_prepare_image.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, i, i, i, i, i, i]
        dp = ctypes.POINTER(ctypes.c_double)
        lib.pf_time_cublas.argtypes = [vp, i, i, i, dp, dp]
        lib.pf_set_stream_k.argtypes = [vp, i]
        lib.pf_set_host_chunks.argtypes = [vp, i]
        lib.pf_gemm_bias_gelu_noalloc.argtypes = [i, i, ctypes.POINTER(Tile), i, i, i, vp, vp, vp, vp, ctypes.c_float,
                                                  ctypes.c_float, vp, ctypes.POINTER(ctypes.c_uint), ctypes.c_char_p,
                                                  ctypes.c_size_t]
        lib.pf_elem_bytes.argtypes = [i]
        lib.pf_elem_bytes.restype = ctypes.c_size_t
        lib.pf_out_bytes.argtypes = [i]
        lib.pf_out_bytes.restype = ctypes.c_size_t
        lib.pf_version.restype = ctypes.c_char_p
        lib.pf_selftest_wait_timeout.argtypes = [vp, ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_uint)]
        for name in ("pf_open", "pf_close", "pf_prepare", "pf_bind", "pf_launch", "pf_time", "pf_attrs",
                     "pf_device_status", "pf_set_wait_timeout", "pf_run_host", "pf_run_host_rows", "pf_shard_rows",
                     "pf_selftest_wait_timeout", "pf_upload", "pf_download", "pf_gemm_bias_gelu_noalloc",
                     "pf_prepare_image", "pf_time_cublas", "pf_set_stream_k", "pf_set_host_chunks"):
            getattr(lib, name).restype = ctypes.c_int
        if path is None:
            _lib = lib
        return lib


def version() -> str:
    return load_library().pf_version().decode()


def shard_rows(M: int, G: int, g: int, align: int = 128) -> tuple[int, int]:
    """Rows [row0, row0 + rows) of the M-row problem that shard g of G owns (pf_shard_rows)."""
    r0, n = ctypes.c_int(), ctypes.c_int()
    rc = load_library().pf_shard_rows(M, G, g, align, ctypes.byref(r0), ctypes.byref(n))
    if rc:
        raise PFError(rc, "pf_shard_rows: bad arguments")
    return r0.value, n.value


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if hasattr(x, "ctypes"):
        return int(x.ctypes.data)
    raise TypeError(f"cannot take a device/host pointer of {type(x)}")


def _stream(s) -> int:
    """A cudaStream_t handle from None (the CUDA default stream), an int or a torch stream."""
    return 0 if s is None else (s if isinstance(s, int) else int(s.cuda_stream))


class Context:
    """One pf_ctx: a GPU, a stream, a prepared kernel variant and bound operands."""

    def __init__(self, device: int = 0, lib: ctypes.CDLL | None = None):
        # `lib`: a library handle from load_library(path) (another build of libpf_b200.so); default the package's.
        self._lib = lib if lib is not None else load_library()
        h = ctypes.c_void_p()
        rc = self._lib.pf_open(device, ctypes.byref(h))
        if rc:
            raise PFError(rc, f"pf_open(device={device}) failed: no sm_100 GPU visible, and this backend "
                              "has no CPU fallback")
        self._h = h
        self.device = device
        self.dtype = None
        self.shape = None
        self.tile = None

    def _check(self, rc: int, what: str):
        if rc:
            raise PFError(rc, f"{what}: {self._lib.pf_last_error(self._h).decode()}")

    def close(self):
        if getattr(self, "_h", None):
            self._lib.pf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def prepare(self, dtype: str, tile, M: int, N: int, K: int):
        t = tile if isinstance(tile, Tile) else Tile(*(tile or default_tile(dtype, M, N, K)))
        self._check(self._lib.pf_prepare(self._h, DTYPES[dtype], ctypes.byref(t), M, N, K), "pf_prepare")
        self.dtype, self.shape, self.tile = dtype, (M, N, K), t
        return self

    def prepare_image(self, image: bytes, kernel: str, grid: tuple[int, int], block: int, M: int, N: int, K: int):
        """Load a PTX/cubin image with the reference kernel ABI (pf_prepare_image, the run_ptx path)."""
        self._check(self._lib.pf_prepare_image(self._h, image, len(image), kernel.encode(), grid[0], grid[1], block,
                                               M, N, K), "pf_prepare_image")
        self.dtype, self.shape, self.tile = "f32", (M, N, K), None
        return self

    def bind(self, A, B, bias, C, scale_a: float = 1.0, scale_b: float = 1.0):
        self._check(self._lib.pf_bind(self._h, _ptr(A), _ptr(B), _ptr(bias), _ptr(C), scale_a, scale_b),
                    "pf_bind")
        return self

    def launch(self, stream=None):
        self._check(self._lib.pf_launch(self._h, _stream(stream)), "pf_launch")

    def time(self, warmup: int = 5, iters: int = 20, reps: int = 5) -> float:
        ms = ctypes.c_double()
        self._check(self._lib.pf_time(self._h, warmup, iters, reps, ctypes.byref(ms)), "pf_time")
        return ms.value

    def time_cublas(self, warmup: int = 5, iters: int = 20, reps: int = 5) -> tuple[float, float]:
        """(cuBLAS GEMM alone, cuBLAS GEMM + separate bias/GELU) in ms on the bound operands (pf_time_cublas).
        C is overwritten with the unfused result."""
        g, u = ctypes.c_double(), ctypes.c_double()
        self._check(self._lib.pf_time_cublas(self._h, warmup, iters, reps, ctypes.byref(g), ctypes.byref(u)),
                    "pf_time_cublas")
        return g.value, u.value

    def attrs(self) -> dict:
        a = Attr()
        self._check(self._lib.pf_attrs(self._h, ctypes.byref(a)), "pf_attrs")
        return a.asdict()

    def status(self) -> int:
        w = ctypes.c_uint()
        self._check(self._lib.pf_device_status(self._h, ctypes.byref(w)), "pf_device_status")
        return w.value

    def set_stream_k(self, mode: int):
        """Stream-K of the CTA-pair kernels (pf_set_stream_k): -1 auto (default), 0 off (whole tiles), 1 the
        stream-K tail, 2 row-band stream-K."""
        self._check(self._lib.pf_set_stream_k(self._h, mode), "pf_set_stream_k")

    def set_host_chunks(self, chunks: int):
        """Row chunks of the host-buffer pipelines: 0 default (8), else 1..64 (pf_set_host_chunks)."""
        self._check(self._lib.pf_set_host_chunks(self._h, chunks), "pf_set_host_chunks")

    def set_wait_timeout(self, ns: int):
        self._check(self._lib.pf_set_wait_timeout(self._h, ns), "pf_set_wait_timeout")

    def run_host(self, hA, hB, hbias, hC, scale_a: float = 1.0, scale_b: float = 1.0):
        """H2D copies of host operands, launch, D2H of C, synchronise (pf_run_host)."""
        self._check(self._lib.pf_run_host(self._h, _ptr(hA), _ptr(hB), _ptr(hbias), _ptr(hC), scale_a, scale_b),
                    "pf_run_host")

    def run_host_rows(self, hA, hC, after_stream=None, copies_after_stream=None):
        """Host rows of A in, launch, C rows out, pipelined in row chunks, with B and bias already on the
        device (bound): kernels after the work queued on `after_stream`, copies of A after the work queued on
        `copies_after_stream` (default: the same stream) (pf_run_host_rows)."""
        s = _stream(after_stream)
        cs = s if copies_after_stream is None else _stream(copies_after_stream)
        self._check(self._lib.pf_run_host_rows(self._h, _ptr(hA), _ptr(hC), s, cs), "pf_run_host_rows")

    def upload(self, hA, hB, hbias, scale_a: float = 1.0, scale_b: float = 1.0):
        """H2D copies into context-owned device operands and bind them (pf_upload)."""
        self._check(self._lib.pf_upload(self._h, _ptr(hA), _ptr(hB), _ptr(hbias), scale_a, scale_b), "pf_upload")

    def download(self, hC):
        """D2H copy of the context-owned C (pf_download)."""
        self._check(self._lib.pf_download(self._h, _ptr(hC)), "pf_download")

    def selftest_wait_timeout(self, ns: int) -> int:
        w = ctypes.c_uint()
        self._check(self._lib.pf_selftest_wait_timeout(self._h, ns, ctypes.byref(w)), "pf_selftest_wait_timeout")
        return w.value


def gemm_bias_gelu_noalloc(device: int, dtype: str, tile, M: int, N: int, K: int, A, B, bias, C,
                           scale_a: float = 1.0, scale_b: float = 1.0, stream=None, sync: bool = True) -> int:
    """pf_gemm_bias_gelu_noalloc: the bf16 / e4m3 kernel on caller-owned device operands, for callers
    that cannot allocate GPU memory at call time (no context, no cudaMalloc; the kernel's scratch is a
    fixed array inside the library).  Torch operands are checked as in gemm_bias_gelu (shapes equal to
    M, N, K, contiguous, element widths of `dtype`, all on `device`; ValueError otherwise), and with no
    `stream` the call goes on torch's current stream of that device.  With sync=True waits for the kernel
    and returns its status word (raising PFError if a bounded device wait ran out); with sync=False returns
    0 after queueing."""
    lib = load_library()
    if all(hasattr(x, "shape") for x in (A, B, bias, C)):
        # torch operands: the same checks as gemm_bias_gelu, before anything reaches the TMA maps
        shape = check_operands(A, B, bias, C, dtype, require_cuda=False)
        if shape != (M, N, K):
            raise ValueError(f"operands are {shape[0]} x {shape[1]} x {shape[2]} (M x N x K), "
                             f"but M, N, K = {M}, {N}, {K}")
        for name, x in (("A", A), ("B", B), ("bias", bias), ("C", C)):
            if not x.is_cuda or x.device.index != device:
                raise ValueError(f"{name} must be a CUDA tensor on device {device}, got {x.device}")
        if stream is None:  # as gemm_bias_gelu: order after the work torch queued on the current stream
            import torch
            stream = torch.cuda.current_stream(A.device)
    t = tile if isinstance(tile, Tile) else Tile(*(tile or default_tile(dtype, M, N, K)))
    s = 0 if stream is None else (stream if isinstance(stream, int) else int(stream.cuda_stream))
    st = ctypes.c_uint(0)
    err = ctypes.create_string_buffer(256)
    rc = lib.pf_gemm_bias_gelu_noalloc(device, DTYPES[dtype], ctypes.byref(t), M, N, K, _ptr(A), _ptr(B),
                                       _ptr(bias), _ptr(C), scale_a, scale_b, s,
                                       ctypes.byref(st) if sync else None, err, len(err))
    if rc:
        raise PFError(rc, "pf_gemm_bias_gelu_noalloc: " + err.value.decode())
    return st.value


def check_operands(A, B, bias, C, dtype: str, require_cuda: bool = True):
    """(M, N, K) of torch operands for `dtype`, or ValueError: the kernels read and write exactly M x K, K x N,
    N and M x N elements of the dtype's sizes through TMA, so a tensor of another size or element width would
    send them past its allocation."""
    if A.dim() != 2 or B.dim() != 2:
        raise ValueError(f"A and B must be matrices, got {tuple(A.shape)} and {tuple(B.shape)}")
    M, K = A.shape
    K2, N = B.shape
    if K2 != K or tuple(bias.shape) != (N,):
        raise ValueError(f"shape mismatch: A {tuple(A.shape)}, B {tuple(B.shape)}, bias {tuple(bias.shape)}")
    if tuple(C.shape) != (M, N):
        raise ValueError(f"C must be {M} x {N}, got {tuple(C.shape)}")
    e, o = ELEM_BYTES[dtype], OUT_BYTES[dtype]
    for name, t, size in (("A", A, e), ("B", B, e), ("bias", bias, 4), ("C", C, o)):
        if require_cuda and not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous (row-major)")
        if t.element_size() != size:
            raise ValueError(f"{name} has {t.element_size()}-byte elements; {dtype} needs {size}")
    if not bias.is_floating_point():
        raise ValueError("bias must be float32")
    return M, N, K


_contexts: dict = {}


def context(device: int = 0) -> Context:
    """A cached Context per device for the convenience functions below."""
    c = _contexts.get(device)
    if c is None:
        c = _contexts[device] = Context(device)
    return c


def gemm_bias_gelu(A, B, bias, C=None, *, dtype: str | None = None, tile=None, scale_a: float = 1.0,
                   scale_b: float = 1.0, stream=None):
    """C = gelu_tanh(scale_a*scale_b * A @ B + bias) for CUDA torch tensors (row-major, contiguous).

    dtype: "f32" (A, B, C float32; SIMT FFMA), "f32_3xtf32" (the same operands on the tensor cores, three
    TF32 products per step), "bf16" (A, B bfloat16, C bfloat16) or "e4m3" (A, B float8_e4m3fn or uint8
    codes, C bfloat16).  bias is float32 [N].  Returns C.
    """
    import torch

    if dtype is None:
        dtype = {torch.float32: "f32", torch.bfloat16: "bf16"}.get(A.dtype, "e4m3")
    if dtype not in DTYPES:
        raise ValueError(f"unknown dtype {dtype!r} (one of {', '.join(DTYPES)})")
    if C is None:
        out_dtype = torch.float32 if OUT_BYTES[dtype] == 4 else torch.bfloat16
        C = torch.empty((A.shape[0], B.shape[-1]), dtype=out_dtype, device=A.device)
    M, N, K = check_operands(A, B, bias, C, dtype)
    ctx = context(A.device.index or 0)
    key = (dtype, tuple(tile) if tile else None, M, N, K)
    if getattr(ctx, "_key", None) != key:
        ctx.prepare(dtype, tile, M, N, K)
        ctx._key = key
    ctx.bind(A, B, bias, C, scale_a, scale_b)
    if stream is None:
        stream = torch.cuda.current_stream(A.device)
    ctx.launch(stream)
    return C
