"""Parity of the sm_100a kernels with the oracle, through the C ABI (needs a B200: -m gpu).

Bars (BASELINE tolerances, metric max |ref - C| / (1 + |ref|) against fp64 of the (dequantised)
inputs, the reference gate's metric core/src/cuda_runner.cpp:196):
    fp32  1e-5        bf16  2e-2        e4m3  5e-2
plus: the fp32 path is bit-identical to the reference's own kernel (kernels/gemm_bias_gelu.cu built for
sm_100a, oracle/_ref/), and at the full BASELINE sizes every output is compared with a plain PyTorch
fp32 computation of the same op (TF32 off), 64 whole rows with the oracle's fp64 result, and the reference
gate's 512 sampled fp64 points.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ptxforge_b200 import workloads as wl  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-5, "bf16": 2e-2, "e4m3": 5e-2}


def _dev(x: np.ndarray, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    if dtype is torch.bfloat16:
        t = t.view(torch.int16).view(torch.bfloat16)
    elif dtype is torch.float8_e4m3fn:
        t = t.view(torch.float8_e4m3fn)
    return t


def device_operands(w, inp):
    if w.dtype == "f32":
        A, B = _dev(inp.A_raw), _dev(inp.B_raw)
        C = torch.full((w.M, w.N), float("nan"), device="cuda", dtype=torch.float32)
    elif w.dtype == "bf16":
        A, B = _dev(inp.A_raw.view(np.int16), torch.bfloat16), _dev(inp.B_raw.view(np.int16), torch.bfloat16)
        C = torch.full((w.M, w.N), float("nan"), device="cuda", dtype=torch.bfloat16)
    else:
        A, B = _dev(inp.A_raw, torch.float8_e4m3fn), _dev(inp.B_raw, torch.float8_e4m3fn)
        C = torch.full((w.M, w.N), float("nan"), device="cuda", dtype=torch.bfloat16)
    return A, B, _dev(inp.bias), C


def run_pf(ctx, w, inp, tile=None, ops=None):
    A, B, bias, C = ops or device_operands(w, inp)
    ctx.prepare(w.dtype, tile, w.M, w.N, w.K)
    ctx.bind(A, B, bias, C, inp.scale_a, inp.scale_b)
    ctx.launch(torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert ctx.status() == 0
    return C


def to_np(C):
    return C.float().cpu().numpy()


def check_full(oracle_mod, w, inp, C):
    ref = oracle_mod.full_f64(inp.A, inp.B, inp.bias, inp.scale_a * inp.scale_b)
    Cn = to_np(C)
    assert int(np.isnan(Cn).sum()) == 0, "unwritten outputs"
    err = oracle_mod.max_rel_err(ref, Cn)
    assert err <= TOL[w.dtype], f"{w.name} {w.M}x{w.N}x{w.K}: max rel err {err:.3e} > {TOL[w.dtype]}"
    return err


def torch_fp32_reference(A, B, bias, scale):
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        x = torch.matmul(A.float(), B.float())
        if scale != 1.0:
            x.mul_(scale)
        x.add_(bias)
        return torch.nn.functional.gelu(x, approximate="tanh")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def max_rel_err_t(ref, C):
    r = ref.double()
    return float(((r - C.double()).abs() / (1.0 + r.abs())).max())


# ---------------------------------------------------------------------------------------------
# fp32 (SIMT) path
# ---------------------------------------------------------------------------------------------
FP32_TILES = [(128, 128, 8, 8, 8, 4), (128, 128, 8, 8, 8, 0), (128, 128, 16, 8, 8, 4), (128, 64, 8, 8, 4, 4),
              (64, 128, 8, 4, 8, 4), (64, 64, 8, 4, 4, 0), (64, 64, 8, 4, 4, 4), (64, 64, 16, 4, 4, 4),
              (32, 64, 8, 2, 4, 4), (32, 32, 8, 2, 2, 0)]
# the TMA-fed kernel (gemm_simt_tma.cuh) on 16-byte-aligned operands, the cp.async kernel of the same tile elsewhere
FP32_TMA_TILES = [(64, 64, 16, 8, 8, 0), (64, 64, 32, 8, 8, 0), (128, 128, 16, 8, 8, 0), (128, 64, 16, 8, 8, 0),
                  (64, 128, 16, 8, 8, 0), (64, 32, 16, 8, 4, 0), (32, 64, 16, 4, 8, 0), (32, 32, 16, 4, 4, 0)]


@pytest.mark.parametrize("tile", FP32_TILES + FP32_TMA_TILES)
def test_fp32_cfg1_every_tile(ctx, oracle_mod, tile):
    w = wl.CONFIGS["cfg1_f32_512"]
    inp = wl.make_inputs(w)
    check_full(oracle_mod, w, inp, run_pf(ctx, w, inp, tile))


@pytest.mark.parametrize("shape", [(200, 136, 72), (1, 8, 4), (129, 257, 33), (77, 5, 9)])
def test_fp32_ragged_shapes(ctx, oracle_mod, shape):
    w = wl.scaled(wl.CONFIGS["cfg1_f32_512"], *shape)
    inp = wl.make_inputs(w, seed=7)
    for tile in [(128, 128, 8, 8, 8, 4), (64, 64, 8, 4, 4, 0), (64, 64, 16, 8, 8, 0), (32, 32, 16, 4, 4, 0)]:
        check_full(oracle_mod, w, inp, run_pf(ctx, w, inp, tile))


@pytest.mark.parametrize("ref_name", ["default", "best5050"])
def test_fp32_bit_identical_to_reference_kernel(ctx, oracle_mod, ref_name):
    path = oracle_mod.ref_kernel_path(ref_name)
    if not os.path.exists(path):
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    ref = oracle_mod.ref_kernel(ref_name)
    for w in (wl.CONFIGS["cfg1_f32_512"], wl.CONFIGS["cfg2_f32_2048"]):
        inp = wl.make_inputs(w)
        A, B, bias, C = device_operands(w, inp)
        C_ref = torch.full_like(C, float("nan"))
        rc = ref.ref_launch(A.data_ptr(), B.data_ptr(), bias.data_ptr(), C_ref.data_ptr(), w.M, w.N, w.K,
                            torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        mine = run_pf(ctx, w, inp, None, (A, B, bias, C))
        torch.cuda.synchronize()
        assert torch.equal(mine, C_ref), f"{w.name}: differs from the reference kernel ({ref_name})"
        for tile in FP32_TMA_TILES[:3] + FP32_TILES[:1]:  # TMA-fed and cp.async kernels, other tiles
            again = torch.full_like(C, float("nan"))
            run_pf(ctx, w, inp, tile, (A, B, bias, again))
            assert torch.equal(again, C_ref), f"{w.name}, tile {tile}: differs from the reference kernel"


def test_fp32_cfg2_gate_and_torch(ctx, oracle_mod):
    w = wl.CONFIGS["cfg2_f32_2048"]
    inp = wl.make_inputs(w)
    A, B, bias, C = device_operands(w, inp)
    run_pf(ctx, w, inp, None, (A, B, bias, C))
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= 1e-5
    assert max_rel_err_t(torch_fp32_reference(A, B, bias, 1.0), C) <= 1e-5


# ---------------------------------------------------------------------------------------------
# bf16 / e4m3 tensor-core path
# ---------------------------------------------------------------------------------------------
BF16_TILES = [(128, 256, 32, 4, 16, 0), (128, 256, 32, 2, 16, 0), (128, 128, 32, 4, 16, 0),
              (128, 128, 32, 8, 8, 0), (128, 64, 32, 8, 16, 0), (128, 64, 32, 4, 2, 0),
              (256, 256, 32, 8, 16, 0), (256, 256, 32, 4, 4, 0), (256, 256, 32, 2, 8, 0),
              (256, 256, 32, 8, 8, 1), (128, 256, 32, 2, 16, 1), (128, 128, 32, 8, 8, 1), (256, 224, 32, 8, 8, 1),
              (256, 224, 32, 3, 2, 1)]
E4M3_TILES = [(128, 256, 32, 4, 16, 0), (128, 256, 32, 2, 16, 0), (128, 128, 32, 4, 16, 0),
              (128, 128, 32, 8, 4, 0), (256, 256, 32, 8, 16, 0), (256, 256, 32, 4, 4, 0),
              (256, 256, 32, 8, 8, 1), (128, 256, 32, 2, 16, 1), (256, 224, 32, 8, 8, 1)]


@pytest.mark.parametrize("tile", BF16_TILES)
@pytest.mark.parametrize("shape", [(256, 512, 320), (200, 136, 72), (128, 256, 64), (1, 8, 8), (300, 1000, 1000)])
def test_bf16_small_vs_oracle(ctx, oracle_mod, tile, shape):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], *shape)
    inp = wl.make_inputs(w, seed=3)
    check_full(oracle_mod, w, inp, run_pf(ctx, w, inp, tile))


@pytest.mark.parametrize("tile", E4M3_TILES)
@pytest.mark.parametrize("shape", [(256, 512, 512), (200, 144, 80), (1, 16, 16), (384, 1024, 768)])
def test_e4m3_small_vs_oracle(ctx, oracle_mod, tile, shape):
    w = wl.scaled(wl.CONFIGS["cfg5_e4m3_16384"], *shape)
    inp = wl.make_inputs(w, seed=5)
    check_full(oracle_mod, w, inp, run_pf(ctx, w, inp, tile))


def test_mlp_shape_small_vs_oracle(ctx, oracle_mod):
    w = wl.scaled(wl.CONFIGS["cfg4_bf16_mlp"], 512, 1792, 512)
    inp = wl.make_inputs(w)
    check_full(oracle_mod, w, inp, run_pf(ctx, w, inp))


@pytest.mark.parametrize("name", ["cfg3_bf16_8192", "cfg4_bf16_mlp", "cfg5_e4m3_16384"])
def test_full_size_gate_torch_and_determinism(ctx, oracle_mod, name):
    w = wl.CONFIGS[name]
    inp = wl.make_inputs(w)
    ops = device_operands(w, inp)
    A, B, bias, C = ops
    run_pf(ctx, w, inp, None, ops)
    Cn = to_np(C)
    assert int(np.isnan(Cn).sum()) == 0
    scale = inp.scale_a * inp.scale_b
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, Cn, scale=scale, samples=512, seed=99)
    assert err <= TOL[w.dtype], f"sampled gate {err:.3e}"
    # whole rows against the oracle's fp64 result: 64 rows spread over every 128-row block of the launch (every
    # column tile, both CTAs of a pair, first and last row), not just the gate's 512 points
    rows = np.unique(np.concatenate([np.linspace(0, w.M - 1, 62).astype(np.int64), [1, w.M - 2]]))
    ref_rows = oracle_mod.full_f64(inp.A[rows], inp.B, inp.bias, scale)
    e_rows = oracle_mod.max_rel_err(ref_rows, Cn[rows])
    assert e_rows <= TOL[w.dtype], f"{len(rows)} whole rows vs the fp64 oracle: {e_rows:.3e}"
    ref = torch_fp32_reference(A, B, bias, scale)
    e2 = max_rel_err_t(ref, C)
    del ref
    assert e2 <= TOL[w.dtype], f"full-matrix error vs torch fp32 {e2:.3e}"
    # a second launch is bit-identical
    C2 = torch.full_like(C, float("nan"))
    run_pf(ctx, w, inp, None, (A, B, bias, C2))
    assert torch.equal(C, C2)


@pytest.mark.parametrize("G", [2, 3, 8])
def test_row_shards_equal_unsharded(ctx, pf, G):
    # Row sharding (the multi-GPU decomposition) on one GPU: each shard is its own launch on a row
    # window of A and C; the concatenation is bit-identical to the single launch (every tile whole:
    # stream-K off, since the tail's split depends on the launch shape).
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 2048, 1024, 768)
    inp = wl.make_inputs(w, seed=9)
    A, B, bias, C = device_operands(w, inp)
    ctx.set_stream_k(0)
    run_pf(ctx, w, inp, None, (A, B, bias, C))
    Cs = torch.full_like(C, float("nan"))
    for g in range(G):
        r0, n = pf.shard_rows(w.M, G, g, 128)
        if n == 0:
            continue
        ctx.prepare("bf16", None, n, w.N, w.K)
        ctx.bind(A[r0:r0 + n], B, bias, Cs[r0:r0 + n])
        ctx.launch(torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert ctx.status() == 0
    ctx.set_stream_k(-1)
    assert torch.equal(C, Cs)


def test_run_host_equals_device_path(ctx, pf):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 384, 512, 256)
    inp = wl.make_inputs(w, seed=2)
    C = run_pf(ctx, w, inp)
    hC = np.empty((w.M, w.N), dtype=np.uint16)
    ctx.prepare("bf16", None, w.M, w.N, w.K)
    ctx.run_host(inp.A_raw, inp.B_raw, inp.bias, hC)
    assert np.array_equal(hC, C.view(torch.int16).cpu().numpy().view(np.uint16))


def test_timing_protocol_and_attrs(ctx):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 1024, 1024, 1024)
    inp = wl.make_inputs(w)
    ctx.set_stream_k(0)  # whole tiles: the grid is min(resident CTAs or pairs, tiles)
    for tile, tiles, per_tile in (((128, 256, 32, 4, 16, 0), (1024 // 128) * (1024 // 256), 1),
                                  ((256, 256, 32, 8, 8, 1), (1024 // 256) * (1024 // 256), 2)):
        run_pf(ctx, w, inp, tile)
        ms = ctx.time(warmup=2, iters=5, reps=3)
        assert 0 < ms < 50
        a = ctx.attrs()
        # local_bytes is the per-thread stack frame (8 B of bookkeeping); ptxas reports 0 bytes of spills
        assert a["threads"] == 192 and a["blocks_per_sm"] == 1 and a["local_bytes"] <= 16
        assert a["num_sms"] == 148 and a["grid"] == min(a["num_sms"] // per_tile, tiles) * per_tile
    ctx.set_stream_k(-1)


def test_invalid_configs_are_errors(ctx, pf):
    with pytest.raises(pf.PFError) as e:
        ctx.prepare("bf16", (64, 256, 32, 4, 16, 0), 256, 256, 256)
    assert e.value.code == pf.PF_ETILE
    with pytest.raises(pf.PFError) as e:
        ctx.prepare("bf16", (128, 256, 16, 4, 16, 0), 256, 256, 256)  # 64-byte k-blocks: not built
    assert e.value.code == pf.PF_ETILE
    with pytest.raises(pf.PFError) as e:
        ctx.prepare("e4m3", (128, 64, 32, 4, 16, 0), 256, 256, 256)  # e4m3 B rows are 128 wide
    assert e.value.code == pf.PF_ETILE
    # TM is a requested pipeline depth, clamped to the deepest compiled variant that fits
    ctx.prepare("bf16", (128, 256, 32, 16, 16, 0), 256, 256, 256)
    with pytest.raises(pf.PFError) as e:
        ctx.prepare("bf16", None, 256, 100, 256)  # 200-byte rows of B and C: not a TMA row
    assert e.value.code == pf.PF_ESHAPE
    with pytest.raises(pf.PFError) as e:
        ctx.prepare("f32", (256, 256, 32, 16, 16, 8), 256, 256, 256)
    assert e.value.code == pf.PF_ETILE
    ctx.prepare("bf16", None, 256, 256, 256)
    with pytest.raises(pf.PFError) as e:
        ctx.launch()
    assert e.value.code == pf.PF_ESTATE


def test_bounded_wait_times_out_and_context_survives(ctx, oracle_mod):
    # A wait on an mbarrier that nothing arrives at runs out after 20 ms; the kernel records it and
    # returns, and the context keeps working.
    assert ctx.selftest_wait_timeout(20_000_000) != 0
    assert ctx.status() == 0
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 256, 256, 256)
    inp = wl.make_inputs(w)
    check_full(oracle_mod, w, inp, run_pf(ctx, w, inp))


def test_torch_convenience_api(pf):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 256, 512, 128)
    inp = wl.make_inputs(w)
    A, B, bias, _ = device_operands(w, inp)
    C = pf.gemm_bias_gelu(A, B, bias)
    torch.cuda.synchronize()
    ref = torch_fp32_reference(A, B, bias, 1.0)
    assert max_rel_err_t(ref, C) <= 2e-2


@pytest.mark.parametrize("name,shape", [("cfg2_f32_2048", None), ("cfg3_bf16_8192", (2048, 2048, 1024)),
                                        ("cfg5_e4m3_16384", (1024, 2048, 1024))])
def test_cublas_comparator(ctx, name, shape):
    # pf_time_cublas: cublasLt GEMM alone and GEMM + separate bias/GELU on the bound operands; the unfused
    # result it leaves in C agrees with the fused kernel within the dtype's tolerance.
    w = wl.CONFIGS[name] if shape is None else wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w)
    A, B, bias, C = device_operands(w, inp)
    fused = run_pf(ctx, w, inp, None, (A, B, bias, C)).clone()
    gemm_ms, unfused_ms = ctx.time_cublas(warmup=2, iters=5, reps=3)
    assert 0 < gemm_ms < unfused_ms
    torch.cuda.synchronize()
    assert max_rel_err_t(fused.float(), C.float()) <= TOL[w.dtype]


@pytest.mark.parametrize("name,shape,tile", [("cfg3_bf16_8192", (2048, 1024, 768), None),
                                             ("cfg3_bf16_8192", (4096, 4096, 512), None),   # 256 tiles: 3.5 waves
                                             ("cfg3_bf16_8192", (4096, 4096, 512), (128, 256, 32, 4, 16, 0)),
                                             ("cfg3_bf16_8192", (1000, 520, 264), (128, 256, 32, 4, 16, 0)),
                                             ("cfg5_e4m3_16384", (1536, 512, 512), None),
                                             ("cfg2_f32_2048", (1030, 256, 128), None)])
def test_pipelined_host_path_equals_device_path(ctx, name, shape, tile):
    # pf_run_host splits rows into chunks whose copies and kernels overlap; the result is the single launch's
    # (stream-K off on the single launch: the chunks run every tile whole).
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=17)
    ctx.set_stream_k(0)
    C = run_pf(ctx, w, inp, tile)
    ctx.set_stream_k(-1)
    hC = np.empty((w.M, w.N), dtype=np.float32 if w.dtype == "f32" else np.uint16)
    ctx.prepare(w.dtype, tile, w.M, w.N, w.K)
    ctx.run_host(inp.A_raw, inp.B_raw, inp.bias, hC, inp.scale_a, inp.scale_b)
    want = C.cpu().numpy() if w.dtype == "f32" else C.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(hC, want)


@pytest.mark.parametrize("chunks", [1, 3, 16, 64])
def test_host_chunks_do_not_change_the_result(ctx, pf, chunks):
    # pf_set_host_chunks: any number of row chunks gives the single launch's bits (stream-K off on the
    # single launch: 256 tiles are 3.5 waves, where the auto tail would split the last tiles' k range)
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 4096, 4096, 512)
    inp = wl.make_inputs(w, seed=19)
    ctx.set_stream_k(0)
    try:
        C = run_pf(ctx, w, inp)
        hC = np.empty((w.M, w.N), dtype=np.uint16)
        ctx.prepare(w.dtype, None, w.M, w.N, w.K)
        ctx.set_host_chunks(chunks)
        ctx.run_host(inp.A_raw, inp.B_raw, inp.bias, hC)
    finally:
        ctx.set_host_chunks(0)
        ctx.set_stream_k(-1)
    assert np.array_equal(hC, C.view(torch.int16).cpu().numpy().view(np.uint16))
    with pytest.raises(pf.PFError):
        ctx.set_host_chunks(65)


# ---------------------------------------------------------------------------------------------
# stream-K tail of the CTA-pair kernel
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name,shape,bn", [("cfg3_bf16_8192", (512, 2048, 4096), 256),    # 16 tiles < 74 pairs
                                           ("cfg3_bf16_8192", (1024, 8192, 2048), 256),   # 128 tiles: 1.73 waves
                                           ("cfg3_bf16_8192", (600, 1000, 1000), 256),    # ragged edges, K tail
                                           ("cfg5_e4m3_16384", (1024, 4096, 2048), 256),
                                           ("cfg3_bf16_8192", (600, 1000, 1000), 224),    # 224-wide tiles, tail box
                                           ("cfg5_e4m3_16384", (512, 2000, 2048), 224)])
def test_stream_k_tail_vs_oracle_and_whole_tiles(ctx, oracle_mod, name, shape, bn):
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=31)
    ops = device_operands(w, inp)
    A, B, bias, C = ops
    tile = (256, bn, 32, 8, 8, 1)
    ctx.set_stream_k(1)
    try:
        run_pf(ctx, w, inp, tile, ops)
        a = ctx.attrs()
        assert a["grid"] == 148  # the tail spreads over every resident pair
        ref = oracle_mod.full_f64(inp.A, inp.B, inp.bias, inp.scale_a * inp.scale_b)
        err = oracle_mod.max_rel_err(ref, to_np(C))
        assert err <= TOL[w.dtype], f"stream-K: {err:.3e}"
        C2 = torch.full_like(C, float("nan"))
        run_pf(ctx, w, inp, tile, (A, B, bias, C2))
        assert torch.equal(C, C2)  # deterministic for a given shape
        ctx.set_stream_k(0)
        C3 = torch.full_like(C, float("nan"))
        run_pf(ctx, w, inp, tile, (A, B, bias, C3))
        assert max_rel_err_t(C3.float(), C.float()) <= TOL[w.dtype]
    finally:
        ctx.set_stream_k(-1)


def test_stream_k_forced_at_full_size(ctx, oracle_mod, pf):
    w = wl.CONFIGS["cfg3_bf16_8192"]
    inp = wl.make_inputs(w)
    A, B, bias, C = device_operands(w, inp)
    ctx.set_stream_k(1)
    try:
        run_pf(ctx, w, inp, pf.DEFAULT_TILES["bf16"], (A, B, bias, C))  # the 256-wide kernel (stream-K tail)
    finally:
        ctx.set_stream_k(-1)
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= 2e-2
    assert max_rel_err_t(torch_fp32_reference(A, B, bias, 1.0), C) <= 2e-2


@pytest.mark.parametrize("name,rows", [("cfg3_bf16_8192", 1024), ("cfg3_bf16_8192", 2048), ("cfg4_bf16_mlp", 2048)])
def test_224_wide_tiles_on_row_shards(ctx, oracle_mod, pf, name, rows):
    # 224-wide pair tiles on the row shards of the 4- and 8-GPU runs; full-K parity on a row sample
    w = wl.CONFIGS[name]
    tile = (256, 224, 32, 8, 8, 1)
    ws = wl.scaled(w, rows, w.N, w.K)
    inp = wl.make_inputs(ws, seed=41)
    A, B, bias, C = device_operands(ws, inp)
    run_pf(ctx, ws, inp, tile, (A, B, bias, C))
    assert ctx.attrs()["grid"] == 2 * min(74, -(-rows // 256) * -(-w.N // 224))
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= TOL[ws.dtype]
    assert max_rel_err_t(torch_fp32_reference(A, B, bias, 1.0), C) <= TOL[ws.dtype]


# ---------------------------------------------------------------------------------------------
# 256 x 512 pair tiles (gemm_tc2w.cuh): one accumulator per CTA, handed back in two halves
# ---------------------------------------------------------------------------------------------
WIDE = (256, 512, 32, 4, 16, 0)      # 4 stages, one staging box per epilogue warp
WIDE8 = (256, 512, 32, 3, 16, 0)     # 3 stages, two staging boxes per epilogue warp (both: 8 epilogue warps)


@pytest.mark.parametrize("name,shape", [("cfg3_bf16_8192", (512, 1024, 512)),
                                        ("cfg3_bf16_8192", (600, 1000, 1000)),   # ragged; last half partly past N
                                        ("cfg3_bf16_8192", (300, 520, 264)),     # boxes wholly past N
                                        ("cfg3_bf16_8192", (256, 512, 64)),      # one k step, fewer than the stages
                                        ("cfg3_bf16_8192", (4096, 8192, 256)),   # 3.5 tiles per pair, 4 k steps each
                                        ("cfg5_e4m3_16384", (1024, 2048, 1024)),
                                        ("cfg5_e4m3_16384", (600, 1008, 1008)),  # e4m3 rows: 16-byte multiples
                                        ("cfg5_e4m3_16384", (4096, 8192, 384))])
@pytest.mark.parametrize("tile", [WIDE, WIDE8])
def test_512_wide_tiles_vs_oracle_and_256_wide(ctx, oracle_mod, name, shape, tile):
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=43)
    A, B, bias, C = device_operands(w, inp)
    run_pf(ctx, w, inp, tile, (A, B, bias, C))
    assert ctx.attrs()["threads"] == 320
    assert ctx.attrs()["grid"] == 2 * min(74, -(-w.M // 256) * -(-w.N // 512))
    if w.M * w.N * w.K <= 2 ** 30:
        check_full(oracle_mod, w, inp, C)
    else:
        err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), inp.scale_a * inp.scale_b, samples=512,
                                            seed=99)
        assert err <= TOL[w.dtype]
    again = torch.full_like(C, float("nan"))
    run_pf(ctx, w, inp, tile, (A, B, bias, again))
    assert torch.equal(C, again)
    narrow = torch.full_like(C, float("nan"))
    run_pf(ctx, w, inp, None, (A, B, bias, narrow))
    assert max_rel_err_t(narrow.float(), C.float()) <= TOL[w.dtype]


@pytest.mark.parametrize("name", ["cfg3_bf16_8192", "cfg4_bf16_mlp"])
@pytest.mark.parametrize("tile", [WIDE, WIDE8])
def test_512_wide_tiles_at_full_size(ctx, oracle_mod, name, tile):
    w = wl.CONFIGS[name]
    inp = wl.make_inputs(w)
    A, B, bias, C = device_operands(w, inp)
    run_pf(ctx, w, inp, tile, (A, B, bias, C))
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= TOL[w.dtype]
    assert max_rel_err_t(torch_fp32_reference(A, B, bias, 1.0), C) <= TOL[w.dtype]


@pytest.mark.parametrize("rows", [1024, 2048])
def test_512_wide_tiles_on_row_shards(ctx, oracle_mod, pf, rows):
    # the 8- and 4-GPU row shards of config 3, where default_tile picks 256 x 512 tiles (whole tiles: row-band
    # stream-K is opt-in), and the same shards with row-band stream-K forced on (4 / 8 bands of 18 / 9 pairs)
    w = wl.CONFIGS["cfg3_bf16_8192"]
    ws = wl.scaled(w, rows, w.N, w.K)
    assert pf.default_tile(ws.dtype, rows, ws.N, ws.K) == pf.WIDE_TILE_DEEP
    inp = wl.make_inputs(ws, seed=53)
    A, B, bias, C = device_operands(ws, inp)
    run_pf(ctx, ws, inp, None, (A, B, bias, C))
    assert ctx.attrs()["threads"] == 320
    assert ctx.attrs()["grid"] == 2 * min(74, (rows // 256) * 16)
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= TOL[ws.dtype]
    ref = torch_fp32_reference(A, B, bias, 1.0)
    assert max_rel_err_t(ref, C) <= TOL[ws.dtype]
    ctx.set_stream_k(2)
    try:
        band = torch.full_like(C, float("nan"))
        run_pf(ctx, ws, inp, None, (A, B, bias, band))
        bands = rows // 256
        assert ctx.attrs()["grid"] == 2 * bands * (74 // bands)
    finally:
        ctx.set_stream_k(-1)
    assert max_rel_err_t(ref, band) <= TOL[ws.dtype]


@pytest.mark.parametrize("tile", [WIDE, WIDE8])
def test_512_wide_tiles_host_path_equals_device_path(ctx, tile):
    # row chunks of 512-wide tiles keep the whole launch's k order: the same bits
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 4096, 4096, 512)
    inp = wl.make_inputs(w, seed=47)
    C = run_pf(ctx, w, inp, tile)
    hC = np.empty((w.M, w.N), dtype=np.uint16)
    ctx.prepare(w.dtype, tile, w.M, w.N, w.K)
    ctx.run_host(inp.A_raw, inp.B_raw, inp.bias, hC)
    assert np.array_equal(hC, C.view(torch.int16).cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("name,shape", [("cfg3_bf16_8192", (2048, 1024, 768)), ("cfg5_e4m3_16384", (1000, 512, 512)),
                                        ("cfg3_bf16_8192", (4096, 4096, 512)),
                                        ("cfg3_bf16_8192", (2048, 4096, 8192)),  # default: 256 x 512 tiles
                                        ("cfg2_f32_2048", (1030, 256, 128))])
def test_run_host_rows_equals_device_path(ctx, name, shape):
    # pf_run_host_rows: B and bias already on the device (bound); host rows of A in, C rows out, in chunks
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=23)
    A, B, bias, C = device_operands(w, inp)
    ctx.set_stream_k(0)
    try:
        run_pf(ctx, w, inp, None, (A, B, bias, C))
        A2, C2 = torch.zeros_like(A), torch.full_like(C, float("nan"))
        ctx.prepare(w.dtype, None, w.M, w.N, w.K)
        if shape == (2048, 4096, 8192):
            assert ctx.tile.BN == 512  # the 4- and 8-GPU e2e path's tiles
        ctx.bind(A2, B, bias, C2, inp.scale_a, inp.scale_b)
        hA = torch.from_numpy(np.ascontiguousarray(inp.A_raw)).pin_memory()
        hC = torch.empty(C.numel() * C.element_size(), dtype=torch.uint8).pin_memory()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        ctx.run_host_rows(hA, hC, after_stream=torch.cuda.current_stream(), copies_after_stream=side)
        assert ctx.status() == 0
    finally:
        ctx.set_stream_k(-1)
    want = C.reshape(-1).view(torch.uint8).cpu()
    assert torch.equal(hC, want)
    assert torch.equal(A2.reshape(-1).view(torch.uint8).cpu(), hA.reshape(-1).view(torch.uint8))


# ---------------------------------------------------------------------------------------------
# row-band stream-K of the pair kernels: each row block of tiles shared by 74 // (row blocks) pairs
# ---------------------------------------------------------------------------------------------
PAIR256 = (256, 256, 32, 8, 16, 1)   # 256 x 256 pair tiles, two k-atoms per stage


@pytest.mark.parametrize("name,shape,tile", [
    ("cfg3_bf16_8192", (512, 2048, 1024), PAIR256),   # 256 x 256 tiles: 2 bands of 37 pairs
    ("cfg3_bf16_8192", (1024, 4096, 1024), PAIR256),  # 4 bands of 18 pairs: 2-3 pairs per tile
    ("cfg3_bf16_8192", (700, 1504, 600), PAIR256),    # ragged M, N and K
    ("cfg5_e4m3_16384", (1024, 2048, 2048), PAIR256),
    ("cfg3_bf16_8192", (512, 2048, 1024), WIDE8),     # 2 bands of 37 pairs, ~1.7 k-blocks each: many contributors
    ("cfg3_bf16_8192", (1024, 4608, 512), WIDE8),     # 4 bands of 18 pairs: 2-3 pairs per tile
    ("cfg3_bf16_8192", (700, 1504, 600), WIDE8),      # ragged M, N and K
    ("cfg3_bf16_8192", (1024, 4608, 512), WIDE),      # 4 stages, one staging box per epilogue warp
    ("cfg3_bf16_8192", (256, 8192, 2048), WIDE8),     # 1 band of 74 pairs
    ("cfg5_e4m3_16384", (512, 2048, 2048), WIDE8),
    ("cfg5_e4m3_16384", (1024, 4608, 1024), WIDE8)])
def test_band_stream_k_vs_oracle_and_whole_tiles(ctx, oracle_mod, name, shape, tile):
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=59)
    A, B, bias, C = device_operands(w, inp)
    ctx.set_stream_k(2)
    try:
        run_pf(ctx, w, inp, tile, (A, B, bias, C))
        bands = -(-w.M // 256)
        assert ctx.attrs()["grid"] == 2 * bands * (74 // bands)
        if w.M * w.N * w.K <= 2 ** 30:
            check_full(oracle_mod, w, inp, C)
        else:
            assert int(torch.isnan(C.float()).sum()) == 0
            err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), inp.scale_a * inp.scale_b,
                                                samples=512, seed=99)
            assert err <= TOL[w.dtype]
            assert max_rel_err_t(torch_fp32_reference(A, B, bias, inp.scale_a * inp.scale_b), C) <= TOL[w.dtype]
        again = torch.full_like(C, float("nan"))
        run_pf(ctx, w, inp, tile, (A, B, bias, again))
        assert torch.equal(C, again)  # deterministic for a given shape
        ctx.set_stream_k(0)
        whole = torch.full_like(C, float("nan"))
        run_pf(ctx, w, inp, tile, (A, B, bias, whole))
        assert ctx.attrs()["grid"] == 2 * min(74, bands * -(-w.N // tile[1]))
        assert max_rel_err_t(whole.float(), C.float()) <= TOL[w.dtype]
    finally:
        ctx.set_stream_k(-1)


def test_band_stream_k_on_the_8_gpu_shard(ctx, oracle_mod, pf):
    # 1,024 x 8192 x 8192 on 256 x 256 tiles: whole tiles need two waves (128 tiles, 74 pairs); row-band mode
    # splits each of the 4 row blocks' k-iterations over 18 pairs instead
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 1024, 8192, 8192)
    inp = wl.make_inputs(w, seed=61)
    A, B, bias, C = device_operands(w, inp)
    run_pf(ctx, w, inp, PAIR256, (A, B, bias, C))
    assert ctx.attrs()["grid"] == 148  # auto: whole tiles
    ctx.set_stream_k(2)
    try:
        run_pf(ctx, w, inp, PAIR256, (A, B, bias, C))
        assert ctx.attrs()["grid"] == 2 * 4 * 18
    finally:
        ctx.set_stream_k(-1)
    err, _, _ = oracle_mod.sampled_gate(inp.A, inp.B, inp.bias, to_np(C), samples=512, seed=99)
    assert err <= TOL[w.dtype]
    assert max_rel_err_t(torch_fp32_reference(A, B, bias, 1.0), C) <= TOL[w.dtype]
