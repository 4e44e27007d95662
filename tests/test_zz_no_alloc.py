"""The no-allocation entry point, pf_gemm_bias_gelu_noalloc, through the C ABI (needs a B200: -m gpu).

Some callers cannot allocate GPU memory at the moment they call this library: a serving process that
reserved nearly all of HBM for its own memory pool at start-up (a cudaMalloc then fails, or forces the
pool to give memory back), or a multi-stream pipeline that cannot take the device-wide synchronisation a
cudaFree brings.  For them the tensor-core kernel also runs without a context: its only scratch, the
device status word, sits in a fixed array compiled into the library.

Checked: two calls in a row produce the same C as the context-based entry point (pf_prepare / pf_bind /
pf_launch) -- within the tolerance the parity tests use, and bit for bit on these shapes, where both run
whole tiles (pf_launch's automatic stream-K tail starts at three waves of tiles; the no-allocation call
never runs it) -- and each is also within tolerance of the oracle's fp64 result on the same inputs; the
calls leave the device's free memory unchanged; requests it cannot serve are refused with a message.  The
file name makes pytest collect it last, so a failure here comes after every other test has run; it also
passes alone.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ptxforge_b200 import workloads as wl  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = {"bf16": 2e-2, "e4m3": 5e-2}


def _operands(w, inp):
    def dev(x):
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        return t.view(torch.int16).view(torch.bfloat16) if w.dtype == "bf16" else t.view(torch.float8_e4m3fn)

    return dev(inp.A_raw), dev(inp.B_raw), torch.from_numpy(inp.bias).cuda()


def _nan_c(w):
    return torch.full((w.M, w.N), float("nan"), device="cuda", dtype=torch.bfloat16)


def _max_rel_err(ref, C):
    r = ref.double()
    return float(((r - C.double()).abs() / (1.0 + r.abs())).max())


CASES = [("cfg3_bf16_8192", (128, 256, 32, 4, 16, 0), (512, 768, 640)),
         ("cfg3_bf16_8192", (256, 256, 32, 8, 16, 0), (512, 768, 640)),
         ("cfg3_bf16_8192", (128, 256, 32, 4, 16, 0), (200, 136, 72)),
         ("cfg5_e4m3_16384", (128, 256, 32, 4, 16, 0), (384, 512, 768)),
         ("cfg3_bf16_8192", (256, 512, 32, 3, 16, 0), (512, 1024, 640)),   # 256 x 512 pair tiles
         ("cfg5_e4m3_16384", (256, 512, 32, 3, 16, 0), (384, 1024, 768))]


@pytest.mark.parametrize("name,tile,shape", CASES)
def test_two_calls_match_the_context_entry_point(pf, ctx, oracle_mod, name, tile, shape):
    w = wl.scaled(wl.CONFIGS[name], *shape)
    inp = wl.make_inputs(w, seed=21)
    A, B, bias = _operands(w, inp)
    stream = torch.cuda.current_stream()
    ref64 = oracle_mod.full_f64(inp.A, inp.B, inp.bias, inp.scale_a * inp.scale_b)

    C_ref = _nan_c(w)
    ctx.prepare(w.dtype, tile, w.M, w.N, w.K)
    ctx.bind(A, B, bias, C_ref, inp.scale_a, inp.scale_b)
    ctx.launch(stream)
    torch.cuda.synchronize()
    assert ctx.status() == 0

    for _ in range(2):  # two calls in a row into fresh outputs
        C = _nan_c(w)
        status = pf.gemm_bias_gelu_noalloc(0, w.dtype, tile, w.M, w.N, w.K, A, B, bias, C, inp.scale_a,
                                           inp.scale_b, stream=stream, sync=True)
        assert status == 0
        assert not torch.isnan(C.float()).any()
        assert _max_rel_err(C_ref.float(), C.float()) <= TOL[w.dtype]
        assert oracle_mod.max_rel_err(ref64, C.float().cpu().numpy()) <= TOL[w.dtype]
        assert torch.equal(C, C_ref)


def test_calls_leave_free_device_memory_unchanged(pf):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 1024, 1024, 512)
    inp = wl.make_inputs(w, seed=22)
    A, B, bias = _operands(w, inp)
    C = _nan_c(w)
    tile = (128, 256, 32, 4, 16, 0)
    pf.gemm_bias_gelu_noalloc(0, "bf16", tile, w.M, w.N, w.K, A, B, bias, C)  # first call: per-device set-up
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        pf.gemm_bias_gelu_noalloc(0, "bf16", tile, w.M, w.N, w.K, A, B, bias, C)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_requests_it_cannot_serve_are_refused(pf):
    w = wl.scaled(wl.CONFIGS["cfg3_bf16_8192"], 128, 256, 64)
    inp = wl.make_inputs(w)
    A, B, bias = _operands(w, inp)
    C = _nan_c(w)
    # the C ABI's own refusals, reached with raw device pointers (a C caller's view: no shapes to check)
    ptrs = [t.data_ptr() for t in (A, B, bias, C)]
    with pytest.raises(pf.PFError) as e:
        pf.gemm_bias_gelu_noalloc(0, "f32", (128, 128, 8, 8, 8, 4), w.M, w.N, w.K, *ptrs)
    assert e.value.code == pf.PF_EINVAL and "tensor-core" in str(e.value)
    with pytest.raises(pf.PFError) as e:
        pf.gemm_bias_gelu_noalloc(0, "bf16", (64, 256, 32, 4, 16, 0), w.M, w.N, w.K, *ptrs)
    assert e.value.code == pf.PF_ETILE and "no tensor-core kernel" in str(e.value)
    with pytest.raises(pf.PFError) as e:
        pf.gemm_bias_gelu_noalloc(0, "bf16", None, w.M, 100, w.K, *ptrs)
    assert e.value.code == pf.PF_ESHAPE
    other = torch.cuda.Stream()  # any stream of this device is accepted
    other.wait_stream(torch.cuda.current_stream())
    assert pf.gemm_bias_gelu_noalloc(0, "bf16", None, w.M, w.N, w.K, A, B, bias, C, stream=other) == 0
    # torch operands whose shapes disagree with M, N, K never reach the C ABI
    with pytest.raises(ValueError, match="but M, N, K"):
        pf.gemm_bias_gelu_noalloc(0, "bf16", None, w.M, 128, w.K, A, B, bias, C)
