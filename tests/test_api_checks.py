"""Host-side operand checks of ptxforge_b200.gemm_bias_gelu (no GPU needed): the kernels read and write
exactly the shapes and element widths of the dtype through TMA, so anything else is refused before a launch."""
import pytest

torch = pytest.importorskip("torch")

import ptxforge_b200 as pf  # noqa: E402


def ops(M=64, N=32, K=48, ab=torch.bfloat16, out=torch.bfloat16):
    return (torch.zeros(M, K, dtype=ab), torch.zeros(K, N, dtype=ab), torch.zeros(N, dtype=torch.float32),
            torch.zeros(M, N, dtype=out))


def check(A, B, bias, C, dtype):
    return pf.check_operands(A, B, bias, C, dtype, require_cuda=False)


def test_valid_operands_give_the_problem_size():
    assert check(*ops(), "bf16") == (64, 32, 48)
    assert check(*ops(ab=torch.uint8), "e4m3") == (64, 32, 48)
    assert check(*ops(ab=torch.float8_e4m3fn), "e4m3") == (64, 32, 48)
    assert check(*ops(ab=torch.float32, out=torch.float32), "f32") == (64, 32, 48)
    assert check(*ops(ab=torch.float32, out=torch.float32), "f32_3xtf32") == (64, 32, 48)


@pytest.mark.parametrize("mutate,needle", [
    (lambda A, B, b, C: (A, B, b, torch.zeros(63, 32, dtype=torch.bfloat16)), "C must be 64 x 32"),
    (lambda A, B, b, C: (A, B, b, torch.zeros(64, 32, dtype=torch.float32)), "C has 4-byte"),
    (lambda A, B, b, C: (A.float(), B, b, C), "A has 4-byte"),
    (lambda A, B, b, C: (A, B[:40], b, C), "shape mismatch"),
    (lambda A, B, b, C: (A, B, b[:31], C), "shape mismatch"),
    (lambda A, B, b, C: (A.t().contiguous().t(), B, b, C), "contiguous"),
    (lambda A, B, b, C: (A, B, b.double(), C), "bias has 8-byte"),
    (lambda A, B, b, C: (A, B, b.int(), C), "bias must be float32"),
    (lambda A, B, b, C: (A.reshape(-1), B, b, C), "matrices"),
])
def test_mismatched_operands_are_refused(mutate, needle):
    with pytest.raises(ValueError, match=needle):
        check(*mutate(*ops()), "bf16")


def test_host_tensors_are_refused_before_any_launch():
    with pytest.raises(ValueError, match="CUDA tensor"):
        pf.gemm_bias_gelu(*ops()[:3], dtype="bf16")
    with pytest.raises(ValueError, match="unknown dtype"):
        pf.gemm_bias_gelu(*ops()[:3], dtype="fp16")


def test_noalloc_checks_torch_operands_before_the_c_abi():
    """pf_gemm_bias_gelu_noalloc's Python view refuses what gemm_bias_gelu refuses, and more: its M, N, K
    arguments must equal the operands' shapes and every operand must sit on `device` -- before the C ABI,
    which would hand the pointers to TMA maps of the stated sizes."""
    A, B, bias, C = ops()
    tile = (128, 256, 32, 4, 16, 0)
    with pytest.raises(ValueError, match="C must be 64 x 32"):
        pf.gemm_bias_gelu_noalloc(0, "bf16", tile, 64, 32, 48, A, B, bias, torch.zeros(32, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="A has 4-byte"):
        pf.gemm_bias_gelu_noalloc(0, "bf16", tile, 64, 32, 48, A.float(), B, bias, C)
    with pytest.raises(ValueError, match="but M, N, K = 128, 32, 48"):
        pf.gemm_bias_gelu_noalloc(0, "bf16", tile, 128, 32, 48, A, B, bias, C)
    with pytest.raises(ValueError, match="CUDA tensor on device 0"):
        pf.gemm_bias_gelu_noalloc(0, "bf16", tile, 64, 32, 48, A, B, bias, C)


def test_timetiles_cli_refuses_unknown_dtypes_before_touching_a_gpu():
    """python -m ptxforge_b200.timetiles: argument errors end the run before any operand or context exists."""
    import pytest
    from ptxforge_b200 import timetiles
    with pytest.raises(SystemExit):
        timetiles.main(["fp64", "16", "16", "16"])
    with pytest.raises(SystemExit):
        timetiles.main(["bf16", "16", "16"])
