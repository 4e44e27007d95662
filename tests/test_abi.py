"""The C-ABI library loads without a GPU and exports exactly what include/pf_b200.h declares (CPU only)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "pf_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pf_[a-z_0-9]+)\s*\(", text)))


def test_header_matches_python_symbol_list(pf):
    assert declared_functions() == sorted(pf.SYMBOLS)


def test_library_exports_every_declared_symbol(pf):
    lib = ctypes.CDLL(pf.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_sizes(pf):
    assert "sm_100a" in pf.version()
    lib = pf.load_library()
    assert [lib.pf_elem_bytes(d) for d in (0, 1, 2, 3)] == [4, 4, 2, 1]
    assert [lib.pf_out_bytes(d) for d in (0, 1, 2, 3)] == [4, 4, 2, 2]
    assert lib.pf_elem_bytes(99) == 0


def test_null_arguments_are_errors_not_crashes(pf):
    lib = pf.load_library()
    assert lib.pf_open(0, None) == pf.PF_EINVAL
    assert lib.pf_close(None) == pf.PF_EINVAL
    assert lib.pf_prepare(None, 2, None, 1, 1, 1) == pf.PF_EINVAL
    assert lib.pf_launch(None, None) == pf.PF_EINVAL
    assert lib.pf_last_error(None) == b"null context"


def test_open_without_gpu_reports_nodev(pf):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(pf.PFError) as e:
        pf.Context(0)
    assert e.value.code == pf.PF_ENODEV


@pytest.mark.parametrize("M,G,align", [(8192, 1, 128), (8192, 2, 128), (8192, 8, 128), (16384, 8, 128),
                                       (1000, 3, 128), (100, 8, 128), (8192, 7, 128), (5, 2, 1)])
def test_shard_rows_partition(pf, M, G, align):
    spans = [pf.shard_rows(M, G, g, align) for g in range(G)]
    pos = 0
    for g, (r0, n) in enumerate(spans):
        assert r0 == pos and n >= 0
        if g < G - 1:
            assert r0 % align == 0 and (r0 + n) % align == 0
        pos += n
    assert pos == M
    sizes = [n for _, n in spans[:-1]]
    if sizes and M >= align * G:
        assert max(sizes) - min(sizes) <= align


def test_shard_rows_rejects_bad_arguments(pf):
    with pytest.raises(pf.PFError):
        pf.shard_rows(100, 2, 2)
    with pytest.raises(pf.PFError):
        pf.shard_rows(0, 1, 0)


def test_default_tile_choice_follows_the_measurements():
    """224-wide pair tiles only where the 256-wide schedule leaves a nearly empty last wave (measured on B200)."""
    import ptxforge_b200 as pf
    assert pf.default_tile("bf16", 2048, 14336)[1] == 224      # MLP shard at 8 GPUs: 448 tiles, 4 in the last wave
    for rows, N in [(1024, 8192), (2048, 8192), (4096, 14336), (8192, 8192), (16384, 14336)]:
        assert pf.default_tile("bf16", rows, N) == pf.DEFAULT_TILES["bf16"], (rows, N)
    assert pf.default_tile("f32", 2048, 2048) == (64, 32, 16, 8, 4, 0)
    # 256 x 512 tiles for long tiles whose waves are full (1 GPU); the 256-wide kernel elsewhere
    assert pf.default_tile("bf16", 8192, 8192, 8192) == pf.WIDE_TILE_DEEP     # 512 tiles, 128 k steps; bf16: 4 stages
    assert pf.default_tile("e4m3", 16384, 16384, 16384) == pf.WIDE_TILE       # 2048 tiles, 128 k steps
    assert pf.default_tile("bf16", 16384, 14336, 4096) == pf.DEFAULT_TILES["bf16"]   # 64 k steps
    # row shards of 8192^3: 512-wide where both widths fill their waves alike (1,024 and 2,048 rows), 256-wide
    # where 512-wide tiles would fill 86.5 % against 98.8 % (4,096 rows)
    assert pf.default_tile("bf16", 1024, 8192, 8192) == pf.WIDE_TILE_DEEP   # 64 tiles: one per pair, 4 stages
    assert pf.default_tile("bf16", 2048, 8192, 8192) == pf.WIDE_TILE_DEEP
    assert pf.default_tile("bf16", 4096, 8192, 8192) == pf.DEFAULT_TILES["bf16"]
    assert pf.default_tile("e4m3", 2048, 16384, 16384) == pf.DEFAULT_TILES["e4m3"]  # 3.5 vs 6.9 waves
    # fp32 SIMT (same bits on every tile): small tiles for small problems, the TMA-fed kernel's 64 x 32 tiles up to
    # ~2900^2 outputs, 128 x 64 above
    assert pf.default_tile("f32", 512, 512) == (32, 32, 32, 4, 2, 2)
    assert pf.default_tile("f32", 1024, 1024) == (64, 32, 16, 8, 4, 0)
    assert pf.default_tile("f32", 1536, 1536) == (64, 32, 16, 8, 4, 0)
    assert pf.default_tile("f32", 4096, 4096) == pf.DEFAULT_TILES["f32"]
    assert pf.default_tile("f32_3xtf32", 512, 512) == pf.DEFAULT_TILES["f32_3xtf32"]
