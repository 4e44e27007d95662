"""python -m ptxforge_b200.timetiles on a B200 (-m gpu): the interleaved A/B that the tile and build comparisons of
this repository were measured with runs, reports every candidate, and compares their outputs bit for bit."""
import pytest

pytestmark = pytest.mark.gpu


def test_timetiles_reports_every_candidate_and_their_bits():
    from ptxforge_b200 import timetiles
    # two SIMT tiles give the same bits (the reference kernel's fmaf chain); two bf16 stage counts too
    line = timetiles.main(["f32", "256", "256", "256", "--tiles", "default", "64,32,16,8,4,0", "--bursts", "2",
                           "--iters", "3", "--pause", "0"])
    assert line["same_bits_as_first"] == [True]
    assert line["status"] == [0, 0]
    assert len(line["us_median"]) == 2 and all(v > 0 for v in line["us_median"].values())
    line = timetiles.main(["bf16", "512", "1024", "512", "--tiles", "256,512,32,4,16,0", "256,512,32,3,16,0",
                           "--bursts", "2", "--iters", "3", "--pause", "0", "--cublas"])
    assert line["same_bits_as_first"] == [True]
    assert line["status"] == [0, 0]
    assert "cublas_gemm" in line["us_median"]
