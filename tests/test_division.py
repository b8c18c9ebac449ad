"""The blend divides each weighted neighbour value by the frame's weight sum
in f64, correctly rounded like the reference's `/`
(crates/vocal-cpu/src/retrieval.rs:73-79).  The CUDA path replaces the
divide instruction sequence by Markstein's refinement with a precomputed
reciprocal (divide_by in vocal-fast-rs_b200/csrc/exact_common.cuh); this
test runs the same IEEE operations on the host (tests/division_check.c)
against the correctly rounded quotient."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_markstein_quotient_is_correctly_rounded(tmp_path):
    exe = tmp_path / "division_check"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", str(exe), os.path.join(HERE, "division_check.c"), "-lm"],
                   check=True)
    out = subprocess.run([str(exe), "8000000"], capture_output=True, text=True)
    cases, mismatches = (int(x) for x in out.stdout.split())
    assert cases > 7_000_000
    assert mismatches == 0, out.stderr
