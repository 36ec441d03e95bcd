"""The reference's own test programs, unchanged, against this library.

oracle/_ref/gemm_test_b200 and elementwise_test_b200 are the reference's tests/gemm_test.cu and
tests/elementwise_test.cu compiled against include/cuvit/kernels.hpp; vit_test_b200 is its
tests/vit_test.cu compiled against include/cuvit/vit.hpp (with the reference's own WeightFile
and CPU reference); all linked with libcuvit_b200.so (oracle/Makefile, target ref-tests). Each
exits 0 and prints PASS only if every check in it holds at the reference's own tolerances.
"""

from __future__ import annotations

import pathlib
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PROGRAMS = ["gemm_test_b200", "elementwise_test_b200", "vit_test_b200"]

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("program", PROGRAMS)
def test_reference_test_program_passes(program, cuda):
    path = ROOT / "oracle" / "_ref" / program
    if not path.exists():
        pytest.skip(f"{path} not built (make -C oracle ref-tests needs the reference sources)")
    result = subprocess.run([str(path)], capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stdout + result.stderr
    assert "PASS" in result.stdout
