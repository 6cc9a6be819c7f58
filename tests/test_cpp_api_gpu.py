"""The C++ drop-in API on the GPU: GPU-queued submit drained by GPU kernels,
WarpSpecSession (single and double buffer), SGWarpSpecSession (host- and
GPU-submitted lists).  Each program checks its own results byte-exact against the
host source (or exact sums) and prints PASS/FAIL per case."""
import os
import subprocess

import pytest

from tests import cpp_build

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def binaries():
    return {os.path.basename(p): p for p in cpp_build.build_all()}


@pytest.mark.parametrize("prog", cpp_build.PROGRAMS)
def test_cpp_program(binaries, prog):
    r = subprocess.run([binaries[prog]], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                       timeout=240)
    print(r.stdout)
    lines = [l for l in r.stdout.splitlines() if l.startswith(("PASS", "FAIL"))]
    assert lines, r.stdout
    assert not [l for l in lines if l.startswith("FAIL")], r.stdout
    assert r.returncode == 0, r.stdout
