"""Drop-in check: the reference's own test programs and examples, compiled unmodified
against include/gfd and libgfd_b200.so (tests/cpp_build.py, build_dropin), run on the
GPU and must report success.  The binaries live in oracle/_ref/dropin/ (built where the
reference checkout exists); without them these tests are skipped."""
import os
import re
import subprocess

import pytest

from tests import cpp_build

pytestmark = pytest.mark.gpu

# order: programs that only use this library's bounded waits first; the two programs
# whose own hand-written kernels spin on the drain's signals come last
ORDER = ["test_db_small_tiles", "test_sg_e2e", "ex02_direct_transfer", "ex01_basic_transfer",
         "ex03_gpu_planned_transfer", "ex07_warp_spec_simple", "test_sg_gpu_submit", "ex09_sg_warp_spec"]


@pytest.mark.parametrize("name", ORDER)
def test_reference_program(name):
    exe = os.path.join(cpp_build.DROPIN_DIR, name)
    if not os.path.exists(exe):
        pytest.skip("reference programs not built here (needs the reference checkout at build time)")
    r = subprocess.run([exe], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=180,
                       cwd=os.path.dirname(exe))
    out = r.stdout
    print(out[-4000:])
    assert r.returncode == 0, out[-2000:]
    assert re.search(r"\bPASS(ED)?\b", out), out[-2000:]
    assert not re.search(r"\bFAIL(ED)?\b", out), out[-2000:]
