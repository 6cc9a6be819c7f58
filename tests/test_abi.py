"""The wire structs in include/gfd/ are byte-compatible with the reference.

tests/golden/abi_layout.json was printed by abi_probe.cpp compiled against the
reference headers (tests/golden/make_golden.py); here the same probe is compiled
against include/gfd and every size, alignment, offset and constant must match.
"""
import json
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def test_wire_layout_matches_reference(tmp_path):
    exe = tmp_path / "abi_ours"
    subprocess.check_call(["g++", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                           "-I", "/usr/local/cuda/include", os.path.join(GOLD, "abi_probe.cpp"),
                           "-o", str(exe)])
    ours = json.loads(subprocess.check_output([str(exe)], text=True))
    ref = json.load(open(os.path.join(GOLD, "abi_layout.json")))
    assert ours == ref


def test_host_headers_compile_standalone(tmp_path):
    # every host header compiles on its own with a plain C++ compiler
    for h in ("gfd.h", "descriptor_queue.h", "tiled_queue.h", "sg_task_queue.h", "copy_engine.h",
              "cpu_polling.h", "warp_spec_session.h", "staging_pool.h", "pcie_topology.h", "log.h"):
        src = tmp_path / "inc.cpp"
        src.write_text(f'#include "gfd/{h}"\nint main() {{ return 0; }}\n')
        subprocess.check_call(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                               "-I", "/usr/local/cuda/include", str(src)])


def test_c_abi_header_is_plain_c(tmp_path):
    src = tmp_path / "c.c"
    src.write_text('#include "gfd_b200.h"\nint main(void) { gfd_sg_entry e; (void)e; return 0; }\n')
    subprocess.check_call(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I",
                           os.path.join(ROOT, "include"), str(src)])
