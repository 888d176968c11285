"""The host-side copy splitter (charsiu_b200/csrc/host_copy.h, cgpu::ParCopy)
on the CPU: the large int8 jobs' operands and outputs and the direct calls'
outputs go through it, cut into 16 KB items for the decode loop's thread pool
(charsiu_b200/host/pool.c). tests/host_copy_check.cpp copies random segment
sets across the item edges, alone and on pools of 1, 3 and 7 workers, and
checks every byte and the guard bytes around each destination."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "charsiu_b200", "csrc")
HOST = os.path.join(ROOT, "charsiu_b200", "host")


@pytest.mark.skipif(shutil.which("g++") is None or shutil.which("gcc") is None,
                    reason="needs gcc and g++")
def test_parcopy_copies_every_segment_exactly(tmp_path):
    pool_o = tmp_path / "pool.o"
    exe = tmp_path / "host_copy_check"
    subprocess.run(["gcc", "-O2", "-std=c11", "-pthread", "-c", os.path.join(HOST, "pool.c"),
                    "-o", str(pool_o)], check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", f"-I{CSRC}",
                    os.path.join(ROOT, "tests", "host_copy_check.cpp"), str(pool_o),
                    "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("ok 400"), out.stdout
