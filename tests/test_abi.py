"""The C-ABI boundary, without a GPU: the library loads, exports exactly what
include/*.h declares, and the struct layouts it reads match charsiu's own
headers byte for byte."""
import os
import re
import subprocess

import pytest

from charsiu_b200 import lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
# the reference's source tree: REF in the environment, else `reference` beside
# this repository (as oracle/Makefile takes it)
REF_INCLUDE = os.path.join(os.environ.get("REF", os.path.join(os.path.dirname(ROOT), "reference")),
                           "include")


def declared():
    names = set()
    for h in os.listdir(INCLUDE):
        if h.endswith(".h"):
            with open(os.path.join(INCLUDE, h)) as f:
                txt = f.read()
            names |= set(re.findall(r"CHARSIU_GPU_API[^;{]*?\b(charsiu_(?:gpu|npu)\w*)\s*\(",
                                    txt))
    return names


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_library_builds_and_loads():
    from charsiu_b200 import build
    build.build()
    lib = L.lib()
    for name, _, _ in L.SIGNATURES:
        assert getattr(lib, name)


def test_exports_are_exactly_the_headers():
    decl = declared()
    assert len(decl) >= 29
    assert decl == exported()
    assert decl == {n for n, _, _ in L.SIGNATURES}


def test_open_without_gpu_returns_null():
    """No GPU here: open must say so and return NULL, never crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert not L.lib().charsiu_gpu_open(2048, 8192, 4)


LAYOUT_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "charsiu.h"
#include "charsiu_llm.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(struct T, f))
int main(void) {
  printf("gguf_tensor %zu\nact %zu\njob %zu\nnpu_tensor %zu\n", sizeof(struct gguf_tensor),
         sizeof(struct charsiu_act), sizeof(struct charsiu_job), sizeof(struct npu_tensor));
  P(gguf_tensor, ne); P(gguf_tensor, type); P(gguf_tensor, data);
  P(charsiu_act, q); P(charsiu_act, d); P(charsiu_act, quantised); P(charsiu_act, n);
  P(charsiu_job, input_scale); P(charsiu_job, input_zero_point); P(charsiu_job, acc_out);
  P(charsiu_act, q1); P(charsiu_act, d1);
  P(npu_tensor, kgroup); P(npu_tensor, kscale); P(npu_tensor, n); P(npu_tensor, k);
  P(npu_tensor, name);
  return 0; }
"""

MIRROR = {
    "gguf_tensor": 152, "act": 64, "job": 64,
    "gguf_tensor.ne": 88, "gguf_tensor.type": 120, "gguf_tensor.data": 136,
    "charsiu_act.q": 16, "charsiu_act.d": 24, "charsiu_act.quantised": 40, "charsiu_act.n": 8,
    "charsiu_job.input_scale": 36, "charsiu_job.input_zero_point": 48, "charsiu_job.acc_out": 60,
    "npu_tensor": 216, "charsiu_act.q1": 48, "charsiu_act.d1": 56,
    "npu_tensor.kgroup": 16, "npu_tensor.kscale": 24, "npu_tensor.n": 80, "npu_tensor.k": 88,
    "npu_tensor.name": 136,
}


@pytest.mark.skipif(not os.path.isdir(REF_INCLUDE), reason="reference headers absent")
def test_struct_layouts_match_reference(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(LAYOUT_PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{REF_INCLUDE}", str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines():
        k, v = ln.rsplit(" ", 1)
        got[k] = int(v)
    assert got == MIRROR
    # and the same numbers are what ref_abi.h asserts at compile time
    with open(os.path.join(ROOT, "charsiu_b200", "csrc", "ref_abi.h")) as f:
        txt = f.read()
    assert "sizeof(RefGgufTensor) == 152" in txt and "sizeof(RefJob) == 64" in txt
