"""The drop-in builds of charsiu's own decode loop (oracle/Makefile), on the
CPU: the routing edit applies to the reference's src/llama.c at exactly one
place each, both builds link to libcharsiu_gpu.so, and where no GPU answers
they stay on the CPU (the layer's NULL open, as an absent NPU) and give the
reference's tokens and logits. tests/test_gpu_dropin.py runs them on a GPU."""
import json
import os
import subprocess
import sys

import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from oracle import oracle as O
from oracle import route_llama

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.environ.get("REF", os.path.join(os.path.dirname(ROOT), "reference"))
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD = json.load(f)


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "src", "llama.c")),
                    reason="the reference tree is not here")
def test_routing_edit_applies_once_each():
    with open(os.path.join(REF, "src", "llama.c")) as f:
        src = f.read()
    out = route_llama.route(src)
    for _, text, _ in route_llama.EDITS:
        assert out.count(text) == 1
    # nothing of the reference's own lines is lost
    assert len(out) == len(src) + sum(len(t) for _, t, _ in route_llama.EDITS)


@pytest.mark.skipif(not (os.path.exists(O.REF_GPU_LIB) and os.path.exists(O.REF_NPU_LIB)),
                    reason="the reference's routed builds (oracle/_ref) were not made")
@pytest.mark.parametrize("build,switches,gold", [
    ("gpu", {"CHARSIU_GPU": "1"}, lambda g: g["tiny_q8"]),
    ("npu", {"CHARSIU_NPU": "1", "CHARSIU_NPU_QUANT": "1"}, lambda g: g["npu"]["tiny_q8"])])
def test_builds_decode_like_the_reference(tmp_path, build, switches, gold):
    spec = W.DECODE["tiny_q8"]
    path = str(tmp_path / "tiny_q8.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"])
    env = {k: v for k, v in os.environ.items() if not k.startswith("CHARSIU_")}
    env.update(switches)
    cp = subprocess.run([sys.executable, "-m", "tests.dropin_child", build, path,
                         json.dumps(GOLD["tiny_q8"]["prompt"]), str(spec["n_gen"]),
                         str(spec["n_ctx"]), str(spec["shape"].n_vocab)],
                        cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert cp.returncode == 0, cp.stderr[-2000:]
    res = json.loads(cp.stdout.strip().splitlines()[-1])
    assert res["tokens"] == gold(GOLD)["tokens"]
    assert res["logits_sha256"] == gold(GOLD)["logits_sha256"]
