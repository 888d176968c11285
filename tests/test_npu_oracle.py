"""The NPU number format (CHARSIU_NPU_QUANT: per-channel int8 weights, one
activation scale) in the oracle: pinned against the reference's own
npu_tensor_build, single-scale activation, npu_matvec and the device path's
arithmetic (tests/npu_ref_pins.py, in a process started with the switch set),
and its greedy decode against the reference's NPU-format decode (golden)."""
import hashlib
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD = json.load(f)["npu"]


@pytest.mark.skipif(not O.have_ref(), reason="the reference build (oracle/_ref) is absent")
def test_npu_restatement_matches_reference():
    env = dict(os.environ, CHARSIU_NPU_QUANT="1")
    r = subprocess.run([sys.executable, os.path.join(HERE, "npu_ref_pins.py")], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "npu pins ok" in r.stdout


def _logits_sha(om, prompt):
    lg = om.logits_after(prompt)
    return hashlib.sha256(np.ascontiguousarray(lg).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_npu_decode_matches_reference(name, tmp_path):
    """The oracle's NPU-format decode with the reference's CPU-model
    arithmetic: the reference's logits bit for bit and its greedy tokens; with
    the device path's arithmetic (what a GPU replacing npudev.c computes): the
    same greedy tokens."""
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    gg = G.GGUFFile(path)
    model = O.OracleModel(gg, n_ctx=spec["n_ctx"], npu=2)
    assert _logits_sha(model, prompt) == gold["logits_sha256"]
    assert model.greedy(prompt, spec["n_gen"]).tolist() == gold["tokens"]
    device = O.OracleModel(gg, n_ctx=spec["n_ctx"], npu=1)
    assert device.greedy(prompt, spec["n_gen"]).tolist() == gold["tokens"]


def test_device_formula_differs_from_the_model_only_in_rounding():
    """The device path computes (float)acc * d1 * scale in float; the CPU model
    rounds once from double. They agree to an ulp or two, not bit for bit --
    which is why the GPU is pinned to the device path's arithmetic and the
    tokens, not the logits, are compared with the CPU model."""
    rng = np.random.default_rng(5)
    blk = G.quant_blocks(rng, G.GGML_Q8_0, 512, 2048)
    q, s, _ = O.npu_tensor_build(G.GGML_Q8_0, blk, 2048, 512)
    q1, d1 = O.act_quantise_one(rng.standard_normal(2048).astype(np.float32))
    y0 = O.npu_matvec(q, s, q1, d1, model=0)
    y1 = O.npu_matvec(q, s, q1, d1, model=1)
    ulp = np.spacing(np.abs(y1).astype(np.float32))
    assert np.all(np.abs(y0 - y1) <= 2 * ulp)
    assert not np.array_equal(y0, y1)
