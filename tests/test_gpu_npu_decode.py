"""The decode loop in charsiu's NPU number format (CHARSIU_NPU_QUANT=1) with
every projection and the head on the GPU through charsiu_npu_*: greedy tokens
identical to the reference's own NPU-format decode (golden), and every
step's logits bit-identical to the oracle's decode with the device path's
arithmetic (src/npudev.c:605, 710)."""
import json
import os

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Llama
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD = json.load(f)["npu"]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def oracle_logits(om, tokens):
    L = O.lib()
    st = L.orc_state_new(O.C.byref(om.m), om.n_ctx)
    out = []
    try:
        for pos, t in enumerate(tokens):
            lp = L.orc_forward(st, int(t), pos)
            out.append(np.ctypeslib.as_array(lp, shape=(om.shape.n_vocab,)).copy())
    finally:
        L.orc_state_free(st)
    return np.stack(out)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_tiny_models(name, tmp_path, monkeypatch):
    monkeypatch.setenv("CHARSIU_NPU_QUANT", "1")
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        calls = m.npu_calls
        assert m.calls == 0                     # nothing went through the GGML layer
    assert toks.tolist() == gold["tokens"]
    # q/k/v and gate/up as one group call each: 4 a layer, and the head
    n_fwd = len(prompt) + spec["n_gen"]
    assert calls == n_fwd * (4 * spec["shape"].n_layer + 1)
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"], npu=1)
    fed = list(prompt) + toks.tolist()
    want = oracle_logits(om, fed[:-1])
    n_p = len(prompt)
    assert np.array_equal(bits(logits), bits(want[n_p - 1:]))


def test_llama_3_2_1b_shape(tmp_path, monkeypatch):
    monkeypatch.setenv("CHARSIU_NPU_QUANT", "1")
    spec, gold = W.DECODE["llama1b_q8"], GOLD["llama1b_q8"]
    path = str(tmp_path / "llama1b.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"])
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
    assert toks.tolist() == gold["tokens"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"], npu=1)
    first = om.logits_after(prompt)
    assert np.array_equal(bits(logits[0]), bits(first))


def npu_step_launches(n_layer):
    """Kernels a token of the device step in the NPU number format: the
    embedding row; per layer the rmsnorm with its single-scale quantiser,
    q/k/v, attention, the attention output's quantiser, o, the rmsnorm, gate/up,
    SiLU, its quantiser, down; then the final rmsnorm, the head, the argmax."""
    return 1 + 10 * n_layer + 3


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_tiny_models_resident(name, tmp_path, monkeypatch):
    """The whole step on the device in the NPU number format
    (charsiu_gpu_decoder_new_npu): the reference's greedy tokens, every step's
    logits (prompt and generated) bit-identical to the oracle's NPU-format
    decode, the argmax-only graph the same tokens, and no host NPU call."""
    monkeypatch.setenv("CHARSIU_NPU_QUANT", "1")
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    with Llama(path, n_ctx=spec["n_ctx"], resident=True) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        toks2, _, _ = m.greedy(prompt, spec["n_gen"], want_logits=False)
        fed = list(prompt) + toks.tolist()
        per_step = np.stack([m.forward(int(t), i) for i, t in enumerate(fed)])
        assert m.step_launches == npu_step_launches(spec["shape"].n_layer)
        assert m.npu_calls == 0 and m.calls == 0
    assert toks.tolist() == gold["tokens"]
    assert toks2.tolist() == gold["tokens"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"], npu=1)
    want = oracle_logits(om, fed)
    assert np.array_equal(bits(per_step), bits(want))
    n_p = len(prompt)
    assert np.array_equal(bits(logits), bits(want[n_p - 1:n_p - 1 + spec["n_gen"]]))


def test_llama_3_2_1b_shape_resident(tmp_path, monkeypatch):
    """The workload in the NPU number format with the step on the device: the
    reference's tokens, every generated step's logits the host-routed NPU
    decode's bits, the first the oracle's."""
    monkeypatch.setenv("CHARSIU_NPU_QUANT", "1")
    spec, gold = W.DECODE["llama1b_q8"], GOLD["llama1b_q8"]
    path = str(tmp_path / "llama1b.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"])
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        host_toks, host_logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        m.set_resident(True)
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        assert m.step_launches == npu_step_launches(16)
    assert host_toks.tolist() == gold["tokens"]
    assert toks.tolist() == gold["tokens"]
    assert np.array_equal(bits(logits), bits(host_logits))
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"], npu=1)
    assert np.array_equal(bits(logits[0]), bits(om.logits_after(prompt)))
