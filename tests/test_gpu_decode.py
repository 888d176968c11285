"""Greedy decode with every projection and the head on the GPU: token ids
identical to the reference's (golden) and logits bit-identical to the oracle's
llama_forward at every step."""
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
    GOLD = json.load(f)


def oracle_step_logits(om, prompt, tokens):
    """The logits each generated token was chosen from, by the oracle."""
    L = O.lib()
    st = L.orc_state_new(O.C.byref(om.m), om.n_ctx)
    out = []
    try:
        lp = None
        pos = 0
        for t in prompt:
            lp = L.orc_forward(st, int(t), pos)
            pos += 1
        for t in tokens:
            out.append(np.ctypeslib.as_array(lp, shape=(om.shape.n_vocab,)).copy())
            lp = L.orc_forward(st, int(t), pos)
            pos += 1
    finally:
        L.orc_state_free(st)
    return np.stack(out)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_tiny_models(name, tmp_path):
    """tiny_q4_q6k is a q4_0 file as llama.cpp writes one: its token_embd, and
    so the tied head, is q6_K (the embedding row and the head both exact)."""
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = np.array(gold["prompt"], np.int32)
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        calls = m.calls
    assert toks.tolist() == gold["tokens"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"])
    want = oracle_step_logits(om, prompt, toks)
    assert np.array_equal(logits.view(np.uint32), want.view(np.uint32))
    # q/k/v and gate/up go as one group each: 4 calls a layer plus the head
    n_fwd = len(prompt) + spec["n_gen"]
    assert calls == n_fwd * (4 * spec["shape"].n_layer + 1)


def test_llama_3_2_1b_shape(tmp_path):
    """The full workload: Llama-3.2-1B architecture, random q8_0 weights, 6
    seeded prompt ids, 24 generated tokens, all 112 projections and the
    128256-wide head on one B200."""
    spec, gold = W.DECODE["llama1b_q8"], GOLD["llama1b_q8"]
    path = str(tmp_path / "llama1b.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"])
    prompt = np.array(gold["prompt"], np.int32)
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
    assert toks.tolist() == gold["tokens"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"])
    first = om.logits_after(prompt)
    assert np.array_equal(logits[0].view(np.uint32), first.view(np.uint32))
