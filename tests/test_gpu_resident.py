"""The decode step with everything on the device (charsiu_gpu_decoder_*, via
charsiu_gpu_llama_set_resident): the embedding row, rmsnorm, RoPE, the KV
cache, attention, SiLU, the residuals, the projections, the head and the
argmax, one CUDA graph a token. Its logits must be the oracle's llama_forward
bit for bit at every step, and its greedy tokens the reference's."""
import json
import os

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer, Llama
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD = json.load(f)


def oracle_logits(om, tokens):
    """The oracle's logits after each of `tokens` at positions 0, 1, ..."""
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


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_tiny_models_every_step(name, tmp_path):
    """Greedy tokens as the reference's; the logits of every step (prompt and
    generated) bit-identical to the oracle's; the argmax-only graph (no logits
    copied back) gives the same tokens."""
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = np.array(gold["prompt"], np.int32)
    with Llama(path, n_ctx=spec["n_ctx"], resident=True) as m:
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        toks2, _, _ = m.greedy(prompt, spec["n_gen"], want_logits=False)
        fed = list(prompt) + toks.tolist()
        per_step = np.stack([m.forward(int(t), i) for i, t in enumerate(fed)])
        # embedding + 8 a layer + final norm, head, argmax
        assert m.step_launches == 1 + 8 * spec["shape"].n_layer + 3
    assert toks.tolist() == gold["tokens"]
    assert toks2.tolist() == gold["tokens"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"])
    want = oracle_logits(om, fed)
    assert np.array_equal(bits(per_step), bits(want))
    n_p = len(prompt)
    assert np.array_equal(bits(logits), bits(want[n_p - 1:n_p - 1 + spec["n_gen"]]))


def test_long_context_attention(tmp_path):
    """More positions than one shared-memory tile of K and V holds (256), so
    scores and outputs run over several tiles, and a softmax sum of 600 terms:
    every step's logits against the oracle."""
    shape = G.TINY
    path = str(tmp_path / "tiny_long.gguf")
    G.write_llama(path, shape, G.GGML_Q8_0, 11)
    rng = np.random.default_rng(12)
    toks = rng.integers(0, shape.n_vocab, size=600).astype(np.int32)
    # n_ctx not a multiple of 4: the tiles after the scores stay 16-byte aligned
    with Llama(path, n_ctx=603, resident=True) as m:
        got = np.stack([m.forward(int(t), i) for i, t in enumerate(toks)])
    om = O.OracleModel(G.GGUFFile(path), n_ctx=603)
    want = oracle_logits(om, toks)
    assert np.array_equal(bits(got), bits(want))


def test_llama_3_2_1b_shape(tmp_path):
    """The full workload on the device: the reference's greedy tokens, every
    generated step's logits bit-identical to the host-routed decode's (itself
    pinned to the oracle), the first step's to the oracle's directly."""
    spec, gold = W.DECODE["llama1b_q8"], GOLD["llama1b_q8"]
    path = str(tmp_path / "llama1b.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"])
    prompt = np.array(gold["prompt"], np.int32)
    with Llama(path, n_ctx=spec["n_ctx"]) as m:
        host_toks, host_logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        m.set_resident(True)
        toks, logits, _ = m.greedy(prompt, spec["n_gen"], want_logits=True)
        assert m.step_launches == 1 + 8 * 16 + 3
    assert host_toks.tolist() == gold["tokens"]
    assert toks.tolist() == gold["tokens"]
    assert np.array_equal(bits(logits), bits(host_logits))
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"])
    first = om.logits_after(prompt)
    assert np.array_equal(bits(logits[0]), bits(first))


@pytest.mark.parametrize("qtype,k,n", [(G.GGML_Q8_0, 2048, 77), (G.GGML_Q4_0, 4096, 33),
                                       (G.GGML_Q6_K, 2048, 41)])
def test_embedding_row(qtype, k, n):
    """charsiu_gpu_row_dev against the oracle's gguf_row_f32, row by row, the
    row index read from device memory; an index past the tensor is a kernel
    error code (the layer then retires) and leaves the output alone."""
    import torch
    rng = np.random.default_rng(k + n)
    blocks = G.quant_blocks(rng, qtype, n, k)
    dev = torch.device("cuda:0")
    with Layer(k, n, 4) as g:
        tid = g.add_blocks(qtype, k, n, blocks, "embd")
        out = torch.empty(k, dtype=torch.float32, device=dev)
        for r in [0, 1, 7, 8, n // 2, n - 1]:
            idx = torch.tensor([r], dtype=torch.int32, device=dev)
            assert g.row_dev(tid, idx.data_ptr(), out.data_ptr(),
                             torch.cuda.current_stream().cuda_stream) == 0
            torch.cuda.synchronize()
            want = O.row_f32(qtype, blocks, k, r)
            assert np.array_equal(bits(out.cpu().numpy()), bits(want)), r
        assert g.kernel_error() == 0
        out.fill_(7.0)
        idx = torch.tensor([n], dtype=torch.int32, device=dev)
        assert g.row_dev(tid, idx.data_ptr(), out.data_ptr(),
                         torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert g.kernel_error() != 0
        assert bool((out == 7.0).all())
        assert g.dead


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4_q6k", "llama1b_q8"])
def test_device_side_greedy_run(name, tmp_path):
    """charsiu_gpu_decoder_generate: the greedy loop with each step's argmax
    fed to the next step on the device, no host round trip between steps.
    Three runs from the prompt in a row (the first warms the step, the second
    captures its graph, the third replays it) each give the reference's
    tokens."""
    spec, gold = W.DECODE[name], GOLD[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    prompt = np.array(gold["prompt"], np.int32)
    n = spec["n_gen"] - 1
    with Llama(path, n_ctx=len(prompt) + n, resident=True) as m:
        for _ in range(3):
            lp = None
            for i, t in enumerate(prompt):
                lp = m.forward(int(t), i)
            first = int(np.argmax(lp))
            toks, ms = m.generate_dev(first, len(prompt), n)
            assert [first] + toks.tolist() == gold["tokens"]
            assert ms > 0
        # embedding + 8 a layer + final norm, head, argmax, and the step that
        # feeds the argmax on
        assert m.step_launches == 1 + 8 * spec["shape"].n_layer + 4
        with pytest.raises(Exception):
            m.generate_dev(first, len(prompt), n + 1)     # past the context: refused
