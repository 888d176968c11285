"""The oracle, pinned: the restatement in oracle/charsiu_oracle.c against the
golden vectors the reference itself produced (tests/golden/), and against the
reference compiled here (oracle/_ref) where that build exists. CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "golden.npz"))
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD_DECODE = json.load(f)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.digest()


@pytest.mark.parametrize("name", list(W.MATVEC_GOLDEN))
def test_act_and_matvec_match_golden(name):
    qt, k, n, _ = W.MATVEC_GOLDEN[name]
    blk, x = GOLD[f"{name}_blocks"], GOLD[f"{name}_x"]
    q, d = O.act_quantise(x)
    assert np.array_equal(q, GOLD[f"{name}_q"])
    assert np.array_equal(bits(d), bits(GOLD[f"{name}_d"]))
    y = O.matvec(qt, blk, k, n, q, d)
    assert np.array_equal(bits(y), bits(GOLD[f"{name}_y"]))
    if f"{name}_dots" in GOLD:
        assert np.array_equal(O.block_dots(qt, blk, k, n, q), GOLD[f"{name}_dots"])


@pytest.mark.parametrize("name", list(W.MATVEC_SEEDED))
def test_workload_matvec_matches_golden(name):
    qt, k, n, seed = W.MATVEC_SEEDED[name]
    blk, x = W.matvec_inputs(qt, k, n, seed)
    assert sha(blk, x) == GOLD[f"{name}_sha"].tobytes(), "input generator drifted"
    q, d = O.act_quantise(x)
    y = O.matvec(qt, blk, k, n, q, d)
    assert np.array_equal(bits(y), bits(GOLD[f"{name}_y"]))


@pytest.mark.parametrize("name", list(W.I8_SHAPES))
def test_int8_matches_golden(name):
    m, k, n, seed = W.I8_SHAPES[name]
    a, w, bias = W.i8_inputs(m, k, n, seed)
    assert sha(a, w, bias) == GOLD[f"{name}_sha"].tobytes(), "input generator drifted"
    sc = tuple(float(v) for v in GOLD[f"{name}_scales"][:3])
    out = O.matmul_i8(a, w, bias, *sc)
    ref = GOLD[f"{name}_out"]
    assert np.array_equal(out, ref)
    # the reference's own readability rule, raised to 60 for this workload
    assert len(np.unique(ref)) >= 60


def test_int8_probes_analytic():
    """The CONST / NEG / IMPULSE constructions of tools/charsiu_matmul.c:275-444,
    whose accumulators are known in closed form."""
    k, n = 64, 64
    mult = np.float32(np.float32(0.02) * np.float32(0.01) / np.float32(0.25))
    # NEG (:331-348): input zp+40, weights of channel c at zp + (c - N/2), zero bias
    a = np.full((1, k), 128 + 40, np.uint8)
    w = np.array([[128 + (c - n // 2)] * k for c in range(n)], np.uint8)
    out = O.matmul_i8(a, w, np.zeros(n, np.int32), 0.02, 0.01, 0.25)
    acc = np.array([40 * k * (c - n // 2) for c in range(n)], np.int64)
    want = np.clip(np.floor(acc.astype(np.float32) * mult + np.float32(0.5)), -128, 127)
    assert np.array_equal(out[0], want.astype(np.int8))
    # CONST (:293-302): input at the zero point, bias ramp -> out = requant(bias)
    a = np.full((1, k), 128, np.uint8)
    rng = np.random.default_rng(3)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    bias = np.array([c * 2000 - 60000 for c in range(n)], np.int32)
    out = O.matmul_i8(a, w, bias, 0.02, 0.01, 0.25)
    want = np.clip(np.floor(bias.astype(np.float32) * mult + np.float32(0.5)), -128, 127)
    assert np.array_equal(out[0], want.astype(np.int8))
    # IMPULSE (:350-424): one live weight (zp + 100) per channel at k = c mod K
    a = np.array([[(128 + (i * 37 % 241) - 120) & 0xff for i in range(k)]], np.uint8)
    w = np.full((n, k), 128, np.uint8)
    for c in range(n):
        w[c, c % k] = 228
    out = O.matmul_i8(a, w, np.zeros(n, np.int32), 0.02, 0.12, 0.25)
    m12 = np.float32(np.float32(0.02) * np.float32(0.12) / np.float32(0.25))
    acc = np.array([(int(a[0, c % k]) - 128) * 100 for c in range(n)], np.int64)
    want = np.clip(np.floor(acc.astype(np.float32) * m12 + np.float32(0.5)), -128, 127)
    assert np.array_equal(out[0], want.astype(np.int8))
    assert len(np.unique(out)) >= 60


@pytest.mark.parametrize("name", list(W.DECODE_EXTRA))
def test_decode_extra_goldens_recorded(name):
    """The decode workloads outside the test matrix (the bench's --model
    choices) have the reference's tokens recorded, for their seeded prompt."""
    spec, gold = W.DECODE_EXTRA[name], GOLD_DECODE[name]
    assert gold["prompt"] == W.prompt_ids(spec["shape"].n_vocab, spec["seed"]).tolist()
    assert len(gold["tokens"]) == spec["n_gen"]
    assert all(0 <= t < spec["shape"].n_vocab for t in gold["tokens"])
    assert len(gold["gguf_sha256"]) == 64 and len(gold["logits_sha256"]) == 64


def test_half_to_float_all_values():
    h = np.arange(65536, dtype=np.uint16)
    lib = O.lib()
    got = np.array([lib.orc_half_to_float(int(v)) for v in h], dtype=np.float32)
    want = h.view(np.float16).astype(np.float32)
    finite = ~np.isnan(want)
    assert np.array_equal(bits(got[finite]), bits(want[finite]))
    assert np.isnan(got[~finite]).all()


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k"])
def test_decode_matches_golden(name, tmp_path):
    spec = W.DECODE[name]
    gold = GOLD_DECODE[name]
    path = str(tmp_path / f"{name}.gguf")
    G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                  embd_qtype=spec.get("embd_qtype"))
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == gold["gguf_sha256"]
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    assert prompt.tolist() == gold["prompt"]
    om = O.OracleModel(G.GGUFFile(path), n_ctx=spec["n_ctx"])
    assert om.greedy(prompt, spec["n_gen"]).tolist() == gold["tokens"]
    lg = om.logits_after(prompt)
    assert hashlib.sha256(lg.tobytes()).hexdigest() == gold["logits_sha256"]


# ---- against the reference compiled here (skipped where the tree is absent) ----

needs_ref = pytest.mark.skipif(not O.have_ref(), reason="reference build absent")


@needs_ref
@pytest.mark.parametrize("qt,k,n,seed", [(G.GGML_Q8_0, 64, 33, 5), (G.GGML_Q4_0, 1024, 40, 6),
                                         (G.GGML_Q8_0, 8192, 16, 7), (G.GGML_Q4_0, 32, 9, 8),
                                         (G.GGML_Q6_K, 256, 9, 21), (G.GGML_Q6_K, 2048, 40, 22),
                                         (G.GGML_Q6_K, 8192, 7, 23)])
def test_restatement_matches_reference_matvec(qt, k, n, seed):
    blk, x = W.matvec_inputs(qt, k, n, seed)
    x[::7] = 0.0                         # blocks with zeros and a few all-zero ones
    x[: min(k, 64)] = 0.0
    yr, qr, dr = O.ref_matvec(qt, blk, k, n, x)
    q, d = O.act_quantise(x)
    assert np.array_equal(q, qr) and np.array_equal(bits(d), bits(dr))
    assert np.array_equal(bits(O.matvec(qt, blk, k, n, q, d)), bits(yr))


@needs_ref
@pytest.mark.parametrize("m,k,n,zp", [(3, 33, 17, (128, 128, 0)), (5, 1, 8, (100, 140, 3)),
                                      (2, 200, 40, (0, 255, -5)), (1, 4096, 8, (128, 128, 0))])
def test_restatement_matches_reference_int8(m, k, n, zp):
    rng = np.random.default_rng(m * 1000 + k)
    a = rng.integers(0, 256, (m, k), dtype=np.uint8)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    bias = rng.integers(-4096, 4097, n, dtype=np.int32)
    for out_scale in (0.05, 0.5, 7.0):
        ref = O.ref_matmul_i8(a, w, bias, 0.02, 0.01, out_scale, *zp)
        assert np.array_equal(O.matmul_i8(a, w, bias, 0.02, 0.01, out_scale, *zp), ref)


@needs_ref
@pytest.mark.parametrize("embd", [None, G.GGML_Q6_K])
def test_restatement_matches_reference_decode(tmp_path, embd):
    shape = G.LlamaShape(256, 2, 4, 2, 256, 300, ctx_train=64)
    path = str(tmp_path / "m.gguf")
    G.write_llama(path, shape, G.GGML_Q4_0, seed=9, embd_qtype=embd)
    prompt = np.array([3, 1, 4, 1, 5, 9], np.int32)
    tr, _, _, lr = O.ref_greedy(path, prompt, 8, n_ctx=32, want_logits=shape.n_vocab)
    om = O.OracleModel(G.GGUFFile(path), n_ctx=32)
    assert om.greedy(prompt, 8).tolist() == tr.tolist()
    assert np.array_equal(bits(om.logits_after(prompt)), bits(lr))
