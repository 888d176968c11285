"""The drop-in, proven with charsiu's own code.

charsiu's decode loop (src/llama.c: llama_forward, matvec_pair, matvec_again;
its structs gguf_tensor, charsiu_act, charsiu_job) is compiled from its own
sources by oracle/Makefile and linked to libcharsiu_gpu.so, two ways:

  gpu  the routing edit of route_llama.py applied (CHARSIU_GPU=1): every
       projection and the head through charsiu_gpu_add / charsiu_gpu_matvec /
       charsiu_gpu_matvec_group on the reference's own structs. The layer is
       bit-exact, so the greedy tokens AND the logits after the prompt are the
       CPU reference's (the goldens).
  npu  the loop unchanged, without src/npudev.c, run with CHARSIU_NPU=1
       CHARSIU_NPU_QUANT=1: its charsiu_npu_* calls land in this library's NPU
       layer. Its float arithmetic differs from the CPU model's double by an
       ulp or two in y, so the tokens (the reference's own acceptance
       criterion for its NPU layer) are what must match.

Each decode runs in a child process, since those switches are read once a
process. The struct-form calls are also checked one by one against the
reference's gguf_matvec and cpu_reference.
"""
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
with open(os.path.join(HERE, "golden", "golden_decode.json")) as f:
    GOLD = json.load(f)

needs_builds = pytest.mark.skipif(
    not (os.path.exists(O.REF_GPU_LIB) and os.path.exists(O.REF_NPU_LIB)),
    reason="the reference's routed builds (oracle/_ref) were not made")


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("dropin")
    out = {}
    for name, spec in W.DECODE.items():
        path = str(d / f"{name}.gguf")
        G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                      embd_qtype=spec.get("embd_qtype"))
        out[name] = path
    return out


def decode(build, name, path, switches):
    spec, gold = W.DECODE[name], GOLD[name]
    env = {k: v for k, v in os.environ.items() if not k.startswith("CHARSIU_")}
    env.update(switches)
    cp = subprocess.run([sys.executable, "-m", "tests.dropin_child", build, path,
                         json.dumps(gold["prompt"]), str(spec["n_gen"]), str(spec["n_ctx"]),
                         str(spec["shape"].n_vocab)],
                        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert cp.returncode == 0, cp.stderr[-2000:]
    return json.loads(cp.stdout.strip().splitlines()[-1]), cp.stderr


def calls_in(report: str, prefix: str) -> int:
    m = re.search(prefix + r"[^\n]*?(\d+) calls", report)
    assert m, report[-2000:]
    return int(m.group(1))


@needs_builds
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q4_q6k", "llama1b_q8"])
def test_reference_loop_routed_to_the_gpu(models, name):
    res, err = decode("gpu", name, models[name], {"CHARSIU_GPU": "1", "CHARSIU_GPU_REPORT": "1"})
    spec, gold = W.DECODE[name], GOLD[name]
    assert "charsiu: GPU open" in err and "NOTHING RAN" not in err, err[-2000:]
    # q/k/v and gate/up as one group call each: 4 calls a layer plus the head
    n_fwd = len(gold["prompt"]) + spec["n_gen"]
    assert calls_in(err, "charsiu GPU:") == n_fwd * (4 * spec["shape"].n_layer + 1)
    assert res["tokens"] == gold["tokens"]
    assert res["logits_sha256"] == gold["logits_sha256"]


@needs_builds
def test_reference_loop_routed_one_call_a_projection(models):
    """CHARSIU_GPU_NOGROUP: the control, every projection its own
    charsiu_gpu_matvec; same bits."""
    name = "tiny_q8"
    res, err = decode("gpu", name, models[name],
                      {"CHARSIU_GPU": "1", "CHARSIU_GPU_REPORT": "1", "CHARSIU_GPU_NOGROUP": "1"})
    spec, gold = W.DECODE[name], GOLD[name]
    n_fwd = len(gold["prompt"]) + spec["n_gen"]
    assert calls_in(err, "charsiu GPU:") == n_fwd * (7 * spec["shape"].n_layer + 1)
    assert res["tokens"] == gold["tokens"]
    assert res["logits_sha256"] == gold["logits_sha256"]


@needs_builds
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "llama1b_q8"])
def test_reference_loop_with_the_npu_layer_on_the_gpu(models, name):
    spec = W.DECODE[name]
    res, err = decode("npu", name, models[name],
                      {"CHARSIU_NPU": "1", "CHARSIU_NPU_QUANT": "1",
                       "CHARSIU_NPU_MAXN": str(spec["shape"].n_vocab)})
    assert "NPU open" in err and "NOTHING RAN" not in err, err[-2000:]
    n_fwd = len(GOLD[name]["prompt"]) + spec["n_gen"]
    # the head too (CHARSIU_NPU_MAXN raised to the vocabulary)
    assert calls_in(err, "charsiu NPU format on the GPU:") == \
        n_fwd * (4 * spec["shape"].n_layer + 1)
    assert res["tokens"] == GOLD["npu"][name]["tokens"]


@needs_builds
@pytest.mark.parametrize("qt,k,n,ntensor,group", [
    (G.GGML_Q8_0, 2048, 300, 3, 1), (G.GGML_Q8_0, 2048, 300, 3, 0),
    (G.GGML_Q4_0, 1024, 77, 2, 1), (G.GGML_Q4_0, 96, 41, 1, 0),
    (G.GGML_Q8_0, 8192, 64, 2, 1)])
def test_struct_form_matvec(qt, k, n, ntensor, group):
    """charsiu_gpu_add(struct gguf_tensor *), charsiu_gpu_matvec(struct
    charsiu_act *) and charsiu_gpu_matvec_group with the reference's structs
    and its charsiu_act_set, against the reference's gguf_matvec."""
    blks, xs = [], None
    for i in range(ntensor):
        blk, x = W.matvec_inputs(qt, k, n, seed=10 + i)
        blks.append(blk)
        xs = x if xs is None else xs
    want = np.stack([O.ref_matvec(qt, b, k, n, xs)[0] for b in blks])
    got = np.zeros((ntensor, n), np.float32)
    import ctypes as C
    ptrs = (C.c_void_p * ntensor)(*[b.ctypes.data for b in blks])
    R = O.ref_routed("gpu")
    rc = R.refgpu_matvec(qt, C.cast(ptrs, C.c_void_p), ntensor, k, n, xs, got, group)
    assert rc == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_builds
@pytest.mark.parametrize("shape", list(W.I8_SHAPES))
def test_struct_form_matmul_i8(shape):
    """charsiu_gpu_matmul_i8(struct charsiu_job *) on a job filled as
    tools/charsiu_matmul.c fills one, byte-exact against cpu_reference."""
    m, k, n, seed = W.I8_SHAPES[shape]
    a, w, bias = W.i8_inputs(m, k, n, seed)
    sc = W.i8_scales(m, k, n, seed)
    out = np.zeros((m, n), np.int8)
    assert O.ref_routed("gpu").refgpu_matmul_i8(m, k, n, a, w, bias, *sc, out) == 0
    want = O.ref_matmul_i8(a, w, bias, *sc)
    assert np.array_equal(out.view(np.uint8).reshape(-1), want.view(np.uint8).reshape(-1))
