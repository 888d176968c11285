"""Generate the golden fixtures from the reference itself.

Run here, where the reference tree is mounted:  python tests/golden/make_golden.py
It builds oracle/_ref/libcharsiu_ref.so (the reference compiled from its own
sources by oracle/Makefile) and records what the reference computes:

  golden.npz         act_set + gguf_matvec (q8_0, q4_0, q6_K), cpu_reference int8
                     outputs at the four int8 workload shapes, and the chosen
                     requant scales;
  golden_decode.json greedy token ids and logit digests of charsiu's own
                     llama_forward on seeded synthetic models: the tiny test
                     models (q8_0; q4_0; q4_0 with a q6_K embedding and head)
                     and the Llama-3.2-1B-shaped one; under "npu", the same
                     in charsiu's NPU number format (CHARSIU_NPU_QUANT=1, its
                     CPU model), added by  python tests/golden/make_golden.py --npu;
                     the decode workloads outside the test matrix
                     (W.DECODE_EXTRA: the 1B shape as a q4_0 file with a q6_K
                     head), added by  python tests/golden/make_golden.py --extra

Inputs are regenerated from the recorded seeds (numpy PCG64); a sha256 of each
input is stored beside it so generator drift is caught rather than trusted.
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from charsiu_b200 import gguf as G  # noqa: E402
from oracle import oracle as O  # noqa: E402
from charsiu_b200 import workloads as W  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main() -> None:
    O.build()
    assert O.have_ref(), "the reference tree is needed to make golden vectors"
    out = {}

    # act_set + gguf_matvec through the reference (small shapes, inputs stored)
    for name, (qt, k, n, seed) in W.MATVEC_GOLDEN.items():
        blk, x = W.matvec_inputs(qt, k, n, seed)
        y, q, d = O.ref_matvec(qt, blk, k, n, x)
        out[f"{name}_blocks"] = blk
        out[f"{name}_x"] = x
        out[f"{name}_y"] = y
        out[f"{name}_q"] = q
        out[f"{name}_d"] = d
        if qt in (G.GGML_Q8_0, G.GGML_Q4_0):        # dots of 32-element blocks
            out[f"{name}_dots"] = O.block_dots(qt, blk, k, n, q)

    # larger matvec shapes: outputs only, inputs from seeds
    for name, (qt, k, n, seed) in W.MATVEC_SEEDED.items():
        blk, x = W.matvec_inputs(qt, k, n, seed)
        y, q, d = O.ref_matvec(qt, blk, k, n, x)
        out[f"{name}_y"] = y
        out[f"{name}_sha"] = np.frombuffer(bytes.fromhex(sha(blk, x)), dtype=np.uint8)

    # cpu_reference at the int8 workload shapes
    for name, (m, k, n, seed) in W.I8_SHAPES.items():
        a, w, bias = W.i8_inputs(m, k, n, seed)
        scales = W.i8_scales(m, k, n, seed)
        ref = O.ref_matmul_i8(a, w, bias, *scales)
        out[f"{name}_out"] = ref
        out[f"{name}_scales"] = np.array(scales, dtype=np.float32)
        out[f"{name}_sha"] = np.frombuffer(bytes.fromhex(sha(a, w, bias)), dtype=np.uint8)
        print(f"{name}: {len(np.unique(ref))} distinct outputs, scales {scales}")

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)

    # the decode loop, by the reference's own llama_forward
    dec = {}
    with tempfile.TemporaryDirectory() as td:
        for name, spec in W.DECODE.items():
            path = os.path.join(td, f"{name}.gguf")
            G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                          embd_qtype=spec.get("embd_qtype"))
            prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
            toks, pm, gm, lg = O.ref_greedy(path, prompt, spec["n_gen"], n_ctx=spec["n_ctx"],
                                            threads=os.cpu_count(),
                                            want_logits=spec["shape"].n_vocab)
            with open(path, "rb") as f:
                fsha = hashlib.sha256(f.read()).hexdigest()
            dec[name] = {"prompt": prompt.tolist(), "tokens": toks.tolist(),
                         "logits_sha256": sha(lg), "logits_head": lg[:8].tolist(),
                         "gguf_sha256": fsha, "gen_ms": gm}
            print(name, toks.tolist(), f"gen {gm:.0f} ms")
    with open(os.path.join(HERE, "golden_decode.json"), "w") as f:
        json.dump(dec, f, indent=1)


def extra() -> None:
    """Add the decode goldens of W.DECODE_EXTRA to golden_decode.json, leaving
    every other entry as it is."""
    O.build()
    assert O.have_ref(), "the reference tree is needed to make golden vectors"
    path = os.path.join(HERE, "golden_decode.json")
    with open(path) as f:
        dec = json.load(f)
    with tempfile.TemporaryDirectory() as td:
        for name, spec in W.DECODE_EXTRA.items():
            gpath = os.path.join(td, f"{name}.gguf")
            G.write_llama(gpath, spec["shape"], spec["qtype"], spec["seed"],
                          embd_qtype=spec.get("embd_qtype"))
            prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
            toks, pm, gm, lg = O.ref_greedy(gpath, prompt, spec["n_gen"], n_ctx=spec["n_ctx"],
                                            threads=os.cpu_count(),
                                            want_logits=spec["shape"].n_vocab)
            with open(gpath, "rb") as f:
                fsha = hashlib.sha256(f.read()).hexdigest()
            dec[name] = {"prompt": prompt.tolist(), "tokens": toks.tolist(),
                         "logits_sha256": sha(lg), "logits_head": lg[:8].tolist(),
                         "gguf_sha256": fsha, "gen_ms": gm}
            print(name, toks.tolist(), f"gen {gm:.0f} ms")
    with open(path, "w") as f:
        json.dump(dec, f, indent=1)


def npu_child(out_path: str) -> None:
    """In a process started with CHARSIU_NPU_QUANT=1: the reference's greedy
    decode in the NPU number format (its CPU model, src/npuquant.c) on every
    decode workload, into out_path as JSON."""
    assert os.environ.get("CHARSIU_NPU_QUANT") == "1"
    res = {}
    with tempfile.TemporaryDirectory() as td:
        for name, spec in W.DECODE.items():
            path = os.path.join(td, f"{name}.gguf")
            G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                          embd_qtype=spec.get("embd_qtype"))
            prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
            toks, pm, gm, lg = O.ref_greedy(path, prompt, spec["n_gen"], n_ctx=spec["n_ctx"],
                                            threads=os.cpu_count(),
                                            want_logits=spec["shape"].n_vocab)
            res[name] = {"tokens": toks.tolist(), "logits_sha256": sha(lg),
                         "logits_head": lg[:8].tolist()}
            print("npu", name, toks.tolist(), f"gen {gm:.0f} ms")
    with open(out_path, "w") as f:
        json.dump(res, f)


def npu() -> None:
    """Add the NPU-format decode goldens ("npu" key) to golden_decode.json,
    leaving every other entry as it is."""
    O.build()
    assert O.have_ref(), "the reference tree is needed to make golden vectors"
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "npu.json")
        env = dict(os.environ, CHARSIU_NPU_QUANT="1")
        subprocess.run([sys.executable, os.path.abspath(__file__), "--npu-child", out], env=env,
                       check=True)
        with open(out) as f:
            res = json.load(f)
    path = os.path.join(HERE, "golden_decode.json")
    with open(path) as f:
        dec = json.load(f)
    dec["npu"] = res
    with open(path, "w") as f:
        json.dump(dec, f, indent=1)


if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[1] == "--npu-child":
        npu_child(sys.argv[2])
    elif len(sys.argv) > 1 and sys.argv[1] == "--npu":
        npu()
    elif len(sys.argv) > 1 and sys.argv[1] == "--extra":
        extra()
    else:
        main()
