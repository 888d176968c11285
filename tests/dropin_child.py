"""Child process of tests/test_gpu_dropin.py: one greedy decode by the
reference's own decode loop (llama_load / llama_forward / llama_argmax)
linked to the GPU layer, in a process started with the switches that build
reads once (CHARSIU_GPU, CHARSIU_NPU, CHARSIU_NPU_QUANT).

    python -m tests.dropin_child BUILD MODEL.gguf PROMPT_JSON N_GEN N_CTX N_VOCAB

BUILD is "gpu" (the routing edit applied) or "npu" (unchanged, without its
NPU device file). Prints one JSON line: the tokens and the sha256 of the
logits after the prompt, as tests/golden/make_golden.py records them.
"""
import hashlib
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from oracle import oracle as O  # noqa: E402


def main() -> None:
    build, path, prompt, n_gen, n_ctx, n_vocab = sys.argv[1:7]
    toks, _, gen_ms, lg = O.ref_greedy(path, np.array(json.loads(prompt), np.int32),
                                       int(n_gen), n_ctx=int(n_ctx), threads=os.cpu_count(),
                                       want_logits=int(n_vocab), build=build)
    print(json.dumps({"tokens": toks.tolist(),
                      "logits_sha256": hashlib.sha256(lg.tobytes()).hexdigest(),
                      "gen_ms": gen_ms}), flush=True)


if __name__ == "__main__":
    main()
