"""Seeded synthetic inputs for every workload shape.

The shapes and distributions are the workload's:
  q8_0 matvec  M=1 K=2048 N=8192 (gate/up shape), q4_0 matvec M=1 K=8192
  N=2048 (down shape): blocks as charsiu_b200.gguf.quant_blocks makes them,
  activation fp32 N(0, 1);
  int8 matmul with the output stage at (M,K,N) = (1,64,64), (1,512,1024),
  (224,64,64), (3136,33,64): a and w uniform u8 around zero point 128 (so
  uniform signed int8), bias uniform in [-4096, 4096], requant scale chosen so
  the output spans at least 60 distinct values;
  Llama-3.2-1B-shaped greedy decode: 6 seeded prompt ids, 24 generated.
All generators are numpy PCG64 with the seeds below.
"""
from __future__ import annotations

import numpy as np

from .gguf import GGML_Q4_0, GGML_Q6_K, GGML_Q8_0, LLAMA_3_2_1B, TINY, quant_blocks

# small shapes whose inputs are stored as fixtures (ragged N and odd nb included)
MATVEC_GOLDEN = {
    "q8_k256_n64": (GGML_Q8_0, 256, 64, 11),
    "q4_k256_n64": (GGML_Q4_0, 256, 64, 12),
    "q8_k96_n40": (GGML_Q8_0, 96, 40, 13),
    "q4_k160_n19": (GGML_Q4_0, 160, 19, 14),
    "q6k_k256_n64": (GGML_Q6_K, 256, 64, 15),
    "q6k_k2048_n41": (GGML_Q6_K, 2048, 41, 16),
}
# the two matvec workload shapes: outputs stored, inputs regenerated from seeds
MATVEC_SEEDED = {
    "q8_k2048_n8192": (GGML_Q8_0, 2048, 8192, 1),
    "q4_k8192_n2048": (GGML_Q4_0, 8192, 2048, 2),
}

# (m, k, n, seed); seeds picked so that each output spans >= 60 distinct values
I8_SHAPES = {
    "i8_1x64x64": (1, 64, 64, 167),
    "i8_1x512x1024": (1, 512, 1024, 0),
    "i8_224x64x64": (224, 64, 64, 0),
    "i8_3136x33x64": (3136, 33, 64, 0),
}
I8_IN_SCALE, I8_WT_SCALE = 0.02, 0.01      # tools/charsiu_matmul.c:184-185

DECODE = {
    "tiny_q8": {"shape": TINY, "qtype": GGML_Q8_0, "seed": 1, "n_gen": 24, "n_ctx": 64},
    "tiny_q4": {"shape": TINY, "qtype": GGML_Q4_0, "seed": 2, "n_gen": 24, "n_ctx": 64},
    "llama1b_q8": {"shape": LLAMA_3_2_1B, "qtype": GGML_Q8_0, "seed": 0, "n_gen": 24,
                   "n_ctx": 64},
    # a q4_0 file as llama.cpp writes one: token_embd (the tied head) in q6_K
    "tiny_q4_q6k": {"shape": TINY, "qtype": GGML_Q4_0, "embd_qtype": GGML_Q6_K, "seed": 3,
                    "n_gen": 24, "n_ctx": 64},
}

# Decode workloads outside the test matrix (their golden tokens are recorded
# all the same, for the bench): the Llama-3.2-1B shape as a llama.cpp q4_0
# file, token_embd and so the tied head in q6_K.
DECODE_EXTRA = {
    "llama1b_q4_q6k": {"shape": LLAMA_3_2_1B, "qtype": GGML_Q4_0, "embd_qtype": GGML_Q6_K,
                       "seed": 0, "n_gen": 24, "n_ctx": 64},
}


def matvec_inputs(qtype: int, k: int, n: int, seed: int):
    rng = np.random.default_rng([seed])
    blocks = quant_blocks(rng, qtype, n, k)
    x = rng.normal(0.0, 1.0, size=k).astype(np.float32)
    return blocks, x


def batch_inputs(qtype: int, k: int, n: int, m: int, seed: int):
    """n rows of weights and m activation rows, for the batched (M>1) path."""
    rng = np.random.default_rng([seed, m])
    blocks = quant_blocks(rng, qtype, n, k)
    x = rng.normal(0.0, 1.0, size=(m, k)).astype(np.float32)
    return blocks, x


def i8_inputs(m: int, k: int, n: int, seed: int):
    rng = np.random.default_rng([seed, m, k, n])
    a = rng.integers(0, 256, size=(m, k), dtype=np.uint8)
    w = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
    bias = rng.integers(-4096, 4097, size=n, dtype=np.int32)
    return a, w, bias


def _i8_acc(a, w, bias):
    return (a.astype(np.int64) - 128) @ (w.astype(np.int64) - 128).T + bias.astype(np.int64)


def i8_scales(m: int, k: int, n: int, seed: int):
    """(in_scale, wt_scale, out_scale, in_zp, wt_zp, out_zp) for a shape.

    out_scale puts the largest |accumulator| at about 120 counts, which fills
    the signed byte without leaning on the rails."""
    a, w, bias = i8_inputs(m, k, n, seed)
    amax = float(np.abs(_i8_acc(a, w, bias)).max())
    mult = 120.0 / amax
    out_scale = float(np.float32(I8_IN_SCALE * I8_WT_SCALE / mult))
    return (I8_IN_SCALE, I8_WT_SCALE, out_scale, 128, 128, 0)


def i8_expected_numpy(a, w, bias, in_scale, wt_scale, out_scale, in_zp=128, wt_zp=128, out_zp=0):
    """numpy form of the output stage, used only to pick seeds and scales."""
    acc = (a.astype(np.int64) - in_zp) @ (w.astype(np.int64) - wt_zp).T + bias.astype(np.int64)
    mult = np.float32(np.float32(in_scale) * np.float32(wt_scale) / np.float32(out_scale))
    v = acc.astype(np.float32) * mult + np.float32(out_zp)
    v = np.floor(v + np.float32(0.5))
    return np.clip(v, -128, 127).astype(np.int8)


def prompt_ids(n_vocab: int, seed: int, n: int = 6) -> np.ndarray:
    return np.random.default_rng([seed, 99]).integers(0, n_vocab, size=n).astype(np.int32)
