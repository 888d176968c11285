"""Pins of the oracle's NPU number format against the reference itself, run
in a process of its own: charsiu_act_set and llama_forward read
CHARSIU_NPU_QUANT once, on their first call, so that process must start with
it set (tests/test_npu_oracle.py runs this file that way). Exits non-zero with
the first mismatch."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from charsiu_b200 import gguf as G  # noqa: E402
from oracle import oracle as O  # noqa: E402

TENSORS = [(G.GGML_Q8_0, 2048, 48, 1), (G.GGML_Q4_0, 256, 33, 2), (G.GGML_Q6_K, 512, 40, 3),
           (G.GGML_Q8_0, 64, 1, 4), (G.GGML_Q4_0, 8192, 9, 5)]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def ref_build(qt, blk, k, n):
    q = np.zeros((n, k), np.int8)
    s = np.zeros(n, np.float32)
    w = np.zeros(n, np.int32)
    assert O.ref().ref_npu_tensor_build(qt, blk.ctypes.data, k, n, q, s, w) == 0
    return q, s, w


def ref_q1(x):
    q1 = np.zeros((x.size + 31) // 32 * 32, np.int8)
    d1 = O.C.c_float()
    assert O.ref().ref_act_q1(x, x.size, q1, O.C.byref(d1)) == 0, "q1 not valid"
    return q1, np.float32(d1.value)


def ref_model(q, s, q1, d1):
    n, k = q.shape
    y = np.zeros(n, np.float32)
    O.ref().ref_npu_matvec(np.ascontiguousarray(q), s, k, n, q1, float(d1), y)
    return y


def main():
    assert os.environ.get("CHARSIU_NPU_QUANT") == "1"
    rng = np.random.default_rng(20)
    for qt, k, n, seed in TENSORS:
        blk = G.quant_blocks(np.random.default_rng(seed), qt, n, k)
        q, s, w = O.npu_tensor_build(qt, blk, k, n)
        rq, rs, rw = ref_build(qt, blk, k, n)
        assert np.array_equal(q, rq) and np.array_equal(bits(s), bits(rs)) and \
            np.array_equal(w, rw), ("npu_tensor_build", qt, k, n)
        xs = [rng.standard_normal(k).astype(np.float32),
              (rng.standard_normal(k) * 1e-3).astype(np.float32), np.zeros(k, np.float32)]
        xs[1][k // 2] = 50.0
        for x in xs:
            q1, d1 = O.act_quantise_one(x)
            rq1, rd1 = ref_q1(x)
            assert np.array_equal(q1, rq1) and bits(d1) == bits(rd1), ("q1", k)
            # the CPU model, bit for bit
            y1 = O.npu_matvec(q, s, q1[:k], d1, model=1)
            assert np.array_equal(bits(y1), bits(ref_model(q, s, q1[:k], d1))), ("model", k)
            # the device path: the reference's integer sums (unit scales, so its
            # double result is the sum itself, exact below 2^24), then its float
            # expression (float)acc * d1 * scale in numpy float32
            acc = ref_model(q, np.ones(n, np.float32), q1[:k], np.float32(1.0))
            assert np.all(np.abs(acc) < 2 ** 24)
            want = (acc.astype(np.float32) * np.float32(d1)) * s
            y0 = O.npu_matvec(q, s, q1[:k], d1, model=0)
            assert np.array_equal(bits(y0), bits(want)), ("device formula", k)
    # ragged activation lengths for q1
    for n_x in (1, 31, 33, 100):
        x = rng.standard_normal(n_x).astype(np.float32)
        q1, d1 = O.act_quantise_one(x)
        rq1, rd1 = ref_q1(x)
        assert np.array_equal(q1, rq1) and bits(d1) == bits(rd1), ("q1 ragged", n_x)
    print("npu pins ok")


if __name__ == "__main__":
    main()
