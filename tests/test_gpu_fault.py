"""Failure handling of the device layer, with the failures made on the host
(charsiu_gpu_inject): no GPU is ever faulted, trapped or hung. The rules are
the NPU layer's (reference src/npudev.c:531-602): a failed launch retires the
layer at once, three slow calls in a row retire it, a good call clears the
count, and a retired layer refuses every later call."""
import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

K, N = 256, 64


def setup_layer():
    L = Layer(max_k=K, max_n=N, max_tensors=4)
    blk, x = W.matvec_inputs(G.GGML_Q8_0, K, N, seed=4)
    tid = L.add_blocks(G.GGML_Q8_0, K, N, blk)
    q, d = O.act_quantise(x)
    return L, tid, q, d, O.matvec(G.GGML_Q8_0, blk, K, N, q, d)


def call(L, tid, q, d):
    y = np.zeros(N, np.float32)
    return L.try_matvec([tid], q, d, K, [y]), y


def test_failed_launch_retires_at_once():
    L, tid, q, d, want = setup_layer()
    with L:
        calls0 = L.L.charsiu_gpu_calls(L.h)
        L.inject(at=3, count=1, kind=1)         # call numbers count add (1) then calls
        assert call(L, tid, q, d)[0] == 0       # call 2
        rc, _ = call(L, tid, q, d)              # call 3: fails
        assert rc == -1 and L.dead
        assert call(L, tid, q, d)[0] == -1      # retired: refuses
        assert L.L.charsiu_gpu_calls(L.h) == calls0 + 1


def test_three_slow_calls_retire_two_do_not():
    L, tid, q, d, want = setup_layer()
    with L:
        L.inject(at=2, count=2, kind=2)         # calls 2, 3 slow, 4 fine
        for _ in range(3):
            rc, y = call(L, tid, q, d)
            assert rc == 0 and np.array_equal(y, want)
        assert not L.dead
        L.inject(at=5, count=3, kind=2)         # 5, 6, 7 slow: the third retires
        assert call(L, tid, q, d)[0] == 0
        assert call(L, tid, q, d)[0] == 0
        assert call(L, tid, q, d)[0] == -1
        assert L.dead


def test_allocation_failure_at_add_keeps_layer_alive():
    L = Layer(max_k=K, max_n=N, max_tensors=4)
    with L:
        blk, x = W.matvec_inputs(G.GGML_Q4_0, K, N, seed=5)
        L.inject(at=1, count=1, kind=3)
        assert L.try_add_blocks(G.GGML_Q4_0, K, N, blk) == -1
        assert not L.dead
        tid = L.add_blocks(G.GGML_Q4_0, K, N, blk)
        q, d = O.act_quantise(x)
        (y,) = L.matvec([tid], q, d, K)
        assert np.array_equal(y, O.matvec(G.GGML_Q4_0, blk, K, N, q, d))
