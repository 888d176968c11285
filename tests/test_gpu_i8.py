"""The int8 matmul with the NPU's output stage on the GPU, through the C ABI:
byte-exact against cpu_reference's golden outputs at the four workload shapes,
the reference's probe constructions, odd K and arbitrary zero points."""
import os

import numpy as np
import pytest

from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "golden.npz"))


@pytest.fixture(scope="module")
def layer():
    with Layer(max_k=64, max_n=64, max_tensors=1) as L:
        yield L


@pytest.mark.parametrize("name", list(W.I8_SHAPES))
def test_workload_shapes_byte_exact(layer, name):
    m, k, n, seed = W.I8_SHAPES[name]
    a, w, bias = W.i8_inputs(m, k, n, seed)
    sc = tuple(float(v) for v in GOLD[f"{name}_scales"][:3])
    out = layer.matmul_i8(a, w, bias, *sc)       # prefilled with a sentinel
    assert np.array_equal(out, GOLD[f"{name}_out"])


def test_probes(layer):
    k, n = 64, 64
    # NEG: a genuinely negative MAC through zero (tools/charsiu_matmul.c:331-348)
    a = np.full((1, k), 168, np.uint8)
    w = np.array([[128 + (c - n // 2)] * k for c in range(n)], np.uint8)
    bias = np.zeros(n, np.int32)
    assert np.array_equal(layer.matmul_i8(a, w, bias, 0.02, 0.01, 0.25),
                          O.matmul_i8(a, w, bias, 0.02, 0.01, 0.25))
    # CONST: input at the zero point, a bias ramp (:293-302)
    a = np.full((1, k), 128, np.uint8)
    w = np.random.default_rng(1).integers(0, 256, (n, k), dtype=np.uint8)
    bias = np.array([c * 2000 - 60000 for c in range(n)], np.int32)
    assert np.array_equal(layer.matmul_i8(a, w, bias, 0.02, 0.01, 0.25),
                          O.matmul_i8(a, w, bias, 0.02, 0.01, 0.25))


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (3, 7, 5), (33, 33, 65), (2, 257, 31),
                                   (64, 4096, 3), (129, 64, 200), (300, 512, 80),
                                   (1, 4096, 1000)])
@pytest.mark.parametrize("zp", [(128, 128, 0), (0, 255, 7), (77, 140, -20)])
def test_shapes_and_zero_points(layer, m, k, n, zp):
    rng = np.random.default_rng(m + 31 * k + 7 * n)
    a = rng.integers(0, 256, (m, k), dtype=np.uint8)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    bias = rng.integers(-4096, 4097, n, dtype=np.int32)
    for out_scale in (0.03, 1.1, 40.0):
        want = O.matmul_i8(a, w, bias, 0.02, 0.01, out_scale, *zp)
        got = layer.matmul_i8(a, w, bias, 0.02, 0.01, out_scale, *zp)
        assert np.array_equal(got, want), out_scale
