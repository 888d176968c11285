"""The algorithm of the rmsnorm's parallel ordered sum, restated step for step
in numpy fp32 (ordered_sum_model.py), against the sequential fp32 sum on the
cases the GPU test uses (ties, crossings, zeros, subnormals, inf, NaN) and on
random squares: the result must be the sequential sum's bits whichever path
(the fast walk, a fallback part way, or all sequential) it takes. CPU only;
the kernel itself is checked on the GPU (test_gpu_ordered_sum.py)."""
import numpy as np
import pytest

from ordered_sum_cases import cases, sequential
from ordered_sum_model import model_sum


def same(a, b):
    a, b = np.float32(a), np.float32(b)
    return (np.isnan(a) and np.isnan(b)) or a.view(np.uint32) == b.view(np.uint32)


@pytest.mark.parametrize("name,a", cases(), ids=[c[0] for c in cases()])
def test_cases(name, a):
    with np.errstate(over="ignore", invalid="ignore"):
        got, _ = model_sum(a)
        want = sequential(a)
    assert same(got, want), (name, got, want)


def test_random_squares_take_the_fast_path():
    rng = np.random.default_rng(5)
    paths = {}
    for _ in range(40):
        n = int(rng.integers(1, 4097))
        x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 4)).astype(np.float32)
        a = x * x
        got, path = model_sum(a)
        paths[path] = paths.get(path, 0) + 1
        assert same(got, sequential(a)), n
    # the walk, not the fallback, is what ordinary squares take
    assert paths.get("fast", 0) >= 35, paths
