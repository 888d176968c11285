"""The device's ordered sums (charsiu_gpu_ordered_sum_dev: the softmax sum's
one-thread form and the rmsnorm's one-CTA form of the decode step) against
the sequential fp32 sum, bit for bit: lengths that do and do not fill its
16-byte words or its threads, ties, binade crossings, zeros, subnormals, inf
and NaN."""
import numpy as np
import pytest

from charsiu_b200.lib import Layer
from ordered_sum_cases import cases, sequential

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def layer():
    with Layer(2048, 2048, 2) as g:
        yield g


@pytest.mark.parametrize("name,a", cases(), ids=[c[0] for c in cases()])
def test_device_sum_is_sequential(layer, name, a):
    import torch
    dev = torch.device("cuda:0")
    at = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)
    out = torch.full((2,), float("nan"), device=dev)
    assert layer.ordered_sum_dev(at.data_ptr(), a.size, out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    want = sequential(a)
    for form, got in zip(("thread", "cta"), out.cpu().numpy()):
        if np.isnan(want):
            assert np.isnan(got), form
        else:
            assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), \
                (form, got, want)


def test_device_sum_random(layer):
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(11)
    out = torch.zeros(2, device=dev)
    for _ in range(300):
        n = int(rng.integers(1, 8193))
        x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 4)).astype(np.float32)
        a = x * x
        at = torch.from_numpy(a).to(dev)
        assert layer.ordered_sum_dev(at.data_ptr(), n, out.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint32)
        assert got[0] == sequential(a).view(np.uint32) and got[1] == got[0], n
