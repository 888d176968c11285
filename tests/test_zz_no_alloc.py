"""The batched matvec for callers that cannot allocate GPU memory while they
run (a server whose memory pool already owns the GPU's free memory, or a
latency-bound loop that must not take cudaMalloc's device synchronisation):
charsiu_gpu_matvec_batch_noalloc keeps its scratch in a fixed 1 MiB array
inside the library instead of growing a buffer.

It must give exactly what charsiu_gpu_matvec_batch_dev gives (the tests' bar
for this path is bit-identity), including on the second of two calls in a row
that reuse the shared array, and it must refuse sizes the array cannot hold
without retiring the layer.
"""
import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer

pytestmark = pytest.mark.gpu


def _device_activations(torch, layer, m, k, seed, dev, stream):
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(seed)).to(dev)
    q = torch.empty((m, k), dtype=torch.int8, device=dev)
    d = torch.empty((m, k // 32), dtype=torch.float32, device=dev)
    assert layer.act_quantise_dev(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(), stream) == 0
    return q, d


def test_noalloc_matches_batch_dev_on_two_calls_in_a_row():
    torch = pytest.importorskip("torch")
    k, n = 2048, 520
    dev = torch.device("cuda:0")
    with Layer(max_k=8192, max_n=n, max_tensors=2) as L:
        blk, _ = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=31)
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk, "noalloc")
        stream = torch.cuda.current_stream().cuda_stream
        cases = []
        # tiles of 32, then of 16 activations; then 1 and 8, which the _dev
        # form sends to the CUDA cores and this one to the tensor cores
        for m, seed in ((48, 1), (9, 2), (1, 3), (8, 4)):
            q, d = _device_activations(torch, L, m, k, seed, dev, stream)
            ref = torch.full((m, n), float("nan"), device=dev)
            assert L.batch_dev(tid, m, q.data_ptr(), d.data_ptr(), ref.data_ptr(), stream) == 0
            cases.append((m, q, d, ref))
        torch.cuda.synchronize()
        outs = []
        before = L.launches
        for m, q, d, _ in cases:                 # the two allocation-free calls, back to back
            y = torch.full((m, n), float("nan"), device=dev)
            assert L.batch_noalloc(tid, m, q.data_ptr(), d.data_ptr(), y.data_ptr(), stream) == 0
            outs.append(y)
        torch.cuda.synchronize()
        # two launches a call: the packing into the library's array, then the
        # tensor-core matvec reading it (never the tensor copies from q and d
        # that the _dev form uses where it can)
        assert L.launches - before == 2 * len(cases)
        for (m, _, _, ref), y in zip(cases, outs):
            a = y.cpu().numpy().view(np.uint32)
            b = ref.cpu().numpy().view(np.uint32)
            assert np.array_equal(a, b), f"m={m}"


def test_noalloc_refuses_what_the_scratch_cannot_hold():
    torch = pytest.importorskip("torch")
    k, n, m = 8192, 64, 200                      # 2.4 MB of packed activations > 1 MiB
    dev = torch.device("cuda:0")
    with Layer(max_k=k, max_n=n, max_tensors=2) as L:
        blk, _ = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=32)
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk)
        q = torch.zeros((m, k), dtype=torch.int8, device=dev)
        d = torch.zeros((m, k // 32), dtype=torch.float32, device=dev)
        y = torch.zeros((m, n), dtype=torch.float32, device=dev)
        assert L.batch_noalloc(tid, m, q.data_ptr(), d.data_ptr(), y.data_ptr()) == -1
        assert "allocation-free" in L.error()
        assert not L.dead


def test_noalloc_at_the_limit_and_one_past_it():
    """The documented largest case, 64 activations at K = 14336 (1,032,192 of
    the 1,048,576 bytes), runs and matches the _dev form; 65 activations are
    refused with the layer left alive."""
    torch = pytest.importorskip("torch")
    k, n = 14336, 40
    dev = torch.device("cuda:0")
    with Layer(max_k=k, max_n=n, max_tensors=2) as L:
        blk, _ = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=33)
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk, "limit")
        stream = torch.cuda.current_stream().cuda_stream
        q, d = _device_activations(torch, L, 65, k, 5, dev, stream)
        ref = torch.full((64, n), float("nan"), device=dev)
        y = torch.full((64, n), float("nan"), device=dev)
        assert L.batch_dev(tid, 64, q.data_ptr(), d.data_ptr(), ref.data_ptr(), stream) == 0
        assert L.batch_noalloc(tid, 64, q.data_ptr(), d.data_ptr(), y.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))
        y65 = torch.zeros((65, n), dtype=torch.float32, device=dev)
        assert L.batch_noalloc(tid, 65, q.data_ptr(), d.data_ptr(), y65.data_ptr(), stream) == -1
        assert "allocation-free" in L.error()
        assert not L.dead
