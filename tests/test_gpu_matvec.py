"""The block-quant matvec on the GPU, through the C ABI, against the oracle and
the reference's golden vectors: y must be bit-identical (the CUDA path sums
blocks in the reference's order), the integer block dots exact."""
import os

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "golden.npz"))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def same(a, b):
    return np.array_equal(bits(a), bits(b))


@pytest.fixture(scope="module")
def layer():
    with Layer(max_k=8256, max_n=128256, max_tensors=200) as L:
        yield L


@pytest.mark.parametrize("name", list(W.MATVEC_GOLDEN))
def test_golden_small_shapes(layer, name):
    qt, k, n, _ = W.MATVEC_GOLDEN[name]
    tid = layer.add_blocks(qt, k, n, GOLD[f"{name}_blocks"], name)
    q, d = GOLD[f"{name}_q"], GOLD[f"{name}_d"]
    (y,) = layer.matvec([tid], q, d, k)
    assert same(y, GOLD[f"{name}_y"])
    if f"{name}_dots" in GOLD:
        assert np.array_equal(layer.block_dots(tid, q), GOLD[f"{name}_dots"])


@pytest.mark.parametrize("name", list(W.MATVEC_SEEDED))
def test_workload_shapes_bit_exact(layer, name):
    qt, k, n, seed = W.MATVEC_SEEDED[name]
    blk, x = W.matvec_inputs(qt, k, n, seed)
    tid = layer.add_blocks(qt, k, n, blk, name)
    q, d = O.act_quantise(x)
    (y,) = layer.matvec([tid], q, d, k)
    assert same(y, GOLD[f"{name}_y"])
    # twice: the second call reuses every staging buffer
    (y2,) = layer.matvec([tid], q, d, k)
    assert same(y2, y)


@pytest.mark.parametrize("qt", [G.GGML_Q8_0, G.GGML_Q4_0])
@pytest.mark.parametrize("k,n", [(32, 1), (32, 7), (64, 9), (96, 40), (544, 31), (2080, 17),
                                 (8192, 8), (8224, 3), (2048, 1000)])
def test_ragged_shapes_vs_oracle(layer, qt, k, n):
    blk, x = W.matvec_inputs(qt, k, n, seed=k * 7 + n)
    x[: min(k, 64)] = 0.0            # all-zero activation blocks (d = 0)
    tid = layer.add_blocks(qt, k, n, blk)
    q, d = O.act_quantise(x)
    (y,) = layer.matvec([tid], q, d, k)
    assert same(y, O.matvec(qt, blk, k, n, q, d))
    assert np.array_equal(layer.block_dots(tid, q), O.block_dots(qt, blk, k, n, q))


@pytest.mark.parametrize("k,n", [(256, 1), (256, 7), (768, 33), (1280, 17), (2048, 40),
                                 (2048, 1000), (4096, 130), (8192, 9), (2048, 128256)])
def test_q6k_vs_oracle(layer, k, n):
    """q6_K (the tied head of llama.cpp's q4_0 files), 256-weight super-blocks,
    ragged N and the 2048 -> 128256 head: bit-exact, as a single call, inside a
    group with a q8_0 tensor, and for three activations."""
    blk, x = W.matvec_inputs(G.GGML_Q6_K, k, n, seed=k + n)
    x[:64] = 0.0
    tid = layer.add_blocks(G.GGML_Q6_K, k, n, blk)
    q, d = O.act_quantise(x)
    want = O.matvec(G.GGML_Q6_K, blk, k, n, q, d)
    (y,) = layer.matvec([tid], q, d, k)
    assert same(y, want)
    if n <= 1000:
        b8, _ = W.matvec_inputs(G.GGML_Q8_0, k, 24, seed=7)
        t8 = layer.add_blocks(G.GGML_Q8_0, k, 24, b8)
        y8, y6 = layer.matvec([t8, tid], q, d, k)
        assert same(y6, want) and same(y8, O.matvec(G.GGML_Q8_0, b8, k, 24, q, d))
        xs = np.random.default_rng(n).normal(size=(3, k)).astype(np.float32)
        qs, ds = zip(*(O.act_quantise(v) for v in xs))
        yb = layer.batch(tid, np.stack(qs), np.stack(ds))
        for i in range(3):
            assert same(yb[i], O.matvec(G.GGML_Q6_K, blk, k, n, qs[i], ds[i])), f"row {i}"


def test_group_equals_singles(layer):
    k = 2048
    shapes = [(G.GGML_Q8_0, 2048), (G.GGML_Q8_0, 512), (G.GGML_Q4_0, 512), (G.GGML_Q8_0, 8192),
              (G.GGML_Q4_0, 40)]
    ids, blks = [], []
    for i, (qt, n) in enumerate(shapes):
        blk, _ = W.matvec_inputs(qt, k, n, seed=100 + i)
        ids.append(layer.add_blocks(qt, k, n, blk, f"g{i}"))
        blks.append((qt, blk, n))
    x = np.random.default_rng(5).normal(size=k).astype(np.float32)
    q, d = O.act_quantise(x)
    ys = layer.matvec(ids, q, d, k)
    for (qt, blk, n), y in zip(blks, ys):
        assert same(y, O.matvec(qt, blk, k, n, q, d))


def test_direct_and_graph_calls_agree(monkeypatch):
    """A host call of one activation runs the direct path (copy-in kernel,
    y written into mapped host memory, a flag raised by the last CTA); with
    CHARSIU_GPU_DIRECT=0 the same call goes through a graph of copies and
    kernels. Both must give the reference's bits, call after call."""
    k = 2048
    shapes = [(G.GGML_Q8_0, 2048), (G.GGML_Q8_0, 520), (G.GGML_Q8_0, 9)]
    blks = [W.matvec_inputs(qt, k, n, seed=500 + i)[0] for i, (qt, n) in enumerate(shapes)]
    xs = np.random.default_rng(8).normal(size=(24, k)).astype(np.float32)
    outs = {}
    for direct in ("1", "0"):
        monkeypatch.setenv("CHARSIU_GPU_DIRECT", direct)
        with Layer(max_k=k, max_n=4096, max_tensors=4) as L:
            ids = [L.add_blocks(qt, k, n, b) for (qt, n), b in zip(shapes, blks)]
            outs[direct] = []
            for x in xs:
                q, d = O.act_quantise(x)
                outs[direct].append(L.matvec(ids, q, d, k))
                outs[direct].append(L.matvec(ids[1:2], q, d, k))
            assert L.calls == 2 * len(xs)
    for j, x in enumerate(xs):
        q, d = O.act_quantise(x)
        for (qt, n), b, y1, y0 in zip(shapes, blks, outs["1"][2 * j], outs["0"][2 * j]):
            ref = O.matvec(qt, b, k, n, q, d)
            assert same(y1, ref) and same(y0, ref), f"activation {j} n={n}"
        assert same(outs["1"][2 * j + 1][0], outs["1"][2 * j][1])


def test_output_head_shape(layer):
    """The 2048 -> 128256 tied head, q8_0: 16032 row groups in one launch."""
    k, n = 2048, 128256
    blk, x = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=77)
    tid = layer.add_blocks(G.GGML_Q8_0, k, n, blk, "output")
    q, d = O.act_quantise(x)
    (y,) = layer.matvec([tid], q, d, k)
    assert same(y, O.matvec(G.GGML_Q8_0, blk, k, n, q, d))


def test_q6k_more_than_one_pass():
    """K = 12288: 48 super-blocks, more than one pass of the 16-warp q6_K
    kernel's 32 (the loads of a later pass issued after the last's dots)."""
    k, n = 12288, 24
    with Layer(max_k=k, max_n=n, max_tensors=1) as L:
        blk, x = W.matvec_inputs(G.GGML_Q6_K, k, n, seed=5)
        tid = L.add_blocks(G.GGML_Q6_K, k, n, blk)
        q, d = O.act_quantise(x)
        (y,) = L.matvec([tid], q, d, k)
        assert same(y, O.matvec(G.GGML_Q6_K, blk, k, n, q, d))


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 13, 32, 64, 100])
@pytest.mark.parametrize("qt", [G.GGML_Q8_0, G.GGML_Q4_0])
@pytest.mark.parametrize("k,n", [(2048, 520), (8192, 136)])
def test_batch_rows_match_single_matvec(layer, m, qt, k, n):
    """M > 1: q8_0 batches of 9 or more run on the tensor cores (tcgen05
    kind::i8, tiles of 16 or 32 activations), smaller ones and every q4_0
    batch on the CUDA cores (qmvm_kernel); every row bit-exact."""
    blk, xs = W.batch_inputs(qt, k, n, m, seed=3)
    tid = layer.add_blocks(qt, k, n, blk)
    qs, ds = zip(*(O.act_quantise(x) for x in xs))
    y = layer.batch(tid, np.stack(qs), np.stack(ds))
    for i in range(m):
        assert same(y[i], O.matvec(qt, blk, k, n, qs[i], ds[i])), f"row {i}"


@pytest.mark.parametrize("m", [2, 3, 5, 8, 13])
@pytest.mark.parametrize("k,n", [(2048, 520), (8192, 136), (544, 40)])
def test_batch_on_cuda_cores_q8(monkeypatch, m, k, n):
    """q8_0 batches below CHARSIU_GPU_QMM_MIN_M run on the CUDA cores
    (qmvm_kernel, chunks of 8/4/2/1 activations): every row bit-exact."""
    monkeypatch.setenv("CHARSIU_GPU_QMM_MIN_M", "65")
    blk, xs = W.batch_inputs(G.GGML_Q8_0, k, n, m, seed=11)
    with Layer(max_k=k, max_n=n, max_tensors=2) as L:
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk)
        qs, ds = zip(*(O.act_quantise(x) for x in xs))
        y = L.batch(tid, np.stack(qs), np.stack(ds))
    for i in range(m):
        assert same(y[i], O.matvec(G.GGML_Q8_0, blk, k, n, qs[i], ds[i])), f"row {i}"


def _dev_acts(torch, xs, dev):
    """q8 activations on the device, quantised by the oracle (checked above)."""
    qs, ds = zip(*(O.act_quantise(x) for x in xs))
    q_t = torch.from_numpy(np.ascontiguousarray(np.stack(qs))).to(dev)
    d_t = torch.from_numpy(np.ascontiguousarray(np.stack(ds))).to(dev)
    return qs, ds, q_t, d_t


@pytest.mark.parametrize("m", [2, 5, 8, 17, 64])
@pytest.mark.parametrize("k", [2048, 2080, 544])
def test_batch_group_dev_one_launch(layer, m, k):
    """Several q8_0 tensors of one K in one launch (as q/k/v and gate/up are
    grouped): on the tensor cores from m = 9; below, on the CUDA cores, one
    launch a chunk of 8, 4 or 2 activations and the M = 1 kernel for a last
    single one (m = 5: 4 + 1). Ragged N (a partial last 128-row tile, a
    partial last group) and K with a partial last segment and chunk; every
    row of every tensor bit-exact."""
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda:0")
    ns = [520, 136, 9, 2048]
    ids, blks = [], []
    for i, n in enumerate(ns):
        blk, _ = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=400 + i)
        ids.append(layer.add_blocks(G.GGML_Q8_0, k, n, blk))
        blks.append(blk)
    xs = np.random.default_rng(m * 31 + k).normal(size=(m, k)).astype(np.float32)
    xs[m // 2, :64] = 0.0                 # zero activation blocks
    qs, ds, q_t, d_t = _dev_acts(torch, xs, dev)
    ys = [torch.full((m, n), float("nan"), device=dev) for n in ns]
    stream = torch.cuda.current_stream().cuda_stream
    assert layer.batch_group_dev(ids, m, q_t.data_ptr(), d_t.data_ptr(),
                                 [y.data_ptr() for y in ys], stream) == 0
    torch.cuda.synchronize()
    for blk, n, y in zip(blks, ns, ys):
        yc = y.cpu().numpy()
        for i in range(m):
            assert same(yc[i], O.matvec(G.GGML_Q8_0, blk, k, n, qs[i], ds[i])), f"n={n} row {i}"


@pytest.mark.parametrize("k,d_off,launches", [(2176, 0, 1), (2080, 0, 2), (2048, 4, 2)])
def test_batch_activation_staging_paths(layer, k, d_off, launches):
    """The tensor-core launch stages the activations by two tiled tensor
    copies straight from q and d when both can be described (16-byte
    aligned, nb a multiple of 4): one launch a group, here with a partial
    last K segment (nb = 68, 4 blocks). Otherwise (nb = 65, or d 4 bytes off
    a 16-byte boundary) a packing launch goes first. Both bit-exact, with a
    ragged last activation tile."""
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda:0")
    m, ns = 21, [520, 9]
    ids, blks = [], []
    for i, n in enumerate(ns):
        blk, _ = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=700 + i)
        ids.append(layer.add_blocks(G.GGML_Q8_0, k, n, blk))
        blks.append(blk)
    xs = np.random.default_rng(k + d_off).normal(size=(m, k)).astype(np.float32)
    qs, ds, q_t, d_t = _dev_acts(torch, xs, dev)
    d_buf = torch.zeros(d_t.numel() + 4, dtype=torch.float32, device=dev)
    d_buf[d_off // 4:d_off // 4 + d_t.numel()].copy_(d_t.reshape(-1))
    ys = [torch.full((m, n), float("nan"), device=dev) for n in ns]
    before = layer.launches
    assert layer.batch_group_dev(ids, m, q_t.data_ptr(), d_buf.data_ptr() + d_off,
                                 [y.data_ptr() for y in ys],
                                 torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert layer.launches - before == launches
    for blk, n, y in zip(blks, ns, ys):
        yc = y.cpu().numpy()
        for i in range(m):
            assert same(yc[i], O.matvec(G.GGML_Q8_0, blk, k, n, qs[i], ds[i])), f"n={n} row {i}"


@pytest.mark.parametrize("na,pre", [("16", "0"), ("16", "1"), ("32", "0"), ("32", "1")])
def test_batch_tile_variants_agree(monkeypatch, na, pre):
    """Every tensor-core tile variant (16 or 32 activations a tile; the int32
    dots converted in the epilogue or accumulated onto the float-bias
    constant in tensor memory) gives the reference's bits, on a tensor with
    more (tile, activation) units than SMs, so CTAs loop."""
    torch = pytest.importorskip("torch")
    monkeypatch.setenv("CHARSIU_GPU_QMM_NA", na)
    monkeypatch.setenv("CHARSIU_GPU_QMM_PRE", pre)
    monkeypatch.setenv("CHARSIU_GPU_QMM_MIN_M", "2")
    dev = torch.device("cuda:0")
    k, n, m = 2048, 20000, 37
    with Layer(max_k=k, max_n=n, max_tensors=2) as L:
        blk, xs = W.batch_inputs(G.GGML_Q8_0, k, n, m, seed=9)
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk)
        qs, ds, q_t, d_t = _dev_acts(torch, xs, dev)
        y = torch.full((m, n), float("nan"), device=dev)
        assert L.batch_dev(tid, m, q_t.data_ptr(), d_t.data_ptr(), y.data_ptr(),
                           torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        yc = y.cpu().numpy()
        for i in (0, 1, 15, 16, 31, 32, 36):
            assert same(yc[i], O.matvec(G.GGML_Q8_0, blk, k, n, qs[i], ds[i])), f"row {i}"


@pytest.mark.parametrize("pre", ["0", "1"])
def test_batch_extreme_blocks(monkeypatch, pre):
    """Blocks at the int8 extremes, where a block's dot is largest
    (32 * 128 * 127), on both epilogues, with ragged K (a partial last
    16-block segment)."""
    torch = pytest.importorskip("torch")
    monkeypatch.setenv("CHARSIU_GPU_QMM_MIN_M", "2")
    monkeypatch.setenv("CHARSIU_GPU_QMM_PRE", pre)
    dev = torch.device("cuda:0")
    k, n, m = 2080, 300, 20
    rng = np.random.default_rng(77)
    blk = G.quant_blocks(rng, G.GGML_Q8_0, n, k)
    b3 = blk.reshape(n, k // 32, 34)
    pattern = rng.choice(np.array([-128, -127, 127], dtype=np.int8), size=(n, k // 32, 32))
    b3[:, :, 2:] = pattern.view(np.uint8)
    xs = rng.normal(size=(m, k)).astype(np.float32)
    xs[:, ::3] *= 40.0                    # many activations quantise to +-127
    with Layer(max_k=k, max_n=n, max_tensors=2) as L:
        tid = L.add_blocks(G.GGML_Q8_0, k, n, blk)
        qs, ds, q_t, d_t = _dev_acts(torch, xs, dev)
        y = torch.full((m, n), float("nan"), device=dev)
        assert L.batch_dev(tid, m, q_t.data_ptr(), d_t.data_ptr(), y.data_ptr(),
                           torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        yc = y.cpu().numpy()
    for i in range(m):
        assert same(yc[i], O.matvec(G.GGML_Q8_0, blk, k, n, qs[i], ds[i])), f"row {i}"


def test_device_forms_and_quantiser(layer):
    torch = pytest.importorskip("torch")
    k, n, m = 8192, 2048, 4
    blk, xs = W.batch_inputs(G.GGML_Q4_0, k, n, m, seed=21)
    xs[1, :96] = 0.0
    tid = layer.add_blocks(G.GGML_Q4_0, k, n, blk)
    dev = torch.device("cuda:0")
    x_t = torch.from_numpy(xs).to(dev)
    q_t = torch.empty((m, k), dtype=torch.int8, device=dev)
    d_t = torch.empty((m, k // 32), dtype=torch.float32, device=dev)
    y_t = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert layer.act_quantise_dev(x_t.data_ptr(), m, k, q_t.data_ptr(), d_t.data_ptr(), stream) == 0
    assert layer.batch_dev(tid, m, q_t.data_ptr(), d_t.data_ptr(), y_t.data_ptr(), stream) == 0
    y1 = torch.full((n,), float("nan"), dtype=torch.float32, device=dev)
    assert layer.matvec_dev([tid], q_t[2].data_ptr(), d_t[2].data_ptr(), [y1.data_ptr()],
                            stream) == 0
    torch.cuda.synchronize()
    qg, dg, yg = q_t.cpu().numpy(), d_t.cpu().numpy(), y_t.cpu().numpy()
    for i in range(m):
        q, d = O.act_quantise(xs[i])
        assert np.array_equal(qg[i], q) and same(dg[i], d), f"quantiser row {i}"
        assert same(yg[i], O.matvec(G.GGML_Q4_0, blk, k, n, q, d)), f"row {i}"
    assert same(y1.cpu().numpy(), yg[2])


def test_rejects_bad_input(layer):
    blk, _ = W.matvec_inputs(G.GGML_Q8_0, 64, 8, seed=1)
    assert layer.try_add_blocks(G.GGML_F32, 64, 8, blk) == -1
    assert layer.try_add_blocks(G.GGML_Q8_0, 48, 8, blk) == -1          # K not a multiple of 32
    assert layer.try_add_blocks(G.GGML_Q8_0, 64, 10 ** 7, blk) == -1    # wider than opened
    tid = layer.add_blocks(G.GGML_Q8_0, 64, 8, blk)
    q = np.zeros(128, np.int8)
    d = np.zeros(4, np.float32)
    y = np.zeros(8, np.float32)
    assert layer.try_matvec([tid], q, d, 128, [y]) == -1                # K mismatch
    assert not layer.dead
