"""charsiu's NPU device layer (charsiu_npu_*) on the GPU: the NPU number
format's matvec, y = (float)acc * d1 * scale with acc the exact int32 dot
(src/npudev.c:605, 710), bit for bit against the oracle's restatement of the
device path, through the flat, struct and device-pointer forms; and the
refusals npudev.c's conventions call for."""
import ctypes as C

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200.lib import NpuActStruct, NpuLayer, NpuTensorStruct
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def npu_tensor(qtype, k, n, seed):
    blk = G.quant_blocks(np.random.default_rng(seed), qtype, n, k)
    q, s, _ = O.npu_tensor_build(qtype, blk, k, n)
    return q, s


def activation(k, seed):
    x = np.random.default_rng(seed).standard_normal(k).astype(np.float32)
    return O.act_quantise_one(x)


@pytest.fixture(scope="module")
def layer():
    with NpuLayer(14336, 128256, 32) as g:
        yield g


# (K, N): the Llama-3.2-1B projection shapes, ragged ones (K not a multiple
# of 16 or 32, N not of the rows a warp takes), the widest K, the head
SHAPES = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (256, 1000), (100, 33),
          (4096, 77), (14336, 64), (2048, 128256)]


@pytest.mark.parametrize("k,n", SHAPES)
def test_matvec_vs_oracle(layer, k, n):
    qt = G.GGML_Q8_0 if k % 32 == 0 else None
    if qt is None:
        rng = np.random.default_rng(k + n)
        q = rng.integers(-127, 128, size=(n, k)).astype(np.int8)
        s = (np.abs(rng.normal(0, 0.02, n)) / 127).astype(np.float32)
    else:
        q, s = npu_tensor(qt, k, n, k + n)
    q1, d1 = activation(k, n)
    tid = layer.add(q, s, f"t{k}x{n}")
    (y,) = layer.matvec([tid], q1, d1, k)
    want = O.npu_matvec(q, s, q1[:k], d1, model=0)
    assert np.array_equal(bits(y), bits(want))


def test_group_is_the_singles(layer):
    """q, k, v of one activation in one launch: each y as its single call."""
    ts = [npu_tensor(G.GGML_Q4_0, 2048, n, 70 + n) for n in (2048, 512, 512)]
    ids = [layer.add(q, s) for q, s in ts]
    q1, d1 = activation(2048, 9)
    ys = layer.matvec(ids, q1, d1, 2048)
    for (q, s), tid, y in zip(ts, ids, ys):
        assert np.array_equal(bits(y), bits(layer.matvec([tid], q1, d1, 2048)[0]))
        assert np.array_equal(bits(y), bits(O.npu_matvec(q, s, q1, d1, model=0)))


def test_struct_forms(layer):
    """charsiu_npu_add / charsiu_npu_matvec / _group on charsiu's own structs."""
    q, s = npu_tensor(G.GGML_Q8_0, 2048, 300, 5)
    x = np.random.default_rng(6).standard_normal(2048).astype(np.float32)
    q1, d1 = O.act_quantise_one(x)
    t = NpuTensorStruct(q=q.ctypes.data, scale=s.ctypes.data, kgroup=2048, n=300, k=2048,
                        name=b"blk.0.attn_q.weight")
    tid = layer.add_struct(t)
    assert tid >= 0
    assert layer.add_struct(t) == tid            # the same tensor: the same id
    a = NpuActStruct(f=x.ctypes.data, n=2048, nb=64, q1=q1.ctypes.data, d1=float(d1), q1_valid=1)
    y = np.empty(300, np.float32)
    assert layer.L.charsiu_npu_matvec(layer.h, tid, C.byref(a), y.ctypes.data) == 0
    want = O.npu_matvec(q, s, q1, d1, model=0)
    assert np.array_equal(bits(y), bits(want))
    y2 = np.empty(300, np.float32)
    ids = (C.c_int * 2)(tid, tid)
    ys = (C.c_void_p * 2)(y.ctypes.data, y2.ctypes.data)
    y[:] = 0
    assert layer.L.charsiu_npu_matvec_group(layer.h, C.addressof(ids), 2, C.byref(a),
                                            C.addressof(ys)) == 0
    assert np.array_equal(bits(y), bits(want)) and np.array_equal(bits(y2), bits(want))


def test_device_form(layer):
    """charsiu_npu_matvec_dev: q1 and y in GPU memory, on a caller's stream."""
    import torch
    dev = torch.device("cuda:0")
    ts = [npu_tensor(G.GGML_Q8_0, 2048, n, 90 + n) for n in (8192, 8192)]
    ids = [layer.add(q, s) for q, s in ts]
    q1, d1 = activation(2048, 11)
    q1_t = torch.from_numpy(q1[:2048].copy()).to(dev)
    ys = [torch.full((8192,), float("nan"), device=dev) for _ in ids]
    st = torch.cuda.current_stream().cuda_stream
    assert layer.matvec_dev(ids, q1_t.data_ptr(), d1, [y.data_ptr() for y in ys], st) == 0
    torch.cuda.synchronize()
    for (q, s), y in zip(ts, ys):
        assert np.array_equal(bits(y.cpu().numpy()), bits(O.npu_matvec(q, s, q1, d1, model=0)))


def test_refusals():
    """The forms the device arithmetic does not cover, a wrong K, and a tensor
    wider than the layer was opened for are refused (-1), not computed."""
    with NpuLayer(2048, 4096, 4) as g:
        q, s = npu_tensor(G.GGML_Q8_0, 2048, 64, 1)
        grouped = NpuTensorStruct(q=q.ctypes.data, scale=s.ctypes.data, kgroup=256, n=64,
                                  k=2048, name=b"grouped")
        assert g.add_struct(grouped) == -1
        kf = np.ones(2048, np.float32)
        kfac = NpuTensorStruct(q=q.ctypes.data, scale=s.ctypes.data, kgroup=0, n=64, k=2048,
                               kscale=kf.ctypes.data, name=b"kfactor")
        assert g.add_struct(kfac) == -1
        wide = np.zeros((8192, 64), np.int8)
        assert g.L.charsiu_npu_add_flat(g.h, wide.ctypes.data, np.ones(8192, np.float32).ctypes.data,
                                        8192, 64, b"wide") == -1
        tid = g.add(q, s)
        q1, d1 = activation(1024, 2)
        idarr = (C.c_int * 1)(tid)
        y = np.empty(64, np.float32)
        yarr = (C.c_void_p * 1)(y.ctypes.data)
        assert g.L.charsiu_npu_matvec_flat(g.h, C.addressof(idarr), 1, q1.ctypes.data, float(d1),
                                           1024, C.addressof(yarr)) == -1
        assert not g.dead
        assert g.calls == 0
