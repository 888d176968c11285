"""The column-split layer on the GPU: each rank's layer holds and computes only
its slab of rows (the split charsiu_b200.shard mirrors), and the slabs,
gathered, equal the unsharded output bit for bit. Ranks are emulated on one
GPU here; with two or more GPUs the same runs as NCCL ranks, one per GPU."""
import datetime
import os
import socket

import numpy as np
import pytest

from charsiu_b200 import gguf as G
from charsiu_b200 import shard
from charsiu_b200 import workloads as W
from charsiu_b200.lib import Layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("qt,k,n", [(G.GGML_Q8_0, 2048, 128256), (G.GGML_Q4_0, 8192, 520)])
def test_slabs_on_one_gpu(world, qt, k, n):
    blk, x = W.matvec_inputs(qt, k, n, seed=world)
    q, d = O.act_quantise(x)
    slabs = []
    for r in range(world):
        with Layer(max_k=k, max_n=n, max_tensors=1, device=0, rank=r, world=world) as L:
            tid = L.add_blocks(qt, k, n, blk)
            assert L.rows(tid) == shard.shard_rows(n, r, world)
            (y,) = L.matvec([tid], q, d, k)
            slab = np.zeros(shard.slab_rows(n, world), np.float32)
            slab[:len(y)] = y
            slabs.append(slab)
    full = shard.assemble(slabs, n, world)
    want = O.matvec(qt, blk, k, n, q, d)
    assert np.array_equal(full.view(np.uint32), want.view(np.uint32))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, result):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        k, n = 2048, 128256
        blk, x = W.matvec_inputs(G.GGML_Q8_0, k, n, seed=11)
        q, d = O.act_quantise(x)
        dev = torch.device("cuda", rank)
        with Layer(max_k=k, max_n=n, max_tensors=1, device=rank, rank=rank, world=world) as L:
            tid = L.add_blocks(G.GGML_Q8_0, k, n, blk)
            qt_ = torch.from_numpy(q).to(dev)
            dt_ = torch.from_numpy(d).to(dev)
            slab = torch.zeros(shard.slab_rows(n, world), dtype=torch.float32, device=dev)
            s = torch.cuda.current_stream().cuda_stream
            assert L.matvec_dev([tid], qt_.data_ptr(), dt_.data_ptr(), [slab.data_ptr()], s) == 0
            full = torch.empty(world * slab.numel(), dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(full, slab)
            torch.cuda.synchronize()
        got = shard.assemble(full.cpu().numpy().reshape(world, -1), n, world)
        want = O.matvec(G.GGML_Q8_0, blk, k, n, q, d)
        result[rank] = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    finally:
        dist.destroy_process_group()


def test_nccl_ranks_one_per_gpu():
    torch = pytest.importorskip("torch")
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("one GPU: ranks are emulated by test_slabs_on_one_gpu")
    import torch.multiprocessing as mp
    world = min(ngpu, 8)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        assert all(result[r] for r in range(world))
