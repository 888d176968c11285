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


def _gather_rank(rank, world, port, result):
    """One rank of the fused matvec + all-gather: the slab's y stored into every
    rank's full output over peer memory, arrivals counted in every rank's sync
    words; the second launch waits for the first's arrivals from every rank."""
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        k = 2048
        shapes = [(2056, 11), (512, 12), (128256, 13)]       # ragged, small, the head
        blks = [W.matvec_inputs(G.GGML_Q8_0, k, n, seed=s)[0] for n, s in shapes]
        x = np.random.default_rng(3).normal(size=k).astype(np.float32)
        q, d = O.act_quantise(x)
        dev = torch.device("cuda", rank)
        ok = True
        with Layer(max_k=k, max_n=128256, max_tensors=4, device=rank, rank=rank,
                   world=world) as L:
            ids = [L.add_blocks(G.GGML_Q8_0, k, n, b) for (n, _), b in zip(shapes, blks)]
            mine = [L.ipc_alloc(4 * n) for n, _ in shapes] + [L.ipc_alloc(64)]
            allh = [None] * world
            dist.all_gather_object(allh, [L.ipc_handle(p) for p in mine])
            bufs = [mine if r == rank else [L.ipc_open(h) for h in allh[r]]
                    for r in range(world)]                 # bufs[r]: rank r's, as seen here
            syncs = [bufs[r][3] for r in range(world)]
            groups = [(n + 7) // 8 for n, _ in shapes]
            qt_ = torch.from_numpy(q).to(dev)
            dt_ = torch.from_numpy(d).to(dev)
            s = torch.cuda.current_stream().cuda_stream
            dist.barrier()                       # every rank's buffers exist and are zero
            ok &= L.gather_epoch_dev(mine[3], s) == 0
            # launch 1: tensors 0 and 1 together; launch 2: the head, after every
            # rank's part of launch 1 has arrived in this rank's sync words
            ok &= L.matvec_gather_dev(ids[:2], qt_.data_ptr(), dt_.data_ptr(),
                                      [bufs[r][i] for r in range(world) for i in (0, 1)],
                                      syncs, signal_idx=1, stream=s) == 0
            ok &= L.matvec_gather_dev(ids[2:], qt_.data_ptr(), dt_.data_ptr(),
                                      [bufs[r][2] for r in range(world)], syncs,
                                      signal_idx=2, wait_idx=1, wait_mult=groups[0] + groups[1],
                                      wait_adj=0, stream=s) == 0
            torch.cuda.synchronize()
            ok &= L.kernel_error() == 0
            dist.barrier()                       # every rank's stores into this rank are done
            for (n, _), b, p in zip(shapes, blks, mine):
                got = L.read_device(p, np.empty(n, dtype=np.float32))
                want = O.matvec(G.GGML_Q8_0, b, k, n, q, d)
                ok &= bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
            counts = L.read_device(mine[3], np.empty(16, dtype=np.uint32))
            ok &= bool(counts[0] == 1 and counts[1] == groups[0] + groups[1]
                       and counts[2] == groups[2])
            dist.barrier()
            for r in range(world):
                if r != rank:
                    for p in bufs[r]:
                        L.ipc_free(p, True)
            dist.barrier()
            for p in mine:
                L.ipc_free(p, False)
        result[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_fused_gather_ranks_one_per_gpu():
    torch = pytest.importorskip("torch")
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("the fused gather waits on other GPUs: needs two or more")
    import torch.multiprocessing as mp
    world = min(ngpu, 8)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_gather_rank, args=(r, world, port, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        assert all(result[r] for r in range(world))


def test_batched_gather_emulated_ranks_on_one_gpu():
    """The batched matvec fused with its all-gather, ranks emulated one after
    another on one GPU with no waits (every 'peer' buffer is this GPU's): each
    rank's launch stores its rows of all m activations into every rank's full
    [m][N] output and adds 1 to every rank's arrival word."""
    torch = pytest.importorskip("torch")
    k, world, m = 2048, 3, 20
    shapes = [(1032, 21), (264, 22)]
    blks = [W.matvec_inputs(G.GGML_Q8_0, k, n, seed=s)[0] for n, s in shapes]
    dev = torch.device("cuda:0")
    xs = np.random.default_rng(4).normal(size=(m, k)).astype(np.float32)
    qd = [O.act_quantise(x) for x in xs]
    q = torch.from_numpy(np.stack([a for a, _ in qd])).to(dev)
    d = torch.from_numpy(np.stack([b for _, b in qd])).to(dev)
    layers = [Layer(max_k=k, max_n=1032, max_tensors=2, device=0, rank=r, world=world)
              for r in range(world)]
    try:
        ids = [[L.add_blocks(G.GGML_Q8_0, k, n, b) for (n, _), b in zip(shapes, blks)]
               for L in layers]
        full = [[torch.full((m, n), float("nan"), device=dev) for n, _ in shapes]
                for _ in range(world)]
        syncs = [torch.zeros(16, dtype=torch.int32, device=dev) for _ in range(world)]
        s = torch.cuda.current_stream().cuda_stream
        for r, L in enumerate(layers):
            assert L.batch_gather_dev(ids[r], m, q.data_ptr(), d.data_ptr(),
                                      [full[rr][i].data_ptr() for rr in range(world)
                                       for i in range(2)],
                                      [sy.data_ptr() for sy in syncs], signal_idx=1,
                                      stream=s) == 0
        torch.cuda.synchronize()
        for r, L in enumerate(layers):
            assert L.kernel_error() == 0
        for i, ((n, _), b) in enumerate(zip(shapes, blks)):
            want = np.stack([O.matvec(G.GGML_Q8_0, b, k, n, a, dd) for a, dd in qd])
            for rr in range(world):
                got = full[rr][i].cpu().numpy()
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        for sy in syncs:
            assert sy.cpu().numpy()[1] == world
    finally:
        for L in layers:
            L.close()


def _batch_gather_rank(rank, world, port, result):
    """One rank of the batched fused gather: two launches, the second waiting
    for every rank's arrival from the first."""
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        k, m = 2048, 33
        shapes = [(2056, 31), (512, 32), (8192, 33)]
        blks = [W.matvec_inputs(G.GGML_Q8_0, k, n, seed=s)[0] for n, s in shapes]
        xs = np.random.default_rng(5).normal(size=(m, k)).astype(np.float32)
        qd = [O.act_quantise(x) for x in xs]
        dev = torch.device("cuda", rank)
        q = torch.from_numpy(np.stack([a for a, _ in qd])).to(dev)
        d = torch.from_numpy(np.stack([b for _, b in qd])).to(dev)
        ok = True
        with Layer(max_k=k, max_n=8192, max_tensors=4, device=rank, rank=rank,
                   world=world) as L:
            ids = [L.add_blocks(G.GGML_Q8_0, k, n, b) for (n, _), b in zip(shapes, blks)]
            mine = [L.ipc_alloc(4 * m * n) for n, _ in shapes] + [L.ipc_alloc(64)]
            allh = [None] * world
            dist.all_gather_object(allh, [L.ipc_handle(p) for p in mine])
            bufs = [mine if r == rank else [L.ipc_open(h) for h in allh[r]]
                    for r in range(world)]
            syncs = [bufs[r][3] for r in range(world)]
            s = torch.cuda.current_stream().cuda_stream
            dist.barrier()
            ok &= L.gather_epoch_dev(mine[3], s) == 0
            ok &= L.batch_gather_dev(ids[:2], m, q.data_ptr(), d.data_ptr(),
                                     [bufs[r][i] for r in range(world) for i in (0, 1)],
                                     syncs, signal_idx=1, stream=s) == 0
            ok &= L.batch_gather_dev(ids[2:], m, q.data_ptr(), d.data_ptr(),
                                     [bufs[r][2] for r in range(world)], syncs,
                                     signal_idx=2, wait_idx=1, wait_mult=world, wait_adj=0,
                                     stream=s) == 0
            torch.cuda.synchronize()
            ok &= L.kernel_error() == 0
            dist.barrier()
            for (n, _), b, p in zip(shapes, blks, mine):
                got = L.read_device(p, np.empty((m, n), dtype=np.float32))
                want = np.stack([O.matvec(G.GGML_Q8_0, b, k, n, a, dd) for a, dd in qd])
                ok &= bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
            counts = L.read_device(mine[3], np.empty(16, dtype=np.uint32))
            ok &= bool(counts[0] == 1 and counts[1] == world and counts[2] == world)
            dist.barrier()
            for r in range(world):
                if r != rank:
                    for p in bufs[r]:
                        L.ipc_free(p, True)
            dist.barrier()
            for p in mine:
                L.ipc_free(p, False)
        result[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_batched_gather_ranks_one_per_gpu():
    torch = pytest.importorskip("torch")
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("the fused gather waits on other GPUs: needs two or more")
    import torch.multiprocessing as mp
    world = min(ngpu, 8)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_batch_gather_rank, args=(r, world, port, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        assert all(result[r] for r in range(world))
