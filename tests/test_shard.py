"""The N-split of a projection over ranks, on the CPU: every row on exactly one
rank, and slabs gathered over a real process group (gloo, world size 2 and 3)
reassemble the full output. The per-rank compute here is the oracle's matvec
of that rank's rows; on the GPU it is the device layer (tests/test_gpu_sharded.py)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from charsiu_b200 import gguf as G
from charsiu_b200 import shard
from charsiu_b200 import workloads as W


@pytest.mark.parametrize("n", [1, 7, 8, 9, 512, 2048, 2049, 128256])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_covers_every_row_once(n, world):
    seen = np.zeros(n, np.int32)
    for r in range(world):
        row0, rows = shard.shard_rows(n, r, world)
        assert rows <= shard.slab_rows(n, world)
        assert row0 % 8 == 0 or rows == 0
        seen[row0:row0 + rows] += 1
    assert (seen == 1).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, qt, k, n, result):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blk, x = W.matvec_inputs(qt, k, n, seed=5)
        q, d = O.act_quantise(x)
        row0, rows = shard.shard_rows(n, rank, world)
        rb = blk.shape[1]
        mine = O.matvec(qt, np.ascontiguousarray(blk[row0:row0 + rows]), k, rows, q, d) \
            if rows else np.zeros(0, np.float32)
        slab = torch.zeros(shard.slab_rows(n, world), dtype=torch.float32)
        slab[:rows] = torch.from_numpy(mine)
        out = [torch.zeros_like(slab) for _ in range(world)]
        dist.all_gather(out, slab)
        full = shard.assemble([o.numpy() for o in out], n, world)
        want = O.matvec(qt, blk, k, n, q, d)
        result[rank] = bool(np.array_equal(full.view(np.uint32), want.view(np.uint32))) \
            and rb == k // 32 * G.BLOCK_BYTES[qt]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,qt,k,n", [(2, G.GGML_Q8_0, 256, 520), (3, G.GGML_Q4_0, 512, 83)])
def test_gathered_slabs_reassemble_the_output(world, qt, k, n):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, qt, k, n, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        assert all(result[r] for r in range(world))
