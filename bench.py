#!/usr/bin/env python
"""Benchmark: Llama-3.2-1B-shaped q8_0 decode, tokens per second.

A step is one greedy decode token: charsiu's whole llama_forward (the
embedding row, 16 layers of rmsnorm, the q/k/v, o, gate/up and down
projections, RoPE, the KV cache, attention, SiLU, the residuals; the final
norm, the 128256-wide tied head and the argmax) on the device. Synthetic
seeded weights with the workload's distributions (no real checkpoint exists on
these machines); the 6 seeded prompt ids of the workload, then greedy tokens
at positions 6..29, checked against the reference's.

  value    tokens/s with the inputs resident in HBM: the greedy steps queued
           back to back with each step's argmax fed to the next on the device
           (charsiu_gpu_decoder_generate), one CUDA graph a step, CUDA events
           around the steps. 1.31 GB of weights a token, far above the 126 MB
           L2, so every token streams its weights from HBM.
  e2e      the same decode through the public C ABI with the host in the loop
           (charsiu_gpu_llama_greedy with the step on the device): each token's
           id and position copied in from pinned host memory and its argmax
           copied back every step. e2e.host_routed is the drop-in form:
           charsiu's CPU rmsnorm/rope/attention/SwiGLU on the host and every
           projection a host-buffer call (charsiu_gpu_llama_forward).
  roofline the block-quant matvec's algorithmic bytes per launch over its
           average launch time, from the token's 65 matvec launches timed
           alone (hot_path), against the measured HBM copy peak.
  configs  the standalone matvec workloads (q8_0 2048x8192, q4_0 8192x2048)
           and the int8 matmul shapes, each beside the reference's CPU code.
  cpu_baseline charsiu's own CPU decode (the reference compiled from its
           sources, oracle/_ref) on this box's host cores.

At N GPUs every GPU decodes its own stream with the whole model (no
collective, weak scaling); `sharded` times the column splits the workload
names -- the 128256-wide head and a token's 65 launches split over the N GPUs
(NCCL all-gathers, and the fused matvec + all-gather over NVLink), and the
batched step at M = 8, 32, 64 -- each checked bit for bit against one GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
  python bench.py --resident | --matvec Q:K:N[:M] | --batch M | --int8 M:K:N | --npu K:N
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from charsiu_b200 import gguf as G  # noqa: E402
from charsiu_b200 import shard  # noqa: E402
from charsiu_b200 import workloads as W  # noqa: E402

METRIC = "Llama-3.2-1B q8_0 decode tok/s"
UNIT = "tok/s"
SPEC = W.DECODE["llama1b_q8"]
SHAPE = SPEC["shape"]
PEAKS_FALLBACK = {"hbm_gbs": 6650.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return PEAKS_FALLBACK["hbm_gbs"], "fallback"


def decode_spec(name: str):
    """The decode workload `name`: the headline llama1b_q8, or one of
    W.DECODE_EXTRA (llama1b_q4_q6k: the same shape as a llama.cpp q4_0 file)."""
    return W.DECODE[name] if name in W.DECODE else W.DECODE_EXTRA[name]


def model_path(rank: int, barrier, name: str = "llama1b_q8") -> str:
    spec = decode_spec(name)
    d = os.path.join(tempfile.gettempdir(), "charsiu_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{name}_seed{spec['seed']}.gguf")
    if rank == 0 and not os.path.exists(path):
        G.write_llama(path, spec["shape"], spec["qtype"], spec["seed"],
                      embd_qtype=spec.get("embd_qtype"))
    barrier()
    return path


# ---- clocks during the timed region ------------------------------------------

CLOCK_Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class Clocks:
    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={CLOCK_Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.2)

    def stop(self):
        if self.p:
            self.p.terminate()
            self.p.wait()
        self.f.flush()
        self.f.seek(0)
        rows = [ln.split(",") for ln in self.f.read().splitlines() if ln.strip()]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4)
                          if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


# ---- the launch plan of one token --------------------------------------------

def launch_groups(shape):
    """[(tensor names, K)] in decode order: 4 launches a layer, then the head."""
    out = []
    for l in range(shape.n_layer):
        b = f"blk.{l}."
        out.append(([b + "attn_q.weight", b + "attn_k.weight", b + "attn_v.weight"], shape.n_embd))
        out.append(([b + "attn_output.weight"], shape.n_embd))
        out.append(([b + "ffn_gate.weight", b + "ffn_up.weight"], shape.n_embd))
        out.append(([b + "ffn_down.weight"], shape.n_ff))
    out.append((["token_embd.weight"], shape.n_embd))
    return out


def algorithmic_bytes(gguf, names, k, rows_of):
    """weights streamed + the q8_0 activation (K + 4K/32) + fp32 outputs."""
    w = sum(rows_of(nm) * (k // 32) * 34 for nm in names)
    return w + k + 4 * (k // 32) + 4 * sum(rows_of(nm) for nm in names)


# ---- our arm -------------------------------------------------------------------

class TokenChain:
    """The 65 launches of one decode token on this GPU, weights resident.

    world == 1: the whole model here. world > 1 (column split): this rank holds
    its slab of every tensor, and each launch group's slabs (one contiguous
    buffer a group) are all-gathered with one NCCL collective -- or, fused,
    every launch stores its rows straight into every rank's full outputs over
    NVLink and the next launch waits on the arrivals
    (charsiu_gpu_matvec_gather_dev)."""

    def __init__(self, gg, dev, rank=0, world=1, dist=None, fused=False, groups=None):
        import torch
        from charsiu_b200.lib import Layer

        self.torch, self.dev, self.world, self.dist = torch, dev, world, dist
        self.gg, self.rank = gg, rank
        self.groups = groups or launch_groups(SHAPE)
        # (a tensor named in several launch groups is added once)
        names = list(dict.fromkeys(nm for g, _ in self.groups for nm in g))
        self.layer = Layer(max_k=max(SHAPE.n_embd, SHAPE.n_ff), max_n=SHAPE.n_vocab,
                           max_tensors=len(names) + 1, device=dev.index, rank=rank, world=world)
        self.ids, self.rows = {}, {}
        for nm in names:
            t = gg.tensors[nm]
            self.ids[nm] = self.layer.add_blocks(t.type, t.k, t.n, np.asarray(gg.data(nm)), nm)
            self.rows[nm] = self.layer.rows(self.ids[nm])[1]
        gen = torch.Generator(device="cpu").manual_seed(1234)
        self.acts = {}
        for k in (SHAPE.n_embd, SHAPE.n_ff):
            x = torch.randn(k, generator=gen).to(dev)
            q = torch.empty(k, dtype=torch.int8, device=dev)
            d = torch.empty(k // 32, dtype=torch.float32, device=dev)
            assert self.layer.act_quantise_dev(x.data_ptr(), 1, k, q.data_ptr(), d.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream) == 0
            self.acts[k] = (q, d)
        # one output buffer a launch group: its tensors' slabs back to back,
        # each padded to the widest rank's slab so a gather moves equal pieces
        self.bufs, self.full = [], []
        for g, _ in self.groups:
            slabs = [shard.slab_rows(gg.tensors[nm].n, world) for nm in g]
            buf = torch.zeros(sum(slabs), dtype=torch.float32, device=dev)
            ptrs, off = [], 0
            for sl in slabs:
                ptrs.append(buf[off:].data_ptr())
                off += sl
            self.bufs.append((buf, ptrs))
            self.full.append(torch.zeros(world * sum(slabs), dtype=torch.float32, device=dev)
                             if world > 1 else None)
        self.bytes_per_token = sum(algorithmic_bytes(gg, g, k, lambda nm: self.rows[nm])
                                   for g, k in self.groups)
        self.fused = fused and world > 1
        if self.fused:
            L = self.layer
            # this rank's full outputs (every tensor of every launch) and its sync
            # words, shared with every rank by IPC handle
            self.mine = [[L.ipc_alloc(4 * gg.tensors[nm].n) for nm in g] for g, _ in self.groups]
            self.mine_sync = L.ipc_alloc(4 * (len(self.groups) + 8))
            own = [[L.ipc_handle(p) for p in row] for row in self.mine] + \
                [[L.ipc_handle(self.mine_sync)]]
            allh = [None] * world
            dist.all_gather_object(allh, own)
            self.peer = {}
            for r in range(world):
                if r != rank:
                    self.peer[r] = [[L.ipc_open(h) for h in row] for row in allh[r]]
            view = lambda r: (self.mine + [[self.mine_sync]]) if r == rank else self.peer[r]
            self.syncs = [view(r)[-1][0] for r in range(world)]
            self.flat = [[view(r)[j][i] for r in range(world) for i in range(len(g))]
                         for j, (g, _) in enumerate(self.groups)]
            self.gsum = [sum((gg.tensors[nm].n + 7) // 8 for nm in g) for g, _ in self.groups]
            dist.barrier()

    def outputs(self):
        """Every tensor's whole output (N floats) as this rank holds it after a
        token: the slabs reassembled (NCCL), or the full buffer the peers
        stored into (fused)."""
        out = []
        for j, (g, _) in enumerate(self.groups):
            ns = [self.gg.tensors[nm].n for nm in g]
            if self.fused:
                for i, n in enumerate(ns):
                    y = np.zeros(n, np.float32)
                    self.layer.read_device(self.mine[j][i], y)
                    out.append(y)
                continue
            buf = (self.full[j] if self.world > 1 else self.bufs[j][0]).cpu().numpy()
            slabs = [shard.slab_rows(n, self.world) for n in ns]
            pieces = buf.reshape(self.world, sum(slabs))
            off = 0
            for n, sl in zip(ns, slabs):
                out.append(shard.assemble(pieces[:, off:off + sl], n, self.world))
                off += sl
        return out

    def token(self, stream):
        if self.fused:
            L, last = self.layer, len(self.groups) - 1
            assert L.gather_epoch_dev(self.mine_sync, stream.cuda_stream) == 0
            for j, (g, k) in enumerate(self.groups):
                q, d = self.acts[k]
                prev = j - 1 if j else last           # launch 0 waits for the last token's head
                rc = L.matvec_gather_dev([self.ids[nm] for nm in g], q.data_ptr(), d.data_ptr(),
                                         self.flat[j], self.syncs, signal_idx=1 + j,
                                         wait_idx=1 + prev, wait_mult=self.gsum[prev],
                                         wait_adj=0 if j else -1, stream=stream.cuda_stream)
                assert rc == 0, L.error()
            return
        for (g, k), (buf, ptrs), full in zip(self.groups, self.bufs, self.full):
            q, d = self.acts[k]
            rc = self.layer.matvec_dev([self.ids[nm] for nm in g], q.data_ptr(), d.data_ptr(),
                                       ptrs, stream.cuda_stream)
            assert rc == 0, self.layer.error()
            if full is not None:
                self.dist.all_gather_into_tensor(full, buf)

    def close(self):
        if self.fused:
            self.torch.cuda.synchronize()
            if self.layer.kernel_error():
                raise RuntimeError("a fused-gather wait gave up: " + self.layer.error())
            self.dist.barrier()
            for rows in self.peer.values():
                for row in rows:
                    for p in row:
                        self.layer.ipc_free(p, True)
            self.dist.barrier()
            for row in self.mine:
                for p in row:
                    self.layer.ipc_free(p, False)
            self.layer.ipc_free(self.mine_sync, False)
        self.layer.close()


class BatchChain:
    """One decode step of M sequences: every projection and the head, grouped
    as the decode groups them, each group one packing of the M activations and
    one tensor-core launch (charsiu_gpu_matvec_batch_group_dev). world > 1:
    every tensor column-split over the ranks (this rank computes its slab of
    rows for all M sequences) and each group's slabs all-gathered with one
    NCCL collective, so every rank holds the whole batch's outputs."""

    def __init__(self, gg, m, dev, rank=0, world=1, dist=None, fused=False):
        import torch
        from charsiu_b200.lib import Layer

        self.torch, self.dist, self.m = torch, dist, m
        self.gg, self.world, self.rank = gg, world, rank
        self.groups = launch_groups(SHAPE)
        names = [nm for g, _ in self.groups for nm in g]
        self.layer = Layer(max_k=max(SHAPE.n_embd, SHAPE.n_ff), max_n=SHAPE.n_vocab,
                           max_tensors=len(names) + 1, device=dev.index, rank=rank, world=world)
        self.ids = {}
        for nm in names:
            t = gg.tensors[nm]
            self.ids[nm] = self.layer.add_blocks(t.type, t.k, t.n, np.asarray(gg.data(nm)), nm)
        self.acts = {}
        for k in (SHAPE.n_embd, SHAPE.n_ff):
            x = torch.randn(m, k, generator=torch.Generator().manual_seed(k)).to(dev)
            q = torch.empty((m, k), dtype=torch.int8, device=dev)
            d = torch.empty((m, k // 32), dtype=torch.float32, device=dev)
            assert self.layer.act_quantise_dev(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream) == 0
            self.acts[k] = (q, d)
        # a group's outputs back to back, each tensor's [M][slab] padded to the
        # widest rank's slab so that a gather moves equal pieces
        self.bufs, self.full = [], []
        for g, _ in self.groups:
            sizes = [m * shard.slab_rows(gg.tensors[nm].n, world) for nm in g]
            buf = torch.zeros(sum(sizes), dtype=torch.float32, device=dev)
            ptrs, off = [], 0
            for sz in sizes:
                ptrs.append(buf[off:].data_ptr())
                off += sz
            self.bufs.append((buf, ptrs))
            self.full.append(torch.zeros(world * sum(sizes), dtype=torch.float32, device=dev)
                             if world > 1 else None)
        self.weight_bytes = sum(gg.tensors[nm].nbytes for nm in names)
        self.fused = fused and world > 1
        if self.fused:
            # this rank's full [M][N] outputs and sync words, shared by IPC
            # handle; every launch stores its rows into every rank's
            L = self.layer
            self.mine = [[L.ipc_alloc(4 * m * gg.tensors[nm].n) for nm in g]
                         for g, _ in self.groups]
            self.mine_sync = L.ipc_alloc(4 * (len(self.groups) + 8))
            own = [[L.ipc_handle(p) for p in row] for row in self.mine] + \
                [[L.ipc_handle(self.mine_sync)]]
            allh = [None] * world
            dist.all_gather_object(allh, own)
            self.peer = {r: [[L.ipc_open(h) for h in row] for row in allh[r]]
                         for r in range(world) if r != rank}
            view = lambda r: (self.mine + [[self.mine_sync]]) if r == rank else self.peer[r]
            self.syncs = [view(r)[-1][0] for r in range(world)]
            self.flat = [[view(r)[j][i] for r in range(world) for i in range(len(g))]
                         for j, (g, _) in enumerate(self.groups)]
            dist.barrier()

    def outputs(self):
        """Every tensor's [M][N] outputs as this rank holds them after a step
        (the gathered slabs reassembled when world > 1)."""
        m, out = self.m, []
        if self.fused:
            for j, (g, _) in enumerate(self.groups):
                for i, nm in enumerate(g):
                    y = np.zeros((m, self.gg.tensors[nm].n), np.float32)
                    self.layer.read_device(self.mine[j][i], y)
                    out.append(y)
            return out
        for (g, _), (buf, _), full in zip(self.groups, self.bufs, self.full):
            ns = [self.gg.tensors[nm].n for nm in g]
            w = self.world
            data = (full if w > 1 else buf).cpu().numpy().reshape(w, -1)
            off = 0
            for n in ns:
                size = m * shard.slab_rows(n, w)
                y = np.empty((m, n), np.float32)
                for r in range(w):
                    row0, rows = shard.shard_rows(n, r, w)
                    y[:, row0:row0 + rows] = data[r, off:off + m * rows].reshape(m, rows)
                out.append(y)
                off += size
        return out

    def token(self, stream):
        if self.fused:
            L, last = self.layer, len(self.groups) - 1
            assert L.gather_epoch_dev(self.mine_sync, stream.cuda_stream) == 0
            for j, (g, k) in enumerate(self.groups):
                q, d = self.acts[k]
                prev = j - 1 if j else last      # launch 0 waits for the last step's head
                rc = L.batch_gather_dev([self.ids[nm] for nm in g], self.m, q.data_ptr(),
                                        d.data_ptr(), self.flat[j], self.syncs,
                                        signal_idx=1 + j, wait_idx=1 + prev,
                                        wait_mult=self.world, wait_adj=0 if j else -1,
                                        stream=stream.cuda_stream)
                assert rc == 0, L.error()
            return
        for (g, k), (buf, ptrs), full in zip(self.groups, self.bufs, self.full):
            q, d = self.acts[k]
            rc = self.layer.batch_group_dev([self.ids[nm] for nm in g], self.m, q.data_ptr(),
                                            d.data_ptr(), ptrs, stream.cuda_stream)
            assert rc == 0, self.layer.error()
            if full is not None:
                self.dist.all_gather_into_tensor(full, buf)

    def close(self):
        if self.fused:
            self.torch.cuda.synchronize()
            if self.layer.kernel_error():
                raise RuntimeError("a fused-gather wait gave up: " + self.layer.error())
            self.dist.barrier()
            for rows in self.peer.values():
                for row in rows:
                    for p in row:
                        self.layer.ipc_free(p, True)
            self.dist.barrier()
            for row in self.mine:
                for p in row:
                    self.layer.ipc_free(p, False)
            self.layer.ipc_free(self.mine_sync, False)
        self.layer.close()


def same_bits(a, b) -> bool:
    return all(x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))
               for x, y in zip(a, b)) and len(a) == len(b)


def all_ranks(flag: bool, world, dist, dev) -> bool:
    """flag on every rank (MIN over ranks)."""
    if world == 1:
        return bool(flag)
    import torch
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def batched_steps(gg, dev, rank, world, dist, barrier, ms=(8, 32, 64), steps=50, warmup=3):
    """tok/s of one batched decode step at each M (M sequences a step, the
    max over ranks of the step time). world > 1: every tensor column-split
    over the world's GPUs and each group's slabs NCCL-all-gathered; the same
    step is timed on one GPU (this rank's, the whole model) and every rank
    checks that its gathered outputs are the one-GPU outputs bit for bit."""
    out = {}
    for m in ms:
        single = BatchChain(gg, m, dev)
        ms_single, _ = time_chain(single, steps, warmup, barrier, dist, world, dev, True, False)
        want = single.outputs() if world > 1 else None
        single.close()
        row = {"value": round(m * 1000.0 / ms_single, 1), "unit": UNIT,
               "ms_per_step": round(ms_single, 5)}
        if world > 1:
            chain = BatchChain(gg, m, dev, rank, world, dist)
            # one CUDA graph a step, the all-gathers included (each rank
            # captures the same collectives in the same order)
            ms_step, _ = time_chain(chain, steps, warmup, barrier, dist, world, dev, True, False)
            ok = all_ranks(same_bits(chain.outputs(), want), world, dist, dev)
            chain.close()
            row = {"value": round(m * 1000.0 / ms_step, 1), "unit": UNIT,
                   "ms_per_step": round(ms_step, 5), "split_matches_single": ok,
                   "single_gpu": row}
            if m >= 9:
                # the same split, the tensor-core epilogue storing every rank's
                # rows over NVLink (no NCCL)
                fz = BatchChain(gg, m, dev, rank, world, dist, fused=True)
                ms_f, _ = time_chain(fz, steps, warmup, barrier, dist, world, dev, True, False)
                okf = all_ranks(same_bits(fz.outputs(), want), world, dist, dev)
                fz.close()
                row["fused"] = {"value": round(m * 1000.0 / ms_f, 1), "unit": UNIT,
                                "ms_per_step": round(ms_f, 5), "split_matches_single": okf}
        out[f"m{m}"] = row
    out["workload"] = ("one decode step of M sequences: the 112 projections and the head as "
                       "grouped batched matvecs (tcgen05 kind::i8 from M = 9, the CUDA cores "
                       f"below), {steps} steps as CUDA graph replays" +
                       (f"; value: every tensor column-split over {world} GPUs and each "
                        "group's slabs NCCL-all-gathered; fused (M >= 9): the tensor-core "
                        "epilogue stores every rank's rows into every rank's outputs over "
                        "NVLink, arrival counters instead of NCCL; each checked bit for bit "
                        "against the one-GPU step (single_gpu)" if world > 1 else ""))
    return out


def head_split(gg, dev, rank, world, dist, barrier, steps=400):
    """The 2048 -> 128256 q8_0 output head alone, column-split over the world's
    GPUs: one GPU with the whole head (each rank's own), the split with an
    NCCL all-gather, and the split whose kernel stores every row into every
    rank's output over NVLink (qmv1_gather_kernel). `steps` heads back to back
    as one CUDA graph, each waiting for the previous one's gather; us a head,
    max over ranks; every rank's gathered head checked bit for bit against its
    one-GPU head."""
    # HEADS heads a graph replay, so a replay's own launch gap is not a
    # head's; every head a launch of its own, each after the last's gather
    heads = 16
    groups = [(["token_embd.weight"], SHAPE.n_embd)] * heads
    reps = max(1, steps // heads)
    single = TokenChain(gg, dev, groups=groups)
    ms1, _ = time_chain(single, reps, 3, barrier, dist, world, dev, True, False)
    ms1 /= heads
    want = single.outputs()
    single.close()
    hbytes = gg.tensors["token_embd.weight"].nbytes
    peak, _ = peaks()
    res = {"single_gpu_us": round(ms1 * 1e3, 3),
           "single_gpu_frac": round(hbytes / (ms1 * 1e-3) / 1e9 / peak, 4)}
    for key, fused in (("nccl", False), ("fused", True)):
        ch = TokenChain(gg, dev, rank, world, dist, fused=fused, groups=groups)
        msn, _ = time_chain(ch, reps, 3, barrier, dist, world, dev, True, False)
        msn /= heads
        ok = all_ranks(same_bits(ch.outputs(), want), world, dist, dev)
        ch.close()
        res[key] = {"us": round(msn * 1e3, 3), "speedup_vs_single": round(ms1 / msn, 3),
                    "split_matches_single": ok}
    res["workload"] = (f"2048 -> 128256 q8_0 head ({hbytes / 1e6:.0f} MB), rows split in 8-row "
                       f"groups over {world} GPUs, {heads} heads a CUDA graph replayed {reps} "
                       "times, each head after the last one's gather; nccl: matvec + "
                       "all_gather_into_tensor; fused: one kernel, peer stores + arrival "
                       "counters over NVLink")
    return res


def time_chain(chain, steps, warmup, barrier, dist, world, dev, graph_ok, sample_clocks):
    """ms a token, the max over ranks; the chain as one CUDA graph when graph_ok."""
    torch = chain.torch
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        chain.token(stream)                     # warm every launch cache first
    torch.cuda.synchronize()
    graph = None
    if graph_ok:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            chain.token(stream)
        torch.cuda.synchronize()
    run = (lambda: graph.replay()) if graph else (lambda: chain.token(stream))
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            run()
    torch.cuda.synchronize()
    barrier()
    clocks = Clocks(dev.index) if sample_clocks else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            run()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop() if clocks else None
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    return ms / steps, clk


def run_decode(path, args, world, dist, dev, sample_clocks, name: str = "llama1b_q8"):
    """The workload's greedy decode with the whole forward on the device and
    the inputs resident in HBM: the 6 prompt ids through the device step
    (untimed), then greedy steps queued back to back with no host round trip
    between them (charsiu_gpu_decoder_generate: each step's argmax is the next
    step's token on the device), timed with CUDA events on the decoder's
    stream. Exactly `args.steps` steps are timed, in runs of at most the
    workload's 24 (positions 6..29), each run from the prompt again. Every
    run's tokens are checked against the reference's. At N GPUs every rank
    decodes its own stream: (ms a token max over ranks, match, clocks,
    kernels a step)."""
    import torch
    from charsiu_b200.lib import Llama

    spec = decode_spec(name)
    n_gen = spec["n_gen"]
    prompt = W.prompt_ids(spec["shape"].n_vocab, spec["seed"])
    with open(os.path.join(ROOT, "tests", "golden", "golden_decode.json")) as f:
        gold = json.load(f)[name]["tokens"]
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    barrier()
    with Llama(path, n_ctx=len(prompt) + n_gen + 1, device=dev.index, resident=True) as m:
        def run(n):
            lp = None
            for i, t in enumerate(prompt):
                lp = m.forward(int(t), i)
            first = int(np.argmax(lp))
            toks, ms = m.generate_dev(first, len(prompt), n)
            return [first] + toks.tolist(), ms

        for _ in range(max(2, min(args.warmup, 4))):      # builds and captures the step graphs
            run(n_gen)
        torch.cuda.synchronize(dev)
        barrier()
        clocks = Clocks(dev.index) if sample_clocks else None
        left, total_ms, match = args.steps, 0.0, True
        while left > 0:
            n = min(left, n_gen)
            toks, ms = run(n)
            total_ms += ms
            left -= n
            k = min(len(toks), len(gold))
            match = match and toks[:k] == gold[:k]
        torch.cuda.synchronize(dev)
        barrier()
        clk = clocks.stop() if clocks else None
        launches = m.step_launches
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    match = all_ranks(match, world, dist, dev)
    return total_ms / args.steps, match, clk, launches


def sharded_paths(gg, dev, rank, world, dist, barrier, args):
    """The column splits of the workload over the world's GPUs, each checked
    bit for bit against one GPU: the 128256-wide head alone, and one stream's
    65 launches, with NCCL all-gathers and with the fused matvec + gather."""
    sharded = {"head": head_split(gg, dev, rank, world, dist, barrier)}
    # one decode stream's hot path, every tensor column-split
    cs = TokenChain(gg, dev, rank, world, dist)
    ms_split, _ = time_chain(cs, max(1, min(args.steps, 200)), 3, barrier, dist, world, dev,
                             True, False)
    cs.close()
    sharded["token_chain_nccl"] = {
        "value": round(1000.0 / ms_split, 2), "unit": UNIT, "ms_per_step": round(ms_split, 5),
        "workload": f"one stream's 65 launches, every tensor column-split over {world} "
                    "GPUs, one NCCL all-gather per launch group, a CUDA graph a token"}
    fused = {"workload": "the same split, each launch storing its rows into every "
                         "rank's outputs over NVLink and waiting on arrival counters "
                         "(matvec and all-gather in one kernel), a CUDA graph a token; "
                         "every output checked against the one-GPU chain"}
    try:
        single = TokenChain(gg, dev)
        time_chain(single, 3, 1, barrier, dist, world, dev, False, False)
        want = single.outputs()
        single.close()
        fz = TokenChain(gg, dev, rank, world, dist, fused=True)
        ms_fused, _ = time_chain(fz, max(1, min(args.steps, 500)), 5, barrier, dist, world,
                                 dev, True, False)
        ok = all_ranks(same_bits(fz.outputs(), want), world, dist, dev)
        fz.close()
        fused.update(value=round(1000.0 / ms_fused, 2), unit=UNIT,
                     ms_per_step=round(ms_fused, 5), split_matches_single=ok)
    except (RuntimeError, AssertionError) as e:   # reported, not fatal to the headline
        fused["error"] = str(e)[:200]
    sharded["token_chain_fused"] = fused

    return sharded


def run_ours(args, rank, world, dist):
    import torch
    from charsiu_b200.lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    path = model_path(rank, barrier)
    gg = G.GGUFFile(path)

    # the headline: greedy decode, whole forward on the device, inputs resident
    ms_per_token, match, clk, step_kernels = run_decode(path, args, world, dist, dev, rank == 0)
    value = world * 1000.0 / ms_per_token

    # the hot path alone: the 65 matvec launches of a token, for the roofline
    chain = TokenChain(gg, dev)
    hot_steps = max(args.steps, 200)
    ms_chain, _ = time_chain(chain, hot_steps, args.warmup, barrier, dist, world, dev, True,
                             False)
    per_token_launches = len(chain.groups)
    tok_bytes = chain.bytes_per_token
    chain.close()
    peak, peak_kind = peaks()
    achieved = tok_bytes / (ms_chain * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(),
                "traffic_source": "ncu DRAM bytes per launch of the same chain, "
                                  "profiles/qmv_decode_llama1b.md",
                "kernel": "cgpu::qmv1_kernel (M=1 block-quant matvec)", "peak_kind": peak_kind,
                "bytes_per_launch": round(tok_bytes / per_token_launches),
                "avg_launch_us": round(ms_chain * 1e3 / per_token_launches, 3),
                "per_gpu": True,
                "timed": f"the token's 65 matvec launches, {hot_steps} tokens as CUDA graph "
                         "replays, CUDA events on the launching stream"}
    hot_path = {"value": round(world * 1000.0 / ms_chain, 2), "unit": UNIT,
                "ms_per_token": round(ms_chain, 5), "gbs": round(achieved, 1),
                "workload": "the hot path of one token alone: 112 projections + the 128256 "
                            "head in 65 matvec launches, fixed activations, 1.31 GB of "
                            "weights a token, no norms/attention between them"}

    sharded = sharded_paths(gg, dev, rank, world, dist, barrier, args) if world > 1 else None

    batched = batched_steps(gg, dev, rank, world, dist, barrier)

    e2e = run_e2e_resident(path, args, world, dist, dev)
    e2e["host_routed"] = run_e2e(path, args, lib, world, dist, dev)
    npu_format = None
    configs = None
    if world == 1:
        # charsiu's NPU number format (CHARSIU_NPU_QUANT): its matvec at the
        # gate/up shape, and the workload's decode with every projection on it
        us, algo, copies, _ = npu_matvec_case(2048, 8192, 200, 10)
        gbs = algo / (us * 1e-6) / 1e9
        npu_format = {"matvec_k2048_n8192": {"value": round(gbs, 1), "unit": "GB/s",
                                             "frac": round(gbs / peak, 4),
                                             "us_per_launch": round(us, 3)},
                      "decode_e2e": npu_decode_e2e(path, args.steps),
                      "decode_e2e_resident": npu_decode_e2e(path, args.steps, resident=True)}
        configs = matvec_configs()
        configs["int8"] = int8_configs()

    out = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_token, 5),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
           "data": "synthetic (seeded random-init Llama-3.2-1B-shaped q8_0 GGUF; no checkpoint)",
           "config": {"workload": "Llama-3.2-1B q8_0 greedy decode (6 seeded prompt ids, then "
                                  "greedy steps at positions 6..29): the whole llama_forward "
                                  "on the device, 112 projections + 128256 tied head + norms, "
                                  "RoPE, attention, SiLU, argmax, one CUDA graph a token, "
                                  "the argmax fed to the next step on the device",
                      "model": "Llama-3.2-1B architecture (16x2048, ffn 8192, 32/8 heads, "
                               "vocab 128256)",
                      "weights_bytes_per_token": tok_bytes, "global_batch": world, "seq_len": 1,
                      "parallelism": f"data-parallel x{world}: one decode stream a GPU, "
                                     "no collective (the column splits are under `sharded`)"
                                     if world > 1 else "single GPU",
                      "l2": "inputs larger than L2 (1.31 GB of weights per step vs 126 MB)",
                      "timed": "CUDA events on the decoder's stream around each run of "
                               "device steps (the prompt outside), summed; max over ranks"},
           "tokens_match_reference": match,
           "roofline": roofline, "hot_path": hot_path, "e2e": e2e,
           "gpu_launches": step_kernels * args.steps, "clocks": clk}
    if sharded:
        out["sharded"] = sharded
    if npu_format:
        out["npu_format"] = npu_format
    out["batched"] = batched
    if configs:
        out["configs"] = configs
    if rank == 0 and world == 1:
        out["cpu_baseline"] = cpu_baseline(path)
    return out


def profile_traffic():
    """DRAM bytes per launch of the matvec from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "qmv_decode_llama1b.md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for ln in f:
            if ln.startswith("traffic_bytes_per_launch:"):
                return int(ln.split(":")[1].strip().split()[0])
    return None


def run_e2e(path, args, lib, world=1, dist=None, dev=None):
    """The public C ABI decode: host buffers in and out on every call. At N GPUs
    every rank decodes its own stream on its own GPU; the rate is the sum over
    ranks, from the slowest rank's time."""
    from charsiu_b200.lib import Llama

    n_gen_timed = min(args.steps, SPEC["n_gen"])
    n_warm = max(3, min(args.warmup, 8))
    prompt = W.prompt_ids(SHAPE.n_vocab, SPEC["seed"])
    n_ctx = len(prompt) + n_warm + n_gen_timed + 1
    L = lib()
    if world > 1:
        dist.barrier()
    with Llama(path, n_ctx=n_ctx, device=dev.index if dev is not None else 0) as m:
        lp = None
        pos = 0
        for t in prompt:
            lp = L.charsiu_gpu_llama_forward(m.h, int(t), pos)
            pos += 1
        tok = L.charsiu_gpu_llama_argmax(lp, m.n_vocab)
        for _ in range(n_warm):
            lp = L.charsiu_gpu_llama_forward(m.h, tok, pos)
            pos += 1
            tok = L.charsiu_gpu_llama_argmax(lp, m.n_vocab)
        calls0 = m.calls
        m.stages(reset=True)
        t0 = time.perf_counter()
        for _ in range(n_gen_timed):
            lp = L.charsiu_gpu_llama_forward(m.h, tok, pos)
            if not lp:
                raise RuntimeError("e2e forward failed")
            pos += 1
            tok = L.charsiu_gpu_llama_argmax(lp, m.n_vocab)
        dt = time.perf_counter() - t0
        calls = (m.calls - calls0) / n_gen_timed
        stages = {k: round(v, 4) for k, v in m.stages().items()}
    if world > 1:
        import torch
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    groups = launch_groups(SHAPE)
    h2d = sum(k + 4 * (k // 32) for _, k in groups)
    d2h = 4 * (SHAPE.n_layer * (SHAPE.n_embd * 2 + 2 * SHAPE.n_head_kv * SHAPE.head_dim
                                + 3 * SHAPE.n_ff) + SHAPE.n_vocab)
    return {"value": round(world * n_gen_timed / dt, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": n_gen_timed, "warmup": n_warm,
            "calls_per_step": calls, "ms_per_step": round(dt * 1e3 / n_gen_timed, 4),
            "stages_ms_per_step": stages,
            "api": "charsiu_gpu_llama_forward (C ABI, host buffers), positions "
                   f"{len(prompt) + n_warm}..{len(prompt) + n_warm + n_gen_timed - 1}"}


def golden_match(toks) -> bool:
    """The timed run's greedy tokens against the reference's (the committed
    fixture: charsiu_run on this model), over the tokens both have."""
    with open(os.path.join(ROOT, "tests", "golden", "golden_decode.json")) as f:
        gold = json.load(f)["llama1b_q8"]["tokens"]
    n = min(len(gold), len(toks))
    return bool(n) and [int(t) for t in toks[:n]] == gold[:n]


def run_e2e_resident(path, args, world=1, dist=None, dev=None):
    """The workload's greedy decode (6 prompt ids, 24 generated tokens) through
    the public C ABI with the whole step on the device
    (charsiu_gpu_llama_set_resident + charsiu_gpu_llama_greedy), repeated from
    the prompt until about K tokens are timed: each timed step copies its
    token and position in from pinned host memory and its argmax token back,
    and replays one CUDA graph. At N GPUs every rank decodes its own stream;
    the rate is the sum over ranks, from the slowest rank's time."""
    from charsiu_b200.lib import Llama

    n_gen = SPEC["n_gen"]
    reps = max(1, min(args.steps, 480) // n_gen)
    prompt = W.prompt_ids(SHAPE.n_vocab, SPEC["seed"])
    n_ctx = len(prompt) + n_gen + 1
    if world > 1:
        dist.barrier()
    total_ms, match = 0.0, True
    with Llama(path, n_ctx=n_ctx, device=dev.index if dev is not None else 0,
               resident=True) as m:
        for _ in range(2):                      # builds and captures the step's graphs
            m.greedy(prompt, n_gen)
        for _ in range(reps):
            toks, _, gen_ms = m.greedy(prompt, n_gen)
            total_ms += gen_ms
            match = match and golden_match(toks)
        launches = m.step_launches
    dt = total_ms / 1e3
    if world > 1:
        import torch
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    steps = reps * n_gen
    return {"value": round(world * steps / dt, 2), "unit": UNIT,
            "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4, "steps": steps,
            "warmup": 2 * (len(prompt) + n_gen), "ms_per_step": round(dt * 1e3 / steps, 4),
            "kernels_per_step": launches, "tokens_match_reference": match,
            "api": "charsiu_gpu_llama_greedy after charsiu_gpu_llama_set_resident(1) (C ABI): "
                   "token + position in (pinned host -> device), argmax token out, one CUDA "
                   f"graph a token; {reps} greedy runs of the workload, positions "
                   f"{len(prompt)}..{len(prompt) + n_gen - 1} timed"}


def cpu_baseline(path):
    """charsiu's own CPU decode on this box's cores: the reference compiled from
    its sources when present (oracle/_ref), else the oracle's restatement."""
    from oracle import oracle as O
    prompt = W.prompt_ids(SHAPE.n_vocab, SPEC["seed"])
    n = 8
    if O.have_ref():
        cores = os.cpu_count()
        toks, stamps = O.ref_greedy_timed(path, prompt, n, n_ctx=64, threads=cores)
        kind = "reference"
    else:
        cores = 1
        toks, stamps = O.port_greedy_timed(G.GGUFFile(path), prompt, n)
        kind = "port"
    rate = (len(stamps) - 1) / ((stamps[-1] - stamps[0]) / 1e3)
    return {"value": round(rate, 3), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"6-token prompt then {n} greedy tokens of the same model; rate over "
                      f"tokens 2..{n} (the first is warm-up)"}


# ---- one matvec on its own -------------------------------------------------------

def matvec_case(qname: str, k: int, n: int, m: int, steps: int, warmup: int):
    """One block-quant matvec shape (M = 1, or the batched matvec of M
    activations), enough copies of the weights rotated that every launch
    streams from HBM (their total at least twice the 126 MB L2), `steps`
    launches replayed as one CUDA graph and timed with CUDA events on the
    launching stream: (us a launch, algorithmic bytes, copies, clocks, weight
    bytes)."""
    import torch
    from charsiu_b200.lib import Layer

    qtype = {"q8_0": G.GGML_Q8_0, "q4_0": G.GGML_Q4_0, "q6_K": G.GGML_Q6_K}[qname]
    blk, _ = W.matvec_inputs(qtype, k, n, seed=1)
    wbytes = blk.nbytes
    copies = max(2, -(-2 * 126 * 2 ** 20 // wbytes))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    with Layer(max_k=k, max_n=n, max_tensors=copies, device=dev.index) as L:
        ids = [L.add_blocks(qtype, k, n, blk, f"copy{i}") for i in range(copies)]
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(7)).to(dev)
        q = torch.empty((m, k), dtype=torch.int8, device=dev)
        d = torch.empty((m, k // 32), dtype=torch.float32, device=dev)
        y = torch.empty((m, n), dtype=torch.float32, device=dev)
        stream = torch.cuda.Stream(device=dev)
        assert L.act_quantise_dev(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(),
                                  stream.cuda_stream) == 0

        def launch(i):
            if m == 1:
                rc = L.matvec_dev([ids[i % copies]], q.data_ptr(), d.data_ptr(), [y.data_ptr()],
                                  stream.cuda_stream)
            else:
                rc = L.batch_dev(ids[i % copies], m, q.data_ptr(), d.data_ptr(), y.data_ptr(),
                                 stream.cuda_stream)
            assert rc == 0, L.error()
        for i in range(warmup):
            launch(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                launch(i)
        graph.replay()
        torch.cuda.synchronize()
        clocks = Clocks(dev.index)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        us = e0.elapsed_time(e1) * 1e3 / steps
        del graph
    algo = wbytes + m * (k + 4 * (k // 32)) + 4 * m * n
    return us, algo, copies, clk, wbytes


def run_matvec_case(args):
    """--matvec q8_0:2048:8192[:M]: one matvec shape (M = 1 unless given)."""
    parts = args.matvec.split(":")
    qname, k, n = parts[0], int(parts[1]), int(parts[2])
    m = int(parts[3]) if len(parts) > 3 else 1
    us, algo, copies, clk, wbytes = matvec_case(qname, k, n, m, args.steps, args.warmup)
    peak, peak_kind = peaks()
    gbs = algo / (us * 1e-6) / 1e9
    return {"metric": "quant matvec HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(us / 1e3, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{qname} matvec M={m} K={k} N={n}", "weight_copies": copies,
                       "l2": f"{copies} weight copies rotated ({copies * wbytes / 1e6:.0f} MB "
                             "> 2x L2)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_launch": algo, "avg_launch_us": round(us, 3)},
            "gpu_launches": args.steps * (1 if m == 1 else 2), "clocks": clk}


# the block-quant matvec workloads: (name, quant type, K, N)
MATVEC_CONFIGS = [("matvec_q8_0_2048x8192", "q8_0", 2048, 8192),
                  ("matvec_q4_0_8192x2048", "q4_0", 8192, 2048)]


def matvec_configs(steps: int = 400):
    """Each block-quant matvec workload on the GPU (M = 1, weights rotated past
    L2), with the reference's charsiu_act_set + gguf_matvec on this box's
    host beside it: one thread, and every core through the decode loop's
    row-split pool (the reference compiled from its sources, oracle/_ref;
    the restated oracle, one thread, if that build is absent)."""
    from oracle import oracle as O
    peak, peak_kind = peaks()
    cores = os.cpu_count() or 1
    out = {}
    for name, qname, k, n in MATVEC_CONFIGS:
        us, algo, copies, _, wbytes = matvec_case(qname, k, n, 1, steps, 10)
        gbs = algo / (us * 1e-6) / 1e9
        row = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
               "peak_kind": peak_kind, "bytes": algo, "launches": steps,
               "weight_copies": copies}
        qtype = {"q8_0": G.GGML_Q8_0, "q4_0": G.GGML_Q4_0}[qname]
        blk, x = W.matvec_inputs(qtype, k, n, seed=1)
        if O.have_ref():
            one = O.ref_matvec_ms(qtype, blk, k, n, x, threads=1, reps=20)
            pool = O.ref_matvec_ms(qtype, blk, k, n, x, threads=cores, reps=50)
            cpu = {"kind": "reference", "us_1_thread": round(one * 1e3, 1),
                   "gbs_1_thread": round(algo / (one * 1e-3) / 1e9, 2),
                   f"us_{cores}_threads": round(pool * 1e3, 1),
                   f"gbs_{cores}_threads": round(algo / (pool * 1e-3) / 1e9, 2), "cores": cores,
                   "sample": "charsiu_act_set + gguf_matvec over all rows (src/gguf.c:829-911, "
                             "1149-1215), 20 calls on 1 thread, 50 through the row-split pool "
                             "of src/llama.c:27-105"}
            row["gpu_vs_cpu_pool"] = round(pool * 1e3 / us, 1)
        else:
            t0 = time.perf_counter()
            for _ in range(5):
                O.matvec(qtype, blk, k, n, *O.act_quantise(x))
            one = (time.perf_counter() - t0) / 5 * 1e3
            cpu = {"kind": "port", "us_1_thread": round(one * 1e3, 1), "cores": 1,
                   "sample": "the restated oracle, 5 calls"}
        row["cpu_baseline"] = cpu
        out[name] = row
    return out


def i8_call_us(L, a, w, bias, sc, steps: int, warm: int = 10):
    """us a call of charsiu_gpu_matmul_i8_flat called straight through ctypes
    on host buffers made once (the reference's own bench times its C function
    the same way), and the output of the last call."""
    from charsiu_b200.lib import _p
    a = np.ascontiguousarray(a, dtype=np.uint8)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    bias = np.ascontiguousarray(bias, dtype=np.int32)
    m, k = a.shape
    n = w.shape[0]
    out = np.full((m, n), 0x5a, dtype=np.int8)
    f = L.L.charsiu_gpu_matmul_i8_flat
    args = (L.h, m, k, n, _p(a), _p(w), _p(bias), *sc, _p(out))
    for _ in range(warm):
        if f(*args):
            raise RuntimeError(L.error())
    rc = 0
    t0 = time.perf_counter()
    for _ in range(steps):
        rc |= f(*args)
    dt = (time.perf_counter() - t0) / steps
    if rc:
        raise RuntimeError(L.error())
    return dt * 1e6, out


def int8_configs(steps: int = 200):
    """The int8 matmul with the NPU output stage at each workload shape
    through the public C ABI (charsiu_gpu_matmul_i8_flat, host buffers: the
    copies inside), us a call on the host clock, byte-exact against the
    reference's cpu_reference; beside it cpu_reference (tools/charsiu_matmul.c:
    41-81) and cpu_us (tools/charsiu_bench.c:74-95) on one host core."""
    from charsiu_b200.lib import Layer
    from oracle import oracle as O
    out = {}
    for name, (m, k, n, seed) in W.I8_SHAPES.items():
        a, w, bias = W.i8_inputs(m, k, n, seed)
        sc = W.i8_scales(m, k, n, seed)
        with Layer(max_k=(max(k, 32) + 31) // 32 * 32, max_n=n, max_tensors=1,
                   device=int(os.environ.get("LOCAL_RANK", 0))) as L:
            l0 = L.launches
            us, got = i8_call_us(L, a, w, bias, sc, steps)
            dt = us * 1e-6
            launches = (L.launches - l0) / (steps + 10)
        have = O.have_ref()
        refmm = O.ref_matmul_i8 if have else O.matmul_i8
        exact = bool(np.array_equal(got, refmm(a, w, bias, *sc)))
        reps = max(3, min(2000, int(0.3 / max(1e-7, m * n * k * 3e-9))))
        t0 = time.perf_counter()
        for _ in range(reps):
            refmm(a, w, bias, *sc)
        cpu_ref = (time.perf_counter() - t0) / reps
        row = {"us_call": round(dt * 1e6, 2), "launches_per_call": launches,
               "byte_exact_vs_reference": exact,
               "cpu_reference_us": round(cpu_ref * 1e6, 2),
               "cpu_kind": "reference" if have else "port", "cpu_cores": 1}
        if have:
            row["cpu_us"] = round(O.ref_cpu_us(a, w, sc[3], sc[4], reps=max(10, reps)), 2)
        out[name] = row
    out["workload"] = ("(M,K,N) = (1,64,64), (1,512,1024), (224,64,64), (3136,33,64): uniform "
                       "u8 operands around zero point 128, bias in [-4096, 4096]; us_call is "
                       f"the mean of {steps} host calls, copies in and out included, "
                       "the C entry called through ctypes on buffers made once")
    return out


# ---- charsiu's NPU number format (CHARSIU_NPU_QUANT) ----------------------------------

def npu_matvec_case(k: int, n: int, steps: int, warmup: int):
    """One NPU-format matvec shape (int8 rows, one scale a row, one activation
    scale) through charsiu_npu_matvec_dev, copies of the weights rotated past
    2x L2, replayed as a CUDA graph: (us a launch, algorithmic bytes, copies,
    clocks)."""
    import torch
    from charsiu_b200.lib import NpuLayer

    # the format's shapes and ranges: int8 rows in [-127, 127], a scale a row
    # of the q8_0 workload's size, an activation quantised to [-127, 127]
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = (np.abs(rng.normal(0.0, 0.02, n)) / 127).astype(np.float32)
    q1 = np.zeros((k + 31) // 32 * 32, np.int8)
    q1[:k] = rng.integers(-127, 128, size=k, dtype=np.int8)
    d1 = np.float32(0.03)
    wbytes = q.nbytes
    copies = max(2, -(-2 * 126 * 2 ** 20 // wbytes))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with NpuLayer(k, n, copies) as L:
        ids = [L.add(q, s, f"copy{i}") for i in range(copies)]
        q1_t = torch.from_numpy(q1[:(k + 15) // 16 * 16].copy()).to(dev)
        y = torch.empty(n, dtype=torch.float32, device=dev)
        stream = torch.cuda.Stream(device=dev)

        def launch(i):
            assert L.matvec_dev([ids[i % copies]], q1_t.data_ptr(), d1, [y.data_ptr()],
                                stream.cuda_stream) == 0, L.error()
        for i in range(warmup):
            launch(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                launch(i)
        graph.replay()
        torch.cuda.synchronize()
        clocks = Clocks(0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        us = e0.elapsed_time(e1) * 1e3 / steps
        del graph
    algo = wbytes + 4 * n + (k + 15) // 16 * 16 + 4 * n
    return us, algo, copies, clk


def npu_decode_e2e(path: str, steps: int, resident: bool = False):
    """The workload's greedy decode in the NPU number format through the C ABI
    (charsiu_gpu_llama_greedy after opening with CHARSIU_NPU_QUANT=1): every
    projection and the head a charsiu_npu_* call with host buffers -- or, with
    `resident`, the whole step on the device in that format
    (charsiu_gpu_llama_set_resident: token and position in, the argmax out)."""
    from charsiu_b200.lib import Llama

    os.environ["CHARSIU_NPU_QUANT"] = "1"
    try:
        prompt = W.prompt_ids(SHAPE.n_vocab, SPEC["seed"])
        n_gen = SPEC["n_gen"]
        reps = max(1, min(steps, 480 if resident else 96) // n_gen)
        total_ms, ok = 0.0, True
        with open(os.path.join(ROOT, "tests", "golden", "golden_decode.json")) as f:
            gold = json.load(f)["npu"]["llama1b_q8"]["tokens"]
        with Llama(path, n_ctx=len(prompt) + n_gen + 1, resident=resident) as m:
            for _ in range(2 if resident else 1):   # (the device step builds its graphs)
                m.greedy(prompt, n_gen)
            for _ in range(reps):
                toks, _, gen_ms = m.greedy(prompt, n_gen)
                total_ms += gen_ms
                ok = ok and toks.tolist() == gold
            calls = m.npu_calls
            launches = m.step_launches
    finally:
        del os.environ["CHARSIU_NPU_QUANT"]
    out = {"value": round(reps * n_gen / (total_ms / 1e3), 2), "unit": UNIT,
           "steps": reps * n_gen, "ms_per_step": round(total_ms / (reps * n_gen), 4),
           "tokens_match_reference": ok, "npu_calls": calls}
    if resident:
        out.update(kernels_per_step=launches,
                   api="charsiu_gpu_llama_greedy after charsiu_gpu_llama_set_resident(1), "
                       "opened with CHARSIU_NPU_QUANT=1: token + position in, argmax out, "
                       "one CUDA graph a token in the NPU number format")
    else:
        out["api"] = ("charsiu_gpu_llama_greedy, opened with CHARSIU_NPU_QUANT=1: each "
                      "projection and the head a charsiu_npu_* host call")
    return out


def run_npu_case(args):
    """--npu K:N: the NPU-format matvec at one shape; with the decode too when
    K:N is the default 2048:8192."""
    k, n = (int(v) for v in args.npu.split(":"))
    us, algo, copies, clk = npu_matvec_case(k, n, args.steps, args.warmup)
    peak, peak_kind = peaks()
    gbs = algo / (us * 1e-6) / 1e9
    return {"metric": "NPU-format int8 matvec HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(us / 1e3, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"NPU-format matvec M=1 K={k} N={n} (int8 rows, one scale "
                                   "a row, one activation scale)", "weight_copies": copies,
                       "l2": f"{copies} weight copies rotated (> 2x L2)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_launch": algo, "avg_launch_us": round(us, 3)},
            "gpu_launches": args.steps, "clocks": clk}


# ---- the int8 matmul with the NPU output stage --------------------------------------

def run_int8_case(args):
    """--int8 M:K:N: the signed-int8 matmul with charsiu's output stage
    (cpu_reference, tools/charsiu_matmul.c:41-81) through the public C ABI
    (charsiu_gpu_matmul_i8_flat, host buffers in and out), K calls timed on
    the host clock; the reference's cpu_reference on the same operands on this
    box's host, one thread, for the baseline. Every call's output is the same
    bytes as the reference's (checked once here; the tests check it fully)."""
    from charsiu_b200.lib import Layer
    from oracle import oracle as O

    m, k, n = (int(v) for v in args.int8.split(":"))
    a, w, bias = W.i8_inputs(m, k, n, 0)
    sc = W.i8_scales(m, k, n, 0)
    with Layer(max_k=(max(k, 32) + 31) // 32 * 32, max_n=n, max_tensors=1) as L:
        l0 = L.launches
        us, out = i8_call_us(L, a, w, bias, sc, args.steps, warm=args.warmup)
        dt = us * 1e-6
        # the timed calls' launches (every call launches the same number)
        launches = (L.launches - l0) * args.steps // (args.steps + args.warmup)
    ref = O.ref_matmul_i8(a, w, bias, *sc) if O.have_ref() else O.matmul_i8(a, w, bias, *sc)
    if not np.array_equal(out, ref):
        raise RuntimeError("int8 matmul differs from the reference")
    reps = max(1, int(0.5 / max(1e-6, m * n * k * 2e-9)))
    t0 = time.perf_counter()
    for _ in range(reps):
        (O.ref_matmul_i8 if O.have_ref() else O.matmul_i8)(a, w, bias, *sc)
    cpu = (time.perf_counter() - t0) / reps
    algo = m * k + n * k + 4 * n + m * n
    return {"metric": "int8 matmul + output stage, us a call", "value": round(dt * 1e6, 2),
            "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 5), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"int8 matmul M={m} K={k} N={n}, zero points 128, "
                                   "NPU output stage", "bytes_per_call": algo,
                       "path": "charsiu_gpu_matmul_i8_flat (host buffers, copies inside)"},
            "byte_exact_vs_reference": True,
            "gpu_launches": launches,
            "cpu_baseline": {"value": round(cpu * 1e6, 2), "unit": "us", "cores": 1,
                             "kind": "reference" if O.have_ref() else "port",
                             "sample": f"{reps} calls of cpu_reference on the same operands"}}


# ---- the batched decode step ------------------------------------------------------

def run_batch_case(args):
    """--batch M: one decode step of M sequences through every projection and
    the head (113 q8_0 tensors), grouped as the decode groups them (q/k/v,
    gate/up), each group one packing of the M activations and one batched
    matvec launch on the tensor cores (tcgen05 kind::i8), as a CUDA graph."""
    import torch
    from charsiu_b200.lib import Layer

    m = args.batch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    path = model_path(0, lambda: None)
    gg = G.GGUFFile(path)
    names = [nm for g, _ in launch_groups(SHAPE) for nm in g]
    with Layer(max_k=max(SHAPE.n_embd, SHAPE.n_ff), max_n=SHAPE.n_vocab,
               max_tensors=len(names) + 1, device=0) as L:
        ids = {}
        for nm in dict.fromkeys(names):
            t = gg.tensors[nm]
            ids[nm] = L.add_blocks(t.type, t.k, t.n, np.asarray(gg.data(nm)), nm)
        stream = torch.cuda.Stream(device=dev)
        acts = {}
        for k in (SHAPE.n_embd, SHAPE.n_ff):
            x = torch.randn(m, k, generator=torch.Generator().manual_seed(k)).to(dev)
            q = torch.empty((m, k), dtype=torch.int8, device=dev)
            d = torch.empty((m, k // 32), dtype=torch.float32, device=dev)
            assert L.act_quantise_dev(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(),
                                      stream.cuda_stream) == 0
            acts[k] = (q, d)
        ys = {nm: torch.empty((m, gg.tensors[nm].n), dtype=torch.float32, device=dev)
              for nm in dict.fromkeys(names)}

        groups = [list(g) for g, _ in launch_groups(SHAPE)]

        def step():
            for grp in groups:
                q, d = acts[gg.tensors[grp[0]].k]
                assert L.batch_group_dev([ids[nm] for nm in grp], m, q.data_ptr(), d.data_ptr(),
                                         [ys[nm].data_ptr() for nm in grp],
                                         stream.cuda_stream) == 0, L.error()
        launches0 = L.launches
        step()
        torch.cuda.synchronize()
        per_step = L.launches - launches0
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        clocks = Clocks(0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        ms = e0.elapsed_time(e1) / args.steps
        del graph
    wbytes = sum(gg.tensors[nm].nbytes for nm in names)
    abytes = sum(m * (gg.tensors[nm].k + gg.tensors[nm].k // 8) + 4 * m * gg.tensors[nm].n
                 for nm in names)
    peak, peak_kind = peaks()
    gbs = (wbytes + abytes) / (ms * 1e-3) / 1e9
    return {"metric": f"Llama-3.2-1B q8_0 batched decode tok/s (M={m})",
            "value": round(m * 1000.0 / ms, 1), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": f"one decode step of {m} sequences: 112 projections + head "
                                   "in 65 grouped tcgen05 kind::i8 batched matvecs",
                       "global_batch": m,
                       "l2": "1.31 GB of weights a step (> L2)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_step": wbytes + abytes},
            "gpu_launches": per_step * args.steps, "clocks": clk}


# ---- the reference arm --------------------------------------------------------

def run_reference(args, rank, world, dist):
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    path = model_path(rank, barrier)
    if rank != 0:
        return None
    from oracle import oracle as O
    prompt = W.prompt_ids(SHAPE.n_vocab, SPEC["seed"])
    n = args.warmup + args.steps
    if O.have_ref():
        cores, kind = os.cpu_count(), "reference"
        toks, stamps = O.ref_greedy_timed(path, prompt, n, n_ctx=len(prompt) + n + 1,
                                          threads=cores)
    else:
        cores, kind = 1, "port"
        toks, stamps = O.port_greedy_timed(G.GGUFFile(path), prompt, n,
                                           n_ctx=len(prompt) + n + 1)
    t_warm = stamps[args.warmup - 1] if args.warmup else 0.0
    ms = (stamps[-1] - t_warm) / args.steps
    value = 1000.0 / ms
    sample = (f"6-token prompt, {args.warmup} warm-up then {args.steps} timed greedy tokens of "
              "the Llama-3.2-1B-shaped q8_0 model, charsiu's llama_forward")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "Llama-3.2-1B q8_0 greedy decode, per token: 112 "
                                   "projections + 128256 tied head (charsiu's llama_forward "
                                   "on the host cores, the rest of the step included)",
                       "model": "Llama-3.2-1B architecture (16x2048, ffn 8192, 32/8 heads, "
                                "vocab 128256)",
                       "global_batch": 1, "seq_len": 1, "parallelism": f"{cores} host threads"},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores,
                             "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=0, metavar="M",
                    help="time one batched decode step of M sequences instead")
    ap.add_argument("--int8", default=None, metavar="M:K:N",
                    help="time the int8 matmul with the NPU output stage (e.g. 224:64:64)")
    ap.add_argument("--npu", default=None, metavar="K:N",
                    help="time the NPU-format (CHARSIU_NPU_QUANT) matvec at one shape")
    ap.add_argument("--resident", action="store_true",
                    help="time only the device-resident greedy decode (the e2e leg)")
    ap.add_argument("--hot-path", action="store_true",
                    help="time only the token's 65 matvec launches (the roofline's chain)")
    ap.add_argument("--decode", action="store_true",
                    help="time only the headline decode (inputs resident, device-side loop)")
    ap.add_argument("--model", default="llama1b_q8", choices=["llama1b_q8", "llama1b_q4_q6k"],
                    help="with --decode: the model (llama1b_q4_q6k: the same shape as a "
                         "llama.cpp q4_0 file, its tied head in q6_K)")
    ap.add_argument("--sharded", action="store_true",
                    help="at N > 1: only the column splits (head, token chain, batched)")
    ap.add_argument("--matvec", default=None, metavar="QTYPE:K:N[:M]",
                    help="time one matvec shape instead of the decode (e.g. q8_0:2048:8192; "
                         "q8_0:2048:8192:64 for 64 activations)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    # the JSON line goes to the original stdout; everything else a library
    # prints there (NCCL's version banner) goes to stderr
    out_fd = os.dup(1)
    os.dup2(2, 1)
    json_out = os.fdopen(out_fd, "w")

    def emit(obj):
        json_out.write(json.dumps(obj) + "\n")
        json_out.flush()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl" if args.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    try:
        if args.matvec:
            emit(run_matvec_case(args))
            return
        if args.batch:
            emit(run_batch_case(args))
            return
        if args.int8:
            emit(run_int8_case(args))
            return
        if args.npu:
            emit(run_npu_case(args))
            return
        if args.sharded and world > 1:
            import torch
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            torch.cuda.set_device(dev)
            barrier = lambda: dist.barrier()
            gg = G.GGUFFile(model_path(rank, barrier))
            out = {"sharded": sharded_paths(gg, dev, rank, world, dist, barrier, args),
                   "batched": batched_steps(gg, dev, rank, world, dist, barrier)}
            if rank == 0:
                emit(out)
            return
        if args.hot_path or args.decode:
            import torch
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            torch.cuda.set_device(dev)
            barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
            path = model_path(rank, barrier, args.model if args.decode else "llama1b_q8")
            if args.decode:
                ms, match, clk, kernels = run_decode(path, args, world, dist, dev, rank == 0,
                                                     args.model)
                out = {"model": args.model,
                       "decode_tok_s": round(world * 1000.0 / ms, 2), "ms_per_token": round(ms, 5),
                       "tokens_match_reference": match, "kernels_per_step": kernels,
                       "clocks": clk}
            else:
                chain = TokenChain(G.GGUFFile(path), dev)
                ms, clk = time_chain(chain, args.steps, args.warmup, barrier, dist, world, dev,
                                     True, rank == 0)
                gbs = chain.bytes_per_token / (ms * 1e-3) / 1e9
                chain.close()
                out = {"hot_path_tok_s": round(world * 1000.0 / ms, 2),
                       "ms_per_token": round(ms, 5), "gbs": round(gbs, 1),
                       "frac": round(gbs / peaks()[0], 4), "clocks": clk}
            if rank == 0:
                emit(out)
            return
        if args.resident:
            import torch
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            torch.cuda.set_device(dev)
            barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
            out = run_e2e_resident(model_path(rank, barrier), args, world, dist, dev)
            if rank == 0:
                emit(out)
            return
        if args.impl == "reference":
            out = run_reference(args, rank, world, dist)
        else:
            out = run_ours(args, rank, world, dist)
        if rank == 0 and out is not None:
            emit(out)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
