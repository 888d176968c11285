"""GGUF v3 files: a seeded synthetic Llama writer and a small reader.

There is no real model on these machines, so every workload is a random-init
GGUF with the Llama-3.2-1B architecture (or a tiny one for fast tests), laid
out exactly as charsiu's reader parses a file (reference src/gguf.c:207-358):
a header, key/value pairs, tensor infos, then the tensor data aligned to 32.

Weights follow the workload's stated distributions:
  q8_0: 32 int8 values uniform in [-127, 127] per block, one fp16 delta drawn
        from |N(0, 0.02)| / 127 (round to nearest even);
  q4_0: 16 bytes of nibbles uniform in 0..15 per block (value = nibble - 8),
        delta from |N(0, 0.02)| / 8;
  norms: f32, 1 + N(0, 0.01).
The tokenizer arrays are present only because charsiu's loader requires them
(reference src/tokenizer.c:269-272, 343-346); the prompt is given as ids.
"""
from __future__ import annotations

import dataclasses
import os
import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q6_K = 0, 1, 2, 8, 14
BLOCK_BYTES = {GGML_Q8_0: 34, GGML_Q4_0: 18, GGML_Q6_K: 210}
BLOCK_ELEMS = {GGML_Q8_0: 32, GGML_Q4_0: 32, GGML_Q6_K: 256}
TYPE_NAMES = {GGML_F32: "f32", GGML_F16: "f16", GGML_Q4_0: "q4_0", GGML_Q8_0: "q8_0",
              GGML_Q6_K: "q6_K"}

# GGUF value types (reference include/charsiu_llm.h:28-32)
V_U32, V_I32, V_F32, V_STRING, V_ARRAY, V_U64 = 4, 5, 6, 8, 9, 10
ALIGN = 32


@dataclasses.dataclass(frozen=True)
class LlamaShape:
    n_embd: int
    n_layer: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_vocab: int
    ctx_train: int = 131072
    rms_eps: float = 1e-5
    rope_base: float = 500000.0

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


LLAMA_3_2_1B = LlamaShape(2048, 16, 32, 8, 8192, 128256)
TINY = LlamaShape(256, 2, 8, 2, 512, 1000, ctx_train=256)

PROJ_NAMES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def proj_shapes(s: LlamaShape):
    """(name, K, N) of the seven projections of one layer."""
    kv = s.n_head_kv * s.head_dim
    return [("attn_q", s.n_embd, s.n_head * s.head_dim), ("attn_k", s.n_embd, kv),
            ("attn_v", s.n_embd, kv), ("attn_output", s.n_embd, s.n_embd),
            ("ffn_gate", s.n_embd, s.n_ff), ("ffn_up", s.n_embd, s.n_ff),
            ("ffn_down", s.n_ff, s.n_embd)]


def quant_blocks(rng: np.random.Generator, qtype: int, n: int, k: int) -> np.ndarray:
    """n rows of k columns as raw GGML blocks: uint8 [n, k/elems*block_bytes].

    q6_K super-blocks (256 weights, 210 bytes: ql[128], qh[64], int8
    scales[16], fp16 d) get uniform 6-bit weights, scales in [-64, 63] and
    d = |N(0, 0.02)| / 2048, so d * scale * q stays near the other types'."""
    if qtype == GGML_Q6_K:
        nsb = k // 256
        blk = np.empty((n, nsb, 210), dtype=np.uint8)
        blk[:, :, 0:192] = rng.integers(0, 256, size=(n, nsb, 192), dtype=np.uint8)
        blk[:, :, 192:208] = rng.integers(-64, 64, size=(n, nsb, 16), dtype=np.int8).view(np.uint8)
        d = (np.abs(rng.normal(0.0, 0.02, size=(n, nsb))) / 2048.0).astype(np.float16)
        blk[:, :, 208:210] = d.view(np.uint8).reshape(n, nsb, 2)
        return blk.reshape(n, nsb * 210)
    nb = k // 32
    if qtype == GGML_Q8_0:
        blk = np.empty((n, nb, 34), dtype=np.uint8)
        d = (np.abs(rng.normal(0.0, 0.02, size=(n, nb))) / 127.0).astype(np.float16)
        blk[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
        blk[:, :, 2:] = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int8).view(np.uint8)
    elif qtype == GGML_Q4_0:
        blk = np.empty((n, nb, 18), dtype=np.uint8)
        d = (np.abs(rng.normal(0.0, 0.02, size=(n, nb))) / 8.0).astype(np.float16)
        blk[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
        blk[:, :, 2:] = rng.integers(0, 256, size=(n, nb, 16), dtype=np.uint8)
    else:
        raise ValueError(f"not a block type: {qtype}")
    return blk.reshape(n, nb * BLOCK_BYTES[qtype])


def _kv_str(key: str, val: str) -> bytes:
    k, v = key.encode(), val.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", V_STRING) + struct.pack("<Q", len(v)) + v


def _kv_u32(key: str, val: int) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<II", V_U32, val)


def _kv_f32(key: str, val: float) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<If", V_F32, val)


def _kv_str_array(key: str, items) -> bytes:
    k = key.encode()
    parts = [struct.pack("<Q", len(k)), k, struct.pack("<IIQ", V_ARRAY, V_STRING, len(items))]
    for it in items:
        b = it.encode()
        parts.append(struct.pack("<Q", len(b)))
        parts.append(b)
    return b"".join(parts)


def _tensor_list(s: LlamaShape, qtype: int, embd_qtype: int):
    """(name, ne0, ne1, type) in file order."""
    out = [("token_embd.weight", s.n_embd, s.n_vocab, embd_qtype),
           ("output_norm.weight", s.n_embd, 1, GGML_F32)]
    for l in range(s.n_layer):
        out.append((f"blk.{l}.attn_norm.weight", s.n_embd, 1, GGML_F32))
        for name, k, n in proj_shapes(s):
            out.append((f"blk.{l}.{name}.weight", k, n, qtype))
        out.append((f"blk.{l}.ffn_norm.weight", s.n_embd, 1, GGML_F32))
    return out


def _nbytes(ne0: int, ne1: int, t: int) -> int:
    if t == GGML_F32:
        return ne0 * ne1 * 4
    return ne0 // BLOCK_ELEMS[t] * BLOCK_BYTES[t] * ne1


def write_llama(path: str, shape: LlamaShape = LLAMA_3_2_1B, qtype: int = GGML_Q8_0,
                seed: int = 0, embd_qtype: int | None = None) -> str:
    """Write a seeded random-init Llama GGUF (tied head, no output.weight).

    embd_qtype: the type of token_embd (and so of the tied head); llama.cpp
    writes q6_K there in q4_0 files. Default: qtype."""
    tensors = _tensor_list(shape, qtype, qtype if embd_qtype is None else embd_qtype)
    kv = [
        _kv_str("general.architecture", "llama"),
        _kv_str("general.name", f"synthetic-llama-seed{seed}"),
        _kv_u32("llama.embedding_length", shape.n_embd),
        _kv_u32("llama.block_count", shape.n_layer),
        _kv_u32("llama.attention.head_count", shape.n_head),
        _kv_u32("llama.attention.head_count_kv", shape.n_head_kv),
        _kv_u32("llama.feed_forward_length", shape.n_ff),
        _kv_u32("llama.context_length", shape.ctx_train),
        _kv_u32("llama.rope.dimension_count", shape.head_dim),
        _kv_f32("llama.attention.layer_norm_rms_epsilon", shape.rms_eps),
        _kv_f32("llama.rope.freq_base", shape.rope_base),
        _kv_str("tokenizer.ggml.model", "gpt2"),
        _kv_str_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(shape.n_vocab)]),
        _kv_str_array("tokenizer.ggml.merges", ["< t"]),
        _kv_u32("tokenizer.ggml.bos_token_id", 0),
        _kv_u32("tokenizer.ggml.eos_token_id", 1),
    ]
    infos, offsets, off = [], [], 0
    for name, ne0, ne1, t in tensors:
        nm = name.encode()
        dims = [ne0] if ne1 == 1 else [ne0, ne1]
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        offsets.append(off)
        infos.append(struct.pack("<Q", len(nm)) + nm + struct.pack("<I", len(dims))
                     + struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", t, off))
        off += _nbytes(ne0, ne1, t)
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)) + b"".join(kv) + b"".join(infos)
    data_start = (len(header) + ALIGN - 1) // ALIGN * ALIGN
    total = data_start + off
    tmp = path + ".part"
    with open(tmp, "wb") as f:
        f.truncate(total)
        f.write(header)
    mm = np.memmap(tmp, dtype=np.uint8, mode="r+", offset=data_start, shape=(off,))
    for idx, ((name, ne0, ne1, t), o) in enumerate(zip(tensors, offsets)):
        rng = np.random.default_rng([seed, idx])
        if t == GGML_F32:
            v = (1.0 + rng.normal(0.0, 0.01, size=ne0 * ne1)).astype(np.float32)
            mm[o:o + v.nbytes] = v.view(np.uint8)
        else:
            rb = ne0 // BLOCK_ELEMS[t] * BLOCK_BYTES[t]
            step = max(1, (64 << 20) // rb)
            for r0 in range(0, ne1, step):
                r1 = min(ne1, r0 + step)
                blk = quant_blocks(rng, t, r1 - r0, ne0)
                mm[o + r0 * rb:o + r1 * rb] = blk.reshape(-1)
    mm.flush()
    del mm
    os.replace(tmp, path)
    return path


# ---- reading -----------------------------------------------------------------

@dataclasses.dataclass
class Tensor:
    name: str
    ne: tuple
    type: int
    offset: int          # absolute, in the file
    nbytes: int

    @property
    def k(self) -> int:
        return self.ne[0]

    @property
    def n(self) -> int:
        return self.ne[1] if len(self.ne) > 1 else 1


class GGUFFile:
    """Header, metadata and a read-only map of the tensor data."""

    def __init__(self, path: str):
        self.path = path
        self.map = np.memmap(path, dtype=np.uint8, mode="r")
        buf = self.map
        p = 0

        def take(n):
            nonlocal p
            b = bytes(buf[p:p + n])
            p += n
            return b

        def u32():
            return struct.unpack("<I", take(4))[0]

        def u64():
            return struct.unpack("<Q", take(8))[0]

        def string():
            return take(u64()).decode("utf-8", "replace")

        if take(4) != b"GGUF":
            raise ValueError(f"{path}: bad magic")
        self.version = u32()
        nt, nkv = u64(), u64()
        self.kv = {}
        fixed = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
        fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B",
               10: "<Q", 11: "<q", 12: "<d"}
        for _ in range(nkv):
            key = string()
            vt = u32()
            if vt == V_STRING:
                self.kv[key] = string()
            elif vt == V_ARRAY:
                at, n = u32(), u64()
                if at == V_STRING:
                    self.kv[key] = [string() for _ in range(n)]
                else:
                    self.kv[key] = np.frombuffer(take(n * fixed[at]), dtype=fmt[at][1:])
            else:
                self.kv[key] = struct.unpack(fmt[vt], take(fixed[vt]))[0]
        infos = []
        for _ in range(nt):
            name = string()
            nd = u32()
            ne = tuple(u64() for _ in range(nd))
            t, off = u32(), u64()
            infos.append((name, ne, t, off))
        align = int(self.kv.get("general.alignment", ALIGN))
        data = (p + align - 1) // align * align
        self.tensors = {}
        for name, ne, t, off in infos:
            ne0 = ne[0]
            ne1 = int(np.prod(ne[1:])) if len(ne) > 1 else 1
            self.tensors[name] = Tensor(name, ne, t, data + off, _nbytes(ne0, ne1, t))

    def data(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self.map[t.offset:t.offset + t.nbytes]

    def shape(self) -> LlamaShape:
        a = self.kv.get("general.architecture", "llama")
        g = lambda k, d=None: self.kv.get(f"{a}.{k}", d)
        n_head = int(g("attention.head_count"))
        return LlamaShape(int(g("embedding_length")), int(g("block_count")), n_head,
                          int(g("attention.head_count_kv", n_head)), int(g("feed_forward_length")),
                          len(self.kv["tokenizer.ggml.tokens"]), int(g("context_length", 2048)),
                          float(g("attention.layer_norm_rms_epsilon", 1e-5)),
                          float(g("rope.freq_base", 10000.0)))
