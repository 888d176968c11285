"""ctypes access to the checkers. TEST INFRASTRUCTURE ONLY.

Libraries built by oracle/Makefile:
  liboracle.so            the restatement in charsiu_oracle.c (always built);
  _ref/libcharsiu_ref.so  the reference compiled from its own sources plus
                          ref_shim.c (built only where the reference tree is);
  _ref/libcharsiu_ref_gpu.so, _ref/libcharsiu_ref_npu.so  the reference's
                          decode loop linked to the GPU layer, routed and
                          unchanged (ref_routed): the drop-in's proof, run by
                          the GPU tests.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs use this module, and only as the checker or the baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libcharsiu_ref.so")
# the reference's decode loop linked to the GPU layer: with the routing edit
# applied (CHARSIU_GPU=1), and unchanged without its NPU device file
REF_GPU_LIB = os.path.join(HERE, "_ref", "libcharsiu_ref_gpu.so")
REF_NPU_LIB = os.path.join(HERE, "_ref", "libcharsiu_ref_npu.so")

_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        L.orc_act_quantise.argtypes = [_f32p, C.c_int, _i8p, _f32p, C.c_void_p]
        L.orc_matvec.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, _i8p, _f32p, _f32p,
                                 C.c_uint64, C.c_uint64]
        L.orc_matvec.restype = C.c_int
        L.orc_block_dots.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _i8p, _i32p]
        L.orc_block_dots.restype = C.c_int
        L.orc_matmul_i8.argtypes = [C.c_uint, C.c_uint, C.c_uint, _u8p, _u8p, _i32p, C.c_float,
                                    C.c_float, C.c_float, C.c_int, C.c_int, C.c_int, _i8p]
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_half_to_float.restype = C.c_float
        L.orc_state_new.argtypes = [C.c_void_p, C.c_int]
        L.orc_state_new.restype = C.c_void_p
        L.orc_state_free.argtypes = [C.c_void_p]
        L.orc_forward.argtypes = [C.c_void_p, C.c_int32, C.c_int]
        L.orc_forward.restype = C.POINTER(C.c_float)
        L.orc_greedy.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p]
        L.orc_greedy.restype = C.c_int
        L.orc_argmax.argtypes = [C.POINTER(C.c_float), C.c_uint32]
        L.orc_argmax.restype = C.c_int32
        L.orc_row_f32.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _f32p]
        L.orc_row_f32.restype = C.c_int
        L.orc_npu_tensor_build.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _i8p,
                                           _f32p, _i32p]
        L.orc_npu_tensor_build.restype = C.c_int
        L.orc_act_quantise_one.argtypes = [_f32p, C.c_int, _i8p, C.POINTER(C.c_float)]
        L.orc_npu_matvec.argtypes = [_i8p, _f32p, C.c_uint64, C.c_uint64, _i8p, C.c_float,
                                     C.c_int, _f32p]
        _lib = L
    return _lib


def have_ref() -> bool:
    return os.path.exists(REF_LIB)


def ref():
    global _ref
    if _ref is None:
        if not have_ref():
            raise FileNotFoundError(REF_LIB)
        R = C.CDLL(REF_LIB)
        R.ref_matmul_i8.argtypes = [C.c_uint, C.c_uint, C.c_uint, _u8p, _u8p, _i32p, C.c_float,
                                    C.c_float, C.c_float, C.c_int, C.c_int, C.c_int, _u8p]
        R.ref_matmul_i8.restype = C.c_int
        R.ref_matvec.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _f32p, _f32p,
                                 _i8p, _f32p]
        R.ref_matvec.restype = C.c_int
        R.ref_greedy.argtypes = [C.c_char_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p,
                                 C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_void_p]
        R.ref_greedy.restype = C.c_int
        R.ref_greedy_timed.argtypes = [C.c_char_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p,
                                       C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_void_p,
                                       C.c_void_p]
        R.ref_greedy_timed.restype = C.c_int
        R.ref_npu_tensor_build.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _i8p,
                                           _f32p, _i32p]
        R.ref_npu_tensor_build.restype = C.c_int
        R.ref_act_q1.argtypes = [_f32p, C.c_int, _i8p, C.POINTER(C.c_float)]
        R.ref_act_q1.restype = C.c_int
        R.ref_npu_matvec.argtypes = [_i8p, _f32p, C.c_uint64, C.c_uint64, _i8p, C.c_float, _f32p]
        R.ref_matvec_time.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _f32p,
                                      C.c_int, C.c_int, C.POINTER(C.c_double)]
        R.ref_matvec_time.restype = C.c_int
        R.ref_cpu_us.argtypes = [C.c_uint, C.c_uint, C.c_uint, _u8p, _u8p, C.c_int, C.c_int,
                                 C.c_uint]
        R.ref_cpu_us.restype = C.c_double
        _ref = R
    return _ref


def _greedy_argtypes(R):
    R.ref_greedy.argtypes = [C.c_char_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p,
                             C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_void_p]
    R.ref_greedy.restype = C.c_int


_routed = {}


def ref_routed(kind: str):
    """The reference's decode loop linked to the GPU layer: kind "gpu" (the
    routing edit, plus the struct-form calls of ref_gpu_calls.c) or "npu"
    (unchanged, its charsiu_npu_* calls resolved by the GPU layer). Each reads
    its switches (CHARSIU_GPU, CHARSIU_NPU, CHARSIU_NPU_QUANT) from the
    environment, some once a process: load it in a process started with them."""
    if kind not in _routed:
        path = {"gpu": REF_GPU_LIB, "npu": REF_NPU_LIB}[kind]
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        R = C.CDLL(path)
        _greedy_argtypes(R)
        if kind == "gpu":
            R.refgpu_matvec.argtypes = [C.c_uint32, C.c_void_p, C.c_uint, C.c_uint64,
                                        C.c_uint64, _f32p, _f32p, C.c_int]
            R.refgpu_matvec.restype = C.c_int
            R.refgpu_matmul_i8.argtypes = [C.c_uint, C.c_uint, C.c_uint, _u8p, _u8p, _i32p,
                                           C.c_float, C.c_float, C.c_float, C.c_int, C.c_int,
                                           C.c_int, _i8p]
            R.refgpu_matmul_i8.restype = C.c_int
        _routed[kind] = R
    return _routed[kind]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---- the restatement ---------------------------------------------------------

def act_quantise(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    nb = (x.size + 31) // 32
    q = np.zeros(nb * 32, dtype=np.int8)
    d = np.zeros(nb, dtype=np.float32)
    lib().orc_act_quantise(x, x.size, q, d, None)
    return q, d


def matvec(qtype: int, blocks: np.ndarray, k: int, n: int, q: np.ndarray, d: np.ndarray):
    y = np.zeros(n, dtype=np.float32)
    rc = lib().orc_matvec(qtype, _ptr(blocks), k, np.ascontiguousarray(q), np.ascontiguousarray(d),
                          y, 0, n)
    assert rc == 0
    return y


def row_f32(qtype: int, blocks: np.ndarray, k: int, row: int) -> np.ndarray:
    """gguf_row_f32 of one row (the embedding lookup)."""
    out = np.empty(k, dtype=np.float32)
    rc = lib().orc_row_f32(qtype, _ptr(blocks), k, row, out)
    assert rc == 0, rc
    return out


def npu_tensor_build(qtype: int, blocks: np.ndarray, k: int, n: int):
    """npu_tensor_build's default form: (q int8 [n, k], scale [n], wsum [n])."""
    q = np.zeros((n, k), dtype=np.int8)
    scale = np.zeros(n, dtype=np.float32)
    wsum = np.zeros(n, dtype=np.int32)
    assert lib().orc_npu_tensor_build(qtype, _ptr(blocks), k, n, q, scale, wsum) == 0
    return q, scale, wsum


def act_quantise_one(x: np.ndarray):
    """charsiu_act_set's single-scale form: (q1 [nb * 32], d1)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q1 = np.zeros((x.size + 31) // 32 * 32, dtype=np.int8)
    d1 = C.c_float()
    lib().orc_act_quantise_one(x, x.size, q1, C.byref(d1))
    return q1, np.float32(d1.value)


def npu_matvec(q: np.ndarray, scale: np.ndarray, q1: np.ndarray, d1, model: int = 0):
    """y in the NPU format: model 0 the device path's arithmetic, 1 the CPU model's."""
    n, k = q.shape
    y = np.zeros(n, dtype=np.float32)
    lib().orc_npu_matvec(np.ascontiguousarray(q), np.ascontiguousarray(scale, dtype=np.float32),
                         k, n, np.ascontiguousarray(q1), float(d1), model, y)
    return y


def block_dots(qtype: int, blocks: np.ndarray, k: int, n: int, q: np.ndarray):
    out = np.zeros((n, k // 32), dtype=np.int32)
    rc = lib().orc_block_dots(qtype, _ptr(blocks), k, n, np.ascontiguousarray(q), out)
    assert rc == 0
    return out


def matmul_i8(a, w, bias, in_scale, wt_scale, out_scale, in_zp=128, wt_zp=128, out_zp=0):
    m, k = a.shape
    n = w.shape[0]
    out = np.zeros((m, n), dtype=np.int8)
    lib().orc_matmul_i8(m, k, n, np.ascontiguousarray(a), np.ascontiguousarray(w),
                        np.ascontiguousarray(bias, dtype=np.int32), in_scale, wt_scale, out_scale,
                        in_zp, wt_zp, out_zp, out)
    return out


class _Layer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("w", C.c_void_p * 7),
                ("type", C.c_uint32 * 7), ("nq", C.c_void_p * 7), ("nscale", C.c_void_p * 7)]


class _Model(C.Structure):
    _fields_ = [("n_embd", C.c_uint32), ("n_layer", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_ff", C.c_uint32), ("n_vocab", C.c_uint32),
                ("head_dim", C.c_uint32), ("rms_eps", C.c_float), ("rope_base", C.c_float),
                ("tok_embd", C.c_void_p), ("tok_type", C.c_uint32), ("output", C.c_void_p),
                ("out_type", C.c_uint32), ("out_norm", C.c_void_p), ("layers", C.c_void_p),
                ("npu", C.c_int), ("out_nq", C.c_void_p), ("out_nscale", C.c_void_p)]


class OracleModel:
    """The restated decode loop over a GGUF file's tensors (mapped, not copied).

    npu = 0: charsiu's default path (gguf_matvec). npu = 1 or 2: the NPU
    format of CHARSIU_NPU_QUANT -- every projection and the head through its
    npu_tensor_build copy (built here), with the device path's arithmetic (1)
    or the CPU model's (2)."""

    def __init__(self, gguf, n_ctx: int = 64, npu: int = 0):
        from charsiu_b200.gguf import PROJ_NAMES
        s = gguf.shape()
        self.gguf, self.shape = gguf, s
        T = gguf.tensors
        self._keep = []

        def npu_copy(name):
            t = T[name]
            k, n = int(t.ne[0]), int(t.ne[1])
            q, scale, _ = npu_tensor_build(t.type, gguf.data(name), k, n)
            self._keep += [q, scale]
            return _ptr(q), _ptr(scale)

        layers = (_Layer * s.n_layer)()
        for l in range(s.n_layer):
            L = layers[l]
            L.attn_norm = _ptr(gguf.data(f"blk.{l}.attn_norm.weight"))
            L.ffn_norm = _ptr(gguf.data(f"blk.{l}.ffn_norm.weight"))
            for i, nm in enumerate(PROJ_NAMES):
                L.w[i] = _ptr(gguf.data(f"blk.{l}.{nm}.weight"))
                L.type[i] = T[f"blk.{l}.{nm}.weight"].type
                if npu:
                    L.nq[i], L.nscale[i] = npu_copy(f"blk.{l}.{nm}.weight")
        out = "output.weight" if "output.weight" in T else "token_embd.weight"
        out_nq, out_nscale = npu_copy(out) if npu else (None, None)
        self._layers = layers
        self.m = _Model(s.n_embd, s.n_layer, s.n_head, s.n_head_kv, s.n_ff, s.n_vocab, s.head_dim,
                        s.rms_eps, s.rope_base, _ptr(gguf.data("token_embd.weight")),
                        T["token_embd.weight"].type, _ptr(gguf.data(out)), T[out].type,
                        _ptr(gguf.data("output_norm.weight")), C.addressof(layers), npu,
                        out_nq, out_nscale)
        self.n_ctx = n_ctx

    def greedy(self, prompt, n_gen: int) -> np.ndarray:
        L = lib()
        st = L.orc_state_new(C.byref(self.m), self.n_ctx)
        assert st
        try:
            out = np.zeros(n_gen, dtype=np.int32)
            p = np.ascontiguousarray(prompt, dtype=np.int32)
            rc = L.orc_greedy(st, p, p.size, n_gen, out)
            assert rc == n_gen, rc
            return out
        finally:
            L.orc_state_free(st)

    def logits_after(self, prompt) -> np.ndarray:
        L = lib()
        st = L.orc_state_new(C.byref(self.m), self.n_ctx)
        try:
            lp = None
            for i, t in enumerate(prompt):
                lp = L.orc_forward(st, int(t), i)
            return np.ctypeslib.as_array(lp, shape=(self.shape.n_vocab,)).copy()
        finally:
            L.orc_state_free(st)


# ---- the reference itself ----------------------------------------------------

def ref_matmul_i8(a, w, bias, in_scale, wt_scale, out_scale, in_zp=128, wt_zp=128, out_zp=0):
    m, k = a.shape
    n = w.shape[0]
    out = np.zeros((m, n), dtype=np.uint8)
    ref().ref_matmul_i8(m, k, n, np.ascontiguousarray(a), np.ascontiguousarray(w),
                        np.ascontiguousarray(bias, dtype=np.int32), in_scale, wt_scale, out_scale,
                        in_zp, wt_zp, out_zp, out)
    return out.view(np.int8)


def ref_matvec(qtype: int, blocks: np.ndarray, k: int, n: int, x: np.ndarray):
    """charsiu_act_set + gguf_matvec of the reference: (y, q, d)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(n, dtype=np.float32)
    q = np.zeros((k + 31) // 32 * 32, dtype=np.int8)
    d = np.zeros((k + 31) // 32, dtype=np.float32)
    rc = ref().ref_matvec(qtype, _ptr(blocks), k, n, x, y, q, d)
    assert rc == 0
    return y, q, d


def ref_matvec_ms(qtype: int, blocks: np.ndarray, k: int, n: int, x: np.ndarray,
                  threads: int = 1, reps: int = 10) -> float:
    """ms a call of the reference's charsiu_act_set + gguf_matvec over all n
    rows, on `threads` host threads splitting the rows as its decode loop's
    pool does (src/llama.c:63-73)."""
    ms = C.c_double()
    rc = ref().ref_matvec_time(qtype, _ptr(blocks), k, n, np.ascontiguousarray(x, np.float32),
                               threads, reps, C.byref(ms))
    if rc:
        raise RuntimeError("ref_matvec_time failed")
    return ms.value


def ref_cpu_us(a, w, in_zp: int = 128, wt_zp: int = 128, reps: int = 10) -> float:
    """The reference's own one-core int8 denominator, cpu_us of
    tools/charsiu_bench.c:74-95 (one activation row against every weight
    row), microseconds a call."""
    m, k = a.shape
    n = w.shape[0]
    return ref().ref_cpu_us(m, k, n, np.ascontiguousarray(a), np.ascontiguousarray(w), in_zp,
                            wt_zp, reps)


def ref_greedy(path: str, prompt, n_gen: int, n_ctx: int = 0, threads: int | None = None,
               want_logits: int = 0, build: str = ""):
    """Greedy decode by the reference's own llama_forward (build "" the
    reference itself; "gpu" or "npu" the builds of ref_routed).

    Returns (tokens, prompt_ms, gen_ms[, logits after the prompt]). The
    reference's pool reads CHARSIU_THREADS once per process."""
    if threads is not None:
        os.environ["CHARSIU_THREADS"] = str(threads)
    out = np.zeros(n_gen, dtype=np.int32)
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    pm, gm = C.c_double(), C.c_double()
    lg = np.zeros(want_logits, dtype=np.float32) if want_logits else None
    R = ref_routed(build) if build else ref()
    n = R.ref_greedy(path.encode(), p, p.size, n_gen, n_ctx, out, C.byref(pm), C.byref(gm),
                     _ptr(lg) if lg is not None else None)
    if n < 0:
        raise RuntimeError(f"reference could not load {path}")
    res = (out[:n], pm.value, gm.value)
    return res + (lg,) if want_logits else res


def ref_greedy_timed(path: str, prompt, n_gen: int, n_ctx: int = 0, threads: int | None = None):
    """(tokens, ms stamps after each generated token's forward pass)."""
    if threads is not None:
        os.environ["CHARSIU_THREADS"] = str(threads)
    out = np.zeros(n_gen, dtype=np.int32)
    stamps = np.zeros(n_gen, dtype=np.float64)
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    pm, gm = C.c_double(), C.c_double()
    n = ref().ref_greedy_timed(path.encode(), p, p.size, n_gen, n_ctx, out, C.byref(pm),
                               C.byref(gm), None, _ptr(stamps))
    if n < 0:
        raise RuntimeError(f"reference could not load {path}")
    return out[:n], stamps[:n]


def port_greedy_timed(gguf, prompt, n_gen: int, n_ctx: int = 64):
    """The restated decode loop, one thread: (tokens, ms stamps)."""
    import time
    om = OracleModel(gguf, n_ctx=n_ctx)
    L = lib()
    st = L.orc_state_new(C.byref(om.m), n_ctx)
    try:
        lp = None
        for i, t in enumerate(prompt):
            lp = L.orc_forward(st, int(t), i)
        pos = len(prompt)
        out = np.zeros(n_gen, dtype=np.int32)
        stamps = np.zeros(n_gen, dtype=np.float64)
        t0 = time.perf_counter()
        for i in range(n_gen):
            out[i] = L.orc_argmax(lp, om.shape.n_vocab)
            lp = L.orc_forward(st, int(out[i]), pos)
            pos += 1
            stamps[i] = (time.perf_counter() - t0) * 1e3
        return out, stamps
    finally:
        L.orc_state_free(st)
