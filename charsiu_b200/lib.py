"""ctypes binding of libcharsiu_gpu.so: the C ABI of include/charsiu_gpu.h and
include/charsiu_gpu_llama.h, one method per entry point.

This is how Python reaches the CUDA path (tests, bench.py, smoke). It never
computes anything itself: if the library is missing it raises, and every
method is a thin call into the shared object.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libcharsiu_gpu.so")

_lib = None

_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_vp = C.c_void_p

# (name, restype, argtypes) of every exported entry point
SIGNATURES = [
    ("charsiu_gpu_open", _vp, [C.c_uint, C.c_uint, C.c_uint]),
    ("charsiu_gpu_open_ex", _vp, [C.c_uint, C.c_uint, C.c_uint, C.c_int, C.c_uint, C.c_uint]),
    ("charsiu_gpu_close", None, [_vp]),
    ("charsiu_gpu_add", C.c_int, [_vp, _vp]),
    ("charsiu_gpu_add_blocks", C.c_int, [_vp, C.c_uint32, C.c_uint64, C.c_uint64, _vp, C.c_char_p]),
    ("charsiu_gpu_rows", C.c_int, [_vp, C.c_int, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    ("charsiu_gpu_matvec", C.c_int, [_vp, C.c_int, _vp, _vp]),
    ("charsiu_gpu_matvec_group", C.c_int, [_vp, _vp, C.c_uint, _vp, _vp]),
    ("charsiu_gpu_matvec_q", C.c_int, [_vp, _vp, C.c_uint, _vp, _vp, C.c_uint, _vp]),
    ("charsiu_gpu_matvec_batch", C.c_int, [_vp, C.c_int, C.c_uint, _vp, _vp, C.c_uint, _vp]),
    ("charsiu_gpu_matmul_i8", C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    ("charsiu_gpu_matmul_i8_flat", C.c_int, [_vp, C.c_uint, C.c_uint, C.c_uint, _vp, _vp, _vp,
                                             C.c_float, C.c_float, C.c_float, C.c_int, C.c_int,
                                             C.c_int, _vp]),
    ("charsiu_gpu_matvec_dev", C.c_int, [_vp, _vp, C.c_uint, _vp, _vp, _vp, _vp]),
    ("charsiu_gpu_matvec_batch_dev", C.c_int, [_vp, C.c_int, C.c_uint, _vp, _vp, _vp, _vp]),
    ("charsiu_gpu_matvec_batch_group_dev", C.c_int,
     [_vp, _vp, C.c_uint, C.c_uint, _vp, _vp, _vp, _vp]),
    ("charsiu_gpu_ipc_alloc", C.c_void_p, [_vp, C.c_size_t]),
    ("charsiu_gpu_ipc_handle", C.c_int, [_vp, _vp, _vp]),
    ("charsiu_gpu_ipc_open", C.c_void_p, [_vp, _vp]),
    ("charsiu_gpu_ipc_free", None, [_vp, _vp, C.c_int]),
    ("charsiu_gpu_gather_epoch_dev", C.c_int, [_vp, _vp, _vp]),
    ("charsiu_gpu_kernel_error", C.c_int, [_vp]),
    ("charsiu_gpu_read_device", C.c_int, [_vp, _vp, _vp, C.c_size_t]),
    ("charsiu_gpu_matvec_gather_dev", C.c_int,
     [_vp, _vp, C.c_uint, _vp, _vp, _vp, _vp, C.c_uint, C.c_uint, C.c_uint, C.c_int, _vp]),
    ("charsiu_gpu_matvec_batch_gather_dev", C.c_int,
     [_vp, _vp, C.c_uint, C.c_uint, _vp, _vp, _vp, _vp, C.c_uint, C.c_uint, C.c_uint, C.c_int,
      _vp]),
    ("charsiu_gpu_matvec_batch_noalloc", C.c_int, [_vp, C.c_int, C.c_uint, _vp, _vp, _vp, _vp]),
    ("charsiu_gpu_act_quantise_dev", C.c_int, [_vp, _vp, C.c_uint, C.c_uint, _vp, _vp, _vp]),
    ("charsiu_gpu_calls", C.c_ulong, [_vp]),
    ("charsiu_gpu_launches", C.c_ulong, [_vp]),
    ("charsiu_gpu_report", None, [_vp]),
    ("charsiu_gpu_error", C.c_char_p, [_vp]),
    ("charsiu_gpu_dead", C.c_int, [_vp]),
    ("charsiu_gpu_block_dots", C.c_int, [_vp, C.c_int, _vp, _vp]),
    ("charsiu_gpu_inject", C.c_int, [_vp, C.c_ulong, C.c_ulong, C.c_int]),
    ("charsiu_gpu_llama_open", _vp, [C.c_char_p, C.c_int, C.c_int]),
    ("charsiu_gpu_llama_close", None, [_vp]),
    ("charsiu_gpu_llama_forward", C.POINTER(C.c_float), [_vp, C.c_int32, C.c_int]),
    ("charsiu_gpu_llama_argmax", C.c_int32, [C.POINTER(C.c_float), C.c_uint32]),
    ("charsiu_gpu_llama_greedy", C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp,
                                           C.POINTER(C.c_double)]),
    ("charsiu_gpu_llama_stages", C.c_int, [_vp, _vp, C.c_int, C.c_int]),
    ("charsiu_gpu_llama_stage_name", C.c_char_p, [C.c_int]),
    ("charsiu_gpu_llama_vocab", C.c_uint32, [_vp]),
    ("charsiu_gpu_llama_layer", _vp, [_vp]),
    ("charsiu_gpu_llama_set_resident", C.c_int, [_vp, C.c_int]),
    ("charsiu_gpu_llama_decoder", _vp, [_vp]),
    ("charsiu_gpu_llama_npu", _vp, [_vp]),
    ("charsiu_gpu_row_dev", C.c_int, [_vp, C.c_int, _vp, _vp, _vp]),
    ("charsiu_gpu_decoder_new", _vp, [_vp, _vp]),
    ("charsiu_gpu_decoder_new_npu", _vp, [_vp, _vp, _vp]),
    ("charsiu_gpu_decoder_free", None, [_vp]),
    ("charsiu_gpu_decoder_step", C.c_int, [_vp, C.c_int32, C.c_int, C.c_int, _vp]),
    ("charsiu_gpu_decoder_logits", C.POINTER(C.c_float), [_vp]),
    ("charsiu_gpu_decoder_generate", C.c_int, [_vp, C.c_int32, C.c_int, C.c_uint, _vp, _vp]),
    ("charsiu_gpu_decoder_launches", C.c_uint, [_vp]),
    ("charsiu_gpu_ordered_sum_dev", C.c_int, [_vp, _vp, C.c_uint, _vp, _vp]),
    ("charsiu_npu_open", _vp, [C.c_uint, C.c_uint, C.c_uint]),
    ("charsiu_npu_open_ex", _vp, [C.c_uint, C.c_uint, C.c_uint, C.c_int]),
    ("charsiu_npu_close", None, [_vp]),
    ("charsiu_npu_add", C.c_int, [_vp, _vp]),
    ("charsiu_npu_matvec", C.c_int, [_vp, C.c_int, _vp, _vp]),
    ("charsiu_npu_matvec_group", C.c_int, [_vp, _vp, C.c_uint, _vp, _vp]),
    ("charsiu_npu_submits", C.c_ulong, [_vp]),
    ("charsiu_npu_report", None, [_vp]),
    ("charsiu_npu_add_flat", C.c_int, [_vp, _vp, _vp, C.c_uint64, C.c_uint64, C.c_char_p]),
    ("charsiu_npu_matvec_flat", C.c_int, [_vp, _vp, C.c_uint, _vp, C.c_float, C.c_uint, _vp]),
    ("charsiu_npu_matvec_dev", C.c_int, [_vp, _vp, C.c_uint, _vp, C.c_float, _vp, _vp]),
    ("charsiu_npu_error", C.c_char_p, [_vp]),
    ("charsiu_npu_dead", C.c_int, [_vp]),
]


def lib():
    """Load libcharsiu_gpu.so. Raises if it was not built: there is no
    fallback implementation to use instead."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m charsiu_b200.build` "
                               "(the CUDA extension is required; there is no CPU path)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class GpuError(RuntimeError):
    pass


class Layer:
    """One charsiu_gpu device layer (one GPU, one column slab)."""

    def __init__(self, max_k: int, max_n: int, max_tensors: int = 16, device: int = 0,
                 rank: int = 0, world: int = 1):
        self.L = lib()
        self.h = self.L.charsiu_gpu_open_ex(max_k, max_n, max_tensors, device, rank, world)
        if not self.h:
            raise GpuError(f"charsiu_gpu_open_ex failed on device {device}")
        self._keep = {}

    def close(self):
        if self.h:
            self.L.charsiu_gpu_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, rc, what):
        if rc != 0:
            raise GpuError(f"{what}: {self.error()}")

    def error(self) -> str:
        return self.L.charsiu_gpu_error(self.h).decode()

    @property
    def calls(self) -> int:
        return self.L.charsiu_gpu_calls(self.h)

    @property
    def launches(self) -> int:
        return self.L.charsiu_gpu_launches(self.h)

    @property
    def dead(self) -> bool:
        return bool(self.L.charsiu_gpu_dead(self.h))

    def report(self):
        self.L.charsiu_gpu_report(self.h)

    def add_blocks(self, qtype: int, k: int, n: int, blocks: np.ndarray, name: str = "") -> int:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        tid = self.L.charsiu_gpu_add_blocks(self.h, qtype, k, n, _p(blocks), name.encode())
        if tid < 0:
            raise GpuError(f"add {name}: {self.error()}")
        return tid

    def try_add_blocks(self, qtype, k, n, blocks, name="") -> int:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        return self.L.charsiu_gpu_add_blocks(self.h, qtype, k, n, _p(blocks), name.encode())

    def rows(self, tid: int):
        r0, nr = C.c_uint64(), C.c_uint64()
        self._check(self.L.charsiu_gpu_rows(self.h, tid, C.byref(r0), C.byref(nr)), "rows")
        return r0.value, nr.value

    def matvec(self, ids, q: np.ndarray, d: np.ndarray, k: int):
        """y for each id (this GPU's rows), host buffers in and out."""
        ids = list(ids)
        ys = [np.empty(self.rows(i)[1], dtype=np.float32) for i in ids]
        rc = self.try_matvec(ids, q, d, k, ys)
        self._check(rc, "matvec")
        return ys

    def try_matvec(self, ids, q, d, k, ys) -> int:
        q = np.ascontiguousarray(q, dtype=np.int8)
        d = np.ascontiguousarray(d, dtype=np.float32)
        idarr = (C.c_int * len(ids))(*ids)
        yarr = (C.c_void_p * len(ids))(*[_p(y) for y in ys])
        return self.L.charsiu_gpu_matvec_q(self.h, C.addressof(idarr), len(ids), _p(q), _p(d), k,
                                           C.addressof(yarr))

    def batch(self, tid: int, q: np.ndarray, d: np.ndarray):
        q = np.ascontiguousarray(q, dtype=np.int8)
        d = np.ascontiguousarray(d, dtype=np.float32)
        m, kq = q.shape
        y = np.empty((m, self.rows(tid)[1]), dtype=np.float32)
        self._check(self.L.charsiu_gpu_matvec_batch(self.h, tid, m, _p(q), _p(d), kq, _p(y)),
                    "batch")
        return y

    def matmul_i8(self, a, w, bias, in_scale, wt_scale, out_scale, in_zp=128, wt_zp=128,
                  out_zp=0):
        a = np.ascontiguousarray(a, dtype=np.uint8)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        bias = np.ascontiguousarray(bias, dtype=np.int32)
        m, k = a.shape
        n = w.shape[0]
        out = np.full((m, n), 0x5a, dtype=np.int8)
        self._check(self.L.charsiu_gpu_matmul_i8_flat(self.h, m, k, n, _p(a), _p(w), _p(bias),
                                                      in_scale, wt_scale, out_scale, in_zp,
                                                      wt_zp, out_zp, _p(out)), "matmul_i8")
        return out

    def block_dots(self, tid: int, q: np.ndarray):
        q = np.ascontiguousarray(q, dtype=np.int8)
        rows = self.rows(tid)[1]
        nb = q.size // 32
        out = np.empty((rows, nb), dtype=np.int32)
        self._check(self.L.charsiu_gpu_block_dots(self.h, tid, _p(q), _p(out)), "block_dots")
        return out

    def inject(self, at: int, count: int, kind: int):
        self._check(self.L.charsiu_gpu_inject(self.h, at, count, kind), "inject")

    # device-pointer forms (pointers are ints, e.g. torch tensor.data_ptr())
    def matvec_dev(self, ids, q_ptr: int, d_ptr: int, y_ptrs, stream: int = 0) -> int:
        ids = list(ids)
        idarr = (C.c_int * len(ids))(*ids)
        yarr = (C.c_void_p * len(ids))(*y_ptrs)
        return self.L.charsiu_gpu_matvec_dev(self.h, C.addressof(idarr), len(ids), q_ptr, d_ptr,
                                             C.addressof(yarr), stream or None)

    def batch_dev(self, tid: int, m: int, q_ptr: int, d_ptr: int, y_ptr: int,
                  stream: int = 0) -> int:
        return self.L.charsiu_gpu_matvec_batch_dev(self.h, tid, m, q_ptr, d_ptr, y_ptr,
                                                   stream or None)

    def batch_group_dev(self, ids, m: int, q_ptr: int, d_ptr: int, y_ptrs,
                        stream: int = 0) -> int:
        ids = list(ids)
        idarr = (C.c_int * len(ids))(*ids)
        yarr = (C.c_void_p * len(ids))(*y_ptrs)
        return self.L.charsiu_gpu_matvec_batch_group_dev(self.h, C.addressof(idarr), len(ids),
                                                         m, q_ptr, d_ptr, C.addressof(yarr),
                                                         stream or None)

    # the matvec fused with its all-gather (one process a GPU, rank/world at open)
    def ipc_alloc(self, nbytes: int) -> int:
        p = self.L.charsiu_gpu_ipc_alloc(self.h, nbytes)
        if not p:
            raise GpuError("ipc_alloc failed")
        return p

    def ipc_handle(self, ptr: int) -> bytes:
        buf = (C.c_ubyte * 64)()
        self._check(self.L.charsiu_gpu_ipc_handle(self.h, ptr, buf), "ipc_handle")
        return bytes(buf)

    def ipc_open(self, handle: bytes) -> int:
        buf = (C.c_ubyte * 64).from_buffer_copy(handle)
        p = self.L.charsiu_gpu_ipc_open(self.h, buf)
        if not p:
            raise GpuError("ipc_open failed")
        return p

    def ipc_free(self, ptr: int, opened: bool):
        self.L.charsiu_gpu_ipc_free(self.h, ptr, int(opened))

    def read_device(self, ptr: int, out: np.ndarray) -> np.ndarray:
        self._check(self.L.charsiu_gpu_read_device(self.h, ptr, _p(out), out.nbytes),
                    "read_device")
        return out

    def gather_epoch_dev(self, sync_ptr: int, stream: int = 0) -> int:
        return self.L.charsiu_gpu_gather_epoch_dev(self.h, sync_ptr, stream or None)

    def kernel_error(self) -> int:
        return self.L.charsiu_gpu_kernel_error(self.h)

    def matvec_gather_dev(self, ids, q_ptr: int, d_ptr: int, full_ptrs, sync_ptrs,
                          signal_idx: int, wait_idx: int = 0, wait_mult: int = 0,
                          wait_adj: int = 0, stream: int = 0) -> int:
        """full_ptrs: rank-major [world][len(ids)] device pointers (peer ones
        from ipc_open); sync_ptrs: [world]."""
        ids = list(ids)
        idarr = (C.c_int * len(ids))(*ids)
        farr = (C.c_void_p * len(full_ptrs))(*full_ptrs)
        sarr = (C.c_void_p * len(sync_ptrs))(*sync_ptrs)
        return self.L.charsiu_gpu_matvec_gather_dev(self.h, C.addressof(idarr), len(ids), q_ptr,
                                                    d_ptr, C.addressof(farr), C.addressof(sarr),
                                                    signal_idx, wait_idx, wait_mult, wait_adj,
                                                    stream or None)

    def batch_gather_dev(self, ids, m: int, q_ptr: int, d_ptr: int, full_ptrs, sync_ptrs,
                         signal_idx: int, wait_idx: int = 0, wait_mult: int = 0,
                         wait_adj: int = 0, stream: int = 0) -> int:
        """The batched matvec fused with its all-gather; full_ptrs rank-major
        [world][len(ids)] device pointers to [m][N] outputs."""
        ids = list(ids)
        idarr = (C.c_int * len(ids))(*ids)
        farr = (C.c_void_p * len(full_ptrs))(*full_ptrs)
        sarr = (C.c_void_p * len(sync_ptrs))(*sync_ptrs)
        return self.L.charsiu_gpu_matvec_batch_gather_dev(
            self.h, C.addressof(idarr), len(ids), m, q_ptr, d_ptr, C.addressof(farr),
            C.addressof(sarr), signal_idx, wait_idx, wait_mult, wait_adj, stream or None)

    def batch_noalloc(self, tid: int, m: int, q_ptr: int, d_ptr: int, y_ptr: int,
                      stream: int = 0) -> int:
        """The batched matvec with no device allocation (fixed 1 MiB scratch)."""
        return self.L.charsiu_gpu_matvec_batch_noalloc(self.h, tid, m, q_ptr, d_ptr, y_ptr,
                                                       stream or None)

    def ordered_sum_dev(self, a_ptr: int, n: int, out_ptr: int, stream: int = 0) -> int:
        """The sequential fp32 sum of n device floats, out_ptr[0] by one
        thread and out_ptr[1] by one CTA (two device floats)."""
        return self.L.charsiu_gpu_ordered_sum_dev(self.h, a_ptr, n, out_ptr, stream or None)

    def row_dev(self, tid: int, row_ptr: int, out_ptr: int, stream: int = 0) -> int:
        """gguf_row_f32 of row *row_ptr (device int32) into out_ptr (device)."""
        return self.L.charsiu_gpu_row_dev(self.h, tid, row_ptr, out_ptr, stream or None)

    def act_quantise_dev(self, x_ptr: int, m: int, k: int, q_ptr: int, d_ptr: int,
                         stream: int = 0) -> int:
        return self.L.charsiu_gpu_act_quantise_dev(self.h, x_ptr, m, k, q_ptr, d_ptr,
                                                   stream or None)


class Llama:
    """charsiu_gpu_llama: the decode loop with every projection on the GPU."""

    def __init__(self, path: str, n_ctx: int = 0, device: int = 0, resident: bool = False):
        self.L = lib()
        self.h = self.L.charsiu_gpu_llama_open(path.encode(), n_ctx, device)
        if not self.h:
            raise GpuError(f"charsiu_gpu_llama_open failed for {path}")
        self.n_vocab = self.L.charsiu_gpu_llama_vocab(self.h)
        if resident:
            try:
                self.set_resident(True)
            except GpuError:
                self.close()
                raise

    def set_resident(self, on: bool = True):
        """Every later forward on the device (charsiu_gpu_llama_set_resident)."""
        if self.L.charsiu_gpu_llama_set_resident(self.h, int(on)):
            msg = self.L.charsiu_gpu_error(self.layer_handle).decode()
            raise GpuError(f"the device decode step would not build: {msg}")

    def close(self):
        if self.h:
            self.L.charsiu_gpu_llama_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def layer_handle(self):
        return self.L.charsiu_gpu_llama_layer(self.h)

    @property
    def npu_calls(self) -> int:
        """Calls of the NPU-format layer (CHARSIU_NPU_QUANT=1 at open), else 0."""
        h = self.L.charsiu_gpu_llama_npu(self.h)
        return self.L.charsiu_npu_submits(h) if h else 0

    @property
    def step_launches(self) -> int:
        """Kernels one device-resident step launches (0 before it is built)."""
        dec = self.L.charsiu_gpu_llama_decoder(self.h)
        return self.L.charsiu_gpu_decoder_launches(dec) if dec else 0

    def report(self):
        self.L.charsiu_gpu_report(self.layer_handle)

    @property
    def launches(self) -> int:
        return self.L.charsiu_gpu_launches(self.layer_handle)

    @property
    def calls(self) -> int:
        return self.L.charsiu_gpu_calls(self.layer_handle)

    def stages(self, reset: bool = False) -> dict:
        """Mean ms a token of each forward-pass stage (reference llama.c:695-705)."""
        ms = np.zeros(32, dtype=np.float64)
        n = self.L.charsiu_gpu_llama_stages(self.h, _p(ms), 32, int(reset))
        return {self.L.charsiu_gpu_llama_stage_name(i).decode(): float(ms[i]) for i in range(n)}

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = self.L.charsiu_gpu_llama_forward(self.h, token, pos)
        if not p:
            raise GpuError(f"forward failed: {self.L.charsiu_gpu_error(self.layer_handle)}")
        return np.ctypeslib.as_array(p, shape=(self.n_vocab,)).copy()

    def generate_dev(self, token: int, pos: int, n: int):
        """n greedy steps on the device from token at pos, no host round trip
        between them (charsiu_gpu_decoder_generate; resident mode only):
        (the n argmax tokens, device ms of the n steps)."""
        dec = self.L.charsiu_gpu_llama_decoder(self.h)
        if not dec:
            raise GpuError("generate_dev needs the device step (set_resident)")
        out = np.zeros(n, dtype=np.int32)
        ms = C.c_float()
        if self.L.charsiu_gpu_decoder_generate(dec, int(token), int(pos), n, _p(out),
                                               C.byref(ms)):
            raise GpuError(f"generate failed: {self.L.charsiu_gpu_error(self.layer_handle)}")
        return out, float(ms.value)

    def greedy(self, prompt, n_gen: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, dtype=np.int32)
        lg = np.zeros((n_gen, self.n_vocab), dtype=np.float32) if want_logits else None
        ms = C.c_double()
        rc = self.L.charsiu_gpu_llama_greedy(self.h, _p(p), p.size, n_gen, _p(out),
                                             _p(lg) if lg is not None else None, C.byref(ms))
        if rc != n_gen:
            raise GpuError(f"greedy failed: {self.L.charsiu_gpu_error(self.layer_handle)}")
        return out, lg, ms.value


class NpuActStruct(C.Structure):
    """struct charsiu_act (include/charsiu_llm.h:100-119), for the struct forms."""
    _fields_ = [("f", C.c_void_p), ("n", C.c_int), ("nb", C.c_int), ("q", C.c_void_p),
                ("d", C.c_void_p), ("bs", C.c_void_p), ("quantised", C.c_int),
                ("q1", C.c_void_p), ("d1", C.c_float), ("q1_valid", C.c_int)]


class NpuTensorStruct(C.Structure):
    """struct npu_tensor (include/charsiu_llm.h:143-161), for the struct forms."""
    _fields_ = [("q", C.c_void_p), ("scale", C.c_void_p), ("kgroup", C.c_uint64),
                ("kscale", C.c_void_p), ("astat", C.c_void_p), ("acalls", C.c_uint64),
                ("acov", C.c_void_p), ("xcal", C.c_void_p), ("nxcal", C.c_uint),
                ("wsum", C.c_void_p), ("n", C.c_uint64), ("k", C.c_uint64),
                ("rms_rel", C.c_double), ("out_scale", C.c_float), ("out_clip", C.c_double),
                ("out_calls", C.c_uint64), ("amax_lo", C.c_float), ("amax_hi", C.c_float),
                ("name", C.c_char * 80)]


class NpuLayer:
    """charsiu_npu_*: charsiu's NPU device layer (the NPU number format) on the GPU."""

    def __init__(self, max_k: int, max_n: int, max_tensors: int = 16):
        self.L = lib()
        self.h = self.L.charsiu_npu_open(max_k, max_n, max_tensors)
        if not self.h:
            raise GpuError("charsiu_npu_open failed")
        self.rows = {}

    def close(self):
        if self.h:
            self.L.charsiu_npu_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def error(self) -> str:
        return self.L.charsiu_npu_error(self.h).decode()

    @property
    def calls(self) -> int:
        return self.L.charsiu_npu_submits(self.h)

    @property
    def dead(self) -> bool:
        return bool(self.L.charsiu_npu_dead(self.h))

    def report(self):
        self.L.charsiu_npu_report(self.h)

    def add(self, q: np.ndarray, scale: np.ndarray, name: str = "") -> int:
        q = np.ascontiguousarray(q, dtype=np.int8)
        scale = np.ascontiguousarray(scale, dtype=np.float32)
        n, k = q.shape
        tid = self.L.charsiu_npu_add_flat(self.h, _p(q), _p(scale), n, k, name.encode())
        if tid < 0:
            raise GpuError(f"add {name}: {self.error()}")
        self.rows[tid] = n
        return tid

    def add_struct(self, t: NpuTensorStruct) -> int:
        tid = self.L.charsiu_npu_add(self.h, C.byref(t))
        if tid >= 0:
            self.rows[tid] = t.n
        return tid

    def matvec(self, ids, q1: np.ndarray, d1, k: int):
        ids = list(ids)
        q1 = np.ascontiguousarray(q1, dtype=np.int8)
        ys = [np.empty(self.rows[i], dtype=np.float32) for i in ids]
        idarr = (C.c_int * len(ids))(*ids)
        yarr = (C.c_void_p * len(ids))(*[_p(y) for y in ys])
        rc = self.L.charsiu_npu_matvec_flat(self.h, C.addressof(idarr), len(ids), _p(q1),
                                            float(d1), k, C.addressof(yarr))
        if rc:
            raise GpuError(f"npu matvec: {self.error()}")
        return ys

    def matvec_dev(self, ids, q1_ptr: int, d1, ys_ptrs, stream: int = 0) -> int:
        ids = list(ids)
        idarr = (C.c_int * len(ids))(*ids)
        yarr = (C.c_void_p * len(ids))(*ys_ptrs)
        return self.L.charsiu_npu_matvec_dev(self.h, C.addressof(idarr), len(ids), q1_ptr,
                                             float(d1), C.addressof(yarr), stream or None)
