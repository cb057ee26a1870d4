"""xqwen35_b200: Python access to libxqwen35.so, the B200 decode library.

The product is the shared library (C ABI in include/xqwen35.h and include/xq_kernels.h);
this module only builds it and binds it with ctypes for tests and benchmarks. Device
memory for the kernel-level entry points may come from any allocator (the tests use torch
tensors); no computation happens in Python.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from typing import Optional

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
# XQ_LIB_PATH: load another build of the library (A/B measurements of build variants).
LIB_PATH = os.environ.get("XQ_LIB_PATH") or os.path.join(PKG_DIR, "lib", "libxqwen35.so")

XQ_OK = 0
XQ_ERR_INVALID_ARGUMENT = -1
XQ_ERR_NOT_READY = -2
XQ_ERR_MODEL = -3
XQ_ERR_RUNTIME = -4
XQ_ERR_BUFFER_TOO_SMALL = -5

# Every symbol the two public headers declare.
ABI_SYMBOLS = [
    "xq_create", "xq_destroy", "xq_prefill", "xq_decode_one", "xq_generate", "xq_reset",
    "xq_get_last_metrics", "xq_get_backend_info", "xq_get_kernel_trace_json", "xq_get_debug_json",
    "xq_get_hidden_state", "xq_run_vulkan_w4a16_selftest", "xq_create_cuda", "xq_cuda_decode_timed",
    "xq_snapshot_size", "xq_snapshot_save", "xq_snapshot_restore", "xq_pack_b200_layout",
    "xq_batch_create", "xq_batch_destroy", "xq_batch_prefill", "xq_batch_decode", "xq_batch_decode_timed",
    "xq_batch_hidden_state", "xq_tp_unique_id", "xq_tp_create", "xq_tp_destroy", "xq_tp_prefill", "xq_tp_decode",
    "xq_tp_hidden_state", "xq_tp_plan", "xq_tp_argmax_combine",
]
KERNEL_SYMBOLS = [
    "xqk_last_error", "xqk_matrix_create", "xqk_matrix_destroy", "xqk_matrix_info", "xqk_gemv_w4a16",
    "xqk_gemv_w4a16_host", "xqk_gemv_w4a16_argmax", "xqk_rmsnorm", "xqk_gated_delta_step",
    "xqk_attention_step", "xqk_attention_step_noalloc", "xqk_gemv_w4a16_mma",
    "xqk_mma_tiles", "xqk_gemv_w4a16_mma_f16", "xqk_prefill_gemm_w4a16",
]


def build(jobs: int = 8) -> str:
    """Compile the CUDA sources for sm_100a into lib/libxqwen35.so (incremental)."""
    subprocess.run(["make", "-s", "-C", CSRC, f"-j{jobs}"], check=True)
    return LIB_PATH


class XqOptions(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("backend", C.c_char_p), ("threads", C.c_int),
                ("quant_bits", C.c_int), ("group_size", C.c_int), ("max_context_tokens", C.c_int),
                ("enable_autotune", C.c_int), ("use_mnn_fallback", C.c_int),
                ("telemetry_path", C.c_char_p)]


class XqMetrics(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("prompt_tokens", C.c_uint64),
                ("generated_tokens", C.c_uint64), ("load_ms", C.c_double), ("prefill_ms", C.c_double),
                ("first_token_ms", C.c_double), ("decode_total_ms", C.c_double),
                ("total_generate_ms", C.c_double), ("prefill_tokens_per_second", C.c_double),
                ("decode_tokens_per_second", C.c_double), ("rss_kb", C.c_uint64), ("pss_kb", C.c_uint64),
                ("backend", C.c_char * 64), ("selected_kernels", C.c_char * 512), ("error", C.c_char * 256)]


class XqCudaOptions(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("device", C.c_int), ("kv_fp16", C.c_int), ("use_graphs", C.c_int),
                ("prefill_batched", C.c_int)]


_lib = None


def lib():
    """Load libxqwen35.so; raises if it has not been built (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is missing: run build() (nvcc, sm_100a)")
    L = C.CDLL(LIB_PATH)
    P = C.c_void_p
    L.xq_create.argtypes = [C.c_char_p, C.POINTER(XqOptions), C.POINTER(P)]
    L.xq_create_cuda.argtypes = [C.c_char_p, C.POINTER(XqOptions), C.POINTER(XqCudaOptions), C.POINTER(P)]
    L.xq_destroy.argtypes = [P]
    L.xq_destroy.restype = None
    L.xq_prefill.argtypes = [P, C.POINTER(C.c_int32), C.c_size_t, C.POINTER(XqMetrics)]
    L.xq_decode_one.argtypes = [P, C.POINTER(C.c_int32), C.POINTER(XqMetrics)]
    L.xq_generate.argtypes = [P, C.POINTER(C.c_int32), C.c_size_t, C.c_size_t, C.POINTER(C.c_int32), C.c_size_t,
                              C.POINTER(XqMetrics)]
    L.xq_reset.argtypes = [P]
    L.xq_get_last_metrics.argtypes = [P, C.POINTER(XqMetrics)]
    for n in ("xq_get_backend_info", "xq_get_kernel_trace_json", "xq_get_debug_json"):
        getattr(L, n).argtypes = [P, C.c_char_p, C.c_size_t]
    L.xq_get_hidden_state.argtypes = [P, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_size_t)]
    L.xq_run_vulkan_w4a16_selftest.argtypes = [C.c_char_p, C.c_size_t]
    L.xq_cuda_decode_timed.argtypes = [P, C.c_size_t, C.POINTER(C.c_int32), C.POINTER(C.c_double)]
    L.xq_snapshot_size.argtypes = [P, C.POINTER(C.c_size_t)]
    L.xq_pack_b200_layout.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
    L.xq_snapshot_save.argtypes = [P, P, C.c_size_t, C.POINTER(C.c_size_t)]
    L.xq_snapshot_restore.argtypes = [P, P, C.c_size_t]
    L.xq_batch_create.argtypes = [C.c_char_p, C.POINTER(XqCudaOptions), C.c_int, C.c_int, C.POINTER(P)]
    L.xq_batch_destroy.argtypes = [P]
    L.xq_batch_destroy.restype = None
    L.xq_batch_prefill.argtypes = [P, C.c_int, C.POINTER(C.c_int32), C.c_size_t]
    L.xq_batch_decode.argtypes = [P, C.POINTER(C.c_int32)]
    L.xq_batch_decode_timed.argtypes = [P, C.c_size_t, C.POINTER(C.c_int32), C.POINTER(C.c_double)]
    L.xq_batch_hidden_state.argtypes = [P, C.c_int, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_size_t)]
    L.xq_tp_unique_id.argtypes = [P, C.c_size_t]
    L.xq_tp_create.argtypes = [C.c_char_p, C.POINTER(XqCudaOptions), C.c_int, C.c_int, P, C.c_int, C.POINTER(P)]
    L.xq_tp_destroy.argtypes = [P]
    L.xq_tp_destroy.restype = None
    L.xq_tp_prefill.argtypes = [P, C.POINTER(C.c_int32), C.c_size_t]
    L.xq_tp_decode.argtypes = [P, C.c_size_t, C.POINTER(C.c_int32), C.POINTER(C.c_double)]
    L.xq_tp_hidden_state.argtypes = [P, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_size_t)]
    L.xq_tp_plan.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.xq_tp_argmax_combine.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_int32)]
    L.xqk_last_error.restype = C.c_char_p
    L.xqk_matrix_create.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(P)]
    L.xqk_matrix_destroy.argtypes = [P]
    L.xqk_matrix_destroy.restype = None
    L.xqk_matrix_info.argtypes = [P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_size_t),
                                  C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.xqk_gemv_w4a16.argtypes = [P, P, P, P]
    L.xqk_gemv_w4a16_mma.argtypes = [P, P, P, P]
    L.xqk_gemv_w4a16_mma_f16.argtypes = [P, P, P, P]
    L.xqk_prefill_gemm_w4a16.argtypes = [P, P, P, C.c_int, P, C.c_int, C.c_int, P]
    L.xqk_mma_tiles.argtypes = [P, P, C.c_int, C.c_int, P, C.c_size_t, C.POINTER(C.c_size_t)]
    L.xqk_gemv_w4a16_host.argtypes = [P, P, P]
    L.xqk_gemv_w4a16_argmax.argtypes = [P, P, P, P, P]
    L.xqk_rmsnorm.argtypes = [P, P, C.c_int, C.c_float, P, P]
    L.xqk_gated_delta_step.argtypes = [P, P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, P]
    L.xqk_attention_step.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_float, C.c_float, P, P]
    L.xqk_attention_step_noalloc.argtypes = L.xqk_attention_step.argtypes
    _lib = L
    return L


def last_error() -> str:
    return (lib().xqk_last_error() or b"").decode()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")


def pack_b200(model_dir: str) -> None:
    """Write the package's weights in the kernels' row layout (xq_pack_b200_layout; host only)."""
    err = C.create_string_buffer(1024)
    st = lib().xq_pack_b200_layout(model_dir.encode(), err, len(err))
    if st != XQ_OK:
        raise RuntimeError(f"xq_pack_b200_layout failed: {st} {err.value.decode()}")


class Matrix:
    """A W4A16 matrix uploaded to the device (xqk_matrix_create)."""

    def __init__(self, packed: np.ndarray, scales: np.ndarray, zeros: np.ndarray, rows: int, cols: int,
                 group: int, version: int = 1, device: int = 0):
        L = lib()
        self._keep = [np.ascontiguousarray(packed, np.uint8), np.ascontiguousarray(scales, np.float32),
                      np.ascontiguousarray(zeros, np.float32)]
        self.h = C.c_void_p()
        check(L.xqk_matrix_create(self._keep[0].ctypes.data, self._keep[1].ctypes.data, self._keep[2].ctypes.data,
                                  rows, cols, group, version, device, C.byref(self.h)), "xqk_matrix_create")
        self.rows, self.cols = rows, cols

    def info(self) -> dict:
        r, c, st, kind, fast = C.c_int(), C.c_int(), C.c_int(), C.c_int(), C.c_int()
        nb = C.c_size_t()
        lib().xqk_matrix_info(self.h, C.byref(r), C.byref(c), C.byref(nb), C.byref(st), C.byref(kind),
                              C.byref(fast))
        return dict(rows=r.value, cols=c.value, bytes=nb.value, row_stride=st.value, kind=kind.value,
                    fast=bool(fast.value))

    def gemv(self, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
        check(lib().xqk_gemv_w4a16(self.h, x_ptr, y_ptr, stream or None), "xqk_gemv_w4a16")

    def gemv_mma(self, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
        """y = W x on the integer tensor cores (xqk_gemv_w4a16_mma)."""
        check(lib().xqk_gemv_w4a16_mma(self.h, x_ptr, y_ptr, stream or None), "xqk_gemv_w4a16_mma")

    def gemv_mma_f16(self, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
        """y = W x with fp16 x and y on the integer tensor cores (xqk_gemv_w4a16_mma_f16)."""
        check(lib().xqk_gemv_w4a16_mma_f16(self.h, x_ptr, y_ptr, stream or None), "xqk_gemv_w4a16_mma_f16")

    def prefill_gemm(self, x_ptr: int, x_lo_ptr: Optional[int], n_tokens: int, y_ptr: int, ldy: int,
                     out_kind: int = 0, stream: int = 0) -> None:
        """Y = X W^T on the tcgen05 tensor cores (xqk_prefill_gemm_w4a16); x bf16 [n_tokens][cols]."""
        check(lib().xqk_prefill_gemm_w4a16(self.h, x_ptr, x_lo_ptr or None, n_tokens, y_ptr, ldy, out_kind,
                                           stream or None), "xqk_prefill_gemm_w4a16")

    def gemv_host(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(self.rows, np.float32)
        check(lib().xqk_gemv_w4a16_host(self.h, x.ctypes.data, y.ctypes.data), "xqk_gemv_w4a16_host")
        return y

    def argmax(self, x_ptr: int, idx_ptr: int, val_ptr: int, stream: int = 0) -> None:
        check(lib().xqk_gemv_w4a16_argmax(self.h, x_ptr, idx_ptr, val_ptr, stream or None), "xqk_gemv_w4a16_argmax")

    def close(self):
        if self.h:
            lib().xqk_matrix_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """One xq_session (the reference C ABI) on a CUDA device."""

    def __init__(self, model_dir: str, device: Optional[int] = None, kv_fp16: bool = False,
                 use_graphs: bool = True, max_context_tokens: int = 0, prefill_batched: Optional[bool] = None):
        L = lib()
        self.L = L
        o = XqOptions()
        o.struct_size = C.sizeof(XqOptions)
        o.backend = b"cuda"
        o.threads = 1
        o.quant_bits = 4
        o.group_size = 64
        o.max_context_tokens = max_context_tokens
        o.use_mnn_fallback = 0
        co = XqCudaOptions()
        co.struct_size = C.sizeof(XqCudaOptions)
        co.device = -1 if device is None else device
        co.kv_fp16 = 1 if kv_fp16 else 0
        co.use_graphs = 1 if use_graphs else 0
        co.prefill_batched = -1 if prefill_batched is None else int(bool(prefill_batched))
        self.h = C.c_void_p()
        st = L.xq_create_cuda(model_dir.encode(), C.byref(o), C.byref(co), C.byref(self.h))
        if st != XQ_OK:
            self.status = st
            raise RuntimeError(f"xq_create_cuda failed: {st} {last_error()}")

    def _m(self):
        m = XqMetrics()
        m.struct_size = C.sizeof(XqMetrics)
        return m

    def prefill(self, ids) -> XqMetrics:
        ids = np.ascontiguousarray(ids, np.int32)
        m = self._m()
        st = self.L.xq_prefill(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size, C.byref(m))
        if st != XQ_OK:
            raise RuntimeError(f"xq_prefill failed: {st} {m.error.decode()}")
        return m

    def decode_one(self) -> int:
        t = C.c_int32()
        m = self._m()
        st = self.L.xq_decode_one(self.h, C.byref(t), C.byref(m))
        if st != XQ_OK:
            raise RuntimeError(f"xq_decode_one failed: {st} {m.error.decode()}")
        return t.value

    def generate(self, ids, max_new: int):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(max_new, np.int32)
        m = self._m()
        st = self.L.xq_generate(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size, max_new,
                                out.ctypes.data_as(C.POINTER(C.c_int32)), out.size, C.byref(m))
        if st != XQ_OK:
            raise RuntimeError(f"xq_generate failed: {st} {m.error.decode()}")
        return out, m

    def decode_timed(self, n: int, want_tokens: bool = False):
        """n decode steps back to back; returns (device_ms, tokens or None)."""
        ms = C.c_double()
        toks = np.zeros(max(1, n), np.int32) if want_tokens else None
        ptr = toks.ctypes.data_as(C.POINTER(C.c_int32)) if want_tokens else None
        st = self.L.xq_cuda_decode_timed(self.h, n, ptr, C.byref(ms))
        if st != XQ_OK:
            raise RuntimeError(f"xq_cuda_decode_timed failed: {st}")
        return ms.value, (toks[:n] if want_tokens else None)

    def snapshot(self) -> bytes:
        """The session's decode state (xq_snapshot_save) as bytes."""
        n = C.c_size_t()
        st = self.L.xq_snapshot_size(self.h, C.byref(n))
        if st != XQ_OK:
            raise RuntimeError(f"xq_snapshot_size failed: {st}")
        buf = C.create_string_buffer(n.value)
        w = C.c_size_t()
        st = self.L.xq_snapshot_save(self.h, buf, n.value, C.byref(w))
        if st != XQ_OK:
            raise RuntimeError(f"xq_snapshot_save failed: {st}")
        return buf.raw[: w.value]

    def restore(self, snap: bytes) -> int:
        """Replace the session's state with a snapshot (xq_snapshot_restore); returns the status."""
        buf = C.create_string_buffer(snap, len(snap))
        return self.L.xq_snapshot_restore(self.h, buf, len(snap))

    def metrics(self) -> XqMetrics:
        m = self._m()
        self.L.xq_get_last_metrics(self.h, C.byref(m))
        return m

    def hidden(self) -> np.ndarray:
        n = C.c_size_t()
        self.L.xq_get_hidden_state(self.h, None, 0, C.byref(n))
        out = np.zeros(n.value, np.float32)
        st = self.L.xq_get_hidden_state(self.h, out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(n))
        if st != XQ_OK:
            raise RuntimeError(f"xq_get_hidden_state failed: {st}")
        return out

    def json(self, which: str) -> str:
        fn = {"backend": self.L.xq_get_backend_info, "trace": self.L.xq_get_kernel_trace_json,
              "debug": self.L.xq_get_debug_json}[which]
        buf = C.create_string_buffer(1 << 20)
        st = fn(self.h, buf, len(buf))
        if st != XQ_OK:
            raise RuntimeError(f"{which} json failed: {st}")
        return buf.value.decode()

    def reset(self) -> int:
        return self.L.xq_reset(self.h)

    def close(self):
        if self.h:
            self.L.xq_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_plan(model_dir: str, world: int, rank: int) -> dict:
    """This rank's tensor-parallel shard ranges (xq_tp_plan), half-open [first, last)."""
    buf = C.create_string_buffer(1024)
    st = lib().xq_tp_plan(model_dir.encode(), world, rank, buf, len(buf))
    if st != XQ_OK:
        raise ValueError(f"xq_tp_plan failed: {st} {last_error()}")
    return json.loads(buf.value.decode())


def tp_argmax_combine(values, indices) -> int:
    """The cross-rank argmax rule (xq_tp_argmax_combine) on host arrays."""
    v = np.ascontiguousarray(values, np.float32)
    i = np.ascontiguousarray(indices, np.int32)
    out = C.c_int32()
    st = lib().xq_tp_argmax_combine(v.ctypes.data_as(C.POINTER(C.c_float)), i.ctypes.data_as(C.POINTER(C.c_int32)),
                                    v.size, C.byref(out))
    if st != XQ_OK:
        raise ValueError(f"xq_tp_argmax_combine failed: {st}")
    return out.value


class Tp:
    """Tensor-parallel decode of one sequence over several GPUs (xq_tp_*): one instance per
    rank process, every rank making the same calls. `uid` is Tp.unique_id() from one rank."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_ubyte * 128)()
        st = lib().xq_tp_unique_id(buf, 128)
        if st != XQ_OK:
            raise RuntimeError(f"xq_tp_unique_id failed: {st} {last_error()}")
        return bytes(buf)

    def __init__(self, model_dir: str, world: int, rank: int, uid: bytes, max_context: int, device: int = 0,
                 kv_fp16: bool = False):
        L = lib()
        self.L = L
        co = XqCudaOptions()
        co.struct_size = C.sizeof(XqCudaOptions)
        co.device = device
        co.kv_fp16 = 1 if kv_fp16 else 0
        co.use_graphs = 1
        co.prefill_batched = -1
        idbuf = (C.c_ubyte * 128).from_buffer_copy(uid[:128])
        self.h = C.c_void_p()
        st = L.xq_tp_create(model_dir.encode(), C.byref(co), world, rank, idbuf, max_context, C.byref(self.h))
        if st != XQ_OK:
            raise RuntimeError(f"xq_tp_create failed: {st} {last_error()}")

    def prefill(self, ids) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        st = self.L.xq_tp_prefill(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size)
        if st != XQ_OK:
            raise RuntimeError(f"xq_tp_prefill failed: {st} {last_error()}")

    def decode(self, steps: int):
        """steps greedy decode steps; returns (this rank's device ms, tokens)."""
        out = np.zeros(steps, np.int32)
        ms = C.c_double()
        st = self.L.xq_tp_decode(self.h, steps, out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(ms))
        if st != XQ_OK:
            raise RuntimeError(f"xq_tp_decode failed: {st} {last_error()}")
        return ms.value, out

    def hidden(self) -> np.ndarray:
        n = C.c_size_t()
        self.L.xq_tp_hidden_state(self.h, None, 0, C.byref(n))
        out = np.zeros(n.value, np.float32)
        st = self.L.xq_tp_hidden_state(self.h, out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(n))
        if st != XQ_OK:
            raise RuntimeError(f"xq_tp_hidden_state failed: {st} {last_error()}")
        return out

    def close(self):
        if self.h:
            self.L.xq_tp_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """Batched decode of several independent sequences (xq_batch_*): one weight pass per step."""

    def __init__(self, model_dir: str, batch: int, max_context: int, device: int = 0, kv_fp16: bool = False):
        L = lib()
        self.L = L
        co = XqCudaOptions()
        co.struct_size = C.sizeof(XqCudaOptions)
        co.device = device
        co.kv_fp16 = 1 if kv_fp16 else 0
        co.use_graphs = 1
        co.prefill_batched = -1
        self.h = C.c_void_p()
        st = L.xq_batch_create(model_dir.encode(), C.byref(co), batch, max_context, C.byref(self.h))
        if st != XQ_OK:
            raise RuntimeError(f"xq_batch_create failed: {st} {last_error()}")
        self.batch = batch

    def prefill(self, seq: int, ids) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        st = self.L.xq_batch_prefill(self.h, seq, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size)
        if st != XQ_OK:
            raise RuntimeError(f"xq_batch_prefill failed: {st} {last_error()}")

    def decode(self) -> np.ndarray:
        out = np.zeros(self.batch, np.int32)
        st = self.L.xq_batch_decode(self.h, out.ctypes.data_as(C.POINTER(C.c_int32)))
        if st != XQ_OK:
            raise RuntimeError(f"xq_batch_decode failed: {st} {last_error()}")
        return out

    def decode_timed(self, steps: int):
        """steps decode steps; returns (device_ms, tokens [steps][batch])."""
        out = np.zeros((steps, self.batch), np.int32)
        ms = C.c_double()
        st = self.L.xq_batch_decode_timed(self.h, steps, out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(ms))
        if st != XQ_OK:
            raise RuntimeError(f"xq_batch_decode_timed failed: {st} {last_error()}")
        return ms.value, out

    def hidden(self, seq: int) -> np.ndarray:
        n = C.c_size_t()
        self.L.xq_batch_hidden_state(self.h, seq, None, 0, C.byref(n))
        out = np.zeros(n.value, np.float32)
        st = self.L.xq_batch_hidden_state(self.h, seq, out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(n))
        if st != XQ_OK:
            raise RuntimeError(f"xq_batch_hidden_state failed: {st}")
        return out

    def close(self):
        if self.h:
            self.L.xq_batch_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
