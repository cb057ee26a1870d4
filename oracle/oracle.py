"""Test infrastructure only: Python access to the two CPU parity checkers.

* ``Port*`` / ``port_*``: the plain-C restatement in ``xq_oracle.c`` (``_build/libxq_oracle.so``).
* ``Ref*`` / ``ref_*``: the reference library compiled from its own sources
  (``_ref/libxqwen35_ref.so``; built only where the reference tree is present, it travels
  to GPU machines as a prebuilt file).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg import this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "_build", "libxq_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libxqwen35_ref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build(reference_dir: Optional[str] = None) -> None:
    """Compile the restatement, and the reference when its source tree is available."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    if reference_dir and os.path.isdir(os.path.join(reference_dir, "customlib")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"XQ_REFERENCE_DIR={reference_dir}"], check=True)


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


# ------------------------------------------------------------------------------------
# ABI structs of the public header (customlib/include/xqwen35.h:30-58)
# ------------------------------------------------------------------------------------
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


class _XoMatrix(C.Structure):
    _fields_ = [("rows", C.c_int), ("cols", C.c_int), ("group_size", C.c_int), ("version", C.c_int),
                ("packed", C.c_void_p), ("scales", C.c_void_p), ("zeros", C.c_void_p)]


_port = None
_ref = None


def port():
    global _port
    if _port is None:
        if not os.path.exists(PORT_LIB):
            build()
        L = C.CDLL(PORT_LIB)
        L.xo_gemv_w4a16.argtypes = [C.POINTER(_XoMatrix), _f32p, _f32p]
        L.xo_gemv_w4a16_argmax.argtypes = [C.POINTER(_XoMatrix), _f32p, C.POINTER(C.c_float)]
        L.xo_gemv_w4a16_argmax.restype = C.c_int
        L.xo_rmsnorm.argtypes = [_f32p, _f32p, C.c_int, C.c_float, _f32p]
        L.xo_head_rmsnorm.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float]
        L.xo_l2norm_heads.argtypes = [_f32p, C.c_int, C.c_int]
        L.xo_gated_head_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_float, _f32p]
        L.xo_rope_partial.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.xo_attention_decode.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        L.xo_conv1d_step.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, _f32p]
        L.xo_gated_delta_decode.argtypes = [_f32p, _f32p, _f32p, C.c_float, C.c_float, C.c_int, C.c_int,
                                            _f32p, _f32p]
        for n in ("xo_silu", "xo_sigmoid", "xo_softplus"):
            getattr(L, n).argtypes = [C.c_float]
            getattr(L, n).restype = C.c_float
        L.xo_model_load.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
        L.xo_model_load.restype = C.c_void_p
        L.xo_model_free.argtypes = [C.c_void_p]
        L.xo_model_reset.argtypes = [C.c_void_p]
        L.xo_model_prefill.argtypes = [C.c_void_p, _i32p, C.c_size_t, C.c_char_p, C.c_size_t]
        L.xo_model_decode_one.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
        for n in ("xo_model_hidden_size", "xo_model_layers", "xo_model_position"):
            getattr(L, n).argtypes = [C.c_void_p]
            getattr(L, n).restype = C.c_int
        L.xo_model_hidden.argtypes = [C.c_void_p, _f32p]
        L.xo_model_logits.argtypes = [C.c_void_p, _f32p]
        for n in ("xo_model_conv_state", "xo_model_recurrent_state"):
            getattr(L, n).argtypes = [C.c_void_p, C.c_int, C.c_void_p]
            getattr(L, n).restype = C.c_size_t
        L.xo_model_kv.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.xo_model_kv.restype = C.c_size_t
        L.xo_set_threads.argtypes = [C.c_int]
        _port = L
    return _port


def ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            raise FileNotFoundError("reference library not built: " + REF_LIB)
        L = C.CDLL(REF_LIB)
        mat = [C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _f32p, _f32p]
        L.ref_gemv_w4a16.argtypes = mat + [_f32p, _f32p]
        L.ref_gemv_w4a16_argmax.argtypes = mat + [_f32p, C.POINTER(C.c_float)]
        L.ref_gemv_w4a16_argmax.restype = C.c_int
        L.ref_gemv_lowbit_reference.argtypes = mat + [_f32p, _f32p]
        L.ref_quantize_w4.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _u8p, _f32p, _f32p]
        L.ref_rmsnorm.argtypes = [_f32p, _f32p, C.c_int, C.c_float, _f32p]
        L.ref_attention_decode.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        L.ref_gated_delta_decode.argtypes = [_f32p, _f32p, _f32p, C.c_float, C.c_float, C.c_int, C.c_int,
                                             _f32p, _f32p]
        declare_abi(L)
        _ref = L
    return _ref


def declare_abi(L) -> None:
    """Argument types of the public C ABI (customlib/include/xqwen35.h:60-77)."""
    P = C.c_void_p
    L.xq_create.argtypes = [C.c_char_p, C.POINTER(XqOptions), C.POINTER(P)]
    L.xq_destroy.argtypes = [P]
    L.xq_destroy.restype = None
    L.xq_prefill.argtypes = [P, C.POINTER(C.c_int32), C.c_size_t, C.POINTER(XqMetrics)]
    L.xq_decode_one.argtypes = [P, C.POINTER(C.c_int32), C.POINTER(XqMetrics)]
    L.xq_generate.argtypes = [P, C.POINTER(C.c_int32), C.c_size_t, C.c_size_t, C.POINTER(C.c_int32),
                              C.c_size_t, C.POINTER(XqMetrics)]
    L.xq_reset.argtypes = [P]
    L.xq_get_last_metrics.argtypes = [P, C.POINTER(XqMetrics)]
    for n in ("xq_get_backend_info", "xq_get_kernel_trace_json", "xq_get_debug_json"):
        getattr(L, n).argtypes = [P, C.c_char_p, C.c_size_t]
    L.xq_get_hidden_state.argtypes = [P, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_size_t)]
    L.xq_run_vulkan_w4a16_selftest.argtypes = [C.c_char_p, C.c_size_t]


# ------------------------------------------------------------------------------------
# Matrices
# ------------------------------------------------------------------------------------
class Matrix:
    """An XQ4 matrix held as numpy arrays (the reference's QuantizedMatrix fields)."""

    def __init__(self, rows, cols, group, version, packed, scales, zeros):
        self.rows, self.cols, self.group, self.version = int(rows), int(cols), int(group), int(version)
        self.packed = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
        self.scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        self.zeros = np.ascontiguousarray(zeros, dtype=np.float32).reshape(-1)

    @classmethod
    def from_xq4(cls, d):
        return cls(d["rows"], d["cols"], d["group"], d["version"], d["packed"], d["scales"], d["zeros"])

    def _xo(self):
        return _XoMatrix(self.rows, self.cols, self.group, self.version, self.packed.ctypes.data,
                         self.scales.ctypes.data, self.zeros.ctypes.data)

    def _refargs(self):
        return (self.rows, self.cols, self.group, self.version, self.packed, self.scales, self.zeros)

    def dequantize(self) -> np.ndarray:
        """Dense fp32 weights, dequantizeValue semantics (ref_gemv.cpp:73-87)."""
        gpr = (self.cols + self.group - 1) // self.group
        p = self.packed.reshape(self.rows, -1)
        codes = np.empty((self.rows, p.shape[1] * 2), dtype=np.float32)
        codes[:, 0::2] = p & 0x0F
        codes[:, 1::2] = p >> 4
        codes = codes[:, : self.cols]
        g = np.arange(self.cols) // self.group
        s = self.scales.reshape(self.rows, gpr)[:, g]
        z = self.zeros.reshape(self.rows, gpr)[:, g]
        if self.version == 2:
            return codes * s + z
        return (codes - z) * s


def port_gemv(m: Matrix, x: np.ndarray) -> np.ndarray:
    y = np.zeros(m.rows, dtype=np.float32)
    xm = m._xo()
    port().xo_gemv_w4a16(C.byref(xm), np.ascontiguousarray(x, np.float32), y)
    return y


def port_argmax(m: Matrix, x: np.ndarray):
    v = C.c_float()
    xm = m._xo()
    i = port().xo_gemv_w4a16_argmax(C.byref(xm), np.ascontiguousarray(x, np.float32), C.byref(v))
    return i, v.value


def ref_gemv(m: Matrix, x: np.ndarray) -> np.ndarray:
    y = np.zeros(m.rows, dtype=np.float32)
    ref().ref_gemv_w4a16(*m._refargs(), np.ascontiguousarray(x, np.float32), y)
    return y


def ref_argmax(m: Matrix, x: np.ndarray):
    v = C.c_float()
    i = ref().ref_gemv_w4a16_argmax(*m._refargs(), np.ascontiguousarray(x, np.float32), C.byref(v))
    return i, v.value


def ref_quantize(w: np.ndarray, group: int) -> Matrix:
    """quantizeLowBit (ref_gemv.cpp:38-71), 4-bit, asymmetric with integer zeros."""
    rows, cols = w.shape
    gpr = (cols + group - 1) // group
    packed = np.zeros(rows * ((cols + 1) // 2), dtype=np.uint8)
    scales = np.zeros(rows * gpr, dtype=np.float32)
    zeros = np.zeros(rows * gpr, dtype=np.float32)
    ref().ref_quantize_w4(np.ascontiguousarray(w, np.float32), rows, cols, group, packed, scales, zeros)
    return Matrix(rows, cols, group, 1, packed, scales, zeros)


# ------------------------------------------------------------------------------------
# Sessions
# ------------------------------------------------------------------------------------
class RefSession:
    """The reference's own C ABI session (custom CPU path, use_mnn_fallback = 0)."""

    def __init__(self, model_dir: str, threads: int = 8):
        L = ref()
        self.L = L
        opts = XqOptions()
        opts.struct_size = C.sizeof(XqOptions)
        opts.backend = b"cpu"
        opts.threads = threads
        opts.quant_bits = 4
        opts.group_size = 64
        opts.use_mnn_fallback = 0
        self.h = C.c_void_p()
        st = L.xq_create(model_dir.encode(), C.byref(opts), C.byref(self.h))
        if st != 0:
            raise RuntimeError(f"reference xq_create failed: {st}")

    def prefill(self, ids) -> XqMetrics:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        m = XqMetrics()
        m.struct_size = C.sizeof(XqMetrics)
        st = self.L.xq_prefill(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size, C.byref(m))
        if st != 0:
            raise RuntimeError(f"reference xq_prefill failed: {st} {m.error}")
        return m

    def decode_one(self) -> int:
        t = C.c_int32()
        m = XqMetrics()
        m.struct_size = C.sizeof(XqMetrics)
        st = self.L.xq_decode_one(self.h, C.byref(t), C.byref(m))
        if st != 0:
            raise RuntimeError(f"reference xq_decode_one failed: {st} {m.error}")
        return t.value

    def hidden(self) -> np.ndarray:
        n = C.c_size_t()
        self.L.xq_get_hidden_state(self.h, None, 0, C.byref(n))
        out = np.zeros(n.value, dtype=np.float32)
        st = self.L.xq_get_hidden_state(self.h, out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(n))
        if st != 0:
            raise RuntimeError(f"reference xq_get_hidden_state failed: {st}")
        return out

    def debug_json(self) -> str:
        buf = C.create_string_buffer(1 << 16)
        self.L.xq_get_debug_json(self.h, buf, len(buf))
        return buf.value.decode()

    def close(self):
        if self.h:
            self.L.xq_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PortModel:
    """The C restatement of CustomModel (custom_model.cpp) with Session positions."""

    def __init__(self, model_dir: str):
        L = port()
        self.L = L
        err = C.create_string_buffer(512)
        self.h = L.xo_model_load(model_dir.encode(), err, len(err))
        if not self.h:
            raise RuntimeError("oracle load failed: " + err.value.decode())

    def prefill(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        err = C.create_string_buffer(512)
        if not self.L.xo_model_prefill(self.h, ids, ids.size, err, len(err)):
            raise RuntimeError(err.value.decode())

    def decode_one(self) -> int:
        t = C.c_int32()
        err = C.create_string_buffer(512)
        if not self.L.xo_model_decode_one(self.h, C.byref(t), err, len(err)):
            raise RuntimeError(err.value.decode())
        return t.value

    @property
    def position(self) -> int:
        return self.L.xo_model_position(self.h)

    def hidden(self) -> np.ndarray:
        out = np.zeros(self.L.xo_model_hidden_size(self.h), dtype=np.float32)
        self.L.xo_model_hidden(self.h, out)
        return out

    def logits(self, vocab: int) -> np.ndarray:
        out = np.zeros(vocab, dtype=np.float32)
        self.L.xo_model_logits(self.h, out)
        return out

    def conv_state(self, layer: int) -> np.ndarray:
        n = self.L.xo_model_conv_state(self.h, layer, None)
        out = np.zeros(n, dtype=np.float32)
        if n:
            self.L.xo_model_conv_state(self.h, layer, out.ctypes.data)
        return out

    def recurrent_state(self, layer: int) -> np.ndarray:
        n = self.L.xo_model_recurrent_state(self.h, layer, None)
        out = np.zeros(n, dtype=np.float32)
        if n:
            self.L.xo_model_recurrent_state(self.h, layer, out.ctypes.data)
        return out

    def kv(self, layer: int):
        n = self.L.xo_model_kv(self.h, layer, None, None)
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        if n:
            self.L.xo_model_kv(self.h, layer, k.ctypes.data, v.ctypes.data)
        return k, v

    def close(self):
        if self.h:
            self.L.xo_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
