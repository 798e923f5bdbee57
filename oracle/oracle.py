"""ctypes binding of the CPU oracle (semantica_oracle.c) — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker. The product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libsemantica_oracle.so")

_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "semantica_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "_build/libsemantica_oracle.so"],
                       check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        f32p, i32p, i8p = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.POINTER(C.c_int8)
        L.orc_f16_runtime.restype = C.c_float
        L.orc_f16_runtime.argtypes = [C.c_uint16]
        L.orc_f16_gguf.restype = C.c_float
        L.orc_f16_gguf.argtypes = [C.c_uint16]
        L.orc_fast_exp.restype = C.c_float
        L.orc_fast_exp.argtypes = [C.c_float]
        L.orc_softmax.argtypes = [f32p, f32p, C.c_int]
        L.orc_gelu_quick_simd.argtypes = [f32p, f32p, C.c_int]
        L.orc_dot_f32.restype = C.c_float
        L.orc_dot_f32.argtypes = [f32p, f32p, C.c_int]
        L.orc_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_float]
        L.orc_quantize_sym_int8.argtypes = [f32p, C.c_int64, i8p, f32p]
        L.orc_matmul_q8_0_int8.argtypes = [f32p, C.c_void_p, f32p, i8p, C.c_float, C.c_int, C.c_int, C.c_int]
        L.orc_set_matmul_path.argtypes = [C.c_int]
        L.orc_set_simd.restype = C.c_int
        L.orc_set_simd.argtypes = [C.c_int]
        L.orc_extract_q8_0_scales.argtypes = [C.c_void_p, C.c_int64, C.c_int, f32p]
        L.orc_model_load.restype = C.c_void_p
        L.orc_model_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_config.argtypes = [C.c_void_p, C.c_void_p]
        L.orc_model_set_faithful.restype = C.c_int
        L.orc_model_set_faithful.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int]
        L.orc_forward.restype = C.c_int
        L.orc_forward.argtypes = [C.c_void_p, i32p, C.c_int, C.c_int, f32p, C.c_char_p, C.c_int]
        L.orc_forward_batch.restype = C.c_int
        L.orc_forward_batch.argtypes = [C.c_void_p, i32p, i32p, C.c_int, C.c_int, f32p, C.c_int,
                                        C.c_char_p, C.c_int]
        L.orc_normalize.argtypes = [f32p, C.c_int]
        L.orc_quantize_int8_vec.argtypes = [f32p, C.c_int, i8p]
        L.orc_quantize_int16_vec.argtypes = [f32p, C.c_int, C.POINTER(C.c_int16)]
        L.orc_dot_int8_ref.restype = C.c_float
        L.orc_dot_int8_ref.argtypes = [i8p, f32p, C.c_int]
        L.orc_dot_int16_ref.restype = C.c_float
        L.orc_dot_int16_ref.argtypes = [C.POINTER(C.c_int16), f32p, C.c_int]
        L.orc_dot_f32_ref.restype = C.c_float
        L.orc_dot_f32_ref.argtypes = [f32p, f32p, C.c_int]
        L.orc_search_ref.restype = C.c_int
        L.orc_search_ref.argtypes = [C.c_int, C.c_void_p, i32p, C.c_int64, C.c_int, f32p, C.c_int, i32p, f32p]
        L.orc_search_exact.restype = C.c_int
        L.orc_search_exact.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_int,
                                       i32p, i32p, f32p]
        L.orc_search_exact_batch.restype = C.c_int
        L.orc_search_exact_batch.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_int,
                                             C.c_int, i32p, i32p, f32p, C.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


class OracleConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("vocab_size", "embed_dim", "num_layers", "num_heads", "num_kv_heads",
                                         "head_dim", "interm_dim", "max_seq_len")] + \
               [(n, C.c_float) for n in ("norm_eps", "rope_base", "attention_scale")]


# ---- scalar kernels ----
def fast_exp(x: float) -> float:
    return lib().orc_fast_exp(x)


def f16_runtime(bits: int) -> float:
    return lib().orc_f16_runtime(bits)


def f16_gguf(bits: int) -> float:
    return lib().orc_f16_gguf(bits)


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_softmax(_p(out, C.c_float), _p(x, C.c_float), x.size)
    return out


def gelu_quick(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_gelu_quick_simd(_p(out, C.c_float), _p(x, C.c_float), x.size)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    o = out.reshape(-1, n)
    for r in range(rows.shape[0]):
        lib().orc_rmsnorm(_p(o[r], C.c_float), _p(rows[r], C.c_float), _p(w, C.c_float), n, eps)
    return out


def quantize_sym_int8(x: np.ndarray) -> tuple[np.ndarray, float]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.empty(x.shape, dtype=np.int8)
    sc = C.c_float(0)
    lib().orc_quantize_sym_int8(_p(x, C.c_float), x.size, _p(codes, C.c_int8), C.byref(sc))
    return codes, sc.value


def extract_q8_0_scales(w_q8: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w_q8 = np.ascontiguousarray(w_q8)
    out = np.empty(rows * ((cols + 31) // 32), dtype=np.float32)
    lib().orc_extract_q8_0_scales(w_q8.ctypes.data, rows, cols, _p(out, C.c_float))
    return out


def matmul_q8_0_int8(w_q8: np.ndarray, codes: np.ndarray, a_scale: float, out_dim: int) -> np.ndarray:
    """Q8_0 weights [out_dim, in/32, 34] bytes x int8 activations [batch, in] -> fp32 [batch, out]."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    batch, in_dim = codes.shape
    w_q8 = np.ascontiguousarray(w_q8)
    scales = extract_q8_0_scales(w_q8, out_dim, in_dim)
    out = np.empty((batch, out_dim), dtype=np.float32)
    lib().orc_matmul_q8_0_int8(_p(out, C.c_float), w_q8.ctypes.data, _p(scales, C.c_float),
                               _p(codes, C.c_int8), a_scale, batch, in_dim, out_dim)
    return out


# ---- model ----
class OracleModel:
    def __init__(self, path: str):
        err = C.create_string_buffer(512)
        self._h = lib().orc_model_load(path.encode(), err, 512)
        if not self._h:
            raise RuntimeError(err.value.decode())
        cfg = OracleConfig()
        lib().orc_model_config(self._h, C.byref(cfg))
        self.config = cfg

    def set_faithful(self, sliding_window: int = 0, swa_pattern: int = 0, rope_base_swa: float = 0.0,
                     dense_head: bool = False) -> None:
        """Model-faithful mode (no reference counterpart): sliding-window
        layers and the dense 2/3 head. Zeros restore the reference's forward."""
        if lib().orc_model_set_faithful(self._h, sliding_window, swa_pattern, rope_base_swa, 1 if dense_head else 0):
            raise ValueError("the model file has no dense_2 / dense_3 weights")

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward_with_dim(self, ids, dim: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(max(dim, 1), dtype=np.float32)
        err = C.create_string_buffer(512)
        rc = lib().orc_forward(self._h, _p(ids, C.c_int32), ids.size, dim, _p(out, C.c_float), err, 512)
        if rc:
            raise ValueError(err.value.decode())
        return out[:dim]

    def forward_batch(self, ids, offsets, dim: int, nthreads: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int32)
        n = offsets.size - 1
        out = np.empty((n, dim), dtype=np.float32)
        err = C.create_string_buffer(512)
        rc = lib().orc_forward_batch(self._h, _p(ids, C.c_int32), _p(offsets, C.c_int32), n, dim,
                                     _p(out, C.c_float), nthreads, err, 512)
        if rc:
            raise ValueError(err.value.decode())
        return out


# ---- brute ----
def normalize(v: np.ndarray) -> np.ndarray:
    v = np.array(v, dtype=np.float32, copy=True)
    rows = v.reshape(-1, v.shape[-1])
    for r in range(rows.shape[0]):
        lib().orc_normalize(_p(rows[r], C.c_float), rows.shape[1])
    return v


def quantize_int8_vec(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.int8)
    lib().orc_quantize_int8_vec(_p(v, C.c_float), v.size, _p(out, C.c_int8))
    return out


def quantize_int16_vec(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.int16)
    lib().orc_quantize_int16_vec(_p(v, C.c_float), v.size, _p(out, C.c_int16))
    return out


def dot_int8_ref(v, q) -> float:
    v = np.ascontiguousarray(v, dtype=np.int8)
    q = np.ascontiguousarray(q, dtype=np.float32)
    return lib().orc_dot_int8_ref(_p(v, C.c_int8), _p(q, C.c_float), v.size)


def dot_int16_ref(v, q) -> float:
    v = np.ascontiguousarray(v, dtype=np.int16)
    q = np.ascontiguousarray(q, dtype=np.float32)
    return lib().orc_dot_int16_ref(_p(v, C.c_int16), _p(q, C.c_float), v.size)


def dot_f32_ref(a, b) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return lib().orc_dot_f32_ref(_p(a, C.c_float), _p(b, C.c_float), a.size)


def search_ref(quant: int, data: np.ndarray, ids: np.ndarray, query_normalized: np.ndarray, topk: int):
    data = np.ascontiguousarray(data)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    q = np.ascontiguousarray(query_normalized, dtype=np.float32)
    count, dim = data.shape
    k = max(1, min(topk, count))
    oi = np.empty(k, dtype=np.int32)
    od = np.empty(k, dtype=np.float32)
    n = lib().orc_search_ref(quant, data.ctypes.data, _p(ids, C.c_int32), count, dim, _p(q, C.c_float), topk,
                             _p(oi, C.c_int32), _p(od, C.c_float))
    return oi[:n], od[:n]


def search_exact_batch(quant: int, data: np.ndarray, qcodes: np.ndarray, topk: int, nthreads: int = 0):
    data = np.ascontiguousarray(data)
    qcodes = np.ascontiguousarray(qcodes)
    count, dim = data.shape
    nq = qcodes.shape[0]
    rows = np.full((nq, topk), -1, dtype=np.int32)
    scores = np.zeros((nq, topk), dtype=np.int32)
    dist = np.zeros((nq, topk), dtype=np.float32)
    n = lib().orc_search_exact_batch(quant, data.ctypes.data, count, dim, qcodes.ctypes.data, nq, topk,
                                     _p(rows, C.c_int32), _p(scores, C.c_int32), _p(dist, C.c_float), nthreads)
    return rows[:, :n], scores[:, :n], dist[:, :n]


def set_simd(on: bool) -> bool:
    """Timing only (bench.py's CPU legs): the Q8_0 inner loop and the float32
    dot product run as AVX512-VNNI / AVX2 intrinsics that are the reference's
    assembly instruction for instruction; results are bit-identical to the
    plain loops. Returns whether the CPU supports it (else the switch stays off)."""
    return bool(lib().orc_set_simd(1 if on else 0))


def set_matmul_path(path: int) -> None:
    """Reference build to follow: 0 amd64 on an AVX512-VNNI host (default),
    1 amd64 on an AVX2-only host, 2 the portable (noasm) build."""
    lib().orc_set_matmul_path(path)
