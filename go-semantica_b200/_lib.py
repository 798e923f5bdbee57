"""ctypes binding of libsemantica_b200.so (declared in include/semantica_b200.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsemantica_b200.so")

SEM_OK, SEM_EINVAL, SEM_EDEVICE, SEM_ENOMEM, SEM_EFORMAT, SEM_ENOTFOUND, SEM_EINTERNAL = range(7)
SEARCH_REFERENCE, SEARCH_EXACT = 0, 1


class SemError(Exception):
    """Error returned by the C ABI; .code is the SEM_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class ModelConfig(C.Structure):
    """Mirrors internal/runtime.ModelConfig (model.go:16-31)."""
    _fields_ = [(n, C.c_int32) for n in ("vocab_size", "embed_dim", "num_layers", "num_heads", "num_kv_heads",
                                         "head_dim", "interm_dim", "max_seq_len")] + \
               [(n, C.c_float) for n in ("norm_eps", "rope_base", "attention_scale")]


class TensorView(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_uint32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("data", C.c_void_p), ("nbytes", C.c_uint64)]


class FaithfulConfig(C.Structure):
    """sem_faithful_config: the model-faithful mode (no reference counterpart)."""
    _fields_ = [("sliding_window", C.c_int32), ("swa_pattern", C.c_int32), ("rope_base_swa", C.c_float),
                ("dense_head", C.c_int32)]


# name -> (restype, argtypes)
_SIGNATURES = {
    "sem_last_error": (C.c_char_p, []),
    "sem_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "sem_context_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "sem_context_destroy": (C.c_int, [C.c_void_p]),
    "sem_context_stream": (C.c_void_p, [C.c_void_p]),
    "sem_model_load": (C.c_int, [C.c_void_p, C.POINTER(ModelConfig), C.POINTER(TensorView), C.c_int32,
                                 C.POINTER(C.c_void_p)]),
    "sem_model_load_gguf": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    "sem_model_config_get": (C.c_int, [C.c_void_p, C.POINTER(ModelConfig)]),
    "sem_model_free": (C.c_int, [C.c_void_p]),
    "sem_embed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "sem_embed_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                   C.c_void_p]),
    "sem_embed_submit": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                                   C.POINTER(C.c_uint64)]),
    "sem_embed_wait": (C.c_int, [C.c_void_p, C.c_uint64, C.c_void_p]),
    "sem_model_check": (C.c_int, [C.c_void_p]),
    "sem_model_set_faithful": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sem_group_load": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(ModelConfig), C.POINTER(TensorView), C.c_int32,
                                 C.POINTER(C.c_void_p)]),
    "sem_group_load_gguf": (C.c_int, [C.c_void_p, C.c_int32, C.c_char_p, C.POINTER(C.c_void_p)]),
    "sem_group_size": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "sem_group_config_get": (C.c_int, [C.c_void_p, C.POINTER(ModelConfig)]),
    "sem_group_set_faithful": (C.c_int, [C.c_void_p, C.c_void_p]),
    "sem_group_embed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "sem_group_free": (C.c_int, [C.c_void_p]),
    "sem_model_profile": (C.c_int, [C.c_void_p, C.c_int32]),
    "sem_model_profile_read": (C.c_int, [C.c_void_p, C.POINTER(C.c_char_p), C.POINTER(C.c_float),
                                         C.POINTER(C.c_int32), C.c_int32, C.POINTER(C.c_int32)]),
    "sem_q8_weight_create": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "sem_q8_weight_free": (C.c_int, [C.c_void_p]),
    "sem_q8_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "sem_q8_gemm_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "sem_q8_matmul_int8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "sem_q8_path": (C.c_int, [C.c_int32]),
    "sem_index_build": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                  C.POINTER(C.c_void_p)]),
    "sem_index_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                   C.POINTER(C.c_void_p)]),
    "sem_index_free": (C.c_int, [C.c_void_p]),
    "sem_index_count": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    "sem_index_dimension": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "sem_index_quantization": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "sem_index_search": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_void_p]),
    "sem_index_search_keys": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int64,
                                        C.c_void_p, C.c_void_p]),
    "sem_topk_merge": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                 C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "sem_quantize_queries": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]),
    "sem_index_vector": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "sem_index_serialize": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "sem_index_deserialize": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
}

_lib = None


def load() -> C.CDLL:
    """The library handle; raises if libsemantica_b200.so has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python go-semantica_b200/build.py` "
                               "(there is no CPU fallback)")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int) -> None:
    if rc != SEM_OK:
        msg = load().sem_last_error()
        raise SemError(rc, msg.decode() if msg else f"status {rc}")


def device_count() -> int:
    n = C.c_int(0)
    rc = load().sem_device_count(C.byref(n))
    return n.value if rc == SEM_OK else 0


class Context:
    """One device, one stream (sem_context)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(load().sem_context_create(device, C.byref(h)))
        self.handle = h
        self.device = device

    @property
    def stream(self) -> int:
        return load().sem_context_stream(self.handle) or 0

    def close(self) -> None:
        if self.handle:
            load().sem_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
