"""Host mirror of go-semantica's search/brute (Builder, Index, Serializer) and
search.Result, over the C ABI. Vectors live on the device; SearchVector
normalises, scans and selects the top-k there.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from _lib import SEARCH_EXACT, SEARCH_REFERENCE, Context, check, load

QuantizeFloat32, QuantizeInt8, QuantizeInt16 = 0, 1, 2  # quant.go:8-15


@dataclass
class Result:
    """search.Result (search/search.go:8-11)."""
    ID: int
    Distance: float


class Builder:
    """brute.Builder (builder.go:14-127); options WithDimension / WithQuantization."""

    def __init__(self, ctx: Context | None = None, dimension: int = 0, quantization: int = QuantizeInt8):
        self.ctx = ctx or Context(0)
        self.dimension = dimension
        self.quantization = quantization
        self._ids: list[int] = []
        self._vecs: list[np.ndarray] = []
        self._idset: set[int] = set()
        self._built = False

    def add_vector(self, id_: int, vec) -> None:
        if self._built:
            raise ValueError("brute: builder already built")
        if id_ in self._idset:
            raise ValueError(f"brute: duplicate id {id_}")
        v = np.asarray(vec, dtype=np.float32)
        if self.dimension == 0:
            self.dimension = v.size
        if v.size != self.dimension:
            raise ValueError(f"brute: vector dimension mismatch: got {v.size} want {self.dimension}")
        self._ids.append(int(id_))
        self._vecs.append(v.copy())
        self._idset.add(int(id_))

    def build(self) -> "Index":
        if self._built:
            raise ValueError("brute: builder already built")
        if not self._vecs:
            raise ValueError("brute: no vectors added")
        idx = Index.build(self.ctx, np.stack(self._vecs), np.asarray(self._ids, dtype=np.int32), self.quantization)
        self._built = True
        return idx


class Index:
    """brute.Index (index.go:12-214)."""

    def __init__(self, ctx: Context, handle):
        self.ctx = ctx
        self.handle = handle

    @classmethod
    def build(cls, ctx: Context, vectors: np.ndarray, ids=None, quantization: int = QuantizeInt8) -> "Index":
        v = np.ascontiguousarray(vectors, dtype=np.float32)
        idp = None if ids is None else np.ascontiguousarray(ids, dtype=np.int32)
        h = C.c_void_p()
        check(load().sem_index_build(ctx.handle, v.shape[1], quantization, v.ctypes.data,
                                     None if idp is None else idp.ctypes.data, v.shape[0], C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def from_codes(cls, ctx: Context, codes: np.ndarray, ids=None, quantization: int | None = None) -> "Index":
        codes = np.ascontiguousarray(codes)
        q = quantization if quantization is not None else {np.dtype(np.float32): 0, np.dtype(np.int8): 1,
                                                           np.dtype(np.int16): 2}[codes.dtype]
        idp = None if ids is None else np.ascontiguousarray(ids, dtype=np.int32)
        h = C.c_void_p()
        check(load().sem_index_create(ctx.handle, codes.shape[1], q, codes.ctypes.data,
                                      None if idp is None else idp.ctypes.data, codes.shape[0], C.byref(h)))
        return cls(ctx, h)

    def close(self):
        if self.handle:
            load().sem_index_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def dimension(self) -> int:
        v = C.c_int32()
        check(load().sem_index_dimension(self.handle, C.byref(v)))
        return v.value

    def count(self) -> int:
        v = C.c_int64()
        check(load().sem_index_count(self.handle, C.byref(v)))
        return v.value

    def quantization(self) -> int:
        v = C.c_int32()
        check(load().sem_index_quantization(self.handle, C.byref(v)))
        return v.value

    def search_batch(self, queries: np.ndarray, top_k: int, mode: int = SEARCH_EXACT, normalize: bool = True):
        """Many queries in one device pass; returns (ids [nq,k], dist [nq,k], scores [nq,k])."""
        q = np.ascontiguousarray(np.atleast_2d(queries), dtype=np.float32)
        nq, dim = q.shape
        k = max(int(top_k), 1)
        ids = np.full((nq, k), -1, dtype=np.int32)
        dist = np.zeros((nq, k), dtype=np.float32)
        scores = np.zeros((nq, k), dtype=np.int32)
        check(load().sem_index_search(self.handle, q.ctypes.data, nq, dim, int(top_k), mode, 1 if normalize else 0,
                                      ids.ctypes.data, dist.ctypes.data, scores.ctypes.data))
        return ids, dist, scores

    def _results(self, ids, dist, top_k):
        n = min(top_k, self.count())
        return [Result(int(ids[0, j]), float(dist[0, j])) for j in range(n)]

    def search_vector(self, vec, top_k: int, mode: int = SEARCH_EXACT) -> list[Result]:
        """SearchVector (index.go:29-42)."""
        ids, dist, _ = self.search_batch(np.asarray(vec, dtype=np.float32)[None, :], top_k, mode, True)
        return self._results(ids, dist, top_k)

    def search_normalized(self, vec, top_k: int, mode: int = SEARCH_EXACT) -> list[Result]:
        """SearchNormalized (index.go:44-53)."""
        ids, dist, _ = self.search_batch(np.asarray(vec, dtype=np.float32)[None, :], top_k, mode, False)
        return self._results(ids, dist, top_k)

    def vector(self, id_: int):
        """Vector (index.go:162-180); None when the id is absent."""
        out = np.empty(self.dimension(), dtype=np.float32)
        rc = load().sem_index_vector(self.handle, id_, out.ctypes.data)
        if rc == 5:
            return None
        check(rc)
        return out


class Serializer:
    """brute.Serializer: BRUT v1 bytes (storage.go:17-153)."""

    @staticmethod
    def serialize(idx: Index) -> bytes:
        n = C.c_size_t()
        check(load().sem_index_serialize(idx.handle, None, 0, C.byref(n)))
        buf = (C.c_uint8 * n.value)()
        check(load().sem_index_serialize(idx.handle, buf, n.value, C.byref(n)))
        return bytes(buf)

    @staticmethod
    def deserialize(data: bytes, ctx: Context | None = None) -> Index:
        ctx = ctx or Context(0)
        b = np.frombuffer(data, dtype=np.uint8)
        h = C.c_void_p()
        check(load().sem_index_deserialize(ctx.handle, b.ctypes.data, b.size, C.byref(h)))
        return Index(ctx, h)


def quantize_queries(q_normalized: np.ndarray, quantization: int) -> np.ndarray:
    q = np.ascontiguousarray(q_normalized, dtype=np.float32)
    out = np.empty(q.shape, dtype=np.int8 if quantization == 1 else np.int16)
    check(load().sem_quantize_queries(q.ctypes.data, q.shape[0], q.shape[1], quantization, out.ctypes.data))
    return out


__all__ = ["Builder", "Index", "Serializer", "Result", "QuantizeFloat32", "QuantizeInt8", "QuantizeInt16",
           "SEARCH_EXACT", "SEARCH_REFERENCE", "quantize_queries"]
