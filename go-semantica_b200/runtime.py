"""Host mirror of go-semantica's internal/runtime over the C ABI.

Model.forward_with_dim keeps the reference signature and errors
((*Model).ForwardWithDim, internal/runtime/model.go:661-666); forward_batch is
the batched call the device path is built for: all sequences of a request in
one sem_embed call instead of one goroutine per sequence
(pkg/ggufembed/api.go:237-295).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

import _lib
from _lib import Context, ModelConfig, TensorView, check, load


class Model:
    def __init__(self, ctx: Context, handle):
        self.ctx = ctx
        self.handle = handle
        cfg = ModelConfig()
        check(load().sem_model_config_get(self.handle, C.byref(cfg)))
        self._config = cfg

    def config(self) -> ModelConfig:
        return self._config

    def close(self) -> None:
        if self.handle:
            load().sem_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- reference surface ----
    def forward(self, token_ids) -> np.ndarray:
        return self.forward_with_dim(token_ids, self._config.embed_dim)

    def forward_with_dim(self, token_ids, target_dim: int) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        return self.forward_batch(ids, np.array([0, ids.size], dtype=np.int32), [target_dim])[0]

    # ---- batched ----
    def forward_batch(self, ids, offsets, dims=None) -> list[np.ndarray]:
        """Packed ids + offsets[B+1]; dims: one int for all, a per-sequence list, or None (embed_dim)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int32)
        n = offsets.size - 1
        if dims is None:
            dims = [self._config.embed_dim] * n
        elif np.isscalar(dims):
            dims = [int(dims)] * n
        d = np.ascontiguousarray(dims, dtype=np.int32)
        out = np.empty(max(int(d[d > 0].sum()) if n else 0, 1), dtype=np.float32)
        check(load().sem_embed(self.handle, ids.ctypes.data, offsets.ctypes.data, n, d.ctypes.data, out.ctypes.data))
        res, o = [], 0
        for k in d:
            res.append(out[o:o + int(k)].copy())
            o += int(k)
        return res

    # ---- request pipeline ----
    def submit(self, ids, offsets, dims=None) -> tuple:
        """sem_embed_submit: enqueues a request and returns its ticket without
        waiting; at most two requests are in flight."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int32)
        n = offsets.size - 1
        if dims is None:
            dims = [self._config.embed_dim] * n
        elif np.isscalar(dims):
            dims = [int(dims)] * n
        d = np.ascontiguousarray(dims, dtype=np.int32)
        t = C.c_uint64()
        check(load().sem_embed_submit(self.handle, ids.ctypes.data, offsets.ctypes.data, n, d.ctypes.data,
                                      C.byref(t)))
        return (t.value, d)

    def wait(self, ticket) -> list[np.ndarray]:
        """sem_embed_wait: the outputs of a submitted request."""
        t, d = ticket
        out = np.empty(max(int(d.sum()) if d.size else 0, 1), dtype=np.float32)
        check(load().sem_embed_wait(self.handle, C.c_uint64(t), out.ctypes.data))
        res, o = [], 0
        for k in d:
            res.append(out[o:o + int(k)].copy())
            o += int(k)
        return res

    def embed_stream(self, requests):
        """Embeds an iterable of (ids, offsets, dims) requests through the
        pipeline, yielding each request's vectors in order. The next request
        is drawn from the iterable (e.g. tokenised) and submitted while the
        device runs the current one."""
        pending = None
        try:
            for ids, offsets, dims in requests:
                t = self.submit(ids, offsets, dims)
                prev, pending = pending, t
                if prev is not None:
                    yield self.wait(prev)
            if pending is not None:
                last, pending = pending, None
                yield self.wait(last)
        finally:
            if pending is not None:  # abandoned or failed: free the slot
                try:
                    self.wait(pending)
                except Exception:
                    pass

    def profile(self, enable: bool) -> None:
        check(load().sem_model_profile(self.handle, 1 if enable else 0))

    def profile_read(self) -> dict:
        """{stage: (total_ms, launches)} since the last read (synchronises)."""
        cap = 32
        names = (C.c_char_p * cap)()
        ms = (C.c_float * cap)()
        n = (C.c_int32 * cap)()
        got = C.c_int32()
        check(load().sem_model_profile_read(self.handle, names, ms, n, cap, C.byref(got)))
        return {names[i].decode(): (ms[i], n[i]) for i in range(got.value)}

    def embed_device(self, d_ids_ptr: int, offsets, n_seqs: int, dim: int, d_out_ptr: int, stream: int = 0) -> None:
        """Device-resident forward (sem_embed_device); offsets stay on the host."""
        offsets = np.ascontiguousarray(offsets, dtype=np.int32)
        check(load().sem_embed_device(self.handle, C.c_void_p(d_ids_ptr), offsets.ctypes.data, n_seqs, dim,
                                      C.c_void_p(d_out_ptr), C.c_void_p(stream or None)))

    def set_faithful(self, sliding_window: int = 0, swa_pattern: int = 0, rope_base_swa: float = 0.0,
                     dense_head: bool = False) -> None:
        """Model-faithful mode (sem_model_set_faithful; no reference
        counterpart): sliding-window layers and the dense 2/3 head. All zero
        restores the reference's forward."""
        cfg = _lib.FaithfulConfig(sliding_window, swa_pattern, rope_base_swa, 1 if dense_head else 0)
        check(load().sem_model_set_faithful(self.handle, C.byref(cfg)))

    def check(self) -> None:
        """Waits for the enqueued device-resident forwards and raises what the
        device recorded (a token id outside the vocabulary, a timed-out
        pipeline wait) since the last check (sem_model_check)."""
        check(load().sem_model_check(self.handle))


class Group:
    """Several devices as one embedding engine (sem_group_*): a model replica
    per device, each request split across them by token count and embedded on
    all devices at once. forward_batch keeps Model.forward_batch's contract."""

    def __init__(self, handle):
        self.handle = handle
        cfg = ModelConfig()
        check(load().sem_group_config_get(self.handle, C.byref(cfg)))
        self._config = cfg
        n = C.c_int32()
        check(load().sem_group_size(self.handle, C.byref(n)))
        self.size = n.value

    def config(self) -> ModelConfig:
        return self._config

    def close(self) -> None:
        if self.handle:
            load().sem_group_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_with_dim(self, token_ids, target_dim: int) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        return self.forward_batch(ids, np.array([0, ids.size], dtype=np.int32), [target_dim])[0]

    def forward_batch(self, ids, offsets, dims=None) -> list[np.ndarray]:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int32)
        n = offsets.size - 1
        if dims is None:
            dims = [self._config.embed_dim] * n
        elif np.isscalar(dims):
            dims = [int(dims)] * n
        d = np.ascontiguousarray(dims, dtype=np.int32)
        out = np.empty(max(int(d[d > 0].sum()) if n else 0, 1), dtype=np.float32)
        check(load().sem_group_embed(self.handle, ids.ctypes.data, offsets.ctypes.data, n, d.ctypes.data,
                                     out.ctypes.data))
        res, o = [], 0
        for k in d:
            res.append(out[o:o + int(k)].copy())
            o += int(k)
        return res

    def set_faithful(self, sliding_window: int = 0, swa_pattern: int = 0, rope_base_swa: float = 0.0,
                     dense_head: bool = False) -> None:
        cfg = _lib.FaithfulConfig(sliding_window, swa_pattern, rope_base_swa, 1 if dense_head else 0)
        check(load().sem_group_set_faithful(self.handle, C.byref(cfg)))


def load_group(path: str, devices) -> Group:
    """The model of a GGUF file on every device in `devices` (sem_group_load_gguf)."""
    devs = np.ascontiguousarray(list(devices), dtype=np.int32)
    h = C.c_void_p()
    check(load().sem_group_load_gguf(devs.ctypes.data, devs.size, path.encode(), C.byref(h)))
    return Group(h)


def load_model(path: str, ctx: Context | None = None) -> Model:
    """LoadModel (model.go:233-246): GGUF file -> device-resident model."""
    ctx = ctx or Context(0)
    h = C.c_void_p()
    check(load().sem_model_load_gguf(ctx.handle, path.encode(), C.byref(h)))
    return Model(ctx, h)


def load_model_from_views(ctx: Context, config: ModelConfig, tensors: dict) -> Model:
    """sem_model_load with tensor views (the path a Go loader takes through cgo).
    tensors: name -> (dtype, dims tuple, numpy buffer)."""
    keep = []
    views = (TensorView * len(tensors))()
    for i, (name, (dtype, dims, buf)) in enumerate(tensors.items()):
        b = np.ascontiguousarray(buf)
        keep.append(b)
        nb = name.encode()
        keep.append(nb)
        views[i].name = nb
        views[i].dtype = dtype
        views[i].n_dims = len(dims)
        for k, dv in enumerate(dims):
            views[i].dims[k] = dv
        views[i].data = b.ctypes.data
        views[i].nbytes = b.nbytes
    h = C.c_void_p()
    check(load().sem_model_load(ctx.handle, C.byref(config), views, len(tensors), C.byref(h)))
    return Model(ctx, h)


class Q8Weight:
    """Isolated Q8_0 projection (QuantizeSymmetricINT8Into + MatMulQ8_0INT8)."""

    def __init__(self, ctx: Context, w_q8: np.ndarray, k_in: int, n_out: int):
        w = np.ascontiguousarray(w_q8)
        h = C.c_void_p()
        check(load().sem_q8_weight_create(ctx.handle, w.ctypes.data, k_in, n_out, C.byref(h)))
        self.handle, self.k_in, self.n_out, self.ctx = h, k_in, n_out, ctx

    def run(self, d_a: int, m: int, d_c: int, d_codes: int, d_absmax: int, stream: int = 0) -> None:
        check(load().sem_q8_gemm(self.handle, C.c_void_p(d_a), m, C.c_void_p(d_c), C.c_void_p(d_codes),
                                 C.c_void_p(d_absmax), C.c_void_p(stream or None)))

    def matmul_int8(self, d_codes: int, d_absmax: int, m: int, d_c: int, stream: int = 0) -> None:
        """MatMulQ8_0INT8 on codes already quantised (fp16-held INT8 codes, absmax bit pattern)."""
        check(load().sem_q8_matmul_int8(self.handle, C.c_void_p(d_codes), C.c_void_p(d_absmax), m, C.c_void_p(d_c),
                                        C.c_void_p(stream or None)))

    def close(self):
        if self.handle:
            load().sem_q8_weight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["Model", "load_model", "load_model_from_views", "Q8Weight", "Context", "_lib"]
