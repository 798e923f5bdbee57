"""Multi-GPU sharding of the two hot paths, one process per GPU.

Embeddings partition by sequence, with no collective on the data path:
split_sequences balances the tokens across ranks, each rank embeds its share
(sem_embed), and embed_sharded gathers every rank's vectors in the caller's
order (the reference fans prompts out over goroutines the same way,
pkg/ggufembed/api.go:237-295).

Search partitions by rows: shard_rows gives each rank a contiguous range of
the corpus; ShardedIndex searches its shard into 64-bit candidate keys
((order-preserving score << 32) | ~global_row, sem_index_search_keys),
all-gathers them over the process group (NCCL between GPUs) and merges them
with sem_topk_merge into the global top-k by (score desc, row asc), the order
of searchNormalized (search/brute/index.go:55-154).

The collectives go through torch.distributed, so the host logic runs the
same with the gloo backend on CPU tensors.
"""
from __future__ import annotations

from typing import Callable, Sequence

import numpy as np


def _group_info(group=None) -> tuple[int, int]:
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_rows(count: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous rows [start, stop) of `rank`: sizes differ by at most one row."""
    if world < 1 or not 0 <= rank < world or count < 0:
        raise ValueError(f"shard_rows: bad arguments count={count} world={world} rank={rank}")
    base, rem = divmod(count, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def split_sequences(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, balanced by token count: longest first to the
    rank holding the fewest tokens (ties to the lower rank, then the lower
    index), each rank's list in ascending order. Deterministic, so every rank
    computes the same split."""
    if world < 1:
        raise ValueError("split_sequences: world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda q: (loads[q], q))
        parts[r].append(i)
        loads[r] += int(lengths[i])
    return [sorted(p) for p in parts]


def embed_sharded(embed_fn: Callable, ids, offsets, dims, group=None) -> list[np.ndarray]:
    """Embeds this rank's share of the sequences with embed_fn(ids, offsets,
    dims) -> list of vectors (on a GPU: Model.forward_batch) and returns every
    sequence's vector, in the caller's order, on every rank."""
    import torch.distributed as dist
    rank, world = _group_info(group)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    lengths = np.diff(offsets)
    n = lengths.size
    dims = [int(dims)] * n if np.isscalar(dims) else [int(d) for d in dims]
    if len(dims) != n:
        raise ValueError(f"embed_sharded: {len(dims)} dims for {n} sequences")
    mine = split_sequences(lengths, world)[rank]
    vecs: list[np.ndarray] = []
    if mine:
        sub_ids = np.concatenate([ids[offsets[i]:offsets[i + 1]] for i in mine]).astype(np.int32)
        sub_offs = np.concatenate([[0], np.cumsum(lengths[mine])]).astype(np.int32)
        vecs = [np.asarray(v, dtype=np.float32) for v in embed_fn(sub_ids, sub_offs, [dims[i] for i in mine])]
    if world == 1:
        shares = [(mine, vecs)]
    else:
        shares = [None] * world
        dist.all_gather_object(shares, (mine, vecs), group=group)
    out: list = [None] * n
    for idxs, vs in shares:
        for i, v in zip(idxs, vs):
            out[i] = v
    return out


def gather_candidates(local_keys, group=None):
    """All ranks' candidate keys ([nq, k] int64 tensors) as one [world, nq, k]
    tensor, rank order, on every rank."""
    import torch
    import torch.distributed as dist
    rank, world = _group_info(group)
    if world == 1:
        return local_keys.unsqueeze(0)
    out = torch.empty((world,) + tuple(local_keys.shape), dtype=local_keys.dtype, device=local_keys.device)
    if local_keys.is_cuda:
        dist.all_gather_into_tensor(out.view(-1), local_keys.contiguous().view(-1), group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, local_keys.contiguous(), group=group)
        out = torch.stack(parts)
    return out


class ShardedIndex:
    """This rank's rows [row_base, row_base + count) of a row-sharded exact
    int8/int16 index on one GPU; search_codes returns the global top-k."""

    def __init__(self, ctx, codes, row_base: int, quantization: int = 1, group=None):
        """codes: this rank's rows as a [count, dim] int8 (1) or int16 (2)
        numpy array or torch tensor (host or device; the index copies them)."""
        import ctypes as C

        import torch
        from _lib import check, load
        self.ctx = ctx
        self.group = group
        self.row_base = int(row_base)
        self.quant = int(quantization)
        if isinstance(codes, torch.Tensor):
            codes = codes.contiguous()
            if codes.is_cuda:
                torch.cuda.current_stream(codes.device).synchronize()  # written on torch's stream
            ptr = codes.data_ptr()
        else:
            codes = np.ascontiguousarray(codes)
            ptr = codes.ctypes.data
        self.count, self.dim = int(codes.shape[0]), int(codes.shape[1])
        h = C.c_void_p()
        check(load().sem_index_create(ctx.handle, self.dim, self.quant, C.c_void_p(ptr), None, self.count,
                                      C.byref(h)))
        self.handle = h
        self._stream = torch.cuda.ExternalStream(ctx.stream)

    def search_codes(self, d_qcodes, k: int):
        """d_qcodes: [nq, dim] device tensor of query codes (quantised like the
        rows), written on the caller's current stream. Returns device tensors
        rows [nq, k] (global; -1 when empty) and scores [nq, k] int32, the same
        on every rank, ready on the caller's stream."""
        import ctypes as C

        import torch
        from _lib import check, load
        lib = load()
        nq = int(d_qcodes.shape[0])
        dev = d_qcodes.device
        caller = torch.cuda.current_stream(dev)
        st = C.c_void_p(self.ctx.stream)
        with torch.cuda.stream(self._stream):  # every step on the library's stream, in order
            self._stream.wait_stream(caller)
            keys = torch.empty((nq, k), dtype=torch.int64, device=dev)  # every key is written
            check(lib.sem_index_search_keys(self.handle, C.c_void_p(d_qcodes.data_ptr()), nq, k, 1, self.row_base,
                                            C.c_void_p(keys.data_ptr()), st))
            allk = gather_candidates(keys, self.group).contiguous()
            rows = torch.empty((nq, k), dtype=torch.int32, device=dev)
            scores = torch.empty((nq, k), dtype=torch.int32, device=dev)
            check(lib.sem_topk_merge(self.ctx.handle, C.c_void_p(allk.data_ptr()), int(allk.shape[0]), nq, k, k, 1,
                                     self.quant, C.c_void_p(rows.data_ptr()), C.c_void_p(scores.data_ptr()), None,
                                     st))
        caller.wait_stream(self._stream)
        for t in (rows, scores):
            t.record_stream(caller)
        return rows, scores

    def close(self) -> None:
        from _lib import load
        if getattr(self, "handle", None):
            load().sem_index_free(self.handle)
            self.handle = None
