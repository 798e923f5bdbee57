"""Host logic of the multi-GPU paths on CPU: the row and sequence partitions,
and two gloo processes (world size 2, 127.0.0.1) that shard a search and an
embedding batch through go-semantica_b200/sharded.py and must reproduce the
single-process results. The per-rank compute here is the oracle; the device
kernels behind it (sem_index_search_keys, sem_topk_merge, sem_embed) are
covered by the -m gpu tests."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import sharded
import synth
from conftest import MODEL_DIR

SEARCH_N, SEARCH_D, SEARCH_Q, SEARCH_K = 3001, 64, 9, 10


def test_shard_rows_partition():
    for count in (0, 1, 7, 100, 3001, 4194304):
        for world in (1, 2, 3, 8):
            ranges = [sharded.shard_rows(count, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == count
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharded.shard_rows(10, 2, 2)


def test_split_sequences_balanced():
    lengths = [int(x) for x in synth.ragged_lengths(5, 37, 1, 600)]
    for world in (1, 2, 3, 8):
        parts = sharded.split_sequences(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(len(lengths)))
        assert all(p == sorted(p) for p in parts)
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)
        assert parts == sharded.split_sequences(lengths, world)  # same split on every rank
    assert sharded.split_sequences([], 2) == [[], []]


def _search_data():
    import oracle
    vecs = oracle.normalize(synth.normal_vectors(41, SEARCH_N, SEARCH_D))
    q = oracle.normalize(synth.normal_vectors(42, SEARCH_Q, SEARCH_D))
    return oracle.quantize_int8_vec(vecs), oracle.quantize_int8_vec(q)


def _keys(rows, scores):
    """The device key format: (order-preserving score << 32) | ~global_row; 0 is empty."""
    k = ((scores.astype(np.int64).astype(np.uint32) ^ np.uint32(0x80000000)).astype(np.uint64) << np.uint64(32)) | \
        (np.uint32(0xFFFFFFFF) - rows.astype(np.uint32)).astype(np.uint64)
    return np.where(rows >= 0, k, np.uint64(0)).astype(np.uint64)


def _merge(keys, k):
    """Best k keys per query over all lists (keys are unique, so descending
    key order is (score desc, row asc))."""
    flat = np.sort(keys.transpose(1, 0, 2).reshape(keys.shape[1], -1), axis=1)[:, ::-1][:, :k]
    rows = np.where(flat == 0, -1, (np.uint64(0xFFFFFFFF) - (flat & np.uint64(0xFFFFFFFF))).astype(np.int64))
    scores = ((flat >> np.uint64(32)).astype(np.uint32) ^ np.uint32(0x80000000)).astype(np.int32)
    return rows.astype(np.int32), np.where(flat == 0, 0, scores)


def _search_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        codes, qcodes = _search_data()
        start, stop = sharded.shard_rows(SEARCH_N, world, rank)
        rows, scores, _ = oracle.search_exact_batch(1, codes[start:stop], qcodes, SEARCH_K)
        local = _keys(np.where(rows >= 0, rows + start, -1), scores).view(np.int64)
        allk = sharded.gather_candidates(torch.from_numpy(np.ascontiguousarray(local)))
        assert tuple(allk.shape) == (world, SEARCH_Q, SEARCH_K)
        q.put((rank, _merge(allk.numpy().view(np.uint64), SEARCH_K)))
    finally:
        dist.destroy_process_group()


def _embed_rank(rank, world, port, path, q):
    import torch.distributed as dist
    import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = oracle.OracleModel(path)
        lengths = [5, 40, 1, 17, 33, 9, 26]
        ids, offs = synth.token_batch(51, lengths, 512)
        dims = [768, 128, 512, 768, 256, 768, 128]
        calls = []

        def embed_fn(sub_ids, sub_offs, sub_dims):
            calls.append(len(sub_dims))
            return [m.forward_with_dim(sub_ids[sub_offs[i]:sub_offs[i + 1]], sub_dims[i]) for i in range(len(sub_dims))]

        out = sharded.embed_sharded(embed_fn, ids, offs, dims)
        m.close()
        q.put((rank, sum(calls), [np.asarray(v) for v in out]))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            item = q.get(timeout=240)
            results[item[0]] = item[1:]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return results


def test_sharded_search_two_ranks_matches_full_scan():
    import oracle
    codes, qcodes = _search_data()
    want_rows, want_scores, _ = oracle.search_exact_batch(1, codes, qcodes, SEARCH_K)
    res = _run(_search_rank, 2)
    for rank in (0, 1):
        (rows, scores), = res[rank]
        np.testing.assert_array_equal(rows, want_rows)
        np.testing.assert_array_equal(scores, want_scores)


def test_sharded_embed_two_ranks_matches_one_process():
    import oracle
    path = synth.cached_gguf(MODEL_DIR, seed=7, vocab_size=512, num_layers=2)
    m = oracle.OracleModel(path)
    lengths = [5, 40, 1, 17, 33, 9, 26]
    ids, offs = synth.token_batch(51, lengths, 512)
    dims = [768, 128, 512, 768, 256, 768, 128]
    want = [m.forward_with_dim(ids[offs[i]:offs[i + 1]], dims[i]) for i in range(len(lengths))]
    m.close()
    res = _run(_embed_rank, 2, path)
    assert res[0][0] + res[1][0] == len(lengths)  # each sequence embedded once, on one rank
    assert res[0][0] > 0 and res[1][0] > 0
    for rank in (0, 1):
        got = res[rank][1]
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w)
