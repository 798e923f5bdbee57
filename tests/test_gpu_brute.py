"""search/brute on the GPU vs the CPU oracle, through the C ABI.

Integer contract: scores and top-k ids bit-exact (ties to the lower row).
Reference float contract: same arithmetic as the reference's AVX2 loops, so
top-k ids and distances are compared exactly too.
"""
import struct

import numpy as np
import pytest

import brute
import oracle
import synth

pytestmark = pytest.mark.gpu


def unit_rows(seed, n, dim):
    return oracle.normalize(synth.normal_vectors(seed, n, dim))


@pytest.mark.parametrize("quant", [1, 2])
@pytest.mark.parametrize("dim", [768, 256, 100, 3])
def test_exact_search_bit_exact(ctx, quant, dim):
    n, nq, k = 3000 if dim > 3 else 500, 37, 10
    vecs = unit_rows(1 + dim, n, dim)
    vecs[7] = vecs[3]  # duplicate rows: ties must go to the lower row
    idx = brute.Index.build(ctx, vecs, quantization=quant)
    conv = oracle.quantize_int8_vec if quant == 1 else oracle.quantize_int16_vec
    codes = conv(oracle.normalize(vecs))  # Build normalises again, as AddVector does (builder.go:65)
    queries = synth.normal_vectors(99 + dim, nq, dim)
    queries[0] = vecs[3] * 2.0
    ids, dist, scores = idx.search_batch(queries, k, brute.SEARCH_EXACT, normalize=True)
    qcodes = conv(oracle.normalize(queries))
    rrows, rscores, rdist = oracle.search_exact_batch(quant, codes, qcodes, k)
    np.testing.assert_array_equal(ids, rrows)
    np.testing.assert_array_equal(scores, rscores)
    np.testing.assert_array_equal(dist, rdist)
    assert ids[0, 0] == 3 and ids[0, 1] == 7


@pytest.mark.parametrize("quant", [0, 1, 2])
def test_reference_float_search_matches(ctx, quant):
    dim, n, nq, k = 64, 256, 20, 10
    vecs = unit_rows(456, n, dim)
    ids_in = np.arange(1000, 1000 + n, dtype=np.int32)
    idx = brute.Index.build(ctx, vecs, ids_in, quantization=quant)
    conv = {0: lambda v: v, 1: oracle.quantize_int8_vec, 2: oracle.quantize_int16_vec}[quant]
    data = conv(oracle.normalize(vecs))
    queries = unit_rows(457, nq, dim)
    gids, gdist, _ = idx.search_batch(queries, k, brute.SEARCH_REFERENCE, normalize=False)
    for i in range(nq):
        rid, rd = oracle.search_ref(quant, data, ids_in, queries[i], k)
        np.testing.assert_array_equal(gids[i], rid)
        np.testing.assert_array_equal(gdist[i], rd)


def test_search_vector_api_and_errors(ctx):
    # search/brute/index_test.go:10-64 (ids 10/11/12, query [1,0,0])
    b = brute.Builder(ctx, dimension=3, quantization=brute.QuantizeInt8)
    for i, v in {10: [1, 0, 0], 11: [0, 1, 0], 12: [0, 0, 1]}.items():
        b.add_vector(i, v)
    with pytest.raises(ValueError, match="duplicate id 10"):
        b.add_vector(10, [1, 1, 1])
    with pytest.raises(ValueError, match="vector dimension mismatch: got 2 want 3"):
        b.add_vector(13, [1, 1])
    idx = b.build()
    res = idx.search_vector([1, 0, 0], 2)
    assert res[0].ID == 10 and len(res) == 2
    assert idx.count() == 3 and idx.dimension() == 3
    res5 = idx.search_vector([1, 0, 0], 5)  # topK > count
    assert [r.ID for r in res5] == [10, 11, 12]
    import _lib
    with pytest.raises(_lib.SemError, match="^brute: topK must be positive$"):
        idx.search_vector([1, 0, 0], 0)
    with pytest.raises(_lib.SemError, match=r"^brute: query dimension mismatch: got 2 want 3$"):
        idx.search_vector([1, 0], 1)


@pytest.mark.parametrize("quant,dt", [(0, np.float32), (1, np.int8), (2, np.int16)])
def test_serializer_round_trip_byte_exact(ctx, quant, dt):
    dim, n = 5, 9
    vecs = unit_rows(77, n, dim)
    ids = np.array([5, 3, 99, 1, 0, 7, 8, 2, 4], dtype=np.int32)
    idx = brute.Index.build(ctx, vecs, ids, quantization=quant)
    blob = brute.Serializer.serialize(idx)
    conv = {0: lambda v: v, 1: oracle.quantize_int8_vec, 2: oracle.quantize_int16_vec}[quant]
    stored = conv(oracle.normalize(vecs)).astype(dt)
    want = b"BRUT" + struct.pack("<HHIB7x", 1, dim, n, quant) + ids.tobytes() + stored.tobytes()
    assert blob == want
    back = brute.Serializer.deserialize(blob, ctx)
    assert back.count() == n and back.dimension() == dim and back.quantization() == quant
    assert brute.Serializer.serialize(back) == blob
    v = back.vector(99)
    assert v is not None and v.shape == (dim,)
    assert back.vector(12345) is None
    import _lib
    with pytest.raises(_lib.SemError, match="invalid magic"):
        brute.Serializer.deserialize(b"XXXX" + blob[4:], ctx)
    with pytest.raises(_lib.SemError, match="unsupported version 2"):
        brute.Serializer.deserialize(blob[:4] + b"\x02\x00" + blob[6:], ctx)


def test_sharded_keys_merge_equals_full_search(ctx):
    import ctypes
    import torch
    import _lib
    dim, n, nq, k = 256, 5000, 24, 10
    vecs = unit_rows(5, n, dim)
    codes = oracle.quantize_int8_vec(vecs)
    bounds = [0, 1700, 3300, n]
    shards = [brute.Index.from_codes(ctx, codes[a:b]) for a, b in zip(bounds, bounds[1:])]
    q = oracle.quantize_int8_vec(unit_rows(6, nq, dim))
    qpad = np.zeros((nq, 256), dtype=np.int8)
    qpad[:, :dim] = q
    d_q = torch.from_numpy(qpad).cuda()
    keys = torch.zeros((3, nq, k), dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    for s, (idx, base) in enumerate(zip(shards, bounds)):
        _lib.check(_lib.load().sem_index_search_keys(idx.handle, ctypes.c_void_p(d_q.data_ptr()), nq, k, 1, base,
                                                     ctypes.c_void_p(keys[s].data_ptr()), None))
    rows = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    st = ctypes.c_void_p(ctx.stream)
    _lib.check(_lib.load().sem_topk_merge(ctx.handle, ctypes.c_void_p(keys.data_ptr()), 3, nq, k, k, 1, 1,
                                          ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(scores.data_ptr()),
                                          None, st))
    torch.cuda.synchronize()
    rrows, rscores, _ = oracle.search_exact_batch(1, codes, q, k)
    np.testing.assert_array_equal(rows.cpu().numpy(), rrows)
    np.testing.assert_array_equal(scores.cpu().numpy(), rscores)


def test_tensor_core_scan_many_parts_and_ties(ctx):
    # int8 rows with D >= 128 take the tensor-core scan: enough rows and queries
    # for several corpus parts of several 256-row tiles and three 128-query
    # tiles; duplicated rows (ties) sit in different parts and tile halves
    dim, n, nq, k = 768, 70000, 300, 16
    codes = oracle.quantize_int8_vec(unit_rows(31, n, dim))
    for a, b in ((5, 60001), (130, 131), (1000, 40000)):
        codes[b] = codes[a]
    q = oracle.quantize_int8_vec(unit_rows(32, nq, dim))
    q[0] = codes[5]
    q[1] = codes[130]
    idx = brute.Index.from_codes(ctx, codes)
    import ctypes
    import torch
    import _lib
    d_q = torch.from_numpy(q).cuda()
    keys = torch.zeros((nq, k), dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    _lib.check(_lib.load().sem_index_search_keys(idx.handle, ctypes.c_void_p(d_q.data_ptr()), nq, k, 1, 0,
                                                 ctypes.c_void_p(keys.data_ptr()), None))
    rows = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    _lib.check(_lib.load().sem_topk_merge(ctx.handle, ctypes.c_void_p(keys.data_ptr()), 1, nq, k, k, 1, 1,
                                          ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(scores.data_ptr()),
                                          None, ctypes.c_void_p(ctx.stream)))
    torch.cuda.synchronize()
    rrows, rscores, _ = oracle.search_exact_batch(1, codes, q, k, nthreads=8)
    np.testing.assert_array_equal(scores.cpu().numpy(), rscores)
    np.testing.assert_array_equal(rows.cpu().numpy(), rrows)
    assert rrows[0, 0] == 5 and rrows[0, 1] == 60001
    assert rrows[1, 0] == 130 and rrows[1, 1] == 131
    idx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("n,nq,k,distinct", [(200_000, 40, 10, 64), (150_000, 1, 1, 0), (150_000, 129, 3, 16),
                                             (90_000, 260, 16, 5)])
def test_tensor_core_scan_shared_bounds_with_ties(ctx, n, nq, k, distinct):
    # The scan publishes each query's k-th best score across tile halves and
    # corpus parts and skips rows below it. Rows drawn from a few distinct
    # vectors make nearly every score tie with the published bounds: the
    # result must still be the lowest rows among equal scores, as the oracle's
    # (score desc, row asc) order gives.
    dim = 768
    if distinct:
        base = oracle.quantize_int8_vec(unit_rows(41, distinct, dim))
        codes = base[np.random.default_rng(42).integers(0, distinct, n)]
    else:
        codes = oracle.quantize_int8_vec(unit_rows(43, n, dim))
    q = oracle.quantize_int8_vec(unit_rows(44, nq, dim))
    idx = brute.Index.from_codes(ctx, codes)
    import ctypes
    import torch
    import _lib
    d_q = torch.from_numpy(q).cuda()
    keys = torch.zeros((nq, k), dtype=torch.int64, device="cuda")
    rows = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    lib = _lib.load()
    for _ in range(2):  # the per-query bounds are reset for every search
        _lib.check(lib.sem_index_search_keys(idx.handle, ctypes.c_void_p(d_q.data_ptr()), nq, k, 1, 0,
                                             ctypes.c_void_p(keys.data_ptr()), None))
        _lib.check(lib.sem_topk_merge(ctx.handle, ctypes.c_void_p(keys.data_ptr()), 1, nq, k, k, 1, 1,
                                      ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(scores.data_ptr()),
                                      None, ctypes.c_void_p(ctx.stream)))
        torch.cuda.synchronize()
        rrows, rscores, _ = oracle.search_exact_batch(1, codes, q, k, nthreads=8)
        np.testing.assert_array_equal(scores.cpu().numpy(), rscores)
        np.testing.assert_array_equal(rows.cpu().numpy(), rrows)
    idx.close()


@pytest.mark.parametrize("row_base", [0, 2500])
def test_sharded_index_single_rank(ctx, row_base):
    # sharded.ShardedIndex without a process group: one shard whose rows are
    # numbered from row_base, searched through keys + sem_topk_merge on the
    # library's stream, against the oracle's scan of the same rows
    import torch
    import sharded
    dim, n, nq, k = 256, 2500, 29, 10
    codes = oracle.quantize_int8_vec(unit_rows(61, n, dim))
    qc = oracle.quantize_int8_vec(unit_rows(62, nq, dim))
    si = sharded.ShardedIndex(ctx, codes, row_base=row_base)
    try:
        rows, scores = si.search_codes(torch.from_numpy(qc).cuda(), k)
        torch.cuda.synchronize()
        want_rows, want_scores, _ = oracle.search_exact_batch(1, codes, qc, k)
        np.testing.assert_array_equal(rows.cpu().numpy(), want_rows + row_base)
        np.testing.assert_array_equal(scores.cpu().numpy(), want_scores)
    finally:
        si.close()


@pytest.mark.parametrize("dim", [768, 256, 200, 128])
def test_tensor_core_int16_scan(ctx, dim):
    # int16 rows with D in [113, 768] take the tensor-core scan on byte planes
    # (high byte signed, low byte unsigned, four kind::i8 products recombined
    # exactly in int32): several corpus parts of 64-row tiles, three 128-query
    # tiles, a partial last K box (D = 200), duplicated rows in different
    # parts, and sign-extreme codes (+-32767: high byte -128 or 127)
    n, nq, k = 70000, 300, 16
    codes = oracle.quantize_int16_vec(unit_rows(51 + dim, n, dim))
    for a, b in ((5, 60001), (130, 131), (1000, 40000)):
        codes[b] = codes[a]
    e0 = np.zeros(dim, dtype=np.float32)
    e0[0] = 1.0
    codes[77] = oracle.quantize_int16_vec(e0[None])[0]       # [32767, 0, ...]
    codes[78] = oracle.quantize_int16_vec(-e0[None])[0]      # [-32767, 0, ...]
    q = oracle.quantize_int16_vec(unit_rows(52 + dim, nq, dim))
    q[0] = codes[5]
    q[1] = codes[130]
    q[2] = codes[77]
    q[3] = codes[78]
    idx = brute.Index.from_codes(ctx, codes)
    import ctypes
    import torch
    import _lib
    lib = _lib.load()
    d_q = torch.from_numpy(q).cuda()
    keys = torch.zeros((nq, k), dtype=torch.int64, device="cuda")
    rows = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    rrows, rscores, _ = oracle.search_exact_batch(2, codes, q, k, nthreads=8)
    for _ in range(2):  # the second search reuses the byte planes built by the first
        _lib.check(lib.sem_index_search_keys(idx.handle, ctypes.c_void_p(d_q.data_ptr()), nq, k, 1, 0,
                                             ctypes.c_void_p(keys.data_ptr()), None))
        _lib.check(lib.sem_topk_merge(ctx.handle, ctypes.c_void_p(keys.data_ptr()), 1, nq, k, k, 1, 2,
                                      ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(scores.data_ptr()),
                                      None, ctypes.c_void_p(ctx.stream)))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(scores.cpu().numpy(), rscores)
        np.testing.assert_array_equal(rows.cpu().numpy(), rrows)
    assert rrows[0, 0] == 5 and rrows[0, 1] == 60001
    assert rrows[2, 0] == 77 and rscores[2, 0] == 32767 * 32767
    assert rrows[3, 0] == 78 and rscores[3, 0] == 32767 * 32767
    idx.close()
