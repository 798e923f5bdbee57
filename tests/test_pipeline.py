"""The request pipeline (sem_embed_submit / sem_embed_wait), the graph cache
of recent batch shapes, and ggufembed.Runtime's batched and streaming
EmbedInputs over a device model.

Every result is compared with sem_embed on the same request: the same kernels
on the same shape, so the vectors are bit-identical whether a request ran
directly, through a replayed graph or through a pipeline slot."""
import numpy as np
import pytest

import synth
from conftest import TEST_VOCAB

pytestmark = pytest.mark.gpu


def _req(seed, lens, dims=None):
    ids, offs = synth.token_batch(seed, lens, TEST_VOCAB)
    return ids, offs, dims if dims is not None else [768] * len(lens)


def _same(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_submit_wait_matches_sem_embed(gpu_model):
    reqs = [_req(201, [64] * 8), _req(202, [512, 300, 40], [768, 256, 128]), _req(203, [5, 127, 1, 90]),
            _req(204, [64] * 8)]
    want = [gpu_model.forward_batch(*r) for r in reqs]
    # two in flight, waited out of submission order once
    t0 = gpu_model.submit(*reqs[0])
    t1 = gpu_model.submit(*reqs[1])
    _same(gpu_model.wait(t1), want[1])
    _same(gpu_model.wait(t0), want[0])
    t2 = gpu_model.submit(*reqs[2])
    t3 = gpu_model.submit(*reqs[3])
    _same(gpu_model.wait(t2), want[2])
    _same(gpu_model.wait(t3), want[3])
    # an empty request completes with nothing
    assert gpu_model.wait(gpu_model.submit(np.zeros(0, np.int32), np.array([0], np.int32))) == []


def test_pipeline_limits_and_errors(gpu_model):
    import _lib
    r = _req(205, [64] * 4)
    t0 = gpu_model.submit(*r)
    t1 = gpu_model.submit(*r)
    with pytest.raises(_lib.SemError, match="two requests in flight"):
        gpu_model.submit(*r)
    a = gpu_model.wait(t0)
    with pytest.raises(_lib.SemError, match="no request in flight"):
        gpu_model.wait(t0)  # each ticket once
    _same(gpu_model.wait(t1), a)
    with pytest.raises(_lib.SemError, match="token ID out of range: 4096"):
        gpu_model.submit(np.array([1, TEST_VOCAB], np.int32), np.array([0, 2], np.int32))
    with pytest.raises(_lib.SemError, match="sequence too long"):
        gpu_model.submit(np.ones(2049, np.int32), np.array([0, 2049], np.int32))
    with pytest.raises(_lib.SemError, match="offsets\\[0\\] must be 0"):
        gpu_model.submit(np.ones(4, np.int32), np.array([1, 3], np.int32))
    # rejected submits take no slot
    _same(gpu_model.wait(gpu_model.submit(*r)), a)


def test_graph_cache_alternating_shapes(gpu_model):
    # shapes that alternate replay their own graphs (metadata re-uploaded for
    # each); every replay equals the first, directly launched, forward
    reqs = [_req(206, [64] * 8), _req(207, [30, 100, 64]), _req(208, [16] * 32), _req(209, [200, 64])]
    first = [gpu_model.forward_batch(*r) for r in reqs]
    for _ in range(3):
        for r, f in zip(reqs, first):
            _same(gpu_model.forward_batch(*r), f)


def test_runtime_embed_inputs_and_stream(gpu_model):
    import ggufembed as ge

    def encode(text):  # a stand-in tokenizer: BOS then one id per byte
        return [2] + [5 + (b * 7919) % (TEST_VOCAB - 10) for b in text.encode()]

    rt = ge.Runtime(gpu_model, encode)
    batches = [[ge.EmbedInput(Task=ge.TaskSearchQuery, Content=f"query number {i} about B200s", Dim=d)
                for i, d in enumerate((768, 512, 256))],
               [],
               [ge.EmbedInput(Task=ge.TaskSearchDocument, Title="t", Content="a document " * 40, Dim=128)],
               [ge.EmbedInput(Task=ge.TaskClustering, Content=f"text {i}", Dim=768) for i in range(9)]]
    want = [rt.embed_inputs(b) for b in batches]
    got = list(rt.embed_inputs_stream(iter(batches)))
    assert len(got) == len(want)
    for g, w in zip(got, want):
        _same(g, w)
    assert [v.shape[0] for v in want[0]] == [768, 512, 256]
    # a stream abandoned part-way frees its slots
    s = rt.embed_inputs_stream(iter(batches))
    next(s)
    s.close()
    t0 = gpu_model.submit(*_req(210, [8]))
    t1 = gpu_model.submit(*_req(211, [8]))
    gpu_model.wait(t0)
    gpu_model.wait(t1)
