"""Host-side logic that needs no GPU: prompt templates, dimension rules, the
C-ABI exports, and the synthetic GGUF layout."""
import ctypes
import os
import re

import numpy as np
import pytest

import ggufembed as ge
from conftest import ROOT

CONTENT = "neural networks are powerful"


@pytest.mark.parametrize("inp,want", [
    # pkg/ggufembed/api_test.go:12-105
    (ge.EmbedInput(Task=ge.TaskNone, Content=CONTENT), CONTENT),
    (ge.EmbedInput(Task=ge.TaskSearchQuery, Content=CONTENT), "task: search result | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskQuestionAnswering, Content=CONTENT), "task: question answering | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskFactVerification, Content=CONTENT), "task: fact checking | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskClassification, Content=CONTENT), "task: classification | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskClustering, Content=CONTENT), "task: clustering | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskSemanticSimilarity, Content=CONTENT), "task: sentence similarity | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskCodeRetrieval, Content=CONTENT), "task: code retrieval | query: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskSearchDocument, Title="Doc", Content=CONTENT), "title: Doc | text: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskSearchDocument, Content=CONTENT), "title: none | text: " + CONTENT),
    (ge.EmbedInput(Task=ge.TaskSemanticSimilarity, Content=CONTENT, CustomTaskDescription="custom"),
     "task: custom | query: " + CONTENT),
])
def test_build_prompt_matches_model_card(inp, want):
    assert ge.build_prompt(inp) == want


def test_build_prompt_errors():
    with pytest.raises(ValueError, match="content must not be empty"):
        ge.build_prompt(ge.EmbedInput(Task=ge.TaskSearchQuery))
    with pytest.raises(ValueError, match="unsupported task"):
        ge.build_prompt(ge.EmbedInput(Task=42, Content=CONTENT))


def test_resolve_dim():
    # tasks.go:101-116
    assert ge.resolve_dim(0) == 512
    for d in (768, 512, 256, 128):
        assert ge.resolve_dim(d) == d
    with pytest.raises(ValueError, match=r"unsupported embed dim 300 \(allowed: 768, 512, 256, 128\)"):
        ge.resolve_dim(300)
    assert ge.supported_dims() == [768, 512, 256, 128]


def header_symbols():
    text = open(os.path.join(ROOT, "include", "semantica_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sem_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)  # loads without a GPU
    syms = header_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.exported_symbols())


def test_no_gpu_calls_fail_cleanly_without_device():
    import _lib
    if _lib.device_count() > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(_lib.SemError):
        _lib.Context(0)


def test_synthetic_gguf_parses_in_oracle(model_path):
    import oracle
    m = oracle.OracleModel(model_path)
    c = m.config
    assert (c.embed_dim, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim, c.interm_dim) == (768, 24, 3, 1, 256, 1152)
    assert c.vocab_size == 4096 and c.max_seq_len == 2048
    assert abs(c.attention_scale - 1 / 16) < 1e-9
    m.close()


def test_token_batch_layout():
    import synth
    ids, offs = synth.token_batch(5, [3, 1, 4], 100)
    assert offs.tolist() == [0, 3, 4, 8]
    assert ids[0] == ids[3] == ids[4] == synth.BOS_ID
    assert (ids[[1, 2, 5, 6, 7]] >= synth.FIRST_NON_SPECIAL).all()


@pytest.mark.parametrize("quant", [1, 2])
def test_quantize_queries_matches_oracle(quant):
    # sem_quantize_queries runs on the host (no device): quantizeInt8 /
    # quantizeInt16 (quant.go:17-41) of normalised queries, clamped to
    # [-1, 1], rounded half away from zero
    import brute
    import oracle
    rng = np.random.default_rng(3)
    q = rng.uniform(-1.25, 1.25, (64, 96)).astype(np.float32)
    scale = 127.0 if quant == 1 else 32767.0
    halves = ((np.arange(-40, 40) + 0.5) / scale).astype(np.float32)  # near-ties of v * scale
    q[1, :80] = halves
    q[2, :80] = np.nextafter(halves, np.float32(2))
    q[0, :6] = [1.0, -1.0, 0.0, -0.0, 1.5, -1.5]
    conv = oracle.quantize_int8_vec if quant == 1 else oracle.quantize_int16_vec
    np.testing.assert_array_equal(brute.quantize_queries(q, quant), conv(q))


class _FakePipelineModel:
    """Host-side stand-in for runtime.Model's submit/wait (no GPU): records
    the order of calls and enforces the two-slot limit."""

    def __init__(self):
        import runtime
        self.log, self.inflight, self.next = [], set(), 1
        self.embed_stream = runtime.Model.embed_stream.__get__(self)

    def submit(self, ids, offsets, dims):
        if len(self.inflight) == 2:
            raise RuntimeError("two requests in flight")
        t = self.next
        self.next += 1
        self.inflight.add(t)
        self.log.append(("submit", t))
        return (t, len(offsets) - 1)

    def wait(self, ticket):
        t, n = ticket
        self.inflight.remove(t)
        self.log.append(("wait", t))
        return [np.full(1, t, np.float32)] * n


def test_embed_stream_overlaps_next_submit_with_current_request():
    m = _FakePipelineModel()
    reqs = [(np.ones(3, np.int32), np.array([0, 3], np.int32), [768]) for _ in range(4)]
    out = list(m.embed_stream(iter(reqs)))
    assert [o[0][0] for o in out] == [1, 2, 3, 4]
    # request i + 1 is submitted before request i is waited for
    assert m.log == [("submit", 1), ("submit", 2), ("wait", 1), ("submit", 3), ("wait", 2), ("submit", 4),
                     ("wait", 3), ("wait", 4)]
    assert not m.inflight


def test_embed_stream_frees_slots_when_abandoned_or_failing():
    m = _FakePipelineModel()
    reqs = [(np.ones(3, np.int32), np.array([0, 3], np.int32), [768]) for _ in range(5)]
    s = m.embed_stream(iter(reqs))
    next(s)
    s.close()
    assert not m.inflight

    def failing():
        yield reqs[0]
        raise ValueError("tokenizer failed")

    with pytest.raises(ValueError, match="tokenizer failed"):
        list(m.embed_stream(failing()))
    assert not m.inflight
