"""Model-faithful mode: EmbeddingGemma's sliding-window layers and dense 2/3
head, which the reference does not implement (it runs full attention in every
layer and has no head, model_int8.go:235-255, :500). Checked against the
oracle with the same settings: sequences under 128 tokens bit-exact, longer
ones within north_star's bound (cosine >= 0.9995; max-abs <= 2e-3, or twice
the spread between the reference's own three builds where that is wider, as
in test_gpu_forward).
"""
import numpy as np
import pytest

import synth
from conftest import MODEL_DIR, TEST_VOCAB, cosine


@pytest.fixture(scope="module")
def dense_path():
    return synth.cached_gguf(MODEL_DIR, seed=1234, vocab_size=TEST_VOCAB, dense_head=True)


def test_oracle_faithful_properties(dense_path, model_path):
    import oracle
    m = oracle.OracleModel(dense_path)
    plain = oracle.OracleModel(model_path)
    try:
        ids, offs = synth.token_batch(31, [40, 300], TEST_VOCAB)
        a = [plain.forward_with_dim(ids[offs[i]:offs[i + 1]], 768) for i in range(2)]
        # the extra tensors change nothing while the mode is off
        for i in range(2):
            np.testing.assert_array_equal(m.forward_with_dim(ids[offs[i]:offs[i + 1]], 768), a[i])
        # a 512-token window covers a 40-token sequence, not a 300-token one
        m.set_faithful(512, 6)
        np.testing.assert_array_equal(m.forward_with_dim(ids[:40], 768), a[0])
        assert not np.array_equal(m.forward_with_dim(ids[40:], 768), a[1])
        # the dense head: unit vectors at every Matryoshka tier, different from the pooled output
        m.set_faithful(512, 6, 0.0, True)
        for d in (768, 128):
            v = m.forward_with_dim(ids[:40], d)
            assert abs(float(np.linalg.norm(v.astype(np.float64))) - 1.0) < 1e-5
        assert cosine(m.forward_with_dim(ids[:40], 768), a[0]) < 0.99
        m.set_faithful()
        np.testing.assert_array_equal(m.forward_with_dim(ids[40:], 768), a[1])
        with pytest.raises(ValueError):
            plain.set_faithful(0, 0, 0.0, True)
    finally:
        m.close()
        plain.close()


def _spread(oracle_model, ids, dim):
    import oracle
    outs = []
    try:
        for path in (0, 1, 2):
            oracle.set_matmul_path(path)
            outs.append(oracle_model.forward_with_dim(ids, dim))
    finally:
        oracle.set_matmul_path(0)
    return outs[0], max(float(np.abs(outs[a] - outs[b]).max()) for a, b in ((0, 1), (0, 2), (1, 2)))


@pytest.mark.gpu
@pytest.mark.parametrize("window,pattern,rope_swa,dense", [(512, 6, 0.0, True), (64, 3, 5e5, True), (96, 2, 0.0, False)])
def test_faithful_forward_matches_oracle(ctx, dense_path, window, pattern, rope_swa, dense):
    import oracle
    import runtime
    gpu = runtime.load_model(dense_path, ctx)
    ref = oracle.OracleModel(dense_path)
    try:
        gpu.set_faithful(window, pattern, rope_swa, dense)
        ref.set_faithful(window, pattern, rope_swa, dense)
        lengths = [3, 40, 127, 128, 400]
        dims = [768, 256, 768, 512, 128]
        ids, offs = synth.token_batch(777 + window, lengths, TEST_VOCAB)
        got = gpu.forward_batch(ids, offs, dims)
        for i, n in enumerate(lengths):
            seq = ids[offs[i]:offs[i + 1]]
            if n < 128:  # the exact kernels: the oracle's bits, window masks included
                np.testing.assert_array_equal(got[i], ref.forward_with_dim(seq, dims[i]), err_msg=f"length {n}")
                continue
            want, spread = _spread(ref, seq, dims[i])
            c, a = cosine(got[i], want), float(np.abs(got[i] - want).max())
            print(f"window {window} len {n}: cosine {c:.7f} max abs {a:.2e} (builds differ by {spread:.2e})")
            assert c >= 0.9995 and a <= max(2e-3, 2 * spread)
        # back to the reference's forward
        gpu.set_faithful()
        plain = gpu.forward_batch(ids[:offs[2]], offs[:3], 768)
        ref.set_faithful()
        for i in range(2):
            np.testing.assert_array_equal(plain[i], ref.forward_with_dim(ids[offs[i]:offs[i + 1]], 768))
    finally:
        gpu.close()
        ref.close()


@pytest.mark.gpu
def test_faithful_errors(gpu_model):
    import _lib
    with pytest.raises(_lib.SemError, match="no dense_2.weight"):
        gpu_model.set_faithful(512, 6, 0.0, True)
    with pytest.raises(_lib.SemError, match="negative"):
        gpu_model.set_faithful(-1, 6)
    gpu_model.set_faithful()
