"""Device groups (sem_group_*): the model on several GPUs of one host, each
request split across them by token count inside the library.

On one GPU the group is a single replica; on a box with two or more GPUs it
spans two and every device takes part in a request. Sequences shorter than 128
tokens run the exact path, so their vectors are bit-identical to a
single-device forward whichever device embeds them; longer ones are held to
the forward's parity bound against the oracle (cosine >= 0.9995; max-abs
<= 2e-3, or twice the spread between the reference's own builds where that
is wider, as for a single device)."""
import numpy as np
import pytest

import synth
from conftest import TEST_VOCAB


def test_group_argument_errors_without_device():
    import _lib
    import runtime
    with pytest.raises(_lib.SemError, match="empty device list"):
        runtime.load_group("unused.gguf", [])
    with pytest.raises(_lib.SemError, match="device 0 listed twice"):
        runtime.load_group("unused.gguf", [0, 1, 0])


def _devices():
    import _lib
    n = _lib.device_count()
    return list(range(min(n, 2)))


@pytest.fixture(scope="module")
def group(model_path):
    import runtime
    g = runtime.load_group(model_path, _devices())
    yield g
    g.close()


@pytest.mark.gpu
def test_group_matches_single_device(group, gpu_model, oracle_model):
    lens = [3, 40, 127, 9, 64, 100, 1, 77, 5, 120, 33, 18]
    ids, offs = synth.token_batch(71, lens, TEST_VOCAB)
    dims = [768, 512, 256, 128, 768, 64, 768, 300, 768, 1, 768, 128]
    got = group.forward_batch(ids, offs, dims)
    one = gpu_model.forward_batch(ids, offs, dims)
    assert group.size == len(_devices())
    for i in range(len(lens)):
        assert got[i].shape == (dims[i],)
        assert np.array_equal(got[i], one[i]), i
    want = oracle_model.forward_with_dim(ids[offs[6]:offs[7]], dims[6])
    assert np.array_equal(got[6], want)


@pytest.mark.gpu
def test_group_long_sequences_within_parity(group, oracle_model):
    from test_gpu_forward import check_parity
    ids, offs = synth.token_batch(72, [512, 300, 129, 700, 64, 256], TEST_VOCAB)
    check_parity(group, oracle_model, ids, offs, [768] * 6, "group")


@pytest.mark.gpu
def test_group_errors_and_empty_request(group):
    import _lib
    with pytest.raises(_lib.SemError, match="token ID out of range: 4096"):
        group.forward_batch(np.array([1, 2, TEST_VOCAB], np.int32), np.array([0, 1, 3], np.int32))
    with pytest.raises(_lib.SemError, match="target dimension 769 out of range"):
        group.forward_batch(np.array([1, 2], np.int32), np.array([0, 2], np.int32), [769])
    with pytest.raises(_lib.SemError, match="empty input"):
        group.forward_batch(np.array([1], np.int32), np.array([0, 1, 1], np.int32))
    assert group.forward_batch(np.zeros(0, np.int32), np.array([0], np.int32)) == []
    # the group still works after rejected requests
    ids, _ = synth.token_batch(3, [5], TEST_VOCAB)
    v = group.forward_with_dim(ids, 768)
    assert abs(float(np.linalg.norm(v)) - 1.0) < 1e-5


@pytest.mark.gpu
def test_group_faithful_mode(group, gpu_model):
    # sem_group_set_faithful sets every replica or none: a setting the model
    # rejects leaves the group's vectors as they were; a sliding window gives
    # the single device's vectors (short sequences: bit-identical), and the
    # default setting restores the first ones exactly
    import _lib
    ids, offs = synth.token_batch(73, [100, 40, 127], TEST_VOCAB)
    base = group.forward_batch(ids, offs)
    with pytest.raises(_lib.SemError, match=r"^device \d+: faithful mode: the model has no dense_2"):
        group.set_faithful(0, 0, 0.0, True)
    assert all(np.array_equal(a, b) for a, b in zip(group.forward_batch(ids, offs), base))
    try:
        group.set_faithful(64, 2)
        gpu_model.set_faithful(64, 2)
        got = group.forward_batch(ids, offs)
        one = gpu_model.forward_batch(ids, offs)
        assert all(np.array_equal(a, b) for a, b in zip(got, one))
        assert not np.array_equal(got[0], base[0])  # 100 tokens reach past the 32-position half window
    finally:
        group.set_faithful()
        gpu_model.set_faithful()
    assert all(np.array_equal(a, b) for a, b in zip(group.forward_batch(ids, offs), base))
