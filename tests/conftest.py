import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "go-semantica_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_DIR = os.environ.get("SEM_TEST_MODEL_DIR", "/tmp/semantica_b200_models")
TEST_VOCAB = 4096


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libsemantica_b200.so")
    config.addinivalue_line("markers", "slow: long-running full-size check")


def gpu_available() -> bool:
    try:
        import _lib
        return _lib.device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_path():
    """Synthetic EmbeddingGemma-shaped GGUF (24 layers, 4096-token vocabulary)."""
    import synth
    return synth.cached_gguf(MODEL_DIR, seed=1234, vocab_size=TEST_VOCAB)


@pytest.fixture(scope="session")
def oracle_model(model_path):
    import oracle
    m = oracle.OracleModel(model_path)
    yield m
    m.close()


@pytest.fixture(scope="session")
def ctx():
    if not gpu_available():
        pytest.fail("GPU test without a CUDA device or without libsemantica_b200.so")
    import _lib
    c = _lib.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def gpu_model(ctx, model_path):
    import runtime
    m = runtime.load_model(model_path, ctx)
    yield m
    m.close()


def cosine(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
