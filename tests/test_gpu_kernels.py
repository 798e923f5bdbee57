"""The product's device helpers against the CPU oracle, element by element,
and the bounded pipeline wait, through a test-only kernel library
(tests/kernels/test_kernels.cu, built by __graft_entry__.build()).

The forward tests check these helpers end to end (sequences under 128 tokens
are bit-exact); these check them on inputs a forward rarely reaches: the
fastExp clamps at +-10 and their neighbouring floats, GELU's sign branches,
subnormal and huge RMSNorm rows.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "libsemantica_testkernels.so")


@pytest.fixture(scope="module")
def tk(ctx):  # ctx: a CUDA device is present
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} missing: run __graft_entry__.build()")
    lib = C.CDLL(LIB)
    f32p = C.POINTER(C.c_float)
    lib.tk_fast_exp.argtypes = lib.tk_gelu_quick.argtypes = [f32p, f32p, C.c_int64]
    lib.tk_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_float]
    lib.tk_bounded_wait.argtypes = [C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
    return lib


def _p(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def edge_inputs(rng, n):
    x = np.concatenate([
        rng.uniform(-12, 12, n).astype(np.float32),
        rng.standard_normal(n // 4).astype(np.float32) * 3,
        np.array([0.0, -0.0, 10.0, -10.0, 1e-30, -1e-30, 87.0, -87.0, 1e30, -1e30], dtype=np.float32),
    ])
    around = np.array([10.0, -10.0, 1.0, -1.0, 0.5, -0.5], dtype=np.float32)
    near = np.concatenate([np.nextafter(around, np.float32(np.inf)), np.nextafter(around, np.float32(-np.inf))])
    return np.concatenate([x, near]).astype(np.float32)


def test_fast_exp_bit_exact(tk):
    # fastExp (activation.go:100-145) on 400k+ inputs incl. both clamps and
    # their neighbouring floats: the branch-free device form gives the
    # reference's bits everywhere
    x = edge_inputs(np.random.default_rng(5), 400_000)
    y = np.empty_like(x)
    assert tk.tk_fast_exp(_p(x), _p(y), x.size) == 0
    ref = np.array([oracle.fast_exp(float(v)) for v in x], dtype=np.float32)
    np.testing.assert_array_equal(y.view(np.uint32), ref.view(np.uint32))


def test_gelu_quick_bit_exact(tk):
    # GELUQuickSIMD (activation.go:47-95): both sign branches, one shared fastExp
    x = edge_inputs(np.random.default_rng(6), 400_000)
    y = np.empty_like(x)
    assert tk.tk_gelu_quick(_p(x), _p(y), x.size) == 0
    ref = oracle.gelu_quick(x)
    np.testing.assert_array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("n", [768, 256])
def test_rmsnorm_rows_bit_exact(tk, n):
    # RMSNorm (norm.go:8-36) with the 8-lane sum-of-squares order and the IEEE
    # float32 root and reciprocal: ordinary, tiny, huge and all-zero rows
    rng = np.random.default_rng(n)
    rows = 301
    x = rng.standard_normal((rows, n)).astype(np.float32)
    x[1] *= np.float32(1e-20)
    x[2] *= np.float32(1e15)
    x[3] = 0.0
    w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    y = np.empty_like(x)
    assert tk.tk_rmsnorm(_p(x), _p(w), _p(y), rows, n, 1e-6) == 0
    ref = oracle.rmsnorm(x, w, 1e-6)
    np.testing.assert_array_equal(y.view(np.uint32), ref.view(np.uint32))


def test_bounded_wait_gives_up_and_reports(tk):
    # A pipeline wait that nothing completes: after its limit (2 s) the waiting
    # thread sets the abort flag and its error bit and returns; the context
    # stays usable (the next kernels run normally).
    import time
    bits = C.c_uint32(0)
    ret = (C.c_uint32 * 2)()
    t0 = time.perf_counter()
    assert tk.tk_bounded_wait(C.byref(bits), ret) == 0
    dt = time.perf_counter() - t0
    assert ret[0] == 1, "the wait must give up, not complete"
    assert ret[1] == 1 and bits.value == 0x10
    assert 1.0 < dt < 30.0
    x = np.linspace(-3, 3, 1000, dtype=np.float32)
    y = np.empty_like(x)
    assert tk.tk_fast_exp(_p(x), _p(y), x.size) == 0
    assert np.isfinite(y).all()
