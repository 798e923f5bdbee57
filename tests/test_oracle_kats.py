"""The CPU oracle against the known-answer tests of the reference's own suite.

The reference's Go tests draw from math/rand streams that cannot be replayed
without Go, so each test below keeps the reference's shapes and tolerances
with seeded numpy draws instead (cited per test).
"""
import math
import struct

import numpy as np
import pytest

import oracle


def f16_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float16).view(np.uint16)[0])


class TestFloat16Decoders:
    def test_normal_values_match_ieee(self):
        # internal/runtime/model_int8_test.go:67-130 (scales 0.01, 1, 10, -0.5 within 1e-3)
        for x in (0.01, 1.0, 10.0, -0.5, 65504.0, -2.0 ** -14, 0.000123):
            b = f16_bits(x)
            exact = float(np.array([b], dtype=np.uint16).view(np.float16)[0])
            assert oracle.f16_runtime(b) == exact
            assert oracle.f16_gguf(b) == exact
            assert abs(oracle.f16_runtime(b) - x) <= max(1e-3, abs(x) * 1e-3)

    def test_zero_inf_nan(self):
        assert oracle.f16_runtime(0x0000) == 0.0
        assert math.copysign(1.0, oracle.f16_runtime(0x8000)) == -1.0
        assert oracle.f16_runtime(0x7C00) == math.inf
        assert oracle.f16_gguf(0xFC00) == -math.inf
        assert math.isnan(oracle.f16_runtime(0x7E00))

    def test_subnormals(self):
        # runtime decoder (model_int8.go:571-597) is exact; the gguf decoder
        # (gguf/tensor.go:207-240) returns half the value for subnormals.
        for b in (0x0001, 0x0002, 0x03FF, 0x8155):
            exact = float(np.array([b], dtype=np.uint16).view(np.float16)[0])
            assert oracle.f16_runtime(b) == exact
            assert oracle.f16_gguf(b) == exact / 2


class TestSoftmax:
    def test_basic_properties(self):
        # internal/kernels/kernels_test.go:66-87
        out = oracle.softmax(np.array([1, 2, 3, 4], dtype=np.float32))
        assert abs(out.sum() - 1) < 1e-5
        assert all(out[i] < out[i + 1] for i in range(3))

    def test_approximation_accuracy(self):
        # internal/kernels/kernels_test.go:89-189: abs <= 6e-4, rel <= 3e-3 (ref > 5e-5), sum within 1e-4
        rng = np.random.default_rng(1234)
        max_abs = max_rel = 0.0
        for n in (1, 2, 3, 4, 8, 16, 32, 64, 128):
            for trial in range(256):
                scale = (1.0, 10.0, 40.0)[trial % 3]
                src = ((rng.random(n) * 2 - 1) * scale).astype(np.float32)
                approx = oracle.softmax(src)
                e = np.exp((src - src.max()).astype(np.float64))
                ref = (e / e.sum()).astype(np.float32)
                d = np.abs(approx.astype(np.float64) - ref)
                max_abs = max(max_abs, d.max())
                mask = np.abs(ref) > 5e-5
                if mask.any():
                    max_rel = max(max_rel, (d[mask] / np.abs(ref[mask])).max())
                assert abs(float(approx.astype(np.float32).sum()) - 1) <= 1e-4
        assert max_abs <= 6e-4
        assert max_rel <= 3e-3


class TestGeluQuick:
    CASES = [
        [0, 0, 0, 0, 0, 0, 0, 0],
        [0.1, 0.5, 1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
        [-0.1, -0.5, -1.0, -2.0, -3.0, -4.0, -5.0, -6.0],
        [-3.0, -2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0],
        [5.0, 6.0, 7.0, 8.0, 9.0, 10.0, 11.0, 12.0],
        [-5.0, -6.0, -7.0, -8.0, -9.0, -10.0, -11.0, -12.0],
        [0.001, 0.01, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6],
        [1.0, 2.0, 3.0, 4.0, 5.0],
    ]

    @pytest.mark.parametrize("vals", CASES)
    def test_simd_matches_scalar(self, vals):
        # internal/kernels/kernels_test.go:304-363: max error < 0.01, RMSE < 0.005 vs x*sigmoid(1.702x)
        x = np.array(vals, dtype=np.float32)
        got = oracle.gelu_quick(x).astype(np.float64)
        exact = x * (1.0 / (1.0 + np.exp(-1.702 * x.astype(np.float64))))
        err = np.abs(got - exact)
        assert err.max() < 0.01
        assert math.sqrt((err ** 2).mean()) < 0.005

    def test_properties(self):
        # kernels_test.go:365-447
        assert abs(oracle.gelu_quick(np.array([0.0]))[0]) < 1e-5
        for x in (5.0, 10.0):
            r = oracle.gelu_quick(np.array([x]))[0] / x
            assert 0.95 <= r <= 1.0
        for x in (-5.0, -10.0):
            assert abs(oracle.gelu_quick(np.array([x]))[0]) <= 0.01
        y = oracle.gelu_quick(np.array([0.0, 0.5, 1.0, 2.0, 3.0, 4.0, 5.0]))
        assert all(y[i] < y[i + 1] for i in range(len(y) - 1))


class TestFastExp:
    def test_clamps(self):
        # activation.go:104-109
        assert oracle.fast_exp(-10.5) == 0.0
        assert oracle.fast_exp(10.5) == np.float32(22026.4657948)
        assert abs(oracle.fast_exp(0.0) - 1.0) < 1e-6

    def test_accuracy(self):
        # activation.go:97-99 documents "accurate to ~0.5%"
        xs = np.linspace(-10, 10, 2001, dtype=np.float32)
        got = np.array([oracle.fast_exp(float(x)) for x in xs])
        rel = np.abs(got - np.exp(xs.astype(np.float64))) / np.exp(xs.astype(np.float64))
        assert rel.max() < 5e-3


class TestNormAndQuant:
    def test_rmsnorm(self):
        # internal/kernels/kernels_test.go:47-64
        x = np.array([1, 2, 3, 4], dtype=np.float32)
        out = oracle.rmsnorm(x, np.ones(4, dtype=np.float32), 1e-6)
        rms = math.sqrt((1 + 4 + 9 + 16) / 4 + 1e-6)
        np.testing.assert_allclose(out, x / rms, rtol=1e-6)

    def test_quantize_round_half_away(self):
        # quantize.go:92-103: absmax 127 -> inv 1, x.5 rounds away from zero
        x = np.array([127.0, 0.5, -0.5, 1.5, -2.5, 126.49], dtype=np.float32)
        codes, scale = oracle.quantize_sym_int8(x)
        assert scale == 1.0
        assert codes.tolist() == [127, 1, -1, 2, -3, 126]

    def test_quantize_zero_buffer(self):
        codes, scale = oracle.quantize_sym_int8(np.zeros(16, dtype=np.float32))
        assert scale == 1.0 and not codes.any()

    def test_matmul_block_math(self):
        # matmul_inner_loop_fallback.go:16-39: sum_b float(int dot) * d_b, then * input scale
        rng = np.random.default_rng(7)
        K, N, M = 96, 8, 3
        qs = rng.integers(-127, 128, size=(N, K // 32, 32)).astype(np.int8)
        d = (rng.random((N, K // 32)) * 0.01).astype(np.float16)
        raw = np.zeros((N, K // 32, 34), dtype=np.uint8)
        raw[:, :, :2] = d.view(np.uint8).reshape(N, K // 32, 2)
        raw[:, :, 2:] = qs.view(np.uint8)
        a = rng.integers(-127, 128, size=(M, K)).astype(np.int8)
        got = oracle.matmul_q8_0_int8(raw, a, 0.5, N)
        bs = np.einsum("mbk,nbk->mnb", a.reshape(M, K // 32, 32).astype(np.int64), qs.astype(np.int64))
        exp = (bs * d.astype(np.float64)[None]).sum(-1) * 0.5
        np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-6)

    def test_avx2_and_vnni_inner_loops_agree_closely(self):
        rng = np.random.default_rng(3)
        K, N = 768, 16
        raw = np.zeros((N, K // 32, 34), dtype=np.uint8)
        raw[:, :, :2] = (rng.random((N, K // 32)) * 0.01).astype(np.float16).view(np.uint8).reshape(N, K // 32, 2)
        raw[:, :, 2:] = rng.integers(-127, 128, size=(N, K // 32, 32)).astype(np.int8).view(np.uint8)
        a = rng.integers(-127, 128, size=(4, K)).astype(np.int8)
        v = oracle.matmul_q8_0_int8(raw, a, 1.0, N)
        oracle.set_matmul_path(1)
        try:
            w = oracle.matmul_q8_0_int8(raw, a, 1.0, N)
        finally:
            oracle.set_matmul_path(0)
        np.testing.assert_allclose(v, w, rtol=1e-4, atol=1e-5)


def _unit(rng, n, dim):
    v = rng.standard_normal((n, dim)).astype(np.float32)
    return oracle.normalize(v)


class TestBruteOracle:
    def test_dot_int8_matches_float32(self):
        # search/brute/index_test.go:105-128: |int8 - f32| <= 0.02 (dim 128, 100 samples)
        rng = np.random.default_rng(123)
        for _ in range(100):
            vec, q = _unit(rng, 1, 128)[0], _unit(rng, 1, 128)[0]
            got = oracle.dot_int8_ref(oracle.quantize_int8_vec(vec), q)
            assert abs(got - oracle.dot_f32_ref(vec, q)) <= 0.02

    def test_dot_int16_matches_float32(self):
        # index_test.go:130-153: <= 0.01
        rng = np.random.default_rng(321)
        for _ in range(100):
            vec, q = _unit(rng, 1, 128)[0], _unit(rng, 1, 128)[0]
            got = oracle.dot_int16_ref(oracle.quantize_int16_vec(vec), q)
            assert abs(got - oracle.dot_f32_ref(vec, q)) <= 0.01

    def test_dot_float32_matches_scalar(self):
        # index_test.go:155-180: <= 1e-5 (dim 256)
        rng = np.random.default_rng(654)
        for _ in range(50):
            vec, q = _unit(rng, 1, 256)[0], _unit(rng, 1, 256)[0]
            want = np.float32(0)
            for a, b in zip(vec, q):
                want = np.float32(want + np.float32(a * b))
            assert abs(oracle.dot_f32_ref(vec, q) - float(want)) <= 1e-5

    def test_search_normalized_matches_float32(self):
        # index_test.go:182-251: top-1 id equal, |dist diff| <= 0.05 (dim 64, 256 rows, 20 queries)
        rng = np.random.default_rng(456)
        data = _unit(rng, 256, 64)
        ids = np.arange(256, dtype=np.int32)
        qs = _unit(rng, 20, 64)
        mismatches = 0
        for q in qs:
            fid, fd = oracle.search_ref(0, data, ids, q, 10)
            for quant, conv, dot_tol in ((1, oracle.quantize_int8_vec, 0.02), (2, oracle.quantize_int16_vec, 0.01)):
                qid, qd = oracle.search_ref(quant, conv(data), ids, q, 10)
                assert abs(fd[0] - qd[0]) <= 0.05
                if fid[0] != qid[0]:
                    # a near-tie under quantisation error: the float scores of the two
                    # winners may differ by at most twice the per-dot error bound
                    mismatches += 1
                    gap = fd[0] - oracle.dot_f32_ref(data[qid[0]], q)
                    assert gap <= 2 * dot_tol
        assert mismatches <= 2

    def test_exact_search_matches_bruteforce_numpy(self):
        rng = np.random.default_rng(9)
        data = oracle.quantize_int8_vec(_unit(rng, 500, 40))
        q = oracle.quantize_int8_vec(_unit(rng, 5, 40))
        rows, scores, _ = oracle.search_exact_batch(1, data, q, 7)
        full = q.astype(np.int64) @ data.astype(np.int64).T
        for i in range(5):
            order = np.lexsort((np.arange(500), -full[i]))[:7]
            assert rows[i].tolist() == order.tolist()
            assert scores[i].tolist() == full[i, order].tolist()

    def test_exact_search_ties_prefer_lower_row(self):
        data = np.array([[1, 0], [0, 1], [1, 0], [1, 0]], dtype=np.int8)
        rows, scores, _ = oracle.search_exact_batch(1, data, np.array([[1, 0]], dtype=np.int8), 2)
        assert rows[0].tolist() == [0, 2]


class TestForwardOracle:
    def test_errors_match_reference_strings(self, oracle_model):
        m = oracle_model
        with pytest.raises(ValueError, match="^empty input$"):
            m.forward_with_dim([], 768)
        with pytest.raises(ValueError, match=r"^sequence too long: 2049 > 2048$"):
            m.forward_with_dim([2] * 2049, 768)
        with pytest.raises(ValueError, match=r"^token ID out of range: 4096$"):
            m.forward_with_dim([2, 4096], 768)
        with pytest.raises(ValueError, match=r"^target dimension 769 out of range \(1\.\.768\)$"):
            m.forward_with_dim([2, 5], 769)

    def test_unit_norm_and_determinism(self, oracle_model):
        # internal/runtime/int8_test.go:51-61 (128-dim output is unit norm), api_test.go:304-349 (determinism)
        ids = [2, 9259 % 4096, 1902, 1]
        a = oracle_model.forward_with_dim(ids, 128)
        b = oracle_model.forward_with_dim(ids, 128)
        assert a.shape == (128,)
        assert abs(np.linalg.norm(a) - 1) < 1e-5
        np.testing.assert_array_equal(a, b)


class TestTimedBuildEqualsChecker:
    """bench.py times the CPU baseline with the oracle's intrinsic inner loops
    (oracle.set_simd): VPDPBUSD / VCVTDQ2PS / VFMADD231PS and the AVX2
    dot product, the reference's assembly instruction for instruction. They
    must give the plain loops' results bit for bit, or the timed baseline
    would not be the checked computation."""

    def test_matmul_and_dot(self):
        import synth
        rng = np.random.default_rng(31)
        if not oracle.set_simd(True):
            oracle.set_simd(False)
            pytest.skip("host CPU has no AVX512-VNNI")
        try:
            for K, N, M in ((768, 256, 9), (1152, 128, 4), (3072, 128, 3)):
                raw = synth.q8_0_blocks(rng, N, K)
                codes, sc = oracle.quantize_sym_int8(rng.standard_normal((M, K)).astype(np.float32))
                fast = oracle.matmul_q8_0_int8(raw, codes, sc, N)
                oracle.set_simd(False)
                plain = oracle.matmul_q8_0_int8(raw, codes, sc, N)
                oracle.set_simd(True)
                np.testing.assert_array_equal(fast, plain)
            for n in (8, 9, 256, 1000):
                a = rng.standard_normal(n).astype(np.float32)
                b = rng.standard_normal(n).astype(np.float32)
                x = oracle.lib().orc_dot_f32(oracle._p(a, oracle.C.c_float), oracle._p(b, oracle.C.c_float), n)
                oracle.set_simd(False)
                y = oracle.lib().orc_dot_f32(oracle._p(a, oracle.C.c_float), oracle._p(b, oracle.C.c_float), n)
                oracle.set_simd(True)
                assert np.float32(x).tobytes() == np.float32(y).tobytes()
        finally:
            oracle.set_simd(False)

    def test_forward(self, model_path):
        import synth
        m = oracle.OracleModel(model_path)
        if not oracle.set_simd(True):
            oracle.set_simd(False)
            pytest.skip("host CPU has no AVX512-VNNI")
        try:
            ids, offs = synth.token_batch(91, [40, 7], m.config.vocab_size)
            fast = m.forward_batch(ids, offs, 768, nthreads=2)
            oracle.set_simd(False)
            plain = m.forward_batch(ids, offs, 768, nthreads=2)
            np.testing.assert_array_equal(fast, plain)
        finally:
            oracle.set_simd(False)
            m.close()
