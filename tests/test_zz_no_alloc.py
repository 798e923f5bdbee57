"""sem_q8_gemm_noalloc: the Q8_0 projection for callers that cannot allocate
device memory (their runtime owns the whole pool, or their memory budget is
fixed up front), checked against sem_q8_gemm with caller-provided scratch.

Kept in its own file that pytest collects last, so a run that stops at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def test_noalloc_matches_scratch_variant_twice(ctx):
    import torch

    import _lib
    import runtime

    lib = _lib.load()
    rng = np.random.default_rng(2024)
    K, N = 768, 256
    w = runtime.Q8Weight(ctx, synth.q8_0_blocks(rng, N, K), K, N)
    stream = ctypes.c_void_p(ctx.stream)
    # two calls in a row with different sizes and activation scales: the static
    # scratch keeps the first call's contents, which must not leak into the second
    for m, scale in ((64, 1.0), (200, 0.25)):
        a = (rng.standard_normal((m, K)) * scale).astype(np.float32)
        d_a = torch.from_numpy(a).cuda()
        ref_out = torch.empty((m, N), dtype=torch.float32, device="cuda")
        codes = torch.empty((m, K), dtype=torch.float16, device="cuda")  # INT8 codes held as fp16
        absmax = torch.zeros(4, dtype=torch.int32, device="cuda")
        got_out = torch.full((m, N), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        w.run(d_a.data_ptr(), m, ref_out.data_ptr(), codes.data_ptr(), absmax.data_ptr(), ctx.stream)
        _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(d_a.data_ptr()), m,
                                           ctypes.c_void_p(got_out.data_ptr()), stream))
        torch.cuda.synchronize()
        ref, got = ref_out.cpu().numpy(), got_out.cpu().numpy()
        assert np.isfinite(got).all()
        # same kernels on the same inputs: equal within the GEMM test tolerance (in practice identical)
        np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-5 * np.abs(ref).max())
    # a size beyond the static maximum is rejected, not truncated
    too_many = (8 << 20) // K + 1
    big = torch.zeros((too_many, K), dtype=torch.float32, device="cuda")
    out = torch.empty((too_many, N), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.SemError, match="above the static maximum"):
        _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(big.data_ptr()), too_many,
                                           ctypes.c_void_p(out.data_ptr()), stream))
    w.close()
