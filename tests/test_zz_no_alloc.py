"""sem_q8_gemm_noalloc: the Q8_0 projection for callers that cannot allocate
device memory (a host runtime that owns the whole device pool, or a request
path whose memory budget is fixed at start-up), checked against the CPU oracle
and against sem_q8_gemm with caller-provided scratch, on two calls in a row.

Kept in its own file that pytest collects last, so a run that stops at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def _run_both(lib, w, ctx, a, N):
    """Returns (sem_q8_gemm output, sem_q8_gemm_noalloc output) for fp32 a."""
    import torch
    import _lib
    m, K = a.shape
    d_a = torch.from_numpy(a).cuda()
    ref_out = torch.empty((m, N), dtype=torch.float32, device="cuda")
    codes = torch.empty((m, K), dtype=torch.float16, device="cuda")  # INT8 codes held as fp16
    absmax = torch.zeros(4, dtype=torch.int32, device="cuda")
    got_out = torch.full((m, N), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    w.run(d_a.data_ptr(), m, ref_out.data_ptr(), codes.data_ptr(), absmax.data_ptr(), ctx.stream)
    _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(d_a.data_ptr()), m,
                                       ctypes.c_void_p(got_out.data_ptr()), ctypes.c_void_p(ctx.stream)))
    torch.cuda.synchronize()
    return ref_out.cpu().numpy(), got_out.cpu().numpy()


@pytest.mark.parametrize("path", [0, 2])
def test_noalloc_matches_oracle_and_scratch_variant_twice(ctx, path):
    import oracle
    import _lib
    import runtime

    lib = _lib.load()
    prev = lib.sem_q8_path(path)  # 2: the split-plane kernel for every m
    rng = np.random.default_rng(2024 + path)
    try:
        # K = 1152 (the down projection) and a shape whose row count takes a
        # tensor-core kernel; two calls per weight with different sizes and
        # activation scales: the static scratch keeps the first call's
        # contents, which must not leak into the second
        for K, N, calls in ((768, 256, ((64, 1.0), (200, 0.25))), (1152, 768, ((127, 3.0), (130, 0.5))),
                            (768, 3072, ((2048, 1.0), (96, 2.0)))):
            raw = synth.q8_0_blocks(rng, N, K)
            w = runtime.Q8Weight(ctx, raw, K, N)
            for m, scale in calls:
                a = (rng.standard_normal((m, K)) * scale).astype(np.float32)
                ref, got = _run_both(lib, w, ctx, a, N)
                assert np.isfinite(got).all()
                # the same kernel as sem_q8_gemm for this m and path: identical outputs
                np.testing.assert_array_equal(got, ref)
                codes, sc = oracle.quantize_sym_int8(a)
                want = oracle.matmul_q8_0_int8(raw, codes, sc, N)
                if m < 128 and path == 0:  # the CUDA-core kernel: the reference's VNNI order exactly
                    np.testing.assert_array_equal(got, want)
                else:  # the GEMM tolerance of the tensor-core kernels
                    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5 * np.abs(want).max())
            w.close()
    finally:
        lib.sem_q8_path(prev)


def test_noalloc_allocates_nothing_and_limits(ctx):
    import torch
    import _lib
    import runtime

    lib = _lib.load()
    rng = np.random.default_rng(77)
    K, N = 768, 256
    w = runtime.Q8Weight(ctx, synth.q8_0_blocks(rng, N, K), K, N)
    stream = ctypes.c_void_p(ctx.stream)
    sizes = (1, 64, 500, 5000)
    bufs = [(torch.from_numpy(rng.standard_normal((m, K)).astype(np.float32)).cuda(),
             torch.empty((m, N), dtype=torch.float32, device="cuda")) for m in sizes]
    # warm-up: the first call on the device resolves the static array's
    # address, and the first launch of each kernel loads its code
    for (a, c), m in zip(bufs, sizes):
        _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(a.data_ptr()), m,
                                           ctypes.c_void_p(c.data_ptr()), stream))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for (a, c), m in zip(bufs, sizes):
            _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(a.data_ptr()), m,
                                               ctypes.c_void_p(c.data_ptr()), stream))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    # an empty batch is a no-op, as for sem_q8_gemm
    _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(bufs[0][0].data_ptr()), 0,
                                       ctypes.c_void_p(bufs[0][1].data_ptr()), stream))
    # a size beyond the static maximum is rejected, not truncated
    too_many = (8 << 20) // K + 1
    big = torch.zeros((too_many, K), dtype=torch.float32, device="cuda")
    out = torch.empty((too_many, N), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.SemError, match="above the static maximum"):
        _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(big.data_ptr()), too_many,
                                           ctypes.c_void_p(out.data_ptr()), stream))
    with pytest.raises(_lib.SemError, match="negative row count"):
        _lib.check(lib.sem_q8_gemm_noalloc(w.handle, ctypes.c_void_p(big.data_ptr()), -1,
                                           ctypes.c_void_p(out.data_ptr()), stream))
    w.close()
