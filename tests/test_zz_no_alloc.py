"""GPU test of b200_dense_f32_noalloc, the entry point for callers that must
not allocate device memory while they run (its scratch is a fixed device array
in the library). It is compared with b200_dense_f32 on two calls in a row.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest

import oracle
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _case(torch, M, N, K, seed):
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b = rng.uniform(-1, 1, (N,)).astype(np.float32)
    return X, W, b, [torch.from_numpy(a).to(dev) for a in (X, W, b)]


def _run(torch, fn_name, tX, tW, tb, Y, M, N, K, act):
    L = _native.lib()
    Y.fill_(float("nan"))
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _native.check(getattr(L, fn_name)(_p(tX), K, _p(tW), N, _p(tb), _p(Y), N, M, N, K, act, 0.0,
                                      s))
    _native.check(L.b200_stream_sync(s))
    return Y.cpu().numpy()


def test_noalloc_matches_dense_on_two_calls(cuda):
    import torch
    L = _native.lib()
    cases = [(700, 900, 1001, 1, 7), (333, 512, 96, 0, 8)]  # different shapes back to back
    for i, (M, N, K, act, seed) in enumerate(cases):
        X, W, b, (tX, tW, tb) = _case(torch, M, N, K, seed)
        Y = torch.empty((M, N), device=tX.device)
        ref_dev = _run(torch, "b200_dense_f32", tX, tW, tb, Y, M, N, K, act)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        got = _run(torch, "b200_dense_f32_noalloc", tX, tW, tb, Y, M, N, K, act)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        bound = oracle.f32_bound(K, X, W)
        assert np.isfinite(got).all()
        assert float(np.max(np.abs(got.astype(np.float64) - ref_dev))) <= bound
        ref = oracle.dense_f32(X, W, b, act=act)
        assert float(np.max(np.abs(got.astype(np.float64) - ref))) <= bound
        if i > 0:  # after the per-device set-up of the first call
            assert free_after == free_before, (free_before, free_after)
    assert L.b200_last_status() == 0


def test_noalloc_rejects_oversized_problem(cuda):
    import torch
    dev = torch.device("cuda:0")
    M, N, K = 4096, 4096, 1028  # needs 8*(M+N)*K > 64 MiB
    X = torch.zeros((M, K), device=dev)
    W = torch.zeros((K, N), device=dev)
    Y = torch.zeros((M, N), device=dev)
    L = _native.lib()
    rc = L.b200_dense_f32_noalloc(_p(X), K, _p(W), N, None, _p(Y), N, M, N, K, 0, 0.0, None)
    assert rc == 7  # B200_ERR_TOO_LARGE
    assert b"scratch" in L.b200_last_error()


def test_noalloc_limit_is_exact(cuda):
    """M = N = 2048: K = 2048 fills the 64 MiB array exactly (four split
    regions of 2048 x 2048 floats) and runs; K = 2049 rounds the split pitch up
    to 2056 and is rejected before anything is launched."""
    import torch
    M = N = 2048
    X, W, b, (tX, tW, tb) = _case(torch, M, N, 2048, 9)
    Y = torch.empty((M, N), device=tX.device)
    ref_dev = _run(torch, "b200_dense_f32", tX, tW, tb, Y, M, N, 2048, 1)
    got = _run(torch, "b200_dense_f32_noalloc", tX, tW, tb, Y, M, N, 2048, 1)
    assert float(np.max(np.abs(got.astype(np.float64) - ref_dev))) <= oracle.f32_bound(2048, X, W)
    L = _native.lib()
    X2 = torch.zeros((M, 2049), device=tX.device)
    W2 = torch.zeros((2049, N), device=tX.device)
    rc = L.b200_dense_f32_noalloc(_p(X2), 2049, _p(W2), N, None, _p(Y), N, M, N, 2049, 0, 0.0,
                                  None)
    assert rc == 7  # B200_ERR_TOO_LARGE
