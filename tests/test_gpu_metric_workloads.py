"""Parity at the metric's own workloads, at full size, on the seeded inputs the
benchmark times (np.random.default_rng; mlir_edsl.workloads restates
oracle.gen_config_inputs):

  dense_65536  relu(X[65536,4096] @ W[4096,4096] + b), U[-0.5,0.5], seed 3
               (the row-sharded layer; the reference times this op in
               benchmarks/bench_dense_layer.py:49-67)
  dense_8192   relu(A[8192,8192] @ B[8192,8192] + b), U[-1,1], seed 2

Each output row depends only on its X row, so the oracle checks a sample of
rows exactly: the first and last row, both sides of every 8-way shard edge,
and random rows, 256 in all. Tolerance (f32 bar of the path):
max|Y - Y_oracle| <= 1e-4 * sqrt(K) * max|X| * max|W|; against float64 the
error must also be f32-level (a tenth of that bound).
"""
import numpy as np
import pytest

import oracle
from gpu_util import max_err, ptr, stream_ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _sample_rows(M, shards=8, total=256, seed=0):
    edges = {0, M - 1}
    step = M // shards
    for k in range(1, shards):
        edges.update((k * step - 1, k * step))
    rest = np.setdiff1d(np.arange(M), sorted(edges))
    extra = np.random.default_rng(seed).choice(rest, total - len(edges), replace=False)
    return np.sort(np.concatenate([np.array(sorted(edges)), extra]))


def _check_rows(X, W, b, got_rows, rows):
    ref = oracle.dense_f32(X[rows], W, b, act=oracle.ACT_RELU)
    bound = oracle.f32_bound(X.shape[1], X, W)
    err = max_err(got_rows, ref)
    assert np.isfinite(got_rows).all()
    assert err <= bound, (err, bound)
    exact = np.maximum(X[rows].astype(np.float64) @ W.astype(np.float64) + b, 0.0)
    err64 = float(np.max(np.abs(got_rows - exact)))
    assert err64 <= bound / 10, (err64, bound)
    return err


def _dense(torch, tX, tW, tb, tY):
    M, K = tX.shape
    N = tW.shape[1]
    L = _native.lib()
    _native.check(L.b200_dense_f32(ptr(tX), tX.stride(0), ptr(tW), N, ptr(tb), ptr(tY),
                                   tY.stride(0), M, N, K, 1, 0.0, stream_ptr(torch)))


def test_dense_65536_full_layer_and_its_shards(cuda):
    import torch
    g = oracle.gen_config_inputs("dense_65536")
    X, W, b = g["X"], g["W"], g["b"]
    M, K = X.shape
    N = W.shape[1]
    tX, tW, tb = (torch.from_numpy(a).to(cuda) for a in (X, W, b))
    tY = torch.full((M, N), float("nan"), device=cuda)
    _dense(torch, tX, tW, tb, tY)
    _native.check(_native.lib().b200_stream_sync(stream_ptr(torch)))
    rows = _sample_rows(M)
    idx = torch.from_numpy(rows).to(cuda)
    _check_rows(X, W, b, tY.index_select(0, idx).cpu().numpy(), rows)
    # The 8 row shards a dp8 run gives its ranks, each as its own call (the
    # split-K schedule of an 8192-row call differs from the 65536-row one).
    tY.fill_(float("nan"))
    step = M // 8
    for k in range(8):
        _dense(torch, tX[k * step:(k + 1) * step], tW, tb, tY[k * step:(k + 1) * step])
    _native.check(_native.lib().b200_stream_sync(stream_ptr(torch)))
    _check_rows(X, W, b, tY.index_select(0, idx).cpu().numpy(), rows)
    assert not torch.isnan(tY).any()


def test_dense_8192_headline_layer(cuda):
    import torch
    g = oracle.gen_config_inputs("dense_8192")
    A, B, b = g["A"], g["B"], g["b"]
    M = A.shape[0]
    tA, tB, tb = (torch.from_numpy(a).to(cuda) for a in (A, B, b))
    tY = torch.full((M, B.shape[1]), float("nan"), device=cuda)
    _dense(torch, tA, tB, tb, tY)
    _native.check(_native.lib().b200_stream_sync(stream_ptr(torch)))
    rows = _sample_rows(M)
    idx = torch.from_numpy(rows).to(cuda)
    _check_rows(A, B, b, tY.index_select(0, idx).cpu().numpy(), rows)
    assert not torch.isnan(tY).any()
