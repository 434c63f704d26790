"""Route A of the integration: each b200_memref_* symbol called through
ctypes.CFUNCTYPE with flattened memref descriptors built the way the
reference's execute_function builds them (alloc, aligned, offset, sizes,
strides per memref; the Python-allocated output descriptor last; void or
scalar return), reference: mlir_edsl/backend.py:37-102, 162-198."""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import max_err
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _desc(a):
    ptr = a.ctypes.data_as(ctypes.c_void_p)
    strides = [s // a.itemsize for s in a.strides]
    types = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] + [ctypes.c_int64] * (2 * a.ndim)
    return types, [ptr, ptr, 0] + list(a.shape) + strides


def _call(sym, ins, out=None, restype=None):
    types, vals = [], []
    for a in ins + ([out] if out is not None else []):
        t, v = _desc(a)
        types += t
        vals += v
    fp = ctypes.cast(getattr(_native.lib(), sym), ctypes.c_void_p).value
    r = ctypes.CFUNCTYPE(restype, *types)(fp)(*vals)
    _native.check_last()
    return r, len(vals)


def _f(rng, *shape):
    return rng.uniform(-1, 1, shape).astype(np.float32)


def test_f32_gemm_symbols(cuda):
    rng = np.random.default_rng(0)
    M, N, K = 130, 70, 90
    X, W, b = _f(rng, M, K), _f(rng, K, N), _f(rng, N)
    bound = oracle.f32_bound(K, X, W)
    cases = [("b200_memref_matmul_f32", [X, W], None, 0, 21),
             ("b200_memref_matmul_relu_f32", [X, W], None, 1, 21),
             ("b200_memref_dense_f32", [X, W, b], b, 0, 26),
             ("b200_memref_dense_relu_f32", [X, W, b], b, 1, 26)]
    for sym, ins, bias, act, nargs in cases:
        Y = np.empty((M, N), np.float32)
        _, n = _call(sym, ins, Y)
        assert n == nargs
        assert max_err(Y, oracle.dense_f32(X, W, bias, act=act)) <= bound, sym


def test_i32_and_elementwise_symbols(cuda):
    rng = np.random.default_rng(1)
    A = rng.integers(-8, 9, (33, 17), dtype=np.int32)
    B = rng.integers(-8, 9, (17, 29), dtype=np.int32)
    bi = rng.integers(-8, 9, (29,), dtype=np.int32)
    C = np.empty((33, 29), np.int32)
    _call("b200_memref_matmul_i32", [A, B], C)
    np.testing.assert_array_equal(C, A @ B)
    _call("b200_memref_dense_i32", [A, B, bi], C)
    np.testing.assert_array_equal(C, A @ B + bi)
    X, b = _f(rng, 40, 24), _f(rng, 24)
    Y = np.empty_like(X)
    _, n = _call("b200_memref_bias_add_f32", [X, b], Y)
    assert n == 19
    np.testing.assert_array_equal(Y, oracle.bias_act_f32(X, b))
    _call("b200_memref_bias_relu_f32", [X, b], Y)
    np.testing.assert_array_equal(Y, oracle.bias_act_f32(X, b, oracle.ACT_RELU))
    _, n = _call("b200_memref_relu_f32", [X], Y)
    assert n == 14
    np.testing.assert_array_equal(Y, oracle.bias_act_f32(X, None, oracle.ACT_RELU))


def test_scalar_symbols(cuda):
    rng = np.random.default_rng(2)
    a, b = _f(rng, 10_001), _f(rng, 10_001)
    r, n = _call("b200_memref_dot_f32", [a, b], restype=ctypes.c_float)
    assert n == 10 and abs(r - np.dot(a.astype(np.float64), b)) <= oracle.sum_bound(a * b)
    r, n = _call("b200_memref_sum_f32", [a], restype=ctypes.c_float)
    assert n == 5 and abs(r - a.astype(np.float64).sum()) <= oracle.sum_bound(a)
    assert _call("b200_memref_max_f32", [a], restype=ctypes.c_float)[0] == a.max()
    assert _call("b200_memref_min_f32", [a], restype=ctypes.c_float)[0] == a.min()
    ai = rng.integers(-100, 100, 999, dtype=np.int32)
    bi = rng.integers(-100, 100, 999, dtype=np.int32)
    assert _call("b200_memref_dot_i32", [ai, bi], restype=ctypes.c_int32)[0] == int(ai @ bi)


def test_shape_mismatch_sets_status(cuda):
    X, W = np.ones((4, 5), np.float32), np.ones((6, 3), np.float32)
    Y = np.empty((4, 3), np.float32)
    types, vals = [], []
    for a in (X, W, Y):
        t, v = _desc(a)
        types += t
        vals += v
    fp = ctypes.cast(_native.lib().b200_memref_matmul_f32, ctypes.c_void_p).value
    ctypes.CFUNCTYPE(None, *types)(fp)(*vals)
    assert _native.lib().b200_last_status() == 1
    assert b"[M,K]x[K,N]" in _native.lib().b200_last_error()
