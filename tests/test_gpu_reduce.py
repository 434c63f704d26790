"""GPU parity of the 1-D reduction and dot kernels against the sequential
CPU oracle: max/min/i32 exact, f32 sums and dots within the reordered-sum
bound n * 2^-24 * sum|terms| (both orders are within it of the exact sum)."""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import ptr, stream_ptr
from mlir_edsl import (Tensor, dot, f32, i32, ml_function, reduce, relu, tensor_max, tensor_min,
                       tensor_sum, to_value)
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _dev_reduce(torch, x, op, init):
    dev = torch.device("cuda:0")
    L = _native.lib()
    tx = torch.from_numpy(x).to(dev)
    if x.dtype == np.float32:
        out = torch.full((1,), 12345.0, device=dev)
        _native.check(L.b200_reduce_f32(ptr(tx), x.size, op, float(init), ptr(out),
                                        stream_ptr(torch)))
    else:
        out = torch.full((1,), 12345, device=dev, dtype=torch.int32)
        _native.check(L.b200_reduce_i32(ptr(tx), x.size, op, int(init), ptr(out),
                                        stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    return out.cpu().numpy()[0]


@pytest.mark.parametrize("n", [1, 7, 4096, 100_003, 1 << 24])
def test_sum_max_min_f32(cuda, n):
    import torch
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    got = _dev_reduce(torch, x, oracle.REDUCE_SUM, 0.0)
    ref = oracle.reduce_f32(x, oracle.REDUCE_SUM)
    exact = float(x.astype(np.float64).sum())
    bound = oracle.sum_bound(x)
    assert abs(got - exact) <= bound and abs(got - ref) <= 2 * bound
    for op in (oracle.REDUCE_MAX, oracle.REDUCE_MIN):
        assert _dev_reduce(torch, x, op, oracle.REDUCE_INIT[op]) == oracle.reduce_f32(x, op)


def test_max_min_with_nan_and_init(cuda):
    import torch
    x = np.array([1.0, np.nan, 5.0, -3.0, np.nan], np.float32)
    assert _dev_reduce(torch, x, oracle.REDUCE_MAX, float("-inf")) == 5.0
    assert _dev_reduce(torch, x, oracle.REDUCE_MIN, float("inf")) == -3.0
    assert _dev_reduce(torch, x, oracle.REDUCE_MAX, 10.0) == 10.0  # init wins
    assert _dev_reduce(torch, np.zeros(0, np.float32), oracle.REDUCE_SUM, 2.5) == 2.5


@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_i32_reductions_exact(cuda, op):
    import torch
    rng = np.random.default_rng(op)
    x = rng.integers(-2**31, 2**31, 1_000_001, dtype=np.int64).astype(np.int32)
    init = {0: 0, 1: 1, 2: -2**31, 3: 2**31 - 1}[op]
    assert _dev_reduce(torch, x, op, init) == oracle.reduce_i32(x, op, init)


def test_product_f32(cuda):
    import torch
    rng = np.random.default_rng(3)
    x = rng.uniform(0.99, 1.01, 10_000).astype(np.float32)
    got = _dev_reduce(torch, x, oracle.REDUCE_PROD, 1.0)
    exact = float(np.prod(x.astype(np.float64)))
    assert abs(got - exact) <= 1e4 * 2 ** -24 * exact  # n * eps relative


@pytest.mark.parametrize("n", [3, 5000, 1 << 22])
def test_dot_f32_and_i32(cuda, n):
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    out = torch.zeros(1, device=dev)
    _native.check(L.b200_dot_f32(ptr(ta), ptr(tb), n, ptr(out), stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    exact = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
    assert abs(out.item() - exact) <= oracle.sum_bound(a * b)
    ai = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    bi = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    r = np.zeros(1, np.int32)
    c = ctypes.c_void_p
    _native.check(L.b200_dot_i32_host(c(ai.ctypes.data), c(bi.ctypes.data), n, c(r.ctypes.data)))
    assert r[0] == oracle.dot_i32(ai, bi)


def test_frontend_reductions_compose(cuda):
    """reference: tests/linalg/test_reduce_execution.py:143-170"""
    @ml_function(target="b200")
    def sum_times_two(a: Tensor[f32, 4]) -> f32:
        return tensor_sum(a) * to_value(2.0)

    @ml_function(target="b200")
    def product(a: Tensor[f32, 4]) -> f32:
        return reduce(a, to_value(1.0), lambda elem, acc: acc * elem)

    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    assert sum_times_two(x) == 20.0
    assert product(x) == 24.0

    @ml_function(target="b200")
    def mix(a: Tensor[f32, 1000], b: Tensor[f32, 1000]) -> f32:
        return tensor_max(relu(a)) + dot(a, b)
    rng = np.random.default_rng(1)
    a, b = rng.standard_normal(1000).astype(np.float32), rng.standard_normal(1000).astype(np.float32)
    exp = float(np.maximum(a, 0).max()) + float(np.dot(a.astype(np.float64), b))
    assert abs(mix(a, b) - exp) <= oracle.sum_bound(a * b) + 1e-6

    @ml_function(target="b200")
    def isum(a: Tensor[i32, 5]) -> i32:
        return tensor_sum(a)
    assert isum(np.array([1, 2, 3, 4, 2**31 - 1], np.int32)) == np.int32(-2**31 + 9)
