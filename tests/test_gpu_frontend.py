"""End-to-end @ml_function(target="b200") on the GPU: the reference's known
answers and dense-net tests, the ragged and 2-layer-MLP benchmark configs,
DYN variants, and the dispatch (fusion / launch count) of each pattern."""
import json
import os

import numpy as np
import pytest

import oracle
from mlir_edsl import (DYN, Tensor, dot, f32, get_backend, i32, leaky_relu, matmul, ml_function,
                       reduce, relu, tensor_max, tensor_min, tensor_sum, to_value)

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")


def _arr(spec):
    return np.array(spec["data"], dtype=spec["dtype"])


def _fn_for(c):
    ins = {k: _arr(v) for k, v in c["inputs"].items()}
    op = c["op"]
    shp = {k: v.shape for k, v in ins.items()}
    if op in ("matmul", "matmul_i32"):
        dt = i32 if op == "matmul_i32" else f32
        (M, K), (_, N) = shp["A"], shp["B"]

        @ml_function(target="b200")
        def fn(A: Tensor[dt, M, K], B: Tensor[dt, K, N]) -> Tensor[dt, M, N]:
            return A @ B
        return fn, [ins["A"], ins["B"]]
    if op == "dense":
        (M, K), (_, N) = shp["X"], shp["W"]

        @ml_function(target="b200")
        def fn(X: Tensor[f32, M, K], W: Tensor[f32, K, N], b: Tensor[f32, N]) -> Tensor[f32, M, N]:
            return X @ W + b
        return fn, [ins["X"], ins["W"], ins["b"]]
    if op in ("dot", "dot_i32"):
        dt = i32 if op == "dot_i32" else f32
        n = shp["a"][0]

        @ml_function(target="b200")
        def fn(a: Tensor[dt, n], b: Tensor[dt, n]) -> dt:
            return dot(a, b)
        return fn, [ins["a"], ins["b"]]
    if op in ("sum", "max", "min", "prod"):
        n = shp["a"][0]
        body = {"sum": tensor_sum, "max": tensor_max, "min": tensor_min,
                "prod": lambda a: reduce(a, to_value(1.0), lambda e, acc: acc * e)}[op]

        @ml_function(target="b200")
        def fn(a: Tensor[f32, n]) -> f32:
            return body(a)
        return fn, [ins["a"]]
    if op == "bias_add":
        M, N = shp["X"]

        @ml_function(target="b200")
        def fn(X: Tensor[f32, M, N], b: Tensor[f32, N]) -> Tensor[f32, M, N]:
            return X + b
        return fn, [ins["X"], ins["b"]]
    dims = shp["X"]
    T = Tensor[(f32,) + tuple(dims)]
    if op == "relu":
        @ml_function(target="b200")
        def fn(X: T) -> T:
            return relu(X)
    else:
        alpha = c["alpha"]

        @ml_function(target="b200")
        def fn(X: T) -> T:
            return leaky_relu(X, alpha=alpha)
    return fn, [ins["X"]]


with open(GOLDEN) as _f:
    _CASES = json.load(_f)["cases"]


@pytest.mark.parametrize("c", _CASES, ids=lambda c: c["name"])
def test_known_answers_through_frontend(cuda, c):
    fn, args = _fn_for(c)
    got = fn(*args)
    exp = np.array(c["expected"])
    if c["op"] in ("matmul_i32", "dot_i32"):
        np.testing.assert_array_equal(got, exp)
    else:
        np.testing.assert_allclose(got, exp, rtol=c["rtol"], atol=max(c["atol"], 1e-6))


def test_bias_on_left_operand(cuda):
    @ml_function(target="b200")
    def f(b: Tensor[f32, 4], x: Tensor[f32, 2, 4]) -> Tensor[f32, 2, 4]:
        return b + x
    b = np.array([1, 2, 3, 4], np.float32)
    np.testing.assert_array_equal(f(b, np.zeros((2, 4), np.float32)), np.tile(b, (2, 1)))


def test_chained_matmul(cuda):
    """(A @ B) @ C with the intermediate kept on the device
    (reference: tests/linalg/test_matmul_execution.py:108-122)."""
    @ml_function(target="b200")
    def chain(A: Tensor[f32, 4, 4], B: Tensor[f32, 4, 4], C: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        return (A @ B) @ C
    rng = np.random.default_rng(1)
    A, B, C = (rng.standard_normal((4, 4)).astype(np.float32) for _ in range(3))
    np.testing.assert_allclose(chain(A, B, C), (A.astype(np.float64) @ B) @ C, rtol=1e-4,
                               atol=1e-5)


@pytest.mark.parametrize("depth", [2, 3])
def test_stacked_dense_nets(cuda, depth):
    """reference: tests/linalg/test_binary_op_execution.py:223-268"""
    rng = np.random.default_rng(depth)
    if depth == 2:
        @ml_function(target="b200")
        def net(X: Tensor[f32, 2, 4], W1: Tensor[f32, 4, 8], b1: Tensor[f32, 8],
                W2: Tensor[f32, 8, 3], b2: Tensor[f32, 3]) -> Tensor[f32, 2, 3]:
            h = relu(X @ W1 + b1)
            return relu(h @ W2 + b2)
        shapes = [(2, 4), (4, 8), (8,), (8, 3), (3,)]
    else:
        @ml_function(target="b200")
        def net(X: Tensor[f32, 4, 8], W1: Tensor[f32, 8, 16], b1: Tensor[f32, 16],
                W2: Tensor[f32, 16, 8], b2: Tensor[f32, 8], W3: Tensor[f32, 8, 4],
                b3: Tensor[f32, 4]) -> Tensor[f32, 4, 4]:
            h1 = relu(X @ W1 + b1)
            h2 = relu(h1 @ W2 + b2)
            return relu(h2 @ W3 + b3)
        shapes = [(4, 8), (8, 16), (16,), (16, 8), (8,), (8, 4), (4,)]
    args = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    got = net(*args)
    h = args[0].astype(np.float64)
    for i in range(depth):
        h = np.maximum(h @ args[1 + 2 * i] + args[2 + 2 * i], 0.0)
    np.testing.assert_allclose(got, h, rtol=1e-4, atol=1e-5)
    from mlir_edsl import _native
    dims = [s[0] for s in shapes[1::2]] + [shapes[-2][1]]  # K of each layer, then last N
    M = shapes[0][0]
    assert get_backend().last_launches == sum(
        _native.dense_launches(M, dims[i + 1], dims[i]) for i in range(depth))


def test_dense_relu_dispatch_is_one_fused_gemm(cuda):
    @ml_function(target="b200")
    def dense(X: Tensor[f32, 64, 96], W: Tensor[f32, 96, 80], b: Tensor[f32, 80]) -> Tensor[f32, 64, 80]:
        return relu(X @ W + b)
    rng = np.random.default_rng(2)
    X, W, b = (rng.standard_normal(s).astype(np.float32) for s in [(64, 96), (96, 80), (80,)])
    got = dense(X, W, b)
    from mlir_edsl import _native
    # W split, X split, one GEMM with fused bias + relu
    assert get_backend().last_launches == _native.dense_launches(64, 80, 96)
    np.testing.assert_allclose(got, np.maximum(X.astype(np.float64) @ W + b, 0), rtol=1e-4,
                               atol=1e-4)


@pytest.mark.parametrize("n", [8, 64, 96, 128, 256, 512, 1024])
def test_matmul_and_dense_sizes(cuda, n):
    """reference: tests/core/test_multicore.py:22-123, tests/gpu/test_gpu_execution.py:55-210,
    tests/gpu/test_gpu_benchmark.py:69-171 (sizes 8..1024, NumPy comparison)."""
    @ml_function(target="b200")
    def mm(A: Tensor[f32, n, n], B: Tensor[f32, n, n]) -> Tensor[f32, n, n]:
        return matmul(A, B)

    @ml_function(target="b200")
    def dense(X: Tensor[f32, n, n], W: Tensor[f32, n, n], b: Tensor[f32, n]) -> Tensor[f32, n, n]:
        return relu(X @ W + b)
    rng = np.random.default_rng(n)
    A, B = rng.random((n, n), dtype=np.float32), rng.random((n, n), dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    np.testing.assert_allclose(mm(A, B), A.astype(np.float64) @ B, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(dense(A, B, b), np.maximum(A.astype(np.float64) @ B + b, 0),
                               rtol=1e-3, atol=1e-4)


def test_dyn_matmul_variants(cuda):
    """reference: tests/linalg/test_linalg_dyn.py:86-95"""
    @ml_function(target="b200")
    def mm(A: Tensor[f32, DYN, DYN], B: Tensor[f32, DYN, DYN]) -> Tensor[f32, DYN, DYN]:
        return matmul(A, B)
    A = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    B = np.array([[5.0, 6.0], [7.0, 8.0]], np.float32)
    np.testing.assert_allclose(mm(A, B), [[19.0, 22.0], [43.0, 50.0]], rtol=1e-3)
    X = np.ones((3, 5), np.float32)
    np.testing.assert_array_equal(mm(X, np.ones((5, 2), np.float32)), np.full((3, 2), 5.0))
    assert len(mm._compiled_variants) == 2


def test_ragged_config_through_frontend(cuda):
    g = oracle.gen_config_inputs("dense_ragged")

    @ml_function(target="b200")
    def dense(X: Tensor[f32, 1000, 1001], W: Tensor[f32, 1001, 999],
              b: Tensor[f32, 999]) -> Tensor[f32, 1000, 999]:
        return relu(X @ W + b)
    got = dense(g["X"], g["W"], g["b"])
    ref = oracle.dense_f32(g["X"], g["W"], g["b"], act=oracle.ACT_RELU)
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= oracle.f32_bound(1001, g["X"], g["W"])


def test_mlp_2layer_config(cuda):
    """cfg5: relu(relu(X @ W1 + b1) @ W2 + b2), X[512,4096], W1[4096,11008],
    W2[11008,4096]; the hidden activation stays on the device."""
    g = oracle.gen_config_inputs("mlp_2layer")

    @ml_function(target="b200")
    def mlp(X: Tensor[f32, 512, 4096], W1: Tensor[f32, 4096, 11008], b1: Tensor[f32, 11008],
            W2: Tensor[f32, 11008, 4096], b2: Tensor[f32, 4096]) -> Tensor[f32, 512, 4096]:
        h = relu(X @ W1 + b1)
        return relu(h @ W2 + b2)
    got = mlp(g["X"], g["W1"], g["b1"], g["W2"], g["b2"])
    from mlir_edsl import _native
    assert get_backend().last_launches == (_native.dense_launches(512, 11008, 4096)
                                           + _native.dense_launches(512, 4096, 11008))
    H = oracle.dense_f32(g["X"], g["W1"], g["b1"], act=oracle.ACT_RELU)
    ref = oracle.dense_f32(H, g["W2"], g["b2"], act=oracle.ACT_RELU)
    bound = oracle.f32_bound(11008, H, g["W2"])
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= bound


def test_i32_dense_and_config(cuda):
    @ml_function(target="b200")
    def d(X: Tensor[i32, 3, 5], W: Tensor[i32, 5, 4], b: Tensor[i32, 4]) -> Tensor[i32, 3, 4]:
        return X @ W + b
    rng = np.random.default_rng(4)
    X = rng.integers(-8, 9, (3, 5), dtype=np.int32)
    W = rng.integers(-8, 9, (5, 4), dtype=np.int32)
    b = rng.integers(-8, 9, (4,), dtype=np.int32)
    np.testing.assert_array_equal(d(X, W, b), X @ W + b)
    g = oracle.gen_config_inputs("matmul_i32_2048")

    @ml_function(target="b200")
    def mm(A: Tensor[i32, 2048, 2048], B: Tensor[i32, 2048, 2048]) -> Tensor[i32, 2048, 2048]:
        return A @ B
    np.testing.assert_array_equal(mm(g["A"], g["B"]), oracle.matmul_i32(g["A"], g["B"]))


def test_leaky_relu_dense_via_host_api(cuda):
    @ml_function(target="b200")
    def f(X: Tensor[f32, 33, 17], W: Tensor[f32, 17, 9]) -> Tensor[f32, 33, 9]:
        return leaky_relu(X @ W, alpha=0.1)
    rng = np.random.default_rng(6)
    X, W = rng.standard_normal((33, 17)).astype(np.float32), rng.standard_normal((17, 9)).astype(np.float32)
    ref = oracle.dense_f32(X, W, act=oracle.ACT_LEAKY_RELU, alpha=0.1)
    assert np.max(np.abs(f(X, W) - ref)) <= oracle.f32_bound(17, X, W)
