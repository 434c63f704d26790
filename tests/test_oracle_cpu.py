"""The CPU oracle against the reference's known answers and NumPy float64."""
import json
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def _arr(spec):
    return np.array(spec["data"], dtype=spec["dtype"])


def run_oracle(c):
    ins = {k: _arr(v) for k, v in c["inputs"].items()}
    op = c["op"]
    if op == "matmul":
        return oracle.dense_f32(ins["A"], ins["B"])
    if op == "matmul_i32":
        return oracle.matmul_i32(ins["A"], ins["B"])
    if op == "dense":
        return oracle.dense_f32(ins["X"], ins["W"], ins["b"])
    if op == "bias_add":
        return oracle.bias_act_f32(ins["X"], ins["b"])
    if op == "dot":
        return oracle.dot_f32(ins["a"], ins["b"])
    if op == "dot_i32":
        return oracle.dot_i32(ins["a"], ins["b"])
    if op in ("sum", "max", "min", "prod"):
        red = {"sum": oracle.REDUCE_SUM, "max": oracle.REDUCE_MAX, "min": oracle.REDUCE_MIN,
               "prod": oracle.REDUCE_PROD}[op]
        return oracle.reduce_f32(ins["a"], red)
    X = ins["X"]
    X2 = X.reshape(1, -1) if X.ndim == 1 else X
    act = oracle.ACT_RELU if op == "relu" else oracle.ACT_LEAKY_RELU
    return oracle.bias_act_f32(X2, None, act, c["alpha"]).reshape(X.shape)


@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["name"])
def test_oracle_known_answers(c):
    got = run_oracle(c)
    exp = np.array(c["expected"])
    if c["op"] in ("matmul_i32", "dot_i32"):
        np.testing.assert_array_equal(got, exp)
    else:
        np.testing.assert_allclose(got, exp, rtol=c["rtol"], atol=c["atol"])


def test_golden_file_is_reproducible(tmp_path):
    """The committed fixture equals what its generator produces."""
    import subprocess
    import sys
    gen = os.path.join(os.path.dirname(__file__), "golden", "make_golden.py")
    before = open(GOLDEN).read()
    subprocess.run([sys.executable, gen], check=True, capture_output=True)
    assert open(GOLDEN).read() == before


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (7, 9, 13), (64, 64, 64), (65, 130, 77),
                                   (200, 100, 300), (128, 256, 1001)])
@pytest.mark.parametrize("mode", [oracle.MODE_FMA, oracle.MODE_MULADD])
def test_oracle_vs_float64(M, N, K, mode):
    rng = np.random.default_rng(M * 1000 + N + K)
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b = rng.uniform(-1, 1, (N,)).astype(np.float32)
    got = oracle.dense_f32(X, W, b, act=oracle.ACT_RELU, mode=mode)
    exact = np.maximum(X.astype(np.float64) @ W.astype(np.float64) + b, 0.0)
    err = np.max(np.abs(got - exact))
    assert err <= oracle.f32_bound(K, X, W) / 20, err  # f32 accumulation, far inside the bound


def test_fma_and_muladd_differ_only_in_rounding():
    rng = np.random.default_rng(5)
    X = rng.uniform(-1, 1, (64, 512)).astype(np.float32)
    W = rng.uniform(-1, 1, (512, 64)).astype(np.float32)
    a = oracle.dense_f32(X, W, mode=oracle.MODE_FMA)
    m = oracle.dense_f32(X, W, mode=oracle.MODE_MULADD)
    assert not np.array_equal(a, m)  # the two rounding sequences are really different
    assert np.max(np.abs(a - m)) < 1e-4


@pytest.mark.parametrize("M,N,K,expected", [
    (256, 256, 256, oracle.MODE_FMA), (1024, 1024, 1024, oracle.MODE_FMA),
    (16, 16, 16, oracle.MODE_FMA), (2, 2, 2, oracle.MODE_MULADD),
    (1000, 999, 1001, oracle.MODE_MULADD), (96, 64, 64, oracle.MODE_MULADD),
    (64, 64, 12, oracle.MODE_MULADD)])
def test_fma_mode_rule(M, N, K, expected):
    assert oracle.fma_mode(M, N, K) == expected


def test_relu_maximumf_semantics():
    X = np.array([[np.nan, -0.0, 0.0, -1.0, 1.0, np.inf, -np.inf]], np.float32)
    Y = oracle.bias_act_f32(X, None, oracle.ACT_RELU)
    assert np.isnan(Y[0, 0])
    assert Y[0, 1] == 0.0 and not np.signbit(Y[0, 1])
    np.testing.assert_array_equal(Y[0, 2:], [0.0, 0.0, 1.0, np.inf, 0.0])


def test_leaky_relu_formula():
    X = np.array([[-2.0, -0.5, 0.0, 3.0, np.nan]], np.float32)
    Y = oracle.bias_act_f32(X, None, oracle.ACT_LEAKY_RELU, 0.25)
    np.testing.assert_array_equal(Y[0, :4], np.array([-0.5, -0.125, 0.0, 3.0], np.float32))
    assert np.isnan(Y[0, 4])


def test_i32_wraps_like_int64_mod_2_32():
    rng = np.random.default_rng(9)
    A = rng.integers(-2**31, 2**31, (17, 33), dtype=np.int64).astype(np.int32)
    B = rng.integers(-2**31, 2**31, (33, 12), dtype=np.int64).astype(np.int32)
    bias = rng.integers(-2**31, 2**31, (12,), dtype=np.int64).astype(np.int32)
    exp = (A.astype(np.int64) @ B.astype(np.int64) + bias) & 0xFFFFFFFF
    exp = exp.astype(np.uint32).view(np.int32)
    np.testing.assert_array_equal(oracle.matmul_i32(A, B, bias), exp)


def test_i32_config_rows_exact():
    g = oracle.gen_config_inputs("matmul_i32_2048")
    A, B = g["A"][:32], g["B"]
    np.testing.assert_array_equal(oracle.matmul_i32(A, B),
                                  (A.astype(np.int64) @ B.astype(np.int64)).astype(np.int32))


@pytest.mark.parametrize("name,shapes", [
    ("matmul_256", {"A": (256, 256), "B": (256, 256)}),
    ("dense_1024", {"X": (1024, 1024), "W": (1024, 1024), "b": (1024,)}),
    ("dense_ragged", {"X": (1000, 1001), "W": (1001, 999), "b": (999,)}),
])
def test_config_inputs_are_seeded(name, shapes):
    g1, g2 = oracle.gen_config_inputs(name), oracle.gen_config_inputs(name)
    for k, shp in shapes.items():
        assert g1[k].shape == shp and g1[k].dtype == np.float32
        np.testing.assert_array_equal(g1[k], g2[k])
        assert g1[k].min() >= -1 and g1[k].max() <= 1


def test_dense_1024_config_within_bound():
    g = oracle.gen_config_inputs("dense_1024")
    Y = oracle.dense_f32(g["X"], g["W"], g["b"], act=oracle.ACT_RELU)
    exact = np.maximum(g["X"].astype(np.float64) @ g["W"] + g["b"], 0)
    assert np.max(np.abs(Y - exact)) <= oracle.f32_bound(1024, g["X"], g["W"])


def test_reductions_match_float64_and_numpy():
    rng = np.random.default_rng(12)
    x = rng.standard_normal(100_003).astype(np.float32)
    y = rng.standard_normal(100_003).astype(np.float32)
    assert abs(oracle.reduce_f32(x, oracle.REDUCE_SUM) - x.astype(np.float64).sum()) <= \
        oracle.sum_bound(x)
    assert oracle.reduce_f32(x, oracle.REDUCE_MAX) == x.max()
    assert oracle.reduce_f32(x, oracle.REDUCE_MIN) == x.min()
    exact = float(np.dot(x.astype(np.float64), y.astype(np.float64)))
    assert abs(oracle.dot_f32(x, y) - exact) <= oracle.sum_bound(x * y)


def test_max_skips_nan_like_the_reference_body():
    x = np.array([1.0, np.nan, 5.0, 2.0], np.float32)
    assert oracle.reduce_f32(x, oracle.REDUCE_MAX) == 5.0  # If(elem > acc, ...) is false for NaN
    assert oracle.reduce_f32(x, oracle.REDUCE_MIN) == 1.0


def test_i32_reductions_wrap():
    x = np.array([2**31 - 1, 1, 5], np.int32)
    assert oracle.reduce_i32(x, oracle.REDUCE_SUM) == np.int32(-2**31 + 5)
    assert oracle.dot_i32(np.array([65536], np.int32), np.array([65536], np.int32)) == 0
