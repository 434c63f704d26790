"""ctypes front end of oracle/ref_linalg.c — TEST INFRASTRUCTURE ONLY.

The C file restates ml-edsl's CPU-pipeline arithmetic for linalg.matmul and
relu(X @ W + b); see its header for the reference lines each step follows.
Parity is pinned to the reference's own known-answer tests (tests/golden/)
and to NumPy float64; the reference's MLIR pipeline cannot be built here, so
bit-level f32 parity against it is unpinned.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

ACT_NONE, ACT_RELU, ACT_LEAKY_RELU = 0, 1, 2
MODE_AUTO, MODE_FMA, MODE_MULADD = -1, 0, 1
REDUCE_SUM, REDUCE_PROD, REDUCE_MAX, REDUCE_MIN = 0, 1, 2, 3
REDUCE_INIT = {REDUCE_SUM: 0.0, REDUCE_PROD: 1.0, REDUCE_MAX: float("-inf"),
               REDUCE_MIN: float("inf")}

_lib = None


def build(force=False):
    src = os.path.join(HERE, "ref_linalg.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-B" if force else "-s", "_build/liboracle.so"], cwd=HERE,
                       check=True)
    return LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        lib = ctypes.CDLL(LIB_PATH)
        i64, f32p, i32p = ctypes.c_int64, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32)
        lib.oracle_dense_f32.argtypes = [f32p, f32p, f32p, f32p, i64, i64, i64, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.oracle_dense_f32.restype = None
        lib.oracle_matmul_i32.argtypes = [i32p, i32p, i32p, i32p, i64, i64, i64, ctypes.c_int]
        lib.oracle_matmul_i32.restype = None
        lib.oracle_bias_act_f32.argtypes = [f32p, f32p, f32p, i64, i64, ctypes.c_int, ctypes.c_float]
        lib.oracle_bias_act_f32.restype = None
        lib.oracle_reduce_f32.argtypes = [f32p, i64, ctypes.c_int, ctypes.c_float]
        lib.oracle_reduce_f32.restype = ctypes.c_float
        lib.oracle_reduce_i32.argtypes = [i32p, i64, ctypes.c_int, ctypes.c_int32]
        lib.oracle_reduce_i32.restype = ctypes.c_int32
        lib.oracle_dot_f32.argtypes = [f32p, f32p, i64]
        lib.oracle_dot_f32.restype = ctypes.c_float
        lib.oracle_dot_i32.argtypes = [i32p, i32p, i64]
        lib.oracle_dot_i32.restype = ctypes.c_int32
        lib.oracle_fma_mode.argtypes = [i64, i64, i64]
        lib.oracle_fma_mode.restype = ctypes.c_int
        _lib = lib
    return _lib


def _p(a, ct):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ct))


def fma_mode(M, N, K):
    return _load().oracle_fma_mode(M, N, K)


def dense_f32(X, W, b=None, act=ACT_NONE, alpha=0.0, mode=MODE_AUTO, threads=0):
    """act(X @ W (+ b)) with the reference CPU pipeline's rounding sequence."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    M, K = X.shape
    K2, N = W.shape
    assert K == K2
    if b is not None:
        b = np.ascontiguousarray(b, dtype=np.float32)
        assert b.shape == (N,)
    Y = np.empty((M, N), np.float32)
    _load().oracle_dense_f32(_p(X, ctypes.c_float), _p(W, ctypes.c_float), _p(b, ctypes.c_float),
                             _p(Y, ctypes.c_float), M, N, K, act, alpha, mode, threads)
    return Y


def matmul_i32(A, B, bias=None, threads=0):
    """A @ B (+ bias) modulo 2^32."""
    A = np.ascontiguousarray(A, dtype=np.int32)
    B = np.ascontiguousarray(B, dtype=np.int32)
    M, K = A.shape
    _, N = B.shape
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.int32)
    C = np.empty((M, N), np.int32)
    _load().oracle_matmul_i32(_p(A, ctypes.c_int32), _p(B, ctypes.c_int32),
                              _p(bias, ctypes.c_int32), _p(C, ctypes.c_int32), M, N, K, threads)
    return C


def bias_act_f32(X, b=None, act=ACT_NONE, alpha=0.0):
    X = np.ascontiguousarray(X, dtype=np.float32)
    M, N = X.shape
    if b is not None:
        b = np.ascontiguousarray(b, dtype=np.float32)
    Y = np.empty_like(X)
    _load().oracle_bias_act_f32(_p(X, ctypes.c_float), _p(b, ctypes.c_float),
                                _p(Y, ctypes.c_float), M, N, act, alpha)
    return Y


def reduce_f32(x, op, init=None):
    """Sequential fold of a 1-D f32 tensor (linalg.reduce semantics)."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    init = REDUCE_INIT[op] if init is None else init
    return np.float32(_load().oracle_reduce_f32(_p(x, ctypes.c_float), x.size, op, init))


def reduce_i32(x, op, init=None):
    x = np.ascontiguousarray(x, dtype=np.int32).ravel()
    if init is None:
        init = {REDUCE_SUM: 0, REDUCE_PROD: 1, REDUCE_MAX: -2**31, REDUCE_MIN: 2**31 - 1}[op]
    return np.int32(_load().oracle_reduce_i32(_p(x, ctypes.c_int32), x.size, op, init))


def dot_f32(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32).ravel()
    b = np.ascontiguousarray(b, dtype=np.float32).ravel()
    return np.float32(_load().oracle_dot_f32(_p(a, ctypes.c_float), _p(b, ctypes.c_float), a.size))


def dot_i32(a, b):
    a = np.ascontiguousarray(a, dtype=np.int32).ravel()
    b = np.ascontiguousarray(b, dtype=np.int32).ravel()
    return np.int32(_load().oracle_dot_i32(_p(a, ctypes.c_int32), _p(b, ctypes.c_int32), a.size))


def sum_bound(x):
    """Tolerance for a reordered f32 sum: both orders are within
    n * 2^-24 * sum|x| of the exact sum (standard recursive-summation bound)."""
    x = np.asarray(x, np.float64).ravel()
    return 2.0 * max(x.size, 1) * 2.0 ** -24 * float(np.sum(np.abs(x))) + 1e-30


def f32_bound(K, A, B):
    """North-star f32 tolerance: 1e-4 * sqrt(K) * max|A| * max|B|."""
    return 1e-4 * np.sqrt(max(K, 1)) * float(np.max(np.abs(A))) * float(np.max(np.abs(B)))


def gen_config_inputs(name):
    """Seeded synthetic inputs of the benchmark configurations.

    Generator: np.random.default_rng(seed); arrays drawn in the listed order;
    f32 as rng.uniform(lo, hi, shape).astype(float32), i32 as
    rng.integers(-8, 9, shape, dtype=int32).
    """
    u = lambda rng, lo, hi, shape: rng.uniform(lo, hi, shape).astype(np.float32)
    if name == "matmul_256":
        rng = np.random.default_rng(0)
        return dict(A=u(rng, -1, 1, (256, 256)), B=u(rng, -1, 1, (256, 256)))
    if name == "dense_1024":
        rng = np.random.default_rng(1)
        return dict(X=u(rng, -1, 1, (1024, 1024)), W=u(rng, -1, 1, (1024, 1024)),
                    b=u(rng, -1, 1, (1024,)))
    if name in ("matmul_4096", "matmul_8192"):
        n = 4096 if name == "matmul_4096" else 8192
        rng = np.random.default_rng(2)
        return dict(A=u(rng, -1, 1, (n, n)), B=u(rng, -1, 1, (n, n)))
    if name == "dense_8192":  # matmul_8192's A and B, then the bias
        rng = np.random.default_rng(2)
        return dict(A=u(rng, -1, 1, (8192, 8192)), B=u(rng, -1, 1, (8192, 8192)),
                    b=u(rng, -1, 1, (8192,)))
    if name == "matmul_i32_2048":
        rng = np.random.default_rng(2)
        return dict(A=rng.integers(-8, 9, (2048, 2048), dtype=np.int32),
                    B=rng.integers(-8, 9, (2048, 2048), dtype=np.int32))
    if name == "dense_65536":
        rng = np.random.default_rng(3)
        return dict(X=u(rng, -0.5, 0.5, (65536, 4096)), W=u(rng, -0.5, 0.5, (4096, 4096)),
                    b=u(rng, -0.5, 0.5, (4096,)))
    if name == "dense_ragged":
        rng = np.random.default_rng(4)
        return dict(X=u(rng, -1, 1, (1000, 1001)), W=u(rng, -1, 1, (1001, 999)),
                    b=u(rng, -1, 1, (999,)))
    if name == "mlp_2layer":
        rng = np.random.default_rng(4)
        return dict(X=u(rng, -1, 1, (512, 4096)), W1=u(rng, -1, 1, (4096, 11008)),
                    b1=u(rng, -1, 1, (11008,)), W2=u(rng, -1, 1, (11008, 4096)),
                    b2=u(rng, -1, 1, (4096,)))
    raise KeyError(name)
