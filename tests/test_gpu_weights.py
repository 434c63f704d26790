"""Weight cache (b200_weights_register): a registered W keeps its device copy
and its tf32 split on the GPU between host calls. Results are bit-identical
to calls that copy and split W every time (the split is the same values),
a new version of W is picked up, and a released W falls back to per-call
copies."""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import max_err, ptr, stream_ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu
c = ctypes.c_void_p


def _host_dense(X, W, b, act=1):
    M, K = X.shape
    N = W.shape[1]
    Y = np.full((M, N), np.nan, np.float32)
    _native.check(_native.lib().b200_dense_f32_host(c(X.ctypes.data), K, c(W.ctypes.data), N,
                                                    c(b.ctypes.data), c(Y.ctypes.data), N, M, N,
                                                    K, act, 0.0, 1))
    return Y


# MN-major B (M <= 4096, N % 32 == 0), K-major B (M > 4096; N % 32 != 0),
# and enough rows for several pipelined slabs
@pytest.mark.parametrize("M,N,K", [(512, 1024, 768), (8192, 256, 512), (700, 999, 1001),
                                   (4608, 512, 2048)])
def test_registered_weights_are_bit_identical_and_track_versions(cuda, M, N, K):
    L = _native.lib()
    rng = np.random.default_rng(M + N + K)
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b = rng.uniform(-1, 1, (N,)).astype(np.float32)
    plain = _host_dense(X, W, b)
    _native.check(L.b200_weights_register(c(W.ctypes.data), N, K, N, 1))
    try:
        first = _host_dense(X, W, b)   # uploads and splits W
        second = _host_dense(X, W, b)  # reuses both
        np.testing.assert_array_equal(first, plain)
        np.testing.assert_array_equal(second, plain)
        # the same version again keeps the copy; a new version is re-read
        W *= -0.5
        _native.check(L.b200_weights_register(c(W.ctypes.data), N, K, N, 1))
        stale = _host_dense(X, W, b)
        np.testing.assert_array_equal(stale, plain)  # the documented contract
        _native.check(L.b200_weights_register(c(W.ctypes.data), N, K, N, 2))
        fresh = _host_dense(X, W, b)
        rows = slice(0, 128)
        assert max_err(fresh[rows], oracle.dense_f32(X[rows], W, b, act=1)) <= \
            oracle.f32_bound(K, X, W)
    finally:
        _native.check(L.b200_weights_release(c(W.ctypes.data)))
    np.testing.assert_array_equal(_host_dense(X, W, b), fresh)  # per-call copies again
    with pytest.raises(_native.B200Error, match="not registered"):
        _native.check(L.b200_weights_release(c(W.ctypes.data)))


def test_registered_weights_device_copy_in_device_calls(cuda):
    """b200_weights_device hands out the kept copy; b200_dense_f32 given it
    reuses the kept split (bit-identical to a plain device call)."""
    import torch
    L = _native.lib()
    M, N, K = 300, 512, 640
    rng = np.random.default_rng(5)
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b = rng.uniform(-1, 1, (N,)).astype(np.float32)
    tX, tW, tb = (torch.from_numpy(a).to(cuda) for a in (X, W, b))
    s = stream_ptr(torch)
    Y1, Y2 = torch.empty((M, N), device=cuda), torch.empty((M, N), device=cuda)
    _native.check(L.b200_dense_f32(ptr(tX), K, ptr(tW), N, ptr(tb), ptr(Y1), N, M, N, K, 1, 0.0,
                                   s))
    _native.check(L.b200_weights_register(c(W.ctypes.data), N, K, N, 0))
    try:
        dW = c()
        _native.check(L.b200_weights_device(c(W.ctypes.data), ctypes.byref(dW)))
        for _ in range(2):
            _native.check(L.b200_dense_f32(ptr(tX), K, dW, N, ptr(tb), ptr(Y2), N, M, N, K, 1,
                                           0.0, s))
            _native.check(L.b200_stream_sync(s))
            assert torch.equal(Y1, Y2)
    finally:
        _native.check(L.b200_weights_release(c(W.ctypes.data)))


def test_frontend_mlp_with_registered_weights(cuda):
    """The 2-layer MLP config through @ml_function with W1 and W2
    registered: same result as unregistered, on repeated calls."""
    from mlir_edsl import Tensor, f32, ml_function, register_weights, relu, release_weights
    g = oracle.gen_config_inputs("mlp_2layer")

    @ml_function(target="b200")
    def mlp(X: Tensor[f32, 512, 4096], W1: Tensor[f32, 4096, 11008], b1: Tensor[f32, 11008],
            W2: Tensor[f32, 11008, 4096], b2: Tensor[f32, 4096]) -> Tensor[f32, 512, 4096]:
        return relu(relu(X @ W1 + b1) @ W2 + b2)

    args = (g["X"], g["W1"], g["b1"], g["W2"], g["b2"])
    plain = np.array(mlp(*args))
    register_weights(g["W1"])
    register_weights(g["W2"])
    try:
        for _ in range(2):
            np.testing.assert_array_equal(np.array(mlp(*args)), plain)
    finally:
        release_weights(g["W1"])
        release_weights(g["W2"])
    with pytest.raises(ValueError):
        release_weights(g["W1"])
