"""GPU parity of the i32 GEMM (tensor-core byte-sliced path, bit-exact modulo
2^32) and the elementwise kernels."""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import ptr, stream_ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _i32_device(torch, A, B, bias=None):
    dev = torch.device("cuda:0")
    tA, tB = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    tb = torch.from_numpy(bias).to(dev) if bias is not None else None
    M, K = A.shape
    N = B.shape[1]
    tC = torch.full((M, N), 12345, dtype=torch.int32, device=dev)
    L = _native.lib()
    _native.check(L.b200_matmul_i32(ptr(tA), K, ptr(tB), N, ptr(tb), ptr(tC), N, M, N, K,
                                    stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    return tC.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (2, 2, 2), (7, 9, 13), (129, 130, 17),
                                   (300, 257, 1000)])
def test_i32_matches_oracle(cuda, M, N, K):
    import torch
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-8, 9, (M, K), dtype=np.int32)
    B = rng.integers(-8, 9, (K, N), dtype=np.int32)
    np.testing.assert_array_equal(_i32_device(torch, A, B), oracle.matmul_i32(A, B))


def test_i32_wraps_mod_2_32(cuda):
    import torch
    rng = np.random.default_rng(1)
    A = rng.integers(-2**31, 2**31, (64, 96), dtype=np.int64).astype(np.int32)
    B = rng.integers(-2**31, 2**31, (96, 80), dtype=np.int64).astype(np.int32)
    bias = rng.integers(-2**31, 2**31, (80,), dtype=np.int64).astype(np.int32)
    np.testing.assert_array_equal(_i32_device(torch, A, B, bias), oracle.matmul_i32(A, B, bias))


def test_i32_2048_config(cuda):
    import torch
    g = oracle.gen_config_inputs("matmul_i32_2048")
    np.testing.assert_array_equal(_i32_device(torch, g["A"], g["B"]),
                                  oracle.matmul_i32(g["A"], g["B"]))


def _full_range(rng, shape):
    return rng.integers(-2**31, 2**31, shape, dtype=np.int64).astype(np.int32)


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (200, 136, 130), (513, 260, 1031),
                                   (64, 64, 9000), (3, 700, 20000)])
def test_i32_full_range_tails_and_split(cuda, M, N, K):
    """Every bit pattern of A and B (the byte planes carry all four bytes),
    M / N tails of the 128 x 128 tile, K tails of the 64-byte stage, and
    K > 8192, which the tensor-core path splits so that no s32 accumulator
    can overflow (partial sums added modulo 2^32)."""
    import torch
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A, B, bias = _full_range(rng, (M, K)), _full_range(rng, (K, N)), _full_range(rng, (N,))
    np.testing.assert_array_equal(_i32_device(torch, A, B, bias), oracle.matmul_i32(A, B, bias))


def test_i32_strided_operands(cuda):
    """Row pitches larger than the rows (lda, ldb, ldc not multiples of 4)."""
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(5)
    M, N, K, lda, ldb, ldc = 150, 90, 77, 81, 93, 95
    Abuf, Bbuf = _full_range(rng, (M, lda)), _full_range(rng, (K, ldb))
    tA, tB = torch.from_numpy(Abuf).to(dev), torch.from_numpy(Bbuf).to(dev)
    tC = torch.full((M, ldc), 7, dtype=torch.int32, device=dev)
    L = _native.lib()
    _native.check(L.b200_matmul_i32(ptr(tA), lda, ptr(tB), ldb, None, ptr(tC), ldc, M, N, K,
                                    stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    C = tC.cpu().numpy()
    np.testing.assert_array_equal(C[:, :N], oracle.matmul_i32(Abuf[:, :K], Bbuf[:, :N]))
    assert (C[:, N:] == 7).all()


def test_i32_host_entry_point(cuda):
    """b200_matmul_i32_host: host buffers, device workspace held by the runtime."""
    rng = np.random.default_rng(9)
    A, B, bias = _full_range(rng, (300, 200)), _full_range(rng, (200, 260)), _full_range(rng, (260,))
    C = np.zeros((300, 260), np.int32)
    L = _native.lib()
    c = ctypes.c_void_p
    _native.check(L.b200_matmul_i32_host(c(A.ctypes.data), 200, c(B.ctypes.data), 260,
                                         c(bias.ctypes.data), c(C.ctypes.data), 260, 300, 260,
                                         200, 1))
    np.testing.assert_array_equal(C, oracle.matmul_i32(A, B, bias))


def test_i32_identity_known_answer(cuda):
    import torch
    I = np.eye(2, dtype=np.int32)
    B = np.array([[5, 6], [7, 8]], np.int32)
    np.testing.assert_array_equal(_i32_device(torch, I, B), B)


@pytest.mark.parametrize("act,alpha", [(0, 0.0), (1, 0.0), (2, 0.01), (2, 0.1)])
@pytest.mark.parametrize("M,N", [(8, 16), (33, 17), (512, 1024)])
def test_bias_act_f32(cuda, act, alpha, M, N):
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(M * N)
    X = rng.standard_normal((M, N)).astype(np.float32)
    X[0, 0] = np.nan
    X[-1, -1] = -0.0
    b = rng.standard_normal(N).astype(np.float32)
    tX, tb = torch.from_numpy(X).to(dev), torch.from_numpy(b).to(dev)
    tY = torch.empty_like(tX)
    L = _native.lib()
    _native.check(L.b200_bias_act_f32(ptr(tX), N, ptr(tb), ptr(tY), N, M, N, act, alpha,
                                      stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    ref = oracle.bias_act_f32(X, b, act, alpha)
    np.testing.assert_array_equal(tY.cpu().numpy(), ref)  # elementwise: bit-exact


def test_act_f32_any_rank(cuda):
    import torch
    dev = torch.device("cuda:0")
    X = np.linspace(-3, 3, 1001, dtype=np.float32)
    tX = torch.from_numpy(X).to(dev)
    tY = torch.empty_like(tX)
    L = _native.lib()
    _native.check(L.b200_act_f32(ptr(tX), ptr(tY), X.size, 1, 0.0, stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    np.testing.assert_array_equal(tY.cpu().numpy(), np.where(X > 0, X, 0).astype(np.float32))


def test_bias_add_i32_host(cuda):
    rng = np.random.default_rng(3)
    X = rng.integers(-2**31, 2**31, (20, 30), dtype=np.int64).astype(np.int32)
    b = rng.integers(-2**31, 2**31, (30,), dtype=np.int64).astype(np.int32)
    Y = np.empty_like(X)
    c = ctypes.c_void_p
    L = _native.lib()
    _native.check(L.b200_bias_add_i32_host(c(X.ctypes.data), 30, c(b.ctypes.data),
                                           c(Y.ctypes.data), 30, 20, 30))
    np.testing.assert_array_equal(Y, (X.astype(np.int64) + b).astype(np.uint32).astype(np.int32)
                                  if False else (X.view(np.uint32) + b.view(np.uint32)).view(np.int32))


def test_staged_copies_round_trip(cuda):
    """b200_memcpy_h2d / _d2h with pageable buffers above the staging
    threshold (several 32 MiB chunks plus a ragged tail) and below it."""
    L = _native.lib()
    c = ctypes.c_void_p
    for nbytes in (100 * (1 << 20) + 12345, 1000):
        src = np.random.default_rng(nbytes).integers(0, 256, nbytes, dtype=np.uint8)
        dst = np.zeros(nbytes, np.uint8)
        d = c()
        _native.check(L.b200_malloc(ctypes.byref(d), nbytes))
        try:
            _native.check(L.b200_memcpy_h2d(d, c(src.ctypes.data), nbytes))
            _native.check(L.b200_memcpy_d2h(c(dst.ctypes.data), d, nbytes))
        finally:
            _native.check(L.b200_free(d))
        np.testing.assert_array_equal(dst, src)


def test_act_f32_host_staged(cuda):
    """A pageable 64 MiB tensor through the host elementwise entry point."""
    L = _native.lib()
    x = np.random.default_rng(5).standard_normal(1 << 24).astype(np.float32)
    y = np.full_like(x, np.nan)
    _native.check(L.b200_act_f32_host(ctypes.c_void_p(x.ctypes.data),
                                      ctypes.c_void_p(y.ctypes.data), x.size, 1, 0.0))
    np.testing.assert_array_equal(y, np.maximum(x, 0) + 0.0)


def test_i32_random_shapes_and_pitches(cuda):
    """30 seeded random i32 problems (M, N, K in [1, 600], full-range values,
    row pitches above the rows, bias or not): bit-exact against the oracle,
    padding columns untouched. Covers the staged and per-thread epilogue
    stores at M / N edges."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    s = stream_ptr(torch)
    rng = np.random.default_rng(77)
    for case in range(30):
        M, N, K = (int(v) for v in rng.integers(1, 601, 3))
        lda, ldb, ldc = (d + int(rng.integers(0, 6)) for d in (K, N, N))
        A, B = _full_range(rng, (M, lda)), _full_range(rng, (K, ldb))
        bias = _full_range(rng, (N,)) if rng.integers(0, 2) else None
        tA, tB = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
        tb = torch.from_numpy(bias).to(dev) if bias is not None else None
        tC = torch.full((M, ldc), 13, dtype=torch.int32, device=dev)
        _native.check(L.b200_matmul_i32(ptr(tA), lda, ptr(tB), ldb, ptr(tb), ptr(tC), ldc, M, N,
                                        K, s))
        _native.check(L.b200_stream_sync(s))
        C = tC.cpu().numpy()
        what = f"case {case}: M={M} N={N} K={K} ld=({lda},{ldb},{ldc}) bias={bias is not None}"
        np.testing.assert_array_equal(C[:, :N], oracle.matmul_i32(A[:, :K], B[:, :N], bias), what)
        assert (C[:, N:] == 13).all(), what
