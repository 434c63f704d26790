"""GPU parity of the 3xTF32 tcgen05 dense kernel against the CPU oracle.

Tolerance (the f32 bar of the path): max|Y_b200 - Y_oracle| <=
1e-4 * sqrt(K) * max|X| * max|W|, checked through the C-ABI.
"""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import dense_device, max_err, ptr, stream_ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, seed, lo=-1.0, hi=1.0):
    rng = np.random.default_rng(seed)
    X = rng.uniform(lo, hi, (M, K)).astype(np.float32)
    W = rng.uniform(lo, hi, (K, N)).astype(np.float32)
    b = rng.uniform(lo, hi, (N,)).astype(np.float32)
    return X, W, b


SHAPES = [
    (128, 256, 32),     # exactly one tile, one k-block
    (1, 1, 1),
    (2, 2, 2),
    (7, 9, 13),
    (129, 257, 63),     # one past every tile edge
    (256, 512, 96),     # multiple tiles, 3 k-blocks (ring wrap-around)
    (300, 500, 1001),   # K not a multiple of 4: padded split path
    (1000, 999, 1001),  # the ragged benchmark shape
]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("act", [0, 1])
def test_dense_matches_oracle(cuda, M, N, K, act):
    import torch
    X, W, b = _inputs(M, N, K, seed=M * 7 + N * 3 + K)
    got = dense_device(torch, X, W, b, act=act)
    ref = oracle.dense_f32(X, W, b, act=act)
    bound = oracle.f32_bound(K, X, W)
    assert np.isfinite(got).all()
    assert max_err(got, ref) <= bound, (max_err(got, ref), bound)


def test_matmul_no_bias(cuda):
    import torch
    X, W, _ = _inputs(384, 640, 200, seed=5)
    got = dense_device(torch, X, W, None, act=0)
    ref = oracle.dense_f32(X, W)
    assert max_err(got, ref) <= oracle.f32_bound(200, X, W)


def test_leaky_relu_epilogue(cuda):
    import torch
    X, W, b = _inputs(200, 300, 64, seed=9)
    got = dense_device(torch, X, W, b, act=2, alpha=0.1)
    ref = oracle.dense_f32(X, W, b, act=2, alpha=0.1)
    assert max_err(got, ref) <= oracle.f32_bound(64, X, W)


def test_precision_is_fp32_level(cuda):
    """3xTF32 must be far tighter than 1xTF32: the error against float64 is
    that of an f32 computation, i.e. within a small factor of the reference
    CPU pipeline's own (sequential f32 FMA) error on the same data."""
    import torch
    X, W, b = _inputs(512, 512, 4096, seed=11)
    got = dense_device(torch, X, W, b, act=0)
    exact = X.astype(np.float64) @ W.astype(np.float64) + b
    err = float(np.max(np.abs(got - exact)))
    ref_err = float(np.max(np.abs(oracle.dense_f32(X, W, b, act=0) - exact)))
    # 1xTF32 gives ~1e-2 here; the f32 reference pipeline ~2e-4
    assert err < 1e-3 and err <= 2 * ref_err, (err, ref_err)


def test_relu_nan_and_signed_zero(cuda):
    """arith.maximumf semantics: NaN propagates, -0 becomes +0."""
    import torch
    X = np.zeros((4, 8), np.float32)
    W = np.zeros((8, 8), np.float32)
    b = np.array([np.nan, -0.0, 0.0, -1.0, 1.0, np.inf, -np.inf, 2.5], np.float32)
    got = dense_device(torch, X, W, b, act=1)
    assert np.isnan(got[:, 0]).all()
    assert (got[:, 1] == 0).all() and not np.signbit(got[:, 1]).any()
    np.testing.assert_array_equal(got[:, 2:], np.tile([0, 0, 1, np.inf, 0, 2.5], (4, 1)))


def test_nan_input_propagates(cuda):
    import torch
    X, W, b = _inputs(64, 64, 16, seed=3)
    X[5, 3] = np.nan
    got = dense_device(torch, X, W, b, act=1)
    assert np.isnan(got[5]).all()
    mask = np.ones(64, bool)
    mask[5] = False
    assert np.isfinite(got[mask]).all()


@pytest.mark.parametrize("name", ["matmul_256", "dense_1024", "dense_ragged"])
def test_benchmark_configs(cuda, name):
    import torch
    g = oracle.gen_config_inputs(name)
    if "X" in g:
        X, W, b, act = g["X"], g["W"], g["b"], 1
    else:
        X, W, b, act = g["A"], g["B"], None, 0
    got = dense_device(torch, X, W, b, act=act)
    ref = oracle.dense_f32(X, W, b, act=act)
    assert max_err(got, ref) <= oracle.f32_bound(X.shape[1], X, W)


def test_strided_views(cuda):
    """Row pitches larger than the row length on every operand."""
    import torch
    dev = torch.device("cuda:0")
    M, N, K = 150, 170, 90
    X, W, b = _inputs(M, N, K, seed=21)
    bigX = torch.zeros((M, K + 13), device=dev)
    bigW = torch.zeros((K, N + 5), device=dev)
    bigY = torch.full((M, N + 7), -7.0, device=dev)
    bigX[:, :K] = torch.from_numpy(X).to(dev)
    bigW[:, :N] = torch.from_numpy(W).to(dev)
    tb = torch.from_numpy(b).to(dev)
    L = _native.lib()
    _native.check(L.b200_dense_f32(ptr(bigX), K + 13, ptr(bigW), N + 5, ptr(tb), ptr(bigY), N + 7,
                                   M, N, K, 1, 0.0, stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    out = bigY.cpu().numpy()
    ref = oracle.dense_f32(X, W, b, act=1)
    assert max_err(out[:, :N], ref) <= oracle.f32_bound(K, X, W)
    assert (out[:, N:] == -7.0).all()  # padding columns untouched


def test_k_zero_gives_bias(cuda):
    import torch
    dev = torch.device("cuda:0")
    b = torch.tensor([-1.0, 2.0, -0.0], device=dev)
    Y = torch.full((4, 3), 9.0, device=dev)
    L = _native.lib()
    _native.check(L.b200_dense_f32(None, 0, None, 3, ptr(b), ptr(Y), 3, 4, 3, 0, 1, 0.0,
                                   stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    np.testing.assert_array_equal(Y.cpu().numpy(), np.tile([0.0, 2.0, 0.0], (4, 1)))


def test_host_api_pipelined_slabs(cuda):
    """Host buffers through b200_dense_f32_host with enough rows to run the
    slab pipeline (H2D / compute / D2H overlap)."""
    M, N, K = 4608, 256, 2048
    X, W, b = _inputs(M, N, K, seed=31)
    Y = np.full((M, N), np.nan, np.float32)
    L = _native.lib()
    c = ctypes.c_void_p
    _native.check(L.b200_dense_f32_host(c(X.ctypes.data), K, c(W.ctypes.data), N,
                                        c(b.ctypes.data), c(Y.ctypes.data), N, M, N, K, 1, 0.0, 1))
    ref = oracle.dense_f32(X, W, b, act=1)
    assert max_err(Y, ref) <= oracle.f32_bound(K, X, W)


def test_host_api_staged_pageable_strided(cuda):
    """Pageable X and Y above the staging threshold with row pitches larger
    than the rows: both go through the pinned staging ring (parallel host
    copies), and the padding columns of Y stay untouched."""
    M, N, K, ldx, ldy = 8192, 1024, 640, 700, 1100
    X, W, b = _inputs(M, N, K, seed=37)
    Xs = np.full((M, ldx), 7.0, np.float32)
    Xs[:, :K] = X
    Y = np.full((M, ldy), np.nan, np.float32)
    L = _native.lib()
    c = ctypes.c_void_p
    _native.check(L.b200_dense_f32_host(c(Xs.ctypes.data), ldx, c(W.ctypes.data), N,
                                        c(b.ctypes.data), c(Y.ctypes.data), ldy, M, N, K, 2,
                                        0.05, 1))
    ref = oracle.dense_f32(X, W, b, act=2, alpha=0.05)
    assert max_err(Y[:, :N], ref) <= oracle.f32_bound(K, X, W)
    assert np.isnan(Y[:, N:]).all()


def test_workspace_entry_point(cuda):
    import torch
    dev = torch.device("cuda:0")
    M, N, K = 200, 300, 130
    X, W, b = _inputs(M, N, K, seed=41)
    L = _native.lib()
    nbytes = L.b200_dense_f32_workspace_bytes(M, N, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    tX, tW, tb = (torch.from_numpy(a).to(dev) for a in (X, W, b))
    tY = torch.empty((M, N), device=dev)
    _native.check(L.b200_dense_f32_ws(ptr(tX), K, ptr(tW), N, ptr(tb), ptr(tY), N, M, N, K, 1, 0.0,
                                      ptr(ws), nbytes, stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    ref = oracle.dense_f32(X, W, b, act=1)
    assert max_err(tY.cpu().numpy(), ref) <= oracle.f32_bound(K, X, W)
    # too-small workspace is rejected with a clear error
    with pytest.raises(_native.B200Error, match="workspace"):
        _native.check(L.b200_dense_f32_ws(ptr(tX), K, ptr(tW), N, ptr(tb), ptr(tY), N, M, N, K, 1,
                                          0.0, ptr(ws), nbytes - 1, stream_ptr(torch)))


@pytest.mark.parametrize("name", ["matmul_4096", "matmul_8192"])
def test_large_matmul_sampled_rows(cuda, name):
    """Full-size cfg3 matmul on the GPU; the oracle checks 128 sampled rows
    (each output row depends only on its X row, so sampling is exact)."""
    import torch
    g = oracle.gen_config_inputs(name)
    A, B = g["A"], g["B"]
    got = dense_device(torch, A, B, None, act=0)
    rows = np.random.default_rng(0).choice(A.shape[0], 128, replace=False)
    ref = oracle.dense_f32(A[rows], B)
    err = max_err(got[rows], ref)
    bound = oracle.f32_bound(A.shape[1], A, B)
    assert err <= bound, (err, bound)
    # fp32-level accuracy, not tf32-level
    exact = A[rows].astype(np.float64) @ B.astype(np.float64)
    assert float(np.max(np.abs(got[rows] - exact))) < bound / 10


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (512, 4096, 11008), (100, 50, 1001)])
def test_split_k_matches_unsplit(cuda, M, N, K):
    """Split-K (chosen for few-tile problems) through b200_dense_f32 against
    the GEMM alone on operands split by the public split entry points; both
    within the f32 bound of the oracle."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    assert L.b200_dense_f32_splits(M, N, K) > 1
    X, W, b = _inputs(M, N, K, seed=K)
    got = dense_device(torch, X, W, b, act=1)
    Kp = _native.split_pitch(K)
    tX, tW, tb = (torch.from_numpy(a).to(dev) for a in (X, W, b))
    xhi, xlo = torch.empty((M, Kp), device=dev), torch.empty((M, Kp), device=dev)
    whi, wlo = torch.empty((N, Kp), device=dev), torch.empty((N, Kp), device=dev)
    Y1 = torch.empty((M, N), device=dev)
    s = stream_ptr(torch)
    _native.check(L.b200_tf32_split_rows(ptr(tX), K, M, K, ptr(xhi), ptr(xlo), s))
    _native.check(L.b200_tf32_split_transpose(ptr(tW), N, K, N, ptr(whi), ptr(wlo), s))
    _native.check(L.b200_gemm_tf32x3_presplit(ptr(xhi), ptr(xlo), ptr(whi), ptr(wlo), ptr(tb),
                                              ptr(Y1), N, M, N, K, 1, 0.0, s))
    _native.check(L.b200_stream_sync(s))
    unsplit = Y1.cpu().numpy()
    bound = oracle.f32_bound(K, X, W)
    assert max_err(got, unsplit) <= bound
    ref = oracle.dense_f32(X[:256], W, b, act=1)
    assert max_err(got[:256], ref) <= bound and max_err(unsplit[:256], ref) <= bound


@pytest.mark.parametrize("M,N,K", [(256, 512, 200), (8192, 4096, 512), (1000, 1000, 1000)])
def test_fused_x_split_matches_split_pass(cuda, M, N, K):
    """b200_dense_f32_wsplit (W pre-split; aligned X is read raw as the tf32
    hi operand and only its lo part is written) against the full split pass +
    GEMM on the same operands."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    X, W, b = _inputs(M, N, K, seed=M + K)
    Kp = _native.split_pitch(K)
    tX, tW, tb = (torch.from_numpy(a).to(dev) for a in (X, W, b))
    xhi, xlo = torch.empty((M, Kp), device=dev), torch.empty((M, Kp), device=dev)
    whi, wlo = torch.empty((N, Kp), device=dev), torch.empty((N, Kp), device=dev)
    Y1, Y2 = torch.empty((M, N), device=dev), torch.empty((M, N), device=dev)
    s = stream_ptr(torch)
    _native.check(L.b200_tf32_split_rows(ptr(tX), K, M, K, ptr(xhi), ptr(xlo), s))
    _native.check(L.b200_tf32_split_transpose(ptr(tW), N, K, N, ptr(whi), ptr(wlo), s))
    _native.check(L.b200_gemm_tf32x3_presplit(ptr(xhi), ptr(xlo), ptr(whi), ptr(wlo), ptr(tb),
                                              ptr(Y1), N, M, N, K, 1, 0.0, s))
    _native.check(L.b200_dense_f32_wsplit(ptr(tX), K, ptr(whi), ptr(wlo), ptr(tb), ptr(Y2), N,
                                          M, N, K, 1, 0.0, s))
    _native.check(L.b200_stream_sync(s))
    a, f = Y1.cpu().numpy(), Y2.cpu().numpy()
    if L.b200_dense_f32_splits(M, N, K) == 1:
        # X read raw as the tf32 hi operand == the split's hi: bit-identical
        np.testing.assert_array_equal(a, f)
    else:
        assert max_err(a, f) <= oracle.f32_bound(K, X, W) / 100
    ref = oracle.dense_f32(X[:128], W, b, act=1)
    assert max_err(f[:128], ref) <= oracle.f32_bound(K, X, W)


def test_host_api_sharded_over_two_devices(cuda):
    """One process, rows sharded over 2 GPUs (one host thread each, W and b
    replicated): same result as on one GPU. Skipped with fewer devices."""
    L = _native.lib()
    if L.b200_device_count() < 2:
        pytest.skip("needs 2 GPUs")
    M, N, K = 5001, 384, 1024
    X, W, b = _inputs(M, N, K, seed=77)
    c = ctypes.c_void_p
    Y1 = np.full((M, N), np.nan, np.float32)
    Y2 = np.full((M, N), np.nan, np.float32)
    for Y, ndev in ((Y1, 1), (Y2, 2)):
        _native.check(L.b200_dense_f32_host(c(X.ctypes.data), K, c(W.ctypes.data), N,
                                            c(b.ctypes.data), c(Y.ctypes.data), N, M, N, K, 1,
                                            0.0, ndev))
    bound = oracle.f32_bound(K, X, W)
    assert max_err(Y1, Y2) <= bound
    assert max_err(Y2[-300:], oracle.dense_f32(X[-300:], W, b, act=1)) <= bound


def test_host_api_two_devices_staged_pageable(cuda):
    """Pageable X and Y large enough that each device's shard is staged
    through the runtime's pinned buffers: both device threads use the shared
    host copy pool at the same time. Skipped with fewer than 2 GPUs."""
    L = _native.lib()
    if L.b200_device_count() < 2:
        pytest.skip("needs 2 GPUs")
    M, N, K = 8192, 1024, 1024  # 16 MiB of X and of Y per device
    X, W, b = _inputs(M, N, K, seed=88)
    Y = np.full((M, N), np.nan, np.float32)
    c = ctypes.c_void_p
    _native.check(L.b200_dense_f32_host(c(X.ctypes.data), K, c(W.ctypes.data), N,
                                        c(b.ctypes.data), c(Y.ctypes.data), N, M, N, K, 1, 0.0,
                                        2))
    rows = np.r_[0:200, 4000:4300, 8000:8192]
    assert max_err(Y[rows], oracle.dense_f32(X[rows], W, b, act=1)) <= oracle.f32_bound(K, X, W)
    assert np.isfinite(Y).all()


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4096, 1, 4096), (8, 8, 16384),
                                   (65536, 8, 32), (3, 2050, 7), (512, 512, 16384)])
def test_edge_shapes(cuda, M, N, K):
    """Single rows / columns, very long K with tiny M and N (split-K at its
    cap), tall-skinny and wide-short shapes."""
    import torch
    X, W, b = _inputs(M, N, K, seed=M + 3 * N + 7 * K)
    got = dense_device(torch, X, W, b, act=1)
    rows = np.arange(M) if M <= 2048 else np.random.default_rng(0).choice(M, 2048, replace=False)
    ref = oracle.dense_f32(X[rows], W, b, act=1)
    bound = oracle.f32_bound(K, X, W)
    assert np.isfinite(got).all()
    assert max_err(got[rows], ref) <= bound
    exact = np.maximum(X[rows].astype(np.float64) @ W.astype(np.float64) + b, 0)
    assert float(np.max(np.abs(got[rows] - exact))) <= bound / 10  # f32-level


# N % 32 == 0 (the MN-major path's condition) with M and K tails, fewer than
# 256 columns, unaligned X rows (K odd: X split path) and split-K.
_WMN_SHAPES = [(512, 512, 4096), (300, 1024, 1001), (1000, 992, 999), (517, 32, 64),
               (512, 11008, 4096), (129, 288, 16), (77, 4096, 37)]


def _wmn_outputs(torch):
    outs = []
    for (M, N, K) in _WMN_SHAPES:
        X, W, b = _inputs(M, N, K, seed=N + K)
        outs.append(dense_device(torch, X, W, b, act=1))
    return outs


def test_w_mn_major_matches_k_major(cuda, tmp_path):
    """The default B operand is the raw row-major W read MN-major (plus a
    row-major lo part); B200_W_MN=0 (child process) selects the transposed
    K-major split. Same tf32 operands, same MMA order: bit-identical output,
    across column-block tails, K tails, unaligned X rows (X split path)
    and split-K."""
    import os
    import subprocess
    import sys
    import torch
    from conftest import PKG_PARENT, ROOT
    out = str(tmp_path / "kmajor.npz")
    script = r"""
import sys, numpy as np, torch
sys.path[:0] = sys.argv[1:4]
import test_gpu_dense as t
np.savez(sys.argv[4], *t._wmn_outputs(torch))
print("ok")
"""
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    mine = _wmn_outputs(torch)
    # B200_W_MN=0: transposed K-major split
    for var in ({"B200_W_MN": "0"},):
        env = dict(os.environ, **var)
        r = subprocess.run([sys.executable, "-c", script, ROOT, PKG_PARENT, tests_dir, out],
                           env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]
        ref = np.load(out)
        for i, (got, shape) in enumerate(zip(mine, _WMN_SHAPES)):
            np.testing.assert_array_equal(got, ref[f"arr_{i}"], err_msg=f"{var} {shape}")
    M, N, K = _WMN_SHAPES[1]
    X, W, b = _inputs(M, N, K, seed=N + K)
    assert max_err(_wmn_outputs(torch)[1], oracle.dense_f32(X, W, b, act=1)) <= \
        oracle.f32_bound(K, X, W)


def test_back_to_back_small_layers_match_synchronised(cuda):
    """Small layers run with programmatic dependent launch (the GEMM's
    prologue overlaps the split pass, the split-K reduction overlaps the GEMM's
    teardown). A chain of dependent layers issued back to back must equal,
    bit for bit, the same chain with a device synchronisation after each
    layer, and stay within the f32 bound of the oracle's chain."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    s = stream_ptr(torch)
    rng = np.random.default_rng(77)
    shapes = [(256, 256, 256), (256, 512, 256), (256, 256, 512), (256, 1024, 256),
              (256, 256, 1024)] * 2 + [(256, 288, 256), (256, 256, 288)]
    Ws = [(rng.uniform(-1, 1, (K, N)) / np.sqrt(K)).astype(np.float32) for (_, N, K) in shapes]
    bs = [rng.uniform(-0.1, 0.1, (N,)).astype(np.float32) for (_, N, _) in shapes]
    X0 = rng.uniform(-1, 1, (256, 256)).astype(np.float32)
    tW = [torch.from_numpy(w).to(dev) for w in Ws]
    tb = [torch.from_numpy(b).to(dev) for b in bs]

    def chain(sync):
        h = torch.from_numpy(X0).to(dev)
        for (M, N, K), w, b in zip(shapes, tW, tb):
            y = torch.empty((M, N), device=dev)
            _native.check(L.b200_dense_f32(ptr(h), K, ptr(w), N, ptr(b), ptr(y), N, M, N, K, 1,
                                           0.0, s))
            if sync:
                _native.check(L.b200_stream_sync(s))
            h = y
        _native.check(L.b200_stream_sync(s))
        return h.cpu().numpy()

    a, b = chain(False), chain(True)
    np.testing.assert_array_equal(a, b)
    h = X0
    for w, bb in zip(Ws, bs):
        h = oracle.dense_f32(h, w, bb, act=1)
    assert max_err(a, h) <= 1e-4 * len(shapes)


def test_whole_and_cut_tiles_in_one_call(cuda):
    """156 output tiles on 148 SMs: one whole wave runs over all of K and the
    8 tiles of the partial wave are cut into K pieces (tile-local partial sums,
    reduced in piece order). Every element, of both kinds of tile, against
    the oracle; the call is deterministic."""
    import torch
    M, N, K = 128 * 13, 256 * 12, 2048
    assert _native.lib().b200_dense_f32_splits(M, N, K) > 1
    X, W, b = _inputs(M, N, K, seed=156)
    got = dense_device(torch, X, W, b, act=1)
    assert max_err(got, oracle.dense_f32(X, W, b, act=1)) <= oracle.f32_bound(K, X, W)
    np.testing.assert_array_equal(got, dense_device(torch, X, W, b, act=1))


@pytest.mark.parametrize("K", [1001, 1004, 1005, 1008, 12, 3])
def test_split_buffers_use_the_32_byte_row_pitch(cuda, K):
    """b200_tf32_split_rows / _transpose write rows of split_pitch(K) = K
    rounded up to 8 floats: pad columns zero, nothing past M * pitch (canary
    words after the buffer stay untouched), and hi + lo is x to 2^-21."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    s = stream_ptr(torch)
    M, N = 37, 29
    kp = _native.split_pitch(K)
    assert kp % 8 == 0 and K <= kp < K + 8
    X, W, _ = _inputs(M, N, K, seed=K)
    tX, tW = torch.from_numpy(X).to(dev), torch.from_numpy(W).to(dev)
    canary = 64
    for rows, call in ((M, lambda hi, lo: L.b200_tf32_split_rows(ptr(tX), K, M, K, ptr(hi),
                                                                   ptr(lo), s)),
                       (N, lambda hi, lo: L.b200_tf32_split_transpose(ptr(tW), N, K, N, ptr(hi),
                                                                        ptr(lo), s))):
        hi = torch.full((rows * kp + canary,), 5.0, device=dev)
        lo = torch.full((rows * kp + canary,), 5.0, device=dev)
        _native.check(call(hi, lo))
        _native.check(L.b200_stream_sync(s))
        h, l = hi.cpu().numpy(), lo.cpu().numpy()
        assert (h[rows * kp:] == 5.0).all() and (l[rows * kp:] == 5.0).all()
        h, l = h[:rows * kp].reshape(rows, kp), l[:rows * kp].reshape(rows, kp)
        assert (h[:, K:] == 0).all() and (l[:, K:] == 0).all()
        src = (X if rows == M else W.T).astype(np.float64)
        # lo is the remainder truncated to tf32: hi + lo is x to 2^-21 relative
        err = np.abs(h[:, :K].astype(np.float64) + l[:, :K] - src)
        assert (err <= np.abs(src) * 2.0 ** -21).all()


def test_split_rule_for_exact_and_non_finite_values(cuda):
    """tf32 split: zero -> (0, 0); a non-zero value exactly representable in
    tf32, and +-Inf -> lo = +-FLT_MIN with the value's sign (so that Inf times
    an exact partner stays Inf); NaN -> hi NaN, lo 0; otherwise hi + lo is x
    to within 2^-21 relative."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    tiny = np.float32(np.finfo(np.float32).tiny)
    x = np.array([[0.0, -0.0, 1.0, -0.5, 3.0, np.inf, -np.inf, np.nan,
                   0.1, -1.2345678, 7.0e-3, 1.0e30]], np.float32)
    tX = torch.from_numpy(x).to(dev)
    kp = _native.split_pitch(12)  # output row pitch
    hi, lo = torch.empty((1, kp), device=dev), torch.empty((1, kp), device=dev)
    _native.check(L.b200_tf32_split_rows(ptr(tX), 12, 1, 12, ptr(hi), ptr(lo), stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    h, l = hi.cpu().numpy()[0, :12], lo.cpu().numpy()[0, :12]
    assert (l[:2] == 0).all() and (h[:2] == 0).all()
    np.testing.assert_array_equal(l[2:7], [tiny, -tiny, tiny, tiny, -tiny])
    np.testing.assert_array_equal(h[2:7], x[0, 2:7])
    assert np.isnan(h[7]) and l[7] == 0
    v = x[0, 8:].astype(np.float64)
    assert np.all(np.abs(h[8:].astype(np.float64) + l[8:] - v) <= np.abs(v) * 2.0 ** -21)


@pytest.mark.parametrize("M,N,K", [(64, 64, 32), (300, 257, 100)])
def test_inf_and_nan_inputs_follow_f32(cuda, M, N, K):
    """Inf and NaN in X and W give the f32 result class of the reference's
    FMA chain element by element: Inf * exact values (1.0, 0.5) and Inf * Inf
    stay +-Inf, Inf * 0 and Inf - Inf give NaN, and finite outputs agree within
    the f32 bound. N = 64 reads W MN-major, N = 257 the K-major split."""
    import torch
    rng = np.random.default_rng(M + N)
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = rng.choice(np.array([1.0, 0.5, -2.0, 0.0, 0.3], np.float32), (K, N))
    X[3, 5] = np.inf
    X[7, 1] = -np.inf
    X[7, 2] = np.inf        # row 7: +Inf and -Inf terms
    X[9, 4] = np.nan
    X[11, :] = 0.0
    W[6, 10] = np.inf       # column 10: Inf weight
    W[8, 12] = -np.inf
    b = rng.uniform(-1, 1, N).astype(np.float32)
    got = dense_device(torch, X, W, b, act=0)
    ref = oracle.dense_f32(X, W, b, act=0)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_array_equal(np.isposinf(got), np.isposinf(ref))
    np.testing.assert_array_equal(np.isneginf(got), np.isneginf(ref))
    fin = np.isfinite(ref)
    assert np.isinf(ref).any() and np.isnan(ref).any()
    Xf, Wf = np.nan_to_num(X, posinf=0, neginf=0), np.nan_to_num(W, posinf=0, neginf=0)
    assert max_err(got[fin], ref[fin]) <= oracle.f32_bound(K, Xf, Wf)


@pytest.mark.parametrize("M,K,N1,N2", [(300, 1001, 512, 256), (5000, 512, 260, 128),
                                       (129, 256, 1024, 64), (64, 96, 4, 32)])
def test_chained_layers_match_separate_calls(cuda, M, K, N1, N2):
    """b200_dense_f32_chain: layer 1's epilogue also stores H's tf32 lo part,
    and layer 2 reads it instead of splitting H again. H, the lo part and Y
    equal the unchained calls and a separate split of H bit for bit, across
    the MN-major and K-major B paths, an unaligned first-layer X (K odd: full
    split), a 4-column layer and cut tiles (lo written by the piece
    reduction)."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    s = stream_ptr(torch)
    X, W1, b1 = _inputs(M, N1, K, seed=M + K)
    _, W2, b2 = _inputs(M, N2, N1, seed=N1 + N2)
    tX, tW1, tb1, tW2, tb2 = (torch.from_numpy(a).to(dev) for a in (X, W1, b1, W2, b2))
    n1p = _native.split_pitch(N1)  # the pitch layer 2 reads Hlo with
    H, Hlo = torch.empty((M, N1), device=dev), torch.full((M, n1p), np.nan, device=dev)
    Y = torch.empty((M, N2), device=dev)
    _native.check(L.b200_dense_f32_chain(ptr(tX), K, None, ptr(tW1), N1, ptr(tb1), ptr(H), N1,
                                         ptr(Hlo), n1p, M, N1, K, 1, 0.0, s))
    _native.check(L.b200_dense_f32_chain(ptr(H), N1, ptr(Hlo), ptr(tW2), N2, ptr(tb2), ptr(Y),
                                         N2, None, 0, M, N2, N1, 1, 0.0, s))
    H2, Y2 = torch.empty_like(H), torch.empty_like(Y)
    _native.check(L.b200_dense_f32(ptr(tX), K, ptr(tW1), N1, ptr(tb1), ptr(H2), N1, M, N1, K,
                                   1, 0.0, s))
    _native.check(L.b200_dense_f32(ptr(H2), N1, ptr(tW2), N2, ptr(tb2), ptr(Y2), N2, M, N2, N1,
                                   1, 0.0, s))
    hhi, hlo = torch.empty((M, n1p), device=dev), torch.empty((M, n1p), device=dev)
    _native.check(L.b200_tf32_split_rows(ptr(H2), N1, M, N1, ptr(hhi), ptr(hlo), s))
    _native.check(L.b200_stream_sync(s))
    np.testing.assert_array_equal(H.cpu().numpy(), H2.cpu().numpy())
    np.testing.assert_array_equal(Hlo.cpu().numpy()[:, :N1], hlo.cpu().numpy()[:, :N1])
    np.testing.assert_array_equal(Y.cpu().numpy(), Y2.cpu().numpy())
    if K % 4:  # a pre-split X needs aligned X rows: rejected before any launch
        assert L.b200_dense_f32_chain(ptr(tX), K, ptr(Hlo), ptr(tW1), N1, None, ptr(H), N1,
                                      None, 0, M, N1, K, 0, 0.0, s) == 1


def test_random_shapes_and_pitches_against_oracle(cuda):
    """40 seeded random problems: M, N, K in [1, 700], row pitches above the
    rows (aligned or not), bias present or not, each activation, through
    b200_dense_f32 and b200_dense_f32_chain (which also writes Y's lo part).
    Covers the staged and per-thread epilogue stores at M / N edges, cut
    tiles, both B layouts and the X split variants."""
    import torch
    dev = torch.device("cuda:0")
    L = _native.lib()
    s = stream_ptr(torch)
    rng = np.random.default_rng(2024)
    for case in range(40):
        M, N, K = (int(v) for v in rng.integers(1, 701, 3))
        ldx = K + int(rng.integers(0, 9)) * int(rng.integers(0, 2))
        ldw = N + int(rng.integers(0, 9)) * int(rng.integers(0, 2))
        ldy = N + int(rng.integers(0, 9)) * int(rng.integers(0, 2))
        act, alpha = int(rng.integers(0, 3)), 0.05
        with_b = bool(rng.integers(0, 2))
        X = rng.uniform(-1, 1, (M, ldx)).astype(np.float32)
        W = rng.uniform(-1, 1, (K, ldw)).astype(np.float32)
        b = rng.uniform(-1, 1, N).astype(np.float32) if with_b else None
        tX, tW = torch.from_numpy(X).to(dev), torch.from_numpy(W).to(dev)
        tb = torch.from_numpy(b).to(dev) if with_b else None
        ref = oracle.dense_f32(X[:, :K], W[:, :N], b, act=act, alpha=alpha)
        bound = oracle.f32_bound(K, X[:, :K], W[:, :N])
        for chain in (False, True):
            tY = torch.full((M, ldy), 7.0, device=dev)
            tlo = torch.full((M, N), 9.0, device=dev)
            if chain:
                rc = L.b200_dense_f32_chain(ptr(tX), ldx, None, ptr(tW), ldw, ptr(tb), ptr(tY),
                                            ldy, ptr(tlo), N, M, N, K, act, alpha, s)
            else:
                rc = L.b200_dense_f32(ptr(tX), ldx, ptr(tW), ldw, ptr(tb), ptr(tY), ldy, M, N, K,
                                      act, alpha, s)
            _native.check(rc)
            _native.check(L.b200_stream_sync(s))
            Y = tY.cpu().numpy()
            what = f"case {case}: M={M} N={N} K={K} ld=({ldx},{ldw},{ldy}) act={act} " \
                   f"bias={with_b} chain={chain}"
            assert max_err(Y[:, :N], ref) <= bound, what
            assert (Y[:, N:] == 7.0).all(), what
            if chain:  # the lo part equals a separate split of Y (pitch roundup(N, 8))
                Np = _native.split_pitch(N)
                hi, lo = torch.empty((M, Np), device=dev), torch.empty((M, Np), device=dev)
                _native.check(L.b200_tf32_split_rows(ptr(tY), ldy, M, N, ptr(hi), ptr(lo), s))
                _native.check(L.b200_stream_sync(s))
                np.testing.assert_array_equal(tlo.cpu().numpy(), lo.cpu().numpy()[:, :N], what)
