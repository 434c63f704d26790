"""Failure detection on the GPU without a GPU fault: a bounded device wait
that runs out is reported as B200_ERR_DEVICE_TIMEOUT and leaves the context
usable; an injected allocation failure surfaces as B200_ERR_OUT_OF_MEMORY and
the next call succeeds."""
import ctypes
import time

import numpy as np
import pytest

import oracle
from gpu_util import dense_device, max_err, stream_ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def test_device_wait_timeout_is_reported_and_context_survives(cuda):
    import torch
    L = _native.lib()
    s = stream_ptr(torch)
    t0 = time.perf_counter()
    _native.check(L.b200_selftest_wait_timeout(50_000_000, s))  # 50 ms, nothing arrives
    rc = L.b200_stream_sync(s)
    elapsed = time.perf_counter() - t0
    assert rc == 5, rc  # B200_ERR_DEVICE_TIMEOUT
    assert b"bounded wait (code 4)" in L.b200_last_error()
    assert 0.04 < elapsed < 5.0
    # the status was read and cleared; the context still computes correctly
    assert L.b200_stream_sync(s) == 0
    rng = np.random.default_rng(0)
    X = rng.uniform(-1, 1, (256, 300)).astype(np.float32)
    W = rng.uniform(-1, 1, (300, 200)).astype(np.float32)
    b = rng.uniform(-1, 1, (200,)).astype(np.float32)
    got = dense_device(torch, X, W, b, act=1)
    assert max_err(got, oracle.dense_f32(X, W, b, act=1)) <= oracle.f32_bound(300, X, W)


def test_injected_allocation_failure(cuda):
    L = _native.lib()
    _native.check(L.b200_release())  # the next host call must allocate again
    rng = np.random.default_rng(1)
    X = rng.uniform(-1, 1, (64, 48)).astype(np.float32)
    W = rng.uniform(-1, 1, (48, 40)).astype(np.float32)
    Y = np.zeros((64, 40), np.float32)
    c = ctypes.c_void_p
    _native.check(L.b200_debug_fail_alloc(1))
    rc = L.b200_dense_f32_host(c(X.ctypes.data), 48, c(W.ctypes.data), 40, None,
                               c(Y.ctypes.data), 40, 64, 40, 48, 0, 0.0, 1)
    assert rc == 6 and b"alloc" in L.b200_last_error()
    rc = L.b200_dense_f32_host(c(X.ctypes.data), 48, c(W.ctypes.data), 40, None,
                               c(Y.ctypes.data), 40, 64, 40, 48, 0, 0.0, 1)
    assert rc == 0
    assert max_err(Y, oracle.dense_f32(X, W)) <= oracle.f32_bound(48, X, W)


def test_release_keeps_the_callers_device(cuda):
    """b200_release visits every initialised device; afterwards the calling
    thread must still be on its own device (a device-pointer call that
    followed on another GPU would read this GPU's buffers from the wrong
    device). With 2 GPUs, a sharded host call first initialises device 1."""
    import torch
    L = _native.lib()
    c = ctypes.c_void_p
    if L.b200_device_count() >= 2:
        X = np.ones((64, 48), np.float32)
        W = np.ones((48, 40), np.float32)
        Y = np.zeros((64, 40), np.float32)
        _native.check(L.b200_dense_f32_host(c(X.ctypes.data), 48, c(W.ctypes.data), 40, None,
                                            c(Y.ctypes.data), 40, 64, 40, 48, 0, 0.0, 2))
        assert (Y == 48).all()
    before = torch.cuda.current_device()
    _native.check(L.b200_release())
    assert torch.cuda.current_device() == before


def _flag_arrays(torch, world):
    """`world` zeroed flag arrays on this GPU standing in for every rank's."""
    fl = torch.zeros((world, 8), dtype=torch.int32, device="cuda:0")
    ptrs = (ctypes.c_void_p * world)(*[fl[r].data_ptr() for r in range(world)])
    return fl, ptrs


def test_peer_barrier_signals_every_peer_and_passes(cuda):
    """One GPU plays rank 1 of 3: the peers' arrivals are already in its own
    flag array, so the barrier passes at once; it stores its epoch into its
    slot of each peer's array and leaves its own slot alone."""
    import torch
    L = _native.lib()
    s = stream_ptr(torch)
    fl, ptrs = _flag_arrays(torch, 3)
    fl[1, 0] = 7
    fl[1, 2] = 8  # a later epoch also counts as reached
    _native.check(L.b200_peer_barrier(ptrs, 3, 1, 7, 1_000_000_000, s))
    assert L.b200_stream_sync(s) == 0
    got = fl.cpu().numpy()
    assert got[0, 1] == 7 and got[2, 1] == 7 and got[1, 1] == 0
    # a lone rank has nobody to wait for
    _native.check(L.b200_peer_barrier(ptrs, 1, 0, 1, 1_000_000, s))
    assert L.b200_stream_sync(s) == 0


def test_peer_barrier_timeout_is_reported_and_context_survives(cuda):
    """Rank 0 of 2 whose peer never arrives (a flag that nothing sets): the
    wait gives up after 50 ms with B200_ERR_DEVICE_TIMEOUT, and the context
    keeps working."""
    import torch
    L = _native.lib()
    s = stream_ptr(torch)
    fl, ptrs = _flag_arrays(torch, 2)
    t0 = time.perf_counter()
    _native.check(L.b200_peer_barrier(ptrs, 2, 0, 1, 50_000_000, s))
    rc = L.b200_stream_sync(s)
    elapsed = time.perf_counter() - t0
    assert rc == 5 and b"code 5" in L.b200_last_error(), (rc, L.b200_last_error())
    assert 0.04 < elapsed < 5.0
    assert int(fl[1, 0].item()) == 1  # it did signal its peer
    assert L.b200_stream_sync(s) == 0
    rng = np.random.default_rng(2)
    X = rng.uniform(-1, 1, (200, 64)).astype(np.float32)
    W = rng.uniform(-1, 1, (64, 96)).astype(np.float32)
    got = dense_device(torch, X, W, None, act=0)
    assert max_err(got, oracle.dense_f32(X, W)) <= oracle.f32_bound(64, X, W)
    with pytest.raises(_native.B200Error):
        _native.check(L.b200_peer_barrier(ptrs, 9, 0, 1, 1000, s))
