"""GPU tests of the host runtime's concurrency rules: two host threads issuing
device-pointer calls on the same stream share that stream's scratch buffer,
which grows (drain the stream, free, allocate) when a larger problem comes
along. A growing thread must never free the buffer while the other thread is
still queueing kernels that use it."""
import ctypes
import threading

import numpy as np
import pytest

from gpu_util import ptr
from mlir_edsl import _native

pytestmark = pytest.mark.gpu


def test_two_threads_one_stream_growing_scratch(cuda):
    import torch
    L = _native.lib()
    L.b200_release()  # start from empty scratch so that every size step grows it
    K, N = 512, 384
    sizes = [64, 96, 160, 256, 384, 640, 1024, 1536, 2304, 3456]
    rng = np.random.default_rng(3)
    W = torch.from_numpy(rng.uniform(-1, 1, (K, N)).astype(np.float32)).to(cuda)
    b = torch.from_numpy(rng.uniform(-1, 1, (N,)).astype(np.float32)).to(cuda)
    X = {t: [torch.from_numpy(rng.uniform(-1, 1, (m, K)).astype(np.float32)).to(cuda)
             for m in sizes] for t in range(2)}
    Y = {t: [torch.full((m, N), float("nan"), device=cuda) for m in sizes] for t in range(2)}
    torch.cuda.synchronize()
    errors = []

    def worker(t):
        try:
            torch.cuda.set_device(cuda)
            order = sizes if t == 0 else sizes[::-1][::2] + sizes[::-1][1::2]
            for m in order:
                i = sizes.index(m)
                # stream NULL: both threads share the legacy default stream
                _native.check(L.b200_dense_f32(ptr(X[t][i]), K, ptr(W), N, ptr(b), ptr(Y[t][i]),
                                               N, m, N, K, 1, 0.0, None))
        except Exception as e:  # pragma: no cover - reported below
            errors.append(repr(e))

    for _ in range(3):
        th = [threading.Thread(target=worker, args=(t,)) for t in range(2)]
        for x in th:
            x.start()
        for x in th:
            x.join()
        _native.check(L.b200_stream_sync(None))
    assert not errors, errors
    # the same calls one at a time give bit-identical rows
    for t in range(2):
        for i, m in enumerate(sizes):
            ref = torch.empty((m, N), device=cuda)
            _native.check(L.b200_dense_f32(ptr(X[t][i]), K, ptr(W), N, ptr(b), ptr(ref), N, m, N,
                                           K, 1, 0.0, None))
            _native.check(L.b200_stream_sync(None))
            assert torch.equal(ref, Y[t][i]), (t, m)
