"""Helpers for the GPU parity tests: call the C-ABI on torch device memory."""
import ctypes

import numpy as np

from mlir_edsl import _native


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream_ptr(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dense_device(torch, X, W, b=None, act=0, alpha=0.0):
    """Runs b200_dense_f32 on device copies of numpy inputs; returns numpy."""
    dev = torch.device("cuda:0")
    tX = torch.from_numpy(np.ascontiguousarray(X)).to(dev)
    tW = torch.from_numpy(np.ascontiguousarray(W)).to(dev)
    tb = torch.from_numpy(np.ascontiguousarray(b)).to(dev) if b is not None else None
    M, K = X.shape
    N = W.shape[1]
    tY = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
    L = _native.lib()
    _native.check(L.b200_dense_f32(ptr(tX), K, ptr(tW), N, ptr(tb), ptr(tY), N, M, N, K, act,
                                   alpha, stream_ptr(torch)))
    _native.check(L.b200_stream_sync(stream_ptr(torch)))
    return tY.cpu().numpy()


def max_err(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64)))) if a.size else 0.0
