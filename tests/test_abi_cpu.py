"""The C-ABI library without a GPU: it loads, exports every function
include/*.h declares, validates arguments, and fails loudly (no fallback)."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from conftest import HAS_GPU, ROOT
from mlir_edsl import _native

HEADERS = glob.glob(os.path.join(ROOT, "include", "*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"#define[^\n]*(\\\n[^\n]*)*", "", src)
        for m in re.finditer(r"\b(b200_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert "b200_dense_f32" in names and "b200_memref_dense_relu_f32" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert declared_functions() == set(_native.EXPORTED_SYMBOLS)


def test_version_and_counters():
    lib = _native.lib()
    assert b"sm_100a" in lib.b200_version()
    assert lib.b200_launch_count() >= 0


def test_split_pitch_agrees_with_the_library():
    """The frontend sizes chained layers' lo buffers with _native.split_pitch;
    the library's scratch formula must use the same pitch (K rounded up to 8)
    for every K residue."""
    lib = _native.lib()
    al = lambda b: (b + 255) // 256 * 256
    M, N = 8192, 8192  # many tiles: no split-K partials in the formula
    for K in range(1001, 1017):
        kp = _native.split_pitch(K)
        assert kp % 8 == 0 and K <= kp < K + 8
        assert lib.b200_dense_f32_splits(M, N, K) == 1
        assert lib.b200_dense_f32_workspace_bytes(M, N, K) == 2 * al(M * kp * 4) + 2 * al(N * kp * 4)


def test_workspace_formula():
    lib = _native.lib()
    al = lambda b: (b + 255) // 256 * 256
    # many tiles: no split-K, scratch = the four split operands
    M, N, K = 8192, 8192, 1001
    Kp = 1008  # split rows are K rounded up to 8 floats
    assert lib.b200_dense_f32_splits(M, N, K) == 1
    assert lib.b200_dense_f32_workspace_bytes(M, N, K) == 2 * al(M * Kp * 4) + 2 * al(N * Kp * 4)
    # one tile, long K: the tile is cut into K pieces whose raw sums are kept
    # tile-local (128 x 256 floats per piece)
    M, N, K = 100, 50, 1001
    s = lib.b200_dense_f32_splits(M, N, K)
    assert 1 < s <= 16
    assert lib.b200_dense_f32_workspace_bytes(M, N, K) == (
        2 * al(M * Kp * 4) + 2 * al(N * Kp * 4) + al(s * 128 * 256 * 4))
    assert lib.b200_dense_f32_workspace_bytes(-1, 2, 3) == -1


@pytest.mark.parametrize("M,N,K,splits", [(8192, 8192, 8192, 1), (65536, 4096, 4096, 1),
                                          (1024, 1024, 1024, 4), (64, 80, 96, 1)])
def test_split_k_choice(M, N, K, splits):
    assert _native.lib().b200_dense_f32_splits(M, N, K) == splits


def test_invalid_arguments_rejected_before_device_use():
    lib = _native.lib()
    rc = lib.b200_dense_f32(None, 4, None, 4, None, None, 4, -1, 4, 4, 1, 0.0, None)
    assert rc == 1 and b"negative" in lib.b200_last_error()
    rc = lib.b200_dense_f32_host(None, 4, None, 4, None, None, 4, 4, 4, 4, 7, 0.0, 1)
    assert rc == 1 and b"activation" in lib.b200_last_error()
    assert lib.b200_set_default_devices(0) == 1
    assert lib.b200_set_default_devices(1) == 0 and lib.b200_get_default_devices() == 1


def test_memref_entry_rejects_strided_innermost():
    lib = _native.lib()
    fn = lib.b200_memref_relu_f32
    X = np.ones((2, 4), np.float32)
    Y = np.empty((2, 4), np.float32)
    vp = ctypes.c_void_p
    i64 = ctypes.c_int64
    fn.argtypes = [vp, vp, i64, i64, i64, i64, i64] * 2
    fn.restype = None
    fn(vp(X.ctypes.data), vp(X.ctypes.data), 0, 2, 2, 4, 2,   # innermost stride 2
       vp(Y.ctypes.data), vp(Y.ctypes.data), 0, 2, 4, 4, 1)
    assert lib.b200_last_status() == 1
    assert b"innermost stride" in lib.b200_last_error()


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device error path")
def test_no_device_fails_loudly():
    lib = _native.lib()
    assert lib.b200_device_count() == 0
    X = np.ones((4, 4), np.float32)
    c = ctypes.c_void_p(X.ctypes.data)
    rc = lib.b200_dense_f32_host(c, 4, c, 4, None, c, 4, 4, 4, 4, 1, 0.0, 1)
    assert rc == 4 and b"no CUDA device" in lib.b200_last_error()
    assert lib.b200_dense_f32_noalloc(c, 4, c, 4, None, c, 4, 4, 4, 4, 1, 0.0, None) == 4


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device error path")
def test_frontend_has_no_cpu_fallback():
    from mlir_edsl import Tensor, f32, ml_function, relu

    @ml_function(target="b200")
    def dense(X: Tensor[f32, 4, 4], W: Tensor[f32, 4, 4], b: Tensor[f32, 4]) -> Tensor[f32, 4, 4]:
        return relu(X @ W + b)
    with pytest.raises(_native.B200Error, match="NO_DEVICE"):
        dense(np.ones((4, 4), np.float32), np.ones((4, 4), np.float32), np.ones(4, np.float32))

    @ml_function(target="b200")
    def net(X: Tensor[f32, 4, 4], W: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        return relu(relu(X @ W) @ W)
    with pytest.raises(_native.B200Error, match="NO_DEVICE"):
        net(np.ones((4, 4), np.float32), np.ones((4, 4), np.float32))


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _native.lib()


def _schedule(kind, M, N, K):
    out = (ctypes.c_int64 * 8)()
    assert _native.lib().b200_debug_schedule(kind, M, N, K, out) == 0
    keys = ("tiles_m", "tiles_n", "whole", "rest", "pieces", "kb", "kbp", "units")
    return dict(zip(keys, list(out)))



@settings(max_examples=300, deadline=None)
@given(kind=st.sampled_from([0, 1]), M=st.integers(1, 70000), N=st.integers(1, 20000),
       K=st.integers(1, 40000))
def test_schedule_invariants(kind, M, N, K):
    """The persistent GEMMs' work schedule (host logic, no GPU): every tile
    is covered once, whole tiles fill whole waves of the 148 SMs, a cut tile's
    pieces are non-empty and cover its K range exactly, an f32 piece spans at
    least one 128-wide K chunk, and no i32 unit covers more than 8192 bytes of
    K (so its s32 accumulators cannot overflow)."""
    s = _schedule(kind, M, N, K)
    bm, bn, bk = (128, 256, 16) if kind == 0 else (128, 128, 64)
    cdiv = lambda a, b: -(-a // b)
    assert s["tiles_m"] == cdiv(M, bm) and s["tiles_n"] == cdiv(N, bn)
    assert s["kb"] == cdiv(K, bk)
    tiles = s["tiles_m"] * s["tiles_n"]
    assert s["whole"] + s["rest"] == tiles
    assert s["units"] == s["whole"] + s["rest"] * s["pieces"]
    if s["rest"] == 0:
        assert s["pieces"] == 1 and s["kbp"] == s["kb"]
    else:
        assert s["pieces"] >= 2
        assert (s["pieces"] - 1) * s["kbp"] < s["kb"] <= s["pieces"] * s["kbp"]
        assert s["whole"] % 148 == 0
        if kind == 0:
            assert s["kbp"] >= 128 // bk
    if kind == 1:
        assert (s["kbp"] if s["rest"] else s["kb"]) * bk <= 8192


def test_schedule_examples():
    """The f32 dense layer: 65536 x 4096 x 4096 runs whole (55 full waves and a
    52-tile tail not worth cutting); 1024^3 cuts its 32 tiles into 4 pieces;
    the MLP's 172-tile layer runs one whole wave and cuts the other 24 tiles.
    i32 at 64 x 64 x 20000 cuts every tile (K over 8192 bytes)."""
    s = _schedule(0, 65536, 4096, 4096)
    assert (s["whole"], s["rest"]) == (8192, 0)
    s = _schedule(0, 1024, 1024, 1024)
    assert (s["whole"], s["rest"], s["pieces"]) == (0, 32, 4)
    s = _schedule(0, 512, 11008, 4096)
    assert (s["whole"], s["rest"]) == (148, 24) and s["pieces"] > 1
    s = _schedule(1, 64, 64, 20000)
    assert s["whole"] == 0 and s["pieces"] >= 3
    assert _native.lib().b200_debug_schedule(2, 1, 1, 1, (ctypes.c_int64 * 8)()) == 1


def test_weights_register_validation_without_a_gpu():
    """Registration is host bookkeeping: argument checks, idempotent
    re-registration and release need no device."""
    import ctypes
    import numpy as np
    lib = _native.lib()
    W = np.zeros((8, 4), np.float32)
    p = ctypes.c_void_p(W.ctypes.data)
    assert lib.b200_weights_register(None, 4, 8, 4, 0) == 1
    assert lib.b200_weights_register(p, 3, 8, 4, 0) == 1  # ldw < N
    assert lib.b200_weights_register(p, 4, 8, 4, 0) == 0
    assert lib.b200_weights_register(p, 4, 8, 4, 0) == 0
    assert lib.b200_weights_register(p, 4, 8, 4, 1) == 0
    assert lib.b200_weights_release(p) == 0
    assert lib.b200_weights_release(p) == 1 and b"not registered" in lib.b200_last_error()
