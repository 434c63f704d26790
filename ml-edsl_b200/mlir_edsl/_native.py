"""ctypes binding of libb200edsl.so (include/b200_edsl.h).

The library is built in-tree (ml-edsl_b200/build.py) and loaded from
ml-edsl_b200/lib/. There is no fallback: if the library is missing or fails
to load, every B200 entry point raises.
"""
import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_PKG_DIR), "lib", "libb200edsl.so")

B200_OK = 0
ERROR_NAMES = {
    1: "B200_ERR_INVALID_ARG",
    2: "B200_ERR_CUDA",
    3: "B200_ERR_DRIVER",
    4: "B200_ERR_NO_DEVICE",
    5: "B200_ERR_DEVICE_TIMEOUT",
    6: "B200_ERR_OUT_OF_MEMORY",
    7: "B200_ERR_TOO_LARGE",
}
ACT_NONE, ACT_RELU, ACT_LEAKY_RELU = 0, 1, 2
REDUCE_SUM, REDUCE_PROD, REDUCE_MAX, REDUCE_MIN = 0, 1, 2, 3

# Every symbol include/b200_edsl.h declares (checked by the CPU test-suite).
EXPORTED_SYMBOLS = [
    "b200_version", "b200_last_error", "b200_last_status", "b200_device_count",
    "b200_launch_count", "b200_set_default_devices", "b200_get_default_devices", "b200_release",
    "b200_dense_f32", "b200_dense_f32_workspace_bytes", "b200_dense_f32_ws",
    "b200_dense_f32_noalloc", "b200_weights_register", "b200_weights_release",
    "b200_weights_device", "b200_dense_f32_splits", "b200_dense_f32_launches", "b200_matmul_i32",
    "b200_bias_act_f32", "b200_act_f32", "b200_bias_add_i32", "b200_stream_sync",
    "b200_tf32_split_rows", "b200_tf32_split_transpose", "b200_gemm_tf32x3_presplit",
    "b200_dense_f32_wsplit",
    "b200_malloc", "b200_free", "b200_memcpy_h2d", "b200_memcpy_d2h",
    "b200_selftest_wait_timeout", "b200_debug_fail_alloc", "b200_debug_schedule", "b200_set_gemm_sm_limit", "b200_dense_f32_chain",
    "b200_dense_f32_peers", "b200_peer_barrier", "b200_dense_f32_multicast",
    "b200_ipc_alloc", "b200_ipc_free", "b200_ipc_open", "b200_ipc_close", "b200_memcpy_d2d_async",
    "b200_host_alloc", "b200_host_free",
    "b200_dense_f32_host", "b200_matmul_i32_host", "b200_bias_act_f32_host",
    "b200_bias_add_i32_host", "b200_act_f32_host",
    "b200_reduce_f32", "b200_reduce_i32", "b200_dot_f32", "b200_dot_i32",
    "b200_reduce_f32_host", "b200_reduce_i32_host", "b200_dot_f32_host", "b200_dot_i32_host",
    "b200_memref_dot_f32", "b200_memref_dot_i32", "b200_memref_sum_f32", "b200_memref_max_f32",
    "b200_memref_min_f32",
    "b200_memref_matmul_f32", "b200_memref_matmul_relu_f32", "b200_memref_dense_f32",
    "b200_memref_dense_relu_f32", "b200_memref_matmul_i32", "b200_memref_dense_i32",
    "b200_memref_bias_add_f32", "b200_memref_bias_relu_f32", "b200_memref_relu_f32",
]

_lib = None


class B200Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code, message):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


def _declare(lib):
    c = ctypes
    i64, i32, f32, vp = c.c_int64, c.c_int, c.c_float, c.c_void_p
    sig = {
        "b200_version": ([], c.c_char_p),
        "b200_last_error": ([], c.c_char_p),
        "b200_last_status": ([], i32),
        "b200_device_count": ([], i32),
        "b200_launch_count": ([], c.c_longlong),
        "b200_set_default_devices": ([i32], i32),
        "b200_get_default_devices": ([], i32),
        "b200_release": ([], i32),
        "b200_dense_f32": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, i32, f32, vp], i32),
        "b200_dense_f32_workspace_bytes": ([i64, i64, i64], i64),
        "b200_dense_f32_ws": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, i32, f32, vp, i64,
                               vp], i32),
        "b200_dense_f32_noalloc": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, i32, f32, vp],
                                   i32),
        "b200_dense_f32_splits": ([i64, i64, i64], i32),
        "b200_weights_register": ([vp, i64, i64, i64, c.c_uint64], i32),
        "b200_weights_release": ([vp], i32),
        "b200_weights_device": ([vp, c.POINTER(vp)], i32),
        "b200_dense_f32_launches": ([i64, i64, i64], i32),
        "b200_matmul_i32": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, vp], i32),
        "b200_bias_act_f32": ([vp, i64, vp, vp, i64, i64, i64, i32, f32, vp], i32),
        "b200_act_f32": ([vp, vp, i64, i32, f32, vp], i32),
        "b200_bias_add_i32": ([vp, i64, vp, vp, i64, i64, i64, vp], i32),
        "b200_stream_sync": ([vp], i32),
        "b200_tf32_split_rows": ([vp, i64, i64, i64, vp, vp, vp], i32),
        "b200_tf32_split_transpose": ([vp, i64, i64, i64, vp, vp, vp], i32),
        "b200_gemm_tf32x3_presplit": ([vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, f32, vp],
                                      i32),
        "b200_dense_f32_wsplit": ([vp, i64, vp, vp, vp, vp, i64, i64, i64, i64, i32, f32, vp],
                                  i32),
        "b200_malloc": ([c.POINTER(vp), i64], i32),
        "b200_selftest_wait_timeout": ([i64, vp], i32),
        "b200_host_alloc": ([c.POINTER(vp), i64], i32),
        "b200_host_free": ([vp], i32),
        "b200_debug_fail_alloc": ([i32], i32),
        "b200_debug_schedule": ([i32, i64, i64, i64, c.POINTER(c.c_int64)], i32),
        "b200_set_gemm_sm_limit": ([i32], i32),
        "b200_dense_f32_chain": ([vp, i64, vp, vp, i64, vp, vp, i64, vp, i64, i64, i64, i64, i32,
                                  f32, vp], i32),
        "b200_dense_f32_peers": ([vp, i64, vp, i64, vp, vp, i64, c.POINTER(vp), i32, i64, i64,
                                  i64, i32, f32, vp], i32),
        "b200_dense_f32_multicast": ([vp, i64, vp, i64, vp, vp, i64, vp, i64, i64, i64, i32,
                                      f32, vp], i32),
        "b200_peer_barrier": ([c.POINTER(vp), i32, i32, c.c_uint32, i64, vp], i32),
        "b200_ipc_alloc": ([c.POINTER(vp), i64, vp], i32),
        "b200_ipc_free": ([vp], i32),
        "b200_ipc_open": ([vp, c.POINTER(vp)], i32),
        "b200_ipc_close": ([vp], i32),
        "b200_memcpy_d2d_async": ([vp, vp, i64, vp], i32),
        "b200_free": ([vp], i32),
        "b200_memcpy_h2d": ([vp, vp, i64], i32),
        "b200_memcpy_d2h": ([vp, vp, i64], i32),
        "b200_dense_f32_host": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, i32, f32, i32],
                                i32),
        "b200_matmul_i32_host": ([vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, i32], i32),
        "b200_bias_act_f32_host": ([vp, i64, vp, vp, i64, i64, i64, i32, f32], i32),
        "b200_bias_add_i32_host": ([vp, i64, vp, vp, i64, i64, i64], i32),
        "b200_act_f32_host": ([vp, vp, i64, i32, f32], i32),
        "b200_reduce_f32": ([vp, i64, i32, f32, vp, vp], i32),
        "b200_reduce_i32": ([vp, i64, i32, c.c_int32, vp, vp], i32),
        "b200_dot_f32": ([vp, vp, i64, vp, vp], i32),
        "b200_dot_i32": ([vp, vp, i64, vp, vp], i32),
        "b200_reduce_f32_host": ([vp, i64, i32, f32, vp], i32),
        "b200_reduce_i32_host": ([vp, i64, i32, c.c_int32, vp], i32),
        "b200_dot_f32_host": ([vp, vp, i64, vp], i32),
        "b200_dot_i32_host": ([vp, vp, i64, vp], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def lib():
    """Returns the loaded library, raising if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"B200 native library not found at {LIB_PATH}; build it with "
                "`python ml-edsl_b200/build.py` (there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        _declare(handle)
        _lib = handle
    return _lib


def check(rc):
    """Raises B200Error for a non-zero status code."""
    if rc != B200_OK:
        raise B200Error(rc, lib().b200_last_error().decode(errors="replace"))


def check_last():
    """Raises if the last void (memref) entry point on this thread failed."""
    check(lib().b200_last_status())


def memref_function(name, nargs):
    """A ctypes function object for a void memref entry point with `nargs`
    flattened descriptor arguments (ptr, ptr, int64...)."""
    return getattr(lib(), name)


def launch_count():
    return int(lib().b200_launch_count())


def split_pitch(K):
    """Row pitch (elements) of the library's tf32 hi/lo split buffers for K
    columns: K rounded up to 8 (32-byte rows), as in csrc/kernels.h."""
    return (K + 7) // 8 * 8


def dense_launches(M, N, K):
    """Kernel launches of one f32 dense layer through b200_dense_f32: one
    split pass (X and W together), the GEMM, and a split-K reduction when the
    problem is split."""
    return int(lib().b200_dense_f32_launches(M, N, K))


def device_count():
    return int(lib().b200_device_count())


def pinned_empty(shape, dtype):
    """An uninitialised numpy array in page-locked memory from the runtime's
    pool; the block returns to the pool when the array (and every view of it)
    is garbage-collected."""
    import weakref
    import numpy as np
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    if nbytes == 0:
        return np.empty(shape, dtype)
    L = lib()
    p = ctypes.c_void_p()
    check(L.b200_host_alloc(ctypes.byref(p), nbytes))
    buf = (ctypes.c_byte * nbytes).from_address(p.value)
    weakref.finalize(buf, L.b200_host_free, ctypes.c_void_p(p.value))
    return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)
