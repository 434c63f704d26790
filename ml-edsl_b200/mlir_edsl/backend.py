"""B200 backend: the drop-in counterpart of the reference's CppMLIRBackend.

Same method names and call shape as the reference (mlir_edsl/backend.py:105-271):
compile_function_from_ast(name, params, return_type, ast_node),
execute_function(name, *args), execute_gpu_function(name, *args),
has_function, list_functions, clear_module, set_optimization_level,
set_target, get_module_ir; get_backend() returns the process-wide instance.

Execution of a compiled plan:
  * a single fused step whose operands are all parameters calls the
    library's memref-descriptor entry point with the reference's flattened
    ctypes ABI (descriptor layout: backend.py:37-102 of the reference;
    output descriptor appended last, void return);
  * multi-step plans (stacked dense layers) run on the device through the
    device-pointer entry points, intermediates never leave HBM;
  * errors surface as the reference's exception types: TypeError for dtype
    mismatches, ValueError for shapes, RuntimeError (B200Error) for device
    failures.
"""
import ctypes
from typing import Dict, List, Tuple, Union

import numpy as np

from . import _native
from .lowering import ACT_LEAKY_RELU, ACT_NONE, ACT_RELU, Plan, Ref, lower
from .types import ScalarType, TensorType, Type

SCALAR_TYPE_TO_NUMPY_DTYPE = {ScalarType.F32: np.float32, ScalarType.I32: np.int32,
                              ScalarType.I1: np.bool_}

try:
    HAS_B200_BACKEND = _native.lib() is not None
except Exception:  # library not built: every call raises through _native.lib()
    HAS_B200_BACKEND = False
HAS_CPP_BACKEND = HAS_B200_BACKEND  # name used by reference-side code

_global_backend = None


def _memref_descriptor(data: np.ndarray, array_type: TensorType):
    """(c_types, c_vals, buffer) of a standard MLIR memref descriptor:
    alloc, aligned, offset, sizes..., strides... (zero-copy)."""
    expected = SCALAR_TYPE_TO_NUMPY_DTYPE[array_type.element_type.kind]
    if data.dtype != expected:
        raise TypeError(f"ndarray dtype {data.dtype} does not match expected {np.dtype(expected)} "
                        f"for {array_type}")
    if not data.flags["C_CONTIGUOUS"]:
        data = np.ascontiguousarray(data)
    ptr = data.ctypes.data_as(ctypes.c_void_p)
    nd = data.ndim
    c_types = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] + [ctypes.c_int64] * (2 * nd)
    c_vals = [ptr, ptr, 0] + list(data.shape) + [s // data.itemsize for s in data.strides]
    return c_types, c_vals, data


# Results of at least this many bytes are returned in page-locked memory.
PINNED_OUTPUT_BYTES = 1 << 20


def _new_output(shape, dtype):
    nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
    if nbytes >= PINNED_OUTPUT_BYTES:
        return _native.pinned_empty(shape, dtype)
    return np.empty(shape, dtype=dtype)


def _output_descriptor(shape, dtype):
    buf = _new_output(shape, dtype)
    ptr = buf.ctypes.data_as(ctypes.c_void_p)
    nd = len(shape)
    strides = [1] * nd
    for i in range(nd - 2, -1, -1):
        strides[i] = strides[i + 1] * shape[i + 1]
    c_types = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] + [ctypes.c_int64] * (2 * nd)
    return c_types, [ptr, ptr, 0] + list(shape) + strides, buf


_DEFAULT_INIT = {0: 0.0, 2: float("-inf"), 3: float("inf")}

# Registered weights: data address -> (array, version). The array is held so
# that its memory cannot be reused by another array while registered.
_WEIGHTS: Dict[int, Tuple[np.ndarray, int]] = {}


def register_weights(W: np.ndarray, version: int = 0) -> None:
    """Declares the 2-D f32 array W unchanged until it is registered again
    with another version or released: the device copy and tf32 split of W
    are then kept on every GPU that runs a function taking it, instead of
    being copied and split in every call (b200_weights_register). Modifying
    W in place without re-registering it leaves later calls on stale data."""
    if not isinstance(W, np.ndarray) or W.dtype != np.float32 or W.ndim != 2:
        raise TypeError("register_weights takes a 2-D float32 ndarray")
    if not W.flags["C_CONTIGUOUS"]:
        raise ValueError("register_weights takes a C-contiguous array")
    _native.check(_native.lib().b200_weights_register(
        ctypes.c_void_p(W.ctypes.data), W.shape[1], W.shape[0], W.shape[1], int(version)))
    _WEIGHTS[W.ctypes.data] = (W, int(version))


def release_weights(W: np.ndarray) -> None:
    """Frees the device copies of a registered array and forgets it."""
    if W.ctypes.data not in _WEIGHTS:
        raise ValueError("array is not registered")
    del _WEIGHTS[W.ctypes.data]
    _native.check(_native.lib().b200_weights_release(ctypes.c_void_p(W.ctypes.data)))


def _registered(a: np.ndarray) -> bool:
    held = _WEIGHTS.get(a.ctypes.data)
    return held is not None and held[0].shape == a.shape and a.dtype == np.float32


def _to_python(v):
    """Scalar results are returned as Python numbers, as the reference's
    ctypes scalar returns are."""
    v = np.asarray(v)
    return float(v) if v.dtype.kind == "f" else int(v)


def _host_binop(op, dtype, a, b):
    """Scalar arithmetic on reduction results: f32 (IEEE single) or i32
    (wrapping; division truncates toward zero like arith.divsi)."""
    if dtype == "f32":
        a, b = np.float32(a), np.float32(b)
        with np.errstate(all="ignore"):
            return [a + b, a - b, a * b, a / b][op]
    a, b = int(a), int(b)
    if op == 3:
        if b == 0:
            raise ZeroDivisionError("i32 division by zero")
        q = abs(a) // abs(b)
        r = q if (a >= 0) == (b >= 0) else -q
    else:
        r = [a + b, a - b, a * b][op]
    r &= 0xFFFFFFFF
    return np.int32(r - (1 << 32) if r >= 1 << 31 else r)


def _memref_symbol(step) -> Union[str, None]:
    """The memref entry point implementing a single step, if one exists."""
    if step.op == "gemm_f32":
        if step.act == ACT_LEAKY_RELU:
            return None
        base = "dense" if step.has_bias else "matmul"
        return f"b200_memref_{base}{'_relu' if step.act == ACT_RELU else ''}_f32"
    if step.op == "gemm_i32":
        return "b200_memref_dense_i32" if step.has_bias else "b200_memref_matmul_i32"
    if step.op == "bias_act_f32" and len(step.shape) == 2:
        if step.has_bias and step.act == ACT_NONE:
            return "b200_memref_bias_add_f32"
        if step.has_bias and step.act == ACT_RELU:
            return "b200_memref_bias_relu_f32"
        if not step.has_bias and step.act == ACT_RELU:
            return "b200_memref_relu_f32"
    return None


class B200Backend:
    """Compiles traced functions to B200 kernel plans and executes them."""

    def __init__(self):
        self._signatures: Dict[str, Tuple[List[Type], Type]] = {}
        self._plans: Dict[str, Plan] = {}
        self._target = "b200"
        self._opt_level = 3
        self.last_launches = 0  # kernels launched by the last execute_function

    # ------------------------------------------------------------ compile
    def compile_function_from_ast(self, name: str, params: list, return_type: Type,
                                  ast_node) -> None:
        plan = lower(ast_node, [n for n, _ in params])
        self._plans[name] = plan
        self._signatures[name] = ([t for _, t in params], return_type)

    # ------------------------------------------------------------ execute
    def execute_function(self, name: str, *args):
        param_types, return_type = self._signatures[name]
        plan = self._plans[name]
        values = []
        for pt, val in zip(param_types, args):
            if isinstance(pt, TensorType):
                expected = SCALAR_TYPE_TO_NUMPY_DTYPE[pt.element_type.kind]
                if val.dtype != expected:
                    raise TypeError(f"ndarray dtype {val.dtype} does not match expected "
                                    f"{np.dtype(expected)} for {pt}")
                values.append(np.ascontiguousarray(val))
            else:
                values.append(SCALAR_TYPE_TO_NUMPY_DTYPE[pt.kind](val))
        before = _native.launch_count()
        try:
            if plan.output.kind == "param":
                v = values[plan.output.index]
                return v.copy() if isinstance(v, np.ndarray) else _to_python(v)
            if plan.output.kind == "const":
                return _to_python(plan.consts[plan.output.index])
            if len(plan.steps) == 1 and all(r.kind == "param" for r in plan.steps[0].inputs):
                step = plan.steps[0]
                if step.shape == ():
                    return self._run_scalar_host(step, values)
                sym = _memref_symbol(step)
                if sym is not None:
                    return self._run_memref(sym, plan, param_types, values)
            return self._run_device(plan, param_types, values)
        finally:
            self.last_launches = _native.launch_count() - before

    execute_gpu_function = execute_function

    def _run_scalar_host(self, step, values):
        """One dot / reduce over parameters: the reference's scalar-returning
        memref ABI where a symbol exists, else the host entry point."""
        L = _native.lib()
        vp = ctypes.c_void_p
        desc1 = lambda a: [vp(a.ctypes.data), vp(a.ctypes.data), 0, a.size, 1]
        ins = [values[r.index] for r in step.inputs]
        f32 = step.dtype == "f32"
        sym, res_t = None, ctypes.c_float if f32 else ctypes.c_int32
        if step.op.startswith("dot"):
            sym = "b200_memref_dot_f32" if f32 else "b200_memref_dot_i32"
        elif f32 and step.init == _DEFAULT_INIT.get(step.red_op):
            sym = {0: "b200_memref_sum_f32", 2: "b200_memref_max_f32",
                   3: "b200_memref_min_f32"}.get(step.red_op)
        if sym is not None:
            args = sum((desc1(a) for a in ins), [])
            types = [vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64] * len(ins)
            fn_ptr = ctypes.cast(getattr(L, sym), ctypes.c_void_p).value
            r = ctypes.CFUNCTYPE(res_t, *types)(fn_ptr)(*args)
            _native.check_last()
            return float(np.float32(r)) if f32 else int(r)
        out = np.zeros(1, np.float32 if f32 else np.int32)
        x = ins[0]
        if f32:
            _native.check(L.b200_reduce_f32_host(vp(x.ctypes.data), x.size, step.red_op,
                                                 float(step.init), vp(out.ctypes.data)))
        else:
            _native.check(L.b200_reduce_i32_host(vp(x.ctypes.data), x.size, step.red_op,
                                                 int(step.init), vp(out.ctypes.data)))
        return _to_python(out[0])

    def _run_memref(self, sym, plan, param_types, arrays):
        step = plan.steps[0]
        c_types, c_vals, live = [], [], []
        for ref in step.inputs:
            ct, cv, buf = _memref_descriptor(arrays[ref.index], param_types[ref.index])
            c_types += ct
            c_vals += cv
            live.append(buf)
        dtype = np.float32 if step.dtype == "f32" else np.int32
        ct, cv, out = _output_descriptor(step.shape, dtype)
        c_types += ct
        c_vals += cv
        fn_ptr = ctypes.cast(getattr(_native.lib(), sym), ctypes.c_void_p).value
        ctypes.CFUNCTYPE(None, *c_types)(fn_ptr)(*c_vals)
        _native.check_last()
        return out

    def _run_device(self, plan: Plan, param_types, arrays):
        L = _native.lib()
        buffers = []

        def dmalloc(nbytes):
            p = ctypes.c_void_p()
            _native.check(L.b200_malloc(ctypes.byref(p), max(int(nbytes), 4)))
            buffers.append(p)
            return p

        try:
            dparams = {}
            needed = {r.index for s in plan.steps for r in s.inputs
                      if r.kind == "param" and s.op != "scalar_op"}
            for i in sorted(needed):
                a = arrays[i]
                if isinstance(a, np.ndarray) and a.ndim == 2 and _registered(a):
                    # the registered weight's kept device copy (and split)
                    p = ctypes.c_void_p()
                    _native.check(L.b200_weights_device(ctypes.c_void_p(a.ctypes.data),
                                                        ctypes.byref(p)))
                    dparams[i] = p
                    continue
                p = dmalloc(a.nbytes)
                _native.check(L.b200_memcpy_h2d(p, a.ctypes.data_as(ctypes.c_void_p), a.nbytes))
                dparams[i] = p
            douts = []
            # f32 GEMM outputs that a later f32 GEMM reads as its A operand:
            # their epilogue also writes the tf32 lo part, so that the next
            # layer does not split them again (b200_dense_f32_chain)
            feeds_a = {st.inputs[0].index for st in plan.steps
                       if st.op == "gemm_f32" and st.inputs[0].kind == "step"}
            lo_of = {}

            def dref(r: Ref):
                return dparams[r.index] if r.kind == "param" else douts[r.index]

            def shape_of(r: Ref):
                return arrays[r.index].shape if r.kind == "param" else plan.steps[r.index].shape

            for s in plan.steps:
                nelem = int(np.prod(s.shape))  # 1 for scalar results
                out = dmalloc(nelem * 4) if s.op != "scalar_op" else None
                douts.append(out)
                if s.op in ("gemm_f32", "gemm_i32"):
                    a, b = s.inputs[0], s.inputs[1]
                    M, K = shape_of(a)
                    N = shape_of(b)[1]
                    bias = dref(s.inputs[2]) if s.has_bias else None
                    if s.op == "gemm_f32":
                        me = len(douts) - 1
                        # the next layer reads this lo part with its split pitch
                        ldylo = _native.split_pitch(N)
                        ylo = dmalloc(M * ldylo * 4) \
                            if (me in feeds_a and N % 4 == 0 and K > 0) else None
                        xlo = lo_of.get(a.index) if a.kind == "step" else None
                        if ylo is not None or xlo is not None:
                            _native.check(L.b200_dense_f32_chain(
                                dref(a), K, xlo, dref(b), N, bias, out, N, ylo,
                                ldylo if ylo is not None else 0, M, N, K, s.act, s.alpha, None))
                            if ylo is not None:
                                lo_of[me] = ylo
                        else:
                            _native.check(L.b200_dense_f32(dref(a), K, dref(b), N, bias, out, N,
                                                           M, N, K, s.act, s.alpha, None))
                    else:
                        _native.check(L.b200_matmul_i32(dref(a), K, dref(b), N, bias, out, N, M,
                                                        N, K, None))
                elif s.op == "bias_act_f32":
                    x = s.inputs[0]
                    bias = dref(s.inputs[1]) if s.has_bias else None
                    if len(s.shape) == 2:
                        M, N = s.shape
                        _native.check(L.b200_bias_act_f32(dref(x), N, bias, out, N, M, N, s.act,
                                                          s.alpha, None))
                    else:
                        _native.check(L.b200_act_f32(dref(x), out, nelem, s.act, s.alpha, None))
                elif s.op == "bias_add_i32":
                    M, N = s.shape
                    _native.check(L.b200_bias_add_i32(dref(s.inputs[0]), N, dref(s.inputs[1]),
                                                      out, N, M, N, None))
                elif s.op in ("dot_f32", "dot_i32"):
                    a, b = s.inputs
                    n = int(np.prod(shape_of(a)))
                    fn = L.b200_dot_f32 if s.dtype == "f32" else L.b200_dot_i32
                    _native.check(fn(dref(a), dref(b), n, out, None))
                elif s.op in ("reduce_f32", "reduce_i32"):
                    x = s.inputs[0]
                    n = int(np.prod(shape_of(x)))
                    if s.dtype == "f32":
                        _native.check(L.b200_reduce_f32(dref(x), n, s.red_op, float(s.init), out,
                                                        None))
                    else:
                        _native.check(L.b200_reduce_i32(dref(x), n, s.red_op, int(s.init), out,
                                                        None))
                elif s.op == "scalar_op":
                    pass  # evaluated on the host below
                else:
                    raise RuntimeError(f"unknown step {s.op}")
            _native.check(L.b200_stream_sync(None))
            host_vals = {}

            def scalar(r: Ref):
                if r.kind == "const":
                    return plan.consts[r.index]
                if r.kind == "param":
                    return arrays[r.index]
                if r.index not in host_vals:
                    st = plan.steps[r.index]
                    if st.op == "scalar_op":
                        host_vals[r.index] = _host_binop(st.scalar_op, st.dtype,
                                                         scalar(st.inputs[0]),
                                                         scalar(st.inputs[1]))
                    else:
                        v = np.zeros(1, np.float32 if st.dtype == "f32" else np.int32)
                        _native.check(L.b200_memcpy_d2h(v.ctypes.data_as(ctypes.c_void_p),
                                                        douts[r.index], v.nbytes))
                        host_vals[r.index] = v[0]
                return host_vals[r.index]

            final = plan.steps[plan.output.index]
            if final.shape == ():
                return _to_python(scalar(plan.output))
            res = _new_output(final.shape, np.float32 if final.dtype == "f32" else np.int32)
            _native.check(L.b200_memcpy_d2h(res.ctypes.data_as(ctypes.c_void_p),
                                            douts[plan.output.index], res.nbytes))
            return res
        finally:
            for p in buffers:
                L.b200_free(p)

    # ------------------------------------------------------------ management
    def has_function(self, name: str) -> bool:
        return name in self._plans

    def list_functions(self) -> List[str]:
        return list(self._plans)

    def get_module_ir(self) -> str:
        """Textual form of every compiled plan (the b200 analogue of module IR)."""
        return "\n\n".join(f"func @{n}:\n{p.describe()}" for n, p in self._plans.items())

    def get_plan(self, name: str) -> Plan:
        return self._plans[name]

    def clear_module(self):
        self._plans.clear()
        self._signatures.clear()

    def set_optimization_level(self, level: int):
        if level not in (0, 2, 3):
            raise ValueError(f"Invalid optimization level {level}. Must be 0, 2, or 3.")
        self._opt_level = level  # kernels are precompiled; accepted for API parity

    def set_target(self, target: str) -> None:
        if target not in ("b200", "gpu"):
            raise ValueError(f"Invalid target '{target}'. This backend implements 'b200' "
                             "('gpu' is accepted as an alias); the reference CPU pipeline "
                             "is not part of it.")
        self._target = "b200"

    @staticmethod
    def set_default_devices(ndev: int):
        """Number of GPUs the memref entry points shard rows over."""
        _native.check(_native.lib().b200_set_default_devices(int(ndev)))


def get_backend():
    """The process-wide backend (None if the native library is missing)."""
    global _global_backend
    if not HAS_B200_BACKEND:
        return None
    if _global_backend is None:
        _global_backend = B200Backend()
    return _global_backend
