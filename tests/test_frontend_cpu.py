"""Frontend behaviour without a GPU: types, validation errors (same exception
types and messages as the reference's tests), DYN specialisation, and the
pattern lowering (which ops fuse into which kernel steps)."""
import numpy as np
import pytest

from mlir_edsl import (DYN, LinalgBinaryOp, Tensor, f32, get_backend, i32, leaky_relu, matmul,
                       ml_function, relu)
from mlir_edsl.ast import Parameter, TENSOR_BIAS_LEFT, TENSOR_BIAS_RIGHT
from mlir_edsl.backend import _memref_descriptor, _memref_symbol
from mlir_edsl.functions import FunctionSignature, validate_function_body
from mlir_edsl.lowering import ACT_LEAKY_RELU, ACT_RELU, lower
from mlir_edsl.types import TensorType


def _plan(fn):
    sig = FunctionSignature.from_callable(fn)
    ast, _ = validate_function_body(fn, sig)
    return lower(ast, sig.param_names)


# ------------------------------------------------------------------ types
def test_tensor_type_syntax():
    t = Tensor[f32, 4, 8]
    assert isinstance(t, TensorType) and t.shape == (4, 8) and t.element_type == f32
    assert Tensor[i32, 5].shape == (5,)
    assert Tensor[f32, DYN, 3].is_dynamic


@pytest.mark.parametrize("bad", [(f32,), (f32, 0), (f32, 1, 2, 3, 4), (3, 4)])
def test_tensor_type_errors(bad):
    with pytest.raises(TypeError):
        Tensor[bad]


def test_missing_hints_raise():
    with pytest.raises(TypeError, match="missing type hint"):
        @ml_function
        def f(A, B: Tensor[f32, 2, 2]) -> Tensor[f32, 2, 2]:
            return A @ B
    with pytest.raises(TypeError, match="missing return type"):
        @ml_function
        def g(A: Tensor[f32, 2, 2]):
            return A


# ------------------------------------------------------------------ AST validation
def test_matmul_rejects_non_2d():
    with pytest.raises(TypeError, match="lhs must be a 2D tensor"):
        matmul(Parameter("a", Tensor[f32, 4]), Parameter("b", Tensor[f32, 4, 4]))


def test_matmul_rejects_mixed_types():
    with pytest.raises(TypeError, match="element types must match"):
        matmul(Parameter("a", Tensor[f32, 4, 4]), Parameter("b", Tensor[i32, 4, 4]))


def test_static_inner_dim_mismatch_raises_at_call():
    """reference: tests/linalg/test_linalg_dyn.py:97-106"""
    @ml_function
    def mm(A: Tensor[f32, 2, 3], B: Tensor[f32, 4, 2]) -> Tensor[f32, 2, 2]:
        return matmul(A, B)
    with pytest.raises(TypeError, match="inner dimensions must match"):
        mm(np.ones((2, 3), np.float32), np.ones((4, 2), np.float32))


def test_dyn_inner_dim_mismatch_raises_at_call():
    """reference: tests/linalg/test_linalg_dyn.py:74-84"""
    @ml_function
    def mm(A: Tensor[f32, DYN, DYN], B: Tensor[f32, DYN, DYN]) -> Tensor[f32, DYN, DYN]:
        return matmul(A, B)
    with pytest.raises(TypeError, match="inner dimensions must match"):
        mm(np.ones((2, 3), np.float32), np.ones((4, 2), np.float32))


def test_bias_broadcast_modes():
    M = Parameter("m", Tensor[f32, 3, 4])
    b = Parameter("b", Tensor[f32, 4])
    assert (M + b).broadcast == TENSOR_BIAS_RIGHT
    assert (b + M).broadcast == TENSOR_BIAS_LEFT
    with pytest.raises(TypeError, match="trailing dims must match"):
        M + Parameter("c", Tensor[f32, 5])
    with pytest.raises(TypeError, match="unsupported tensor shapes"):
        M + Parameter("d", Tensor[f32, 4, 3])


def test_activation_requires_tensor():
    from mlir_edsl.ast import Constant
    with pytest.raises(TypeError, match="input must be a tensor"):
        relu(Constant(1.0))


def test_return_type_mismatch():
    @ml_function
    def f(A: Tensor[f32, 2, 3], B: Tensor[f32, 3, 4]) -> Tensor[f32, 2, 3]:
        return A @ B
    with pytest.raises(TypeError, match="Return type mismatch"):
        f(np.ones((2, 3), np.float32), np.ones((3, 4), np.float32))


# ------------------------------------------------------------------ runtime arg validation
def _mm():
    @ml_function
    def mm(A: Tensor[f32, 2, 2], B: Tensor[f32, 2, 2]) -> Tensor[f32, 2, 2]:
        return A @ B
    return mm


def test_wrong_ndim_raises_valueerror():
    with pytest.raises(ValueError, match="expected 2D tensor"):
        _mm()(np.ones(4, np.float32), np.ones((2, 2), np.float32))


def test_wrong_shape_raises_valueerror():
    with pytest.raises(ValueError, match="expected shape"):
        _mm()(np.ones((3, 2), np.float32), np.ones((2, 2), np.float32))


def test_non_array_raises_typeerror():
    with pytest.raises(TypeError, match="expected ndarray"):
        _mm()([[1, 2], [3, 4]], np.ones((2, 2), np.float32))


def test_wrong_dtype_raises_typeerror():
    with pytest.raises(TypeError, match="does not match expected"):
        _mm()(np.ones((2, 2), np.float64), np.ones((2, 2), np.float32))


# ------------------------------------------------------------------ lowering / fusion
def test_dense_relu_is_one_fused_step():
    def dense(X: Tensor[f32, 8, 4], W: Tensor[f32, 4, 3], b: Tensor[f32, 3]) -> Tensor[f32, 8, 3]:
        return relu(X @ W + b)
    p = _plan(dense)
    assert len(p.steps) == 1
    s = p.steps[0]
    assert s.op == "gemm_f32" and s.has_bias and s.act == ACT_RELU
    assert _memref_symbol(s) == "b200_memref_dense_relu_f32"


def test_bias_on_the_left_also_fuses():
    def dense(X: Tensor[f32, 8, 4], W: Tensor[f32, 4, 3], b: Tensor[f32, 3]) -> Tensor[f32, 8, 3]:
        return b + X @ W
    p = _plan(dense)
    assert len(p.steps) == 1 and p.steps[0].has_bias and p.steps[0].inputs[2].index == 2


def test_two_layer_net_two_steps():
    def net(X: Tensor[f32, 2, 4], W1: Tensor[f32, 4, 8], b1: Tensor[f32, 8],
            W2: Tensor[f32, 8, 3], b2: Tensor[f32, 3]) -> Tensor[f32, 2, 3]:
        h = relu(X @ W1 + b1)
        return relu(h @ W2 + b2)
    p = _plan(net)
    assert [s.op for s in p.steps] == ["gemm_f32", "gemm_f32"]
    assert all(s.has_bias and s.act == ACT_RELU for s in p.steps)
    assert p.steps[1].inputs[0].kind == "step"


def test_shared_value_is_not_fused():
    """m is used twice: relu must not be folded into the gemm producing m."""
    def f(X: Tensor[f32, 4, 4], W: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        m = X @ W
        return relu(m) @ m
    p = _plan(f)
    assert [s.op for s in p.steps] == ["gemm_f32", "bias_act_f32", "gemm_f32"]
    assert p.steps[0].act == 0 and p.steps[1].act == ACT_RELU


def test_leaky_relu_fuses_with_alpha():
    def f(X: Tensor[f32, 4, 4], W: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        return leaky_relu(X @ W, alpha=0.2)
    p = _plan(f)
    assert p.steps[0].act == ACT_LEAKY_RELU and abs(p.steps[0].alpha - 0.2) < 1e-12
    assert _memref_symbol(p.steps[0]) is None  # leaky runs through the host API


def test_elementwise_patterns():
    def bias(X: Tensor[f32, 3, 4], b: Tensor[f32, 4]) -> Tensor[f32, 3, 4]:
        return relu(X + b)
    p = _plan(bias)
    assert len(p.steps) == 1 and p.steps[0].op == "bias_act_f32"
    assert _memref_symbol(p.steps[0]) == "b200_memref_bias_relu_f32"

    def r1(X: Tensor[f32, 7]) -> Tensor[f32, 7]:
        return relu(X)
    p = _plan(r1)
    assert p.steps[0].op == "bias_act_f32" and not p.steps[0].has_bias


def test_i32_dense_and_relu_rejected():
    def d(X: Tensor[i32, 4, 4], W: Tensor[i32, 4, 4], b: Tensor[i32, 4]) -> Tensor[i32, 4, 4]:
        return X @ W + b
    p = _plan(d)
    assert p.steps[0].op == "gemm_i32" and p.steps[0].has_bias
    assert _memref_symbol(p.steps[0]) == "b200_memref_dense_i32"

    def r(X: Tensor[i32, 4, 4], W: Tensor[i32, 4, 4]) -> Tensor[i32, 4, 4]:
        return relu(X @ W)
    with pytest.raises(TypeError, match="float tensor"):
        _plan(r)


@pytest.mark.parametrize("body", ["X * 2.0", "X - X", "X + X"])
def test_ops_outside_the_path_raise(body):
    ns = {}
    exec(f"def f(X: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:\n    return {body}\n",
         {"Tensor": Tensor, "f32": f32}, ns)
    with pytest.raises(NotImplementedError, match="b200 target"):
        _plan(ns["f"])


def test_nested_ml_function_inlines():
    @ml_function
    def layer(X: Tensor[f32, 4, 4], W: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        return relu(X @ W)

    def net(X: Tensor[f32, 4, 4], W1: Tensor[f32, 4, 4], W2: Tensor[f32, 4, 4]) -> Tensor[f32, 4, 4]:
        return layer(layer(X, W1), W2)
    p = _plan(net)
    assert [s.op for s in p.steps] == ["gemm_f32", "gemm_f32"]


# ------------------------------------------------------------------ backend API
def test_backend_management_api():
    be = get_backend()
    assert be is not None
    with pytest.raises(ValueError, match="Invalid target"):
        be.set_target("cpu")
    be.set_target("gpu")  # alias of b200
    with pytest.raises(ValueError, match="optimization level"):
        be.set_optimization_level(1)
    be.set_optimization_level(3)

    @ml_function(target="b200")
    def dense(X: Tensor[f32, 8, 4], W: Tensor[f32, 4, 3], b: Tensor[f32, 3]) -> Tensor[f32, 8, 3]:
        return relu(X @ W + b)
    sig = dense.signature
    ast, _ = validate_function_body(dense.func, sig)
    be.compile_function_from_ast(sig.name, sig.make_param_list(), sig.return_type, ast)
    assert be.has_function(sig.name) and sig.name in be.list_functions()
    assert "gemm_f32(X, W, b, act=relu)" in be.get_module_ir()
    be.clear_module()
    assert not be.has_function(sig.name)


def test_dense_memref_descriptor_has_26_args():
    """The flattened ABI of relu(X @ W + b): 7 + 7 + 5 + 7 arguments."""
    from mlir_edsl.backend import _output_descriptor
    X, W, b = np.ones((3, 4), np.float32), np.ones((4, 5), np.float32), np.ones(5, np.float32)
    n = sum(len(_memref_descriptor(a, TensorType(a.shape, f32))[0]) for a in (X, W, b))
    n += len(_output_descriptor((3, 5), np.float32)[0])
    assert n == 26
    ct, cv, _ = _memref_descriptor(X, TensorType((3, 4), f32))
    assert cv[2:] == [0, 3, 4, 4, 1]


def test_variant_cache_per_dyn_shape():
    """DYN shapes compile one variant per concrete shape (reference:
    mlir_edsl/functions/decorator.py:67-99); execution needs a GPU, so only the
    compile side is checked here."""
    @ml_function
    def mm(A: Tensor[f32, DYN, DYN], B: Tensor[f32, DYN, DYN]) -> Tensor[f32, DYN, DYN]:
        return A @ B
    for shp in [(2, 3, 4), (5, 6, 7)]:
        M, K, N = shp
        try:
            mm(np.ones((M, K), np.float32), np.ones((K, N), np.float32))
        except RuntimeError:
            pass  # no GPU here: execution fails loudly, compilation already happened
    assert set(mm._compiled_variants) == {((2, 3), (3, 4)), ((5, 6), (6, 7))}
    names = {v.name for v in mm._compiled_variants.values()}
    assert all("__" in n for n in names)


# ------------------------------------------------------------------ dot / reduce
def test_dot_validation():
    """reference: tests/linalg/test_dot_execution.py:84-100"""
    from mlir_edsl import dot
    from mlir_edsl.ast import Constant
    with pytest.raises(TypeError, match="1D tensor"):
        dot(Constant(5), Constant(5))
    with pytest.raises(TypeError, match="element types must match"):
        dot(Parameter("a", Tensor[f32, 2]), Parameter("b", Tensor[i32, 2]))
    with pytest.raises(TypeError, match="lengths must match"):
        dot(Parameter("a", Tensor[f32, 3]), Parameter("b", Tensor[f32, 4]))


def test_reduce_validation():
    """reference: tests/linalg/test_reduce_execution.py:173-197"""
    from mlir_edsl import reduce, to_value
    with pytest.raises(TypeError, match="1D tensor"):
        reduce(Parameter("a", Tensor[f32, 2, 2]), to_value(0.0), lambda e, a: a + e)
    with pytest.raises(TypeError, match="init must be a scalar"):
        reduce(Parameter("a", Tensor[f32, 3]), to_value(0), lambda e, a: a + e)
    with pytest.raises(TypeError, match="body must return element type"):
        reduce(Parameter("a", Tensor[f32, 3]), to_value(0.0), lambda e, a: to_value(1))


@pytest.mark.parametrize("body,red", [
    ("tensor_sum(a)", 0), ("tensor_max(a)", 2), ("tensor_min(a)", 3),
    ("reduce(a, to_value(1.0), lambda e, acc: acc * e)", 1),
    ("reduce(a, to_value(0.0), lambda e, acc: e + acc)", 0),
    ("reduce(a, to_value(0.0), lambda e, acc: If(acc < e, e, acc))", 2),
])
def test_reduce_bodies_lower(body, red):
    import mlir_edsl as m
    ns = {}
    exec(f"def f(a: Tensor[f32, 8]) -> f32:\n    return {body}\n", vars(m), ns)
    p = _plan(ns["f"])
    assert p.steps[0].op == "reduce_f32" and p.steps[0].red_op == red


def test_unsupported_reduce_body_raises():
    import mlir_edsl as m
    ns = {}
    exec("def f(a: Tensor[f32, 8]) -> f32:\n"
         "    return reduce(a, to_value(0.0), lambda e, acc: acc + e * e)\n", vars(m), ns)
    with pytest.raises(NotImplementedError, match="reduce bodies"):
        _plan(ns["f"])


def test_scalar_tail_is_a_host_step():
    from mlir_edsl import tensor_sum, to_value

    def f(a: Tensor[f32, 4]) -> f32:
        return tensor_sum(a) * to_value(2.0)
    p = _plan(f)
    assert [s.op for s in p.steps] == ["reduce_f32", "scalar_op"]
    assert p.consts == [2.0]


def test_host_binop_i32_semantics():
    from mlir_edsl.backend import _host_binop
    assert _host_binop(0, "i32", 2**31 - 1, 1) == -2**31
    assert _host_binop(3, "i32", -7, 2) == -3  # truncates toward zero
    assert _host_binop(2, "f32", 0.1, 3.0) == np.float32(np.float32(0.1) * np.float32(3.0))
