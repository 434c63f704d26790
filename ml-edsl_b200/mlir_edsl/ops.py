"""User-facing ops of the dense-layer path.

Same names, arguments and dispatch as the reference:
  matmul      mlir_edsl/ops/linalg.py:28-46
  relu        mlir_edsl/ops/linalg.py:70-85
  leaky_relu  mlir_edsl/ops/linalg.py:178-194
  add/sub/mul/div with tensor -> LinalgBinaryOp dispatch
              mlir_edsl/ops/arithmetic.py:14-43
"""
from .ast import (ADD, DIV, LEAKY_RELU, MUL, RELU, SUB, BinaryOp, LinalgActivation,
                  LinalgBinaryOp, LinalgMatmul, Value, to_value)
from .types import ScalarType, TensorType


def matmul(A: Value, B: Value) -> LinalgMatmul:
    """Matrix product of two 2-D tensors: [M,K] @ [K,N] -> [M,N]."""
    return LinalgMatmul(A, B)


def relu(arr: Value) -> LinalgActivation:
    """max(x, 0) element-wise (NaN propagates, -0 becomes +0)."""
    return LinalgActivation(arr, RELU)


def leaky_relu(arr: Value, alpha: float = 0.01) -> LinalgActivation:
    """max(x,0) + alpha*min(x,0) element-wise."""
    return LinalgActivation(arr, LEAKY_RELU, float(alpha))


def _dispatch_binary_op(op: int, left: Value, right: Value):
    lt, rt = left.infer_type(), right.infer_type()
    if isinstance(lt, TensorType) or isinstance(rt, TensorType):
        return LinalgBinaryOp(op, left, right)
    if isinstance(lt, ScalarType) and isinstance(rt, ScalarType):
        return BinaryOp(op, left, right)
    raise TypeError(f"Arithmetic not supported for operand types {lt} and {rt}.")


def add(left, right):
    return _dispatch_binary_op(ADD, to_value(left), to_value(right))


def sub(left, right):
    return _dispatch_binary_op(SUB, to_value(left), to_value(right))


def mul(left, right):
    return _dispatch_binary_op(MUL, to_value(left), to_value(right))


def div(left, right):
    return _dispatch_binary_op(DIV, to_value(left), to_value(right))


# --------------------------------------------------------------------------
# Comparisons, If, dot and reductions
# (reference: mlir_edsl/ops/comparison.py, ops/control_flow.py,
#  ops/linalg.py:7-25 dot, :88-175 reduce / tensor_sum / tensor_max / tensor_min)
def _cmp(pred, left, right):
    from .ast import CompareOp
    return CompareOp(pred, to_value(left), to_value(right))


def lt(left, right):
    return _cmp("lt", left, right)


def le(left, right):
    return _cmp("le", left, right)


def gt(left, right):
    return _cmp("gt", left, right)


def ge(left, right):
    return _cmp("ge", left, right)


def eq(left, right):
    return _cmp("eq", left, right)


def ne(left, right):
    return _cmp("ne", left, right)


def If(cond, then_value, else_value):
    """Value selection (the value form of the reference's If)."""
    from .ast import IfOp
    return IfOp(cond, to_value(then_value), to_value(else_value))


def dot(a: Value, b: Value):
    """Dot product of two 1-D tensors -> scalar."""
    from .ast import LinalgDot
    return LinalgDot(a, b)


def reduce(arr: Value, init: Value, fn):
    """Fold a 1-D tensor: acc = init; acc = fn(element, acc) for each element."""
    from .ast import LinalgReduce
    return LinalgReduce(arr, to_value(init), fn)


def tensor_sum(arr: Value):
    """Sum of a 1-D tensor (init 0)."""
    from .ast import Constant, LinalgReduce
    zero = Constant(0.0) if arr.infer_type().element_type.is_float() else Constant(0)
    return LinalgReduce(arr, zero, lambda elem, acc: acc + elem)


def tensor_max(arr: Value):
    """Maximum of a 1-D f32 tensor (init -inf; NaN elements never win)."""
    from .ast import Constant, IfOp, LinalgReduce
    return LinalgReduce(arr, Constant(float("-inf")),
                        lambda elem, acc: IfOp(elem > acc, elem, acc))


def tensor_min(arr: Value):
    """Minimum of a 1-D f32 tensor (init +inf)."""
    from .ast import Constant, IfOp, LinalgReduce
    return LinalgReduce(arr, Constant(float("inf")),
                        lambda elem, acc: IfOp(elem < acc, elem, acc))
