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
