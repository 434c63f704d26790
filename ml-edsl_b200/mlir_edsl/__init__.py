"""B200 (sm_100a) implementation of ml-edsl's dense-layer path.

Drop-in for the reference package's user surface on this path
(reference: mlir_edsl/__init__.py:11-94):

    from mlir_edsl import ml_function, Tensor, f32, relu

    @ml_function(target="b200")
    def dense(X: Tensor[f32, 1024, 1024], W: Tensor[f32, 1024, 1024],
              b: Tensor[f32, 1024]) -> Tensor[f32, 1024, 1024]:
        return relu(X @ W + b)

Functions are traced symbolically, pattern-matched to fused kernels
(lowering.py) and run through libb200edsl.so (include/b200_edsl.h).
"""
from .ast import (ADD, DIV, MUL, SUB, BinaryOp, Constant, LinalgActivation, LinalgBinaryOp,
                  LinalgMatmul, Parameter, Value)
from .functions import MLFunction, ml_function
from .ops import (If, add, div, dot, eq, ge, gt, le, leaky_relu, lt, matmul, mul, ne, reduce,
                  relu, sub, tensor_max, tensor_min, tensor_sum)
from .ast import CompareOp, IfOp, LinalgDot, LinalgReduce, to_value
from .types import DYN, Tensor, TensorType, ScalarType, f32, i1, i32

try:
    from .backend import (HAS_B200_BACKEND, HAS_CPP_BACKEND, get_backend, register_weights,
                          release_weights)
except Exception:  # pragma: no cover - import-time failure of ctypes itself
    HAS_B200_BACKEND = HAS_CPP_BACKEND = False

    def get_backend():
        return None

__version__ = "0.1.0"

__all__ = [
    "ml_function", "MLFunction",
    "i32", "f32", "i1", "DYN", "Tensor", "TensorType", "ScalarType",
    "add", "sub", "mul", "div", "matmul", "relu", "leaky_relu",
    "dot", "reduce", "tensor_sum", "tensor_max", "tensor_min", "If",
    "lt", "le", "gt", "ge", "eq", "ne", "to_value", "CompareOp", "IfOp", "LinalgDot",
    "LinalgReduce",
    "ADD", "SUB", "MUL", "DIV",
    "Value", "Constant", "Parameter", "BinaryOp", "LinalgMatmul", "LinalgBinaryOp",
    "LinalgActivation",
    "get_backend", "HAS_B200_BACKEND", "HAS_CPP_BACKEND", "register_weights",
    "release_weights",
]
