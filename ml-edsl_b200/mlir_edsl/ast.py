"""AST nodes of the dense-layer path, built by symbolic execution.

Mirrors the reference nodes the path uses, with the same validation rules and
error messages:
  Value + operator overloads    reference: mlir_edsl/ast/base.py:19-88,
                                           mlir_edsl/ast/operators.py:12-60
  Parameter                     mlir_edsl/ast/nodes/functions.py:19-36
  Constant (scalar literal)     mlir_edsl/ast/nodes/scalars.py
  LinalgMatmul                  mlir_edsl/ast/nodes/linalg.py:75-138
  LinalgBinaryOp (broadcasts)   mlir_edsl/ast/nodes/linalg.py:141-257
  LinalgActivation              mlir_edsl/ast/nodes/linalg.py:331-363
Nodes are plain Python objects; the b200 backend pattern-matches them
directly (lowering.py) instead of serialising to protobuf.
"""
from .types import ScalarType, TensorType, Type, f32, i1, i32

# Binary operation and broadcast codes (names as in the reference schema).
ADD, SUB, MUL, DIV = 0, 1, 2, 3
OP_NAMES = {ADD: "add", SUB: "sub", MUL: "mul", DIV: "div"}
NONE, SCALAR_RIGHT, SCALAR_LEFT, TENSOR_BIAS_RIGHT, TENSOR_BIAS_LEFT = 0, 1, 2, 3, 4
RELU, LEAKY_RELU = 0, 1


class Value:
    """Base class of AST values; every node gets a unique id."""

    _next_id = 0

    def __init__(self):
        self.id = Value._next_id
        Value._next_id += 1

    def infer_type(self) -> Type:
        raise NotImplementedError

    def get_children(self):
        return []

    # arithmetic
    def __add__(self, other):
        from .ops import add
        return add(self, other)

    def __radd__(self, other):
        from .ops import add
        return add(other, self)

    def __sub__(self, other):
        from .ops import sub
        return sub(self, other)

    def __rsub__(self, other):
        from .ops import sub
        return sub(other, self)

    def __mul__(self, other):
        from .ops import mul
        return mul(self, other)

    def __rmul__(self, other):
        from .ops import mul
        return mul(other, self)

    def __truediv__(self, other):
        from .ops import div
        return div(self, other)

    def __rtruediv__(self, other):
        from .ops import div
        return div(other, self)

    def __matmul__(self, other):
        from .ops import matmul
        return matmul(self, other)

    # comparisons (scalar values inside reduce bodies); == and != keep Python
    # identity semantics here, use ops.eq / ops.ne instead
    def __lt__(self, other):
        from .ops import lt
        return lt(self, other)

    def __le__(self, other):
        from .ops import le
        return le(self, other)

    def __gt__(self, other):
        from .ops import gt
        return gt(self, other)

    def __ge__(self, other):
        from .ops import ge
        return ge(self, other)

    def __rmatmul__(self, other):
        from .ops import matmul
        return matmul(other, self)

    __hash__ = object.__hash__

    def dump(self, indent=0) -> str:
        pad = "  " * indent
        lines = [f"{pad}{self._describe()} : {self.infer_type()!r}"]
        for c in self.get_children():
            lines.append(c.dump(indent + 1))
        return "\n".join(lines)

    def _describe(self) -> str:
        return type(self).__name__


def to_value(x):
    """Python scalars become Constant nodes; Values pass through."""
    return x if isinstance(x, Value) else Constant(x)


class Parameter(Value):
    """A named function parameter (symbolic argument)."""

    def __init__(self, name: str, value_type: Type):
        super().__init__()
        self.name = name
        self.value_type = value_type

    def infer_type(self):
        return self.value_type

    def _describe(self):
        return f"Parameter({self.name})"


class Constant(Value):
    """A scalar literal: int -> i32, float -> f32, bool -> i1."""

    def __init__(self, value, value_type: Type = None):
        super().__init__()
        if value_type is None:
            if isinstance(value, bool):
                value_type = i1
            elif isinstance(value, int):
                value_type = i32
            elif isinstance(value, float):
                value_type = f32
            else:
                raise TypeError(f"Unsupported constant type: {type(value).__name__}")
        self.value = value
        self.value_type = value_type

    def infer_type(self):
        return self.value_type

    def _describe(self):
        return f"Constant({self.value})"


class LinalgMatmul(Value):
    """C[M,N] = A[M,K] @ B[K,N] (linalg.fill(0) + linalg.matmul)."""

    def __init__(self, lhs: Value, rhs: Value):
        super().__init__()
        self.lhs, self.rhs = lhs, rhs
        lt, rt = lhs.infer_type(), rhs.infer_type()
        if not isinstance(lt, TensorType) or lt.ndim != 2:
            raise TypeError(f"linalg.matmul: lhs must be a 2D tensor, got {lt}")
        if not isinstance(rt, TensorType) or rt.ndim != 2:
            raise TypeError(f"linalg.matmul: rhs must be a 2D tensor, got {rt}")
        if lt.element_type != rt.element_type:
            raise TypeError(f"linalg.matmul: operand element types must match, "
                            f"got {lt.element_type} and {rt.element_type}")
        M, K_lhs = lt.shape
        K_rhs, N = rt.shape
        if K_lhs != -1 and K_rhs != -1 and K_lhs != K_rhs:
            raise TypeError(f"linalg.matmul: inner dimensions must match, "
                            f"got lhs shape {lt.shape} and rhs shape {rt.shape}")
        self._out_type = TensorType((M, N), lt.element_type)

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.lhs, self.rhs]


class LinalgBinaryOp(Value):
    """Element-wise tensor op with the reference's broadcast rules:
    same shape -> NONE, tensor op scalar -> SCALAR_RIGHT, scalar op tensor ->
    SCALAR_LEFT, [M,N] op [N] -> TENSOR_BIAS_RIGHT, [N] op [M,N] ->
    TENSOR_BIAS_LEFT."""

    def __init__(self, op: int, lhs: Value, rhs: Value):
        super().__init__()
        self.op, self.lhs, self.rhs = op, lhs, rhs
        lt, rt = lhs.infer_type(), rhs.infer_type()
        lten, rten = isinstance(lt, TensorType), isinstance(rt, TensorType)
        if lten and rten:
            if lt.shape == rt.shape:
                if lt.element_type != rt.element_type:
                    raise TypeError(f"LinalgBinaryOp: element types must match, "
                                    f"got {lt.element_type} and {rt.element_type}")
                self.broadcast, self._out_type = NONE, lt
            elif lt.ndim == 2 and rt.ndim == 1:
                n_l, (n_r,) = lt.shape[1], rt.shape
                if n_l != -1 and n_r != -1 and n_l != n_r:
                    raise TypeError(f"LinalgBinaryOp TENSOR_BIAS_RIGHT: trailing dims must "
                                    f"match, got {lt.shape} and {rt.shape}")
                if lt.element_type != rt.element_type:
                    raise TypeError(f"LinalgBinaryOp: element types must match, "
                                    f"got {lt.element_type} and {rt.element_type}")
                self.broadcast, self._out_type = TENSOR_BIAS_RIGHT, lt
            elif lt.ndim == 1 and rt.ndim == 2:
                (n_l,), n_r = lt.shape, rt.shape[1]
                if n_l != -1 and n_r != -1 and n_l != n_r:
                    raise TypeError(f"LinalgBinaryOp TENSOR_BIAS_LEFT: trailing dims must "
                                    f"match, got {lt.shape} and {rt.shape}")
                if lt.element_type != rt.element_type:
                    raise TypeError(f"LinalgBinaryOp: element types must match, "
                                    f"got {lt.element_type} and {rt.element_type}")
                self.broadcast, self._out_type = TENSOR_BIAS_LEFT, rt
            else:
                raise TypeError(f"LinalgBinaryOp: unsupported tensor shapes {lt.shape} and "
                                f"{rt.shape}. Supported: same shape, or [M,N]+[N] bias "
                                f"broadcast.")
        elif lten and isinstance(rt, ScalarType):
            if lt.element_type != rt:
                raise TypeError(f"LinalgBinaryOp: scalar type {rt} must match tensor element "
                                f"type {lt.element_type}")
            self.broadcast, self._out_type = SCALAR_RIGHT, lt
        elif isinstance(lt, ScalarType) and rten:
            if rt.element_type != lt:
                raise TypeError(f"LinalgBinaryOp: scalar type {lt} must match tensor element "
                                f"type {rt.element_type}")
            self.broadcast, self._out_type = SCALAR_LEFT, rt
        else:
            raise TypeError(f"LinalgBinaryOp requires at least one tensor operand, "
                            f"got {lt} and {rt}")

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.lhs, self.rhs]

    def _describe(self):
        return f"LinalgBinaryOp({OP_NAMES[self.op]}, broadcast={self.broadcast})"


class LinalgActivation(Value):
    """relu / leaky_relu applied element-wise to a tensor."""

    def __init__(self, input: Value, act_type: int, alpha: float = 0.0):
        super().__init__()
        self.input, self.act_type, self.alpha = input, act_type, float(alpha)
        it = input.infer_type()
        if not isinstance(it, TensorType):
            raise TypeError(f"activation: input must be a tensor, got {it}")
        self._out_type = it

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.input]

    def _describe(self):
        return "relu" if self.act_type == RELU else f"leaky_relu(alpha={self.alpha})"


class BinaryOp(Value):
    """Scalar arithmetic between two scalar values (kept for operator
    completeness; the b200 target only lowers tensor patterns)."""

    def __init__(self, op: int, lhs: Value, rhs: Value):
        super().__init__()
        self.op, self.lhs, self.rhs = op, lhs, rhs
        lt, rt = lhs.infer_type(), rhs.infer_type()
        if lt != rt:
            raise TypeError(f"Type mismatch in {OP_NAMES[op]}: {lt} vs {rt}")
        self._out_type = lt

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.lhs, self.rhs]


# ----------------------------------------------------------------------------
# Comparisons, value selection, dot and reduce (1-D reductions).
# reference: mlir_edsl/ops/comparison.py, mlir_edsl/ast/nodes/control_flow.py
# (IfOp), mlir_edsl/ast/nodes/linalg.py:15-72 (LinalgDot), :366-475
# (LinalgReduce and its element / accumulator placeholders).
LT, LE, GT, GE, EQ, NE = "lt", "le", "gt", "ge", "eq", "ne"


class CompareOp(Value):
    """Scalar comparison producing i1."""

    def __init__(self, pred: str, lhs: Value, rhs: Value):
        super().__init__()
        self.pred, self.lhs, self.rhs = pred, lhs, rhs
        lt, rt = lhs.infer_type(), rhs.infer_type()
        if not (isinstance(lt, ScalarType) and isinstance(rt, ScalarType)):
            raise TypeError(f"comparison requires scalar operands, got {lt} and {rt}")
        if lt != rt:
            raise TypeError(f"Type mismatch in comparison: {lt} vs {rt}")

    def infer_type(self):
        return i1

    def get_children(self):
        return [self.lhs, self.rhs]

    def _describe(self):
        return f"CompareOp({self.pred})"


class IfOp(Value):
    """Value selection: then_value if cond else else_value."""

    def __init__(self, cond: Value, then_value: Value, else_value: Value):
        super().__init__()
        self.cond, self.then_value, self.else_value = cond, then_value, else_value
        if cond.infer_type() != i1:
            raise TypeError(f"If condition must be i1, got {cond.infer_type()}")
        tt, et = then_value.infer_type(), else_value.infer_type()
        if tt != et:
            raise TypeError(f"If branches must have the same type, got {tt} and {et}")
        self._out_type = tt

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.cond, self.then_value, self.else_value]


class LinalgDot(Value):
    """Dot product of two 1-D tensors; returns a scalar of the element type."""

    def __init__(self, lhs: Value, rhs: Value):
        super().__init__()
        self.lhs, self.rhs = lhs, rhs
        lt, rt = lhs.infer_type(), rhs.infer_type()
        if not isinstance(lt, TensorType) or lt.ndim != 1:
            raise TypeError(f"linalg.dot: lhs must be a 1D tensor, got {lt}")
        if not isinstance(rt, TensorType) or rt.ndim != 1:
            raise TypeError(f"linalg.dot: rhs must be a 1D tensor, got {rt}")
        if lt.element_type != rt.element_type:
            raise TypeError(f"linalg.dot: operand element types must match, "
                            f"got {lt.element_type} and {rt.element_type}")
        if lt.shape[0] != -1 and rt.shape[0] != -1 and lt.shape[0] != rt.shape[0]:
            raise TypeError(f"linalg.dot: operand lengths must match, "
                            f"got {lt.shape} and {rt.shape}")
        self._out_type = lt.element_type

    def infer_type(self):
        return self._out_type

    def get_children(self):
        return [self.lhs, self.rhs]


class LinalgReduceElement(Value):
    """Placeholder for the current element in a reduce body."""

    def __init__(self, element_type):
        super().__init__()
        self._t = element_type

    def infer_type(self):
        return self._t


class LinalgReduceAccumulator(Value):
    """Placeholder for the running accumulator in a reduce body."""

    def __init__(self, element_type):
        super().__init__()
        self._t = element_type

    def infer_type(self):
        return self._t


class LinalgReduce(Value):
    """Fold of a 1-D tensor: acc = init; acc = fn(element, acc) per element."""

    def __init__(self, input: Value, init: Value, fn):
        super().__init__()
        self.input, self.init = input, init
        it = input.infer_type()
        if not isinstance(it, TensorType) or it.ndim != 1:
            raise TypeError(f"linalg.reduce: input must be a 1D tensor, got {it}")
        self._element_type = it.element_type
        init_t = init.infer_type()
        if not isinstance(init_t, ScalarType) or init_t != self._element_type:
            raise TypeError(f"linalg.reduce: init must be a scalar of element type "
                            f"{self._element_type}, got {init_t}")
        self.element = LinalgReduceElement(self._element_type)
        self.accumulator = LinalgReduceAccumulator(self._element_type)
        self.body = fn(self.element, self.accumulator)
        bt = self.body.infer_type()
        if bt != self._element_type:
            raise TypeError(f"linalg.reduce body must return element type "
                            f"{self._element_type}, got {bt}")

    def infer_type(self):
        return self._element_type

    def get_children(self):
        # the body refers to placeholders only; it is matched, not executed
        return [self.input, self.init]
