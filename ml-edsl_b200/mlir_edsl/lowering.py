"""Pattern lowering of a traced function body to B200 kernel steps.

The reference builds linalg IR for the body (cpp/src/builders/LinalgBuilder.cpp)
and relies on linalg-fuse-elementwise-ops plus tiling passes to fuse
bias_add + relu (cpp/src/MLIRLowering.cpp:355-434). The b200 target
recognises the same op chains directly on the AST and binds each chain to
one fused kernel step:

  matmul(A, B)                         -> gemm (f32: 3xTF32 tcgen05; i32: byte-sliced int8 tcgen05)
  matmul(A, B) + b        (either side)  -> gemm with fused bias
  relu / leaky_relu(gemm)                -> gemm with fused activation
  X + b, relu(X + b), relu(X), leaky(X)  -> bias_act (HBM-bound elementwise)
  dot(a, b), tensor_sum/max/min, reduce  -> dot / reduce (HBM-bound, two-pass)
  scalar arithmetic on those results     -> a host step after the device work

A producer is folded into its consumer only when the consumer is its sole
use (SSA values used twice stay materialised). Chains of layers become
several steps whose intermediates stay on the device. Anything else raises
NotImplementedError: there is no CPU fallback on this target.
"""
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from .ast import (ADD, MUL, LEAKY_RELU, RELU, TENSOR_BIAS_LEFT, TENSOR_BIAS_RIGHT, BinaryOp,
                  CompareOp, Constant, IfOp, LinalgActivation, LinalgBinaryOp, LinalgDot,
                  LinalgMatmul, LinalgReduce, OP_NAMES, Parameter, Value)
from .types import ScalarType, TensorType

ACT_NONE, ACT_RELU, ACT_LEAKY_RELU = 0, 1, 2
REDUCE_SUM, REDUCE_PROD, REDUCE_MAX, REDUCE_MIN = 0, 1, 2, 3
REDUCE_NAMES = {REDUCE_SUM: "sum", REDUCE_PROD: "prod", REDUCE_MAX: "max", REDUCE_MIN: "min"}


@dataclass
class Ref:
    """An operand: a function parameter or the output of an earlier step."""
    kind: str  # "param" | "step" | "const"
    index: int


@dataclass
class Step:
    op: str                 # "gemm_f32" | "gemm_i32" | "bias_act_f32" | "bias_add_i32" |
                            # "dot_{f32,i32}" | "reduce_{f32,i32}" | "scalar_op" (host)
    inputs: List[Ref]       # gemm: [A, B(, bias)]; bias_act: [X(, bias)]; dot: [a, b]
    shape: Tuple[int, ...]  # output shape (() for scalars)
    dtype: str              # "f32" | "i32"
    has_bias: bool = False
    act: int = ACT_NONE
    alpha: float = 0.0
    red_op: int = REDUCE_SUM   # reduce: the fold
    init: float = 0.0          # reduce: initial accumulator
    scalar_op: int = ADD       # scalar_op: ADD/SUB/MUL/DIV

    def describe(self, names) -> str:
        args = ", ".join(names(r) for r in self.inputs)
        if self.op.startswith("reduce"):
            return (f"{self.op}({args}, {REDUCE_NAMES[self.red_op]}, init={self.init}) "
                    f"-> {self.dtype}")
        if self.op == "scalar_op":
            return f"host {OP_NAMES[self.scalar_op]}({args}) -> {self.dtype}"
        act = {ACT_NONE: "", ACT_RELU: ", act=relu",
               ACT_LEAKY_RELU: f", act=leaky_relu({self.alpha})"}[self.act]
        return f"{self.op}({args}{act}) -> {self.dtype}{list(self.shape)}"


@dataclass
class Plan:
    params: List[str]
    steps: List[Step] = field(default_factory=list)
    output: Optional[Ref] = None
    consts: List[float] = field(default_factory=list)

    def describe(self) -> str:
        def names(r):
            if r.kind == "const":
                return repr(self.consts[r.index])
            return self.params[r.index] if r.kind == "param" else f"%{r.index}"
        lines = [f"%{i} = {s.describe(names)}" for i, s in enumerate(self.steps)]
        lines.append(f"return {names(self.output)}")
        return "\n".join(lines)


def _dtype(t) -> str:
    el = t.element_type if isinstance(t, TensorType) else t
    if el.kind == ScalarType.F32:
        return "f32"
    if el.kind == ScalarType.I32:
        return "i32"
    raise NotImplementedError(f"b200 target: element type {el} is not supported")


def _use_counts(root: Value) -> Dict[int, int]:
    counts: Dict[int, int] = {}
    seen = set()
    stack = [root]
    while stack:
        node = stack.pop()
        for child in node.get_children():
            counts[child.id] = counts.get(child.id, 0) + 1
            if child.id not in seen:
                seen.add(child.id)
                stack.append(child)
    return counts


def _match_reduce_body(node: LinalgReduce) -> int:
    """Maps a reduce body to a fold the kernels implement: acc + elem, acc *
    elem (either operand order), If(elem > acc, elem, acc) (max) and
    If(elem < acc, elem, acc) (min), comparisons in either orientation."""
    e, a, body = node.element, node.accumulator, node.body
    if isinstance(body, BinaryOp) and {body.lhs.id, body.rhs.id} == {e.id, a.id}:
        if body.op == ADD:
            return REDUCE_SUM
        if body.op == MUL:
            return REDUCE_PROD
    if (isinstance(body, IfOp) and isinstance(body.cond, CompareOp)
            and body.then_value is e and body.else_value is a):
        c = body.cond
        e_gt_a = (c.pred == "gt" and c.lhs is e and c.rhs is a) or \
                 (c.pred == "lt" and c.lhs is a and c.rhs is e)
        e_lt_a = (c.pred == "lt" and c.lhs is e and c.rhs is a) or \
                 (c.pred == "gt" and c.lhs is a and c.rhs is e)
        if e_gt_a:
            return REDUCE_MAX
        if e_lt_a:
            return REDUCE_MIN
    raise NotImplementedError(
        "b200 target: reduce bodies supported are acc + elem, acc * elem, "
        "If(elem > acc, elem, acc) and If(elem < acc, elem, acc)")


def lower(root: Value, param_names: List[str]) -> Plan:
    """Lowers a traced body to a Plan; raises NotImplementedError for ops
    outside the dense-layer path."""
    plan = Plan(params=list(param_names))
    uses = _use_counts(root)
    memo: Dict[int, Ref] = {}

    def step_of(ref: Ref) -> Optional[Step]:
        return plan.steps[ref.index] if ref.kind == "step" else None

    def single_use(node: Value) -> bool:
        return uses.get(node.id, 0) <= 1

    def emit(step: Step) -> Ref:
        plan.steps.append(step)
        return Ref("step", len(plan.steps) - 1)

    def visit(node: Value) -> Ref:
        if node.id in memo:
            return memo[node.id]
        ref = _visit(node)
        memo[node.id] = ref
        return ref

    def _visit(node: Value) -> Ref:
        if isinstance(node, Parameter):
            return Ref("param", plan.params.index(node.name))
        if isinstance(node, LinalgMatmul):
            a, b = visit(node.lhs), visit(node.rhs)
            t = node.infer_type()
            dt = _dtype(t)
            return emit(Step("gemm_f32" if dt == "f32" else "gemm_i32", [a, b], t.shape, dt))
        if isinstance(node, LinalgBinaryOp):
            if node.op != ADD or node.broadcast not in (TENSOR_BIAS_RIGHT, TENSOR_BIAS_LEFT):
                raise NotImplementedError(
                    f"b200 target: {OP_NAMES[node.op]} with broadcast mode {node.broadcast} is "
                    "not on the dense-layer path (supported: [M,N] + [N] bias add)")
            if node.broadcast == TENSOR_BIAS_RIGHT:
                mat_node, bias_node = node.lhs, node.rhs
            else:
                bias_node, mat_node = node.lhs, node.rhs
            t = node.infer_type()
            dt = _dtype(t)
            mat, bias = visit(mat_node), visit(bias_node)
            s = step_of(mat)
            # Fold into a producing gemm that has no bias/activation yet.
            if (s is not None and s.op.startswith("gemm") and not s.has_bias
                    and s.act == ACT_NONE and single_use(mat_node)):
                s.inputs.append(bias)
                s.has_bias = True
                return mat
            if dt == "i32":
                return emit(Step("bias_add_i32", [mat, bias], t.shape, dt, has_bias=True))
            return emit(Step("bias_act_f32", [mat, bias], t.shape, dt, has_bias=True))
        if isinstance(node, LinalgActivation):
            t = node.infer_type()
            dt = _dtype(t)
            if dt != "f32":
                raise TypeError(f"activation: input must be a float tensor, got {t}")
            act = ACT_RELU if node.act_type == RELU else ACT_LEAKY_RELU
            src = visit(node.input)
            s = step_of(src)
            if (s is not None and s.op in ("gemm_f32", "bias_act_f32") and s.act == ACT_NONE
                    and single_use(node.input)):
                s.act, s.alpha = act, node.alpha
                return src
            return emit(Step("bias_act_f32", [src], t.shape, dt, act=act, alpha=node.alpha))
        if isinstance(node, LinalgDot):
            a, b = visit(node.lhs), visit(node.rhs)
            dt = _dtype(node.infer_type())
            return emit(Step(f"dot_{dt}", [a, b], (), dt))
        if isinstance(node, LinalgReduce):
            if not isinstance(node.init, Constant):
                raise NotImplementedError("b200 target: reduce init must be a constant")
            op = _match_reduce_body(node)
            x = visit(node.input)
            dt = _dtype(node.infer_type())
            return emit(Step(f"reduce_{dt}", [x], (), dt, red_op=op, init=node.init.value))
        if isinstance(node, BinaryOp):
            a, b = visit(node.lhs), visit(node.rhs)
            dt = _dtype(node.infer_type())
            return emit(Step("scalar_op", [a, b], (), dt, scalar_op=node.op))
        if isinstance(node, Constant):
            plan.consts.append(node.value)
            return Ref("const", len(plan.consts) - 1)
        raise NotImplementedError(
            f"b200 target: {type(node).__name__} is not on the dense-layer path")

    plan.output = visit(root)
    return plan
