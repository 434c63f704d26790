"""@ml_function: signature parsing, symbolic execution, per-shape variants.

Mirrors the reference's mlir_edsl/functions package for the path:
  FunctionSignature      functions/signature.py:9-122 (type hints, arg
                         ordering, runtime validation, DYN specialisation)
  symbolic_execution     functions/context.py:7-29
  validate_function_body functions/validation.py:10-39
  compile_function       functions/compilation.py:37-77
  MLFunction/ml_function functions/decorator.py:14-133 (per-shape variant
                         cache, name = f"{func.__name__}_{id}")
Differences: the default target is "b200" (the only one this package
implements; "gpu" is an alias), and calling another @ml_function inside a
function body inlines its body instead of emitting a call node.
"""
import inspect
from contextvars import ContextVar
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Tuple, get_type_hints

from .ast import Parameter, Value
from .types import DYN, TYPE_HINT_NAMESPACE, Tensor, TensorType, Type, TypeSystem

DEFAULT_TARGET = "b200"

_symbolic: ContextVar[bool] = ContextVar("symbolic", default=False)


class symbolic_execution:
    """While active, @ml_function calls build AST instead of executing."""

    def __enter__(self):
        self._token = _symbolic.set(True)
        return self

    def __exit__(self, *exc):
        _symbolic.reset(self._token)


def in_symbolic_context() -> bool:
    return _symbolic.get()


def _get_type_hints(func: Callable) -> dict:
    localns = {**TYPE_HINT_NAMESPACE, "Tensor": Tensor, "TensorType": TensorType}
    return get_type_hints(func, globalns={"int": int, "float": float, "bool": bool},
                          localns=localns)


@dataclass
class FunctionSignature:
    name: str
    param_names: List[str]
    param_types: Dict[str, Type]
    return_type: Type

    @classmethod
    def from_callable(cls, func: Callable) -> "FunctionSignature":
        sig = inspect.signature(func)
        hints = _get_type_hints(func)
        names, types = [], {}
        for pname, p in sig.parameters.items():
            if p.annotation == inspect.Parameter.empty:
                raise TypeError(f"@ml_function '{func.__name__}' parameter '{pname}' "
                                f"missing type hint")
            names.append(pname)
            types[pname] = TypeSystem.parse_type_hint(hints[pname], f"parameter '{pname}'")
        if sig.return_annotation == inspect.Signature.empty:
            raise TypeError(f"@ml_function '{func.__name__}' missing return type")
        ret = TypeSystem.parse_type_hint(hints["return"], "return type")
        return cls(name=func.__name__, param_names=names, param_types=types, return_type=ret)

    def _combine(self, args: tuple, kwargs: dict) -> dict:
        combined = {}
        for i, val in enumerate(args):
            if i < len(self.param_names):
                combined[self.param_names[i]] = val
        combined.update(kwargs)
        return combined

    def order_args(self, args: tuple, kwargs: dict) -> List[Any]:
        combined = self._combine(args, kwargs)
        return [combined[n] for n in self.param_names]

    def validate_runtime_args(self, args: tuple, kwargs: dict):
        for name, value in self._combine(args, kwargs).items():
            TypeSystem.validate_value_matches_type(value, self.param_types[name], name)

    def make_param_list(self) -> List[Tuple[str, Type]]:
        return [(n, self.param_types[n]) for n in self.param_names]

    def specialize(self, concrete_shapes: Dict[str, tuple]) -> "FunctionSignature":
        new_types = {}
        for n in self.param_names:
            t = self.param_types[n]
            if isinstance(t, TensorType) and t.is_dynamic and n in concrete_shapes:
                new_types[n] = TensorType(concrete_shapes[n], t.element_type)
            else:
                new_types[n] = t
        suffix = "__".join("_".join(str(d) for d in concrete_shapes[n])
                           for n in self.param_names if n in concrete_shapes)
        return FunctionSignature(name=f"{self.name}__{suffix}" if suffix else self.name,
                                 param_names=self.param_names, param_types=new_types,
                                 return_type=self.return_type)


def validate_function_body(func: Callable, signature: FunctionSignature):
    """Runs `func` on Parameter placeholders; returns (ast, inferred type)."""
    args = [Parameter(n, signature.param_types[n]) for n in signature.param_names]
    with symbolic_execution():
        result = func(*args)
    if not isinstance(result, Value):
        raise TypeError(f"'{signature.name}' must return an EDSL value, got "
                        f"{type(result).__name__}")
    inferred = result.infer_type()
    ok, msg = TypeSystem.types_match(inferred, signature.return_type)
    if not ok:
        raise TypeError(f"Return type mismatch in '{signature.name}':\n{msg}")
    return result, inferred


class CompiledFunction:
    """A compiled shape variant, executable through the backend."""

    def __init__(self, name: str, signature: FunctionSignature, backend, target: str):
        self.name, self.signature, self._backend, self._target = name, signature, backend, target

    def execute(self, args: tuple, kwargs: dict):
        self.signature.validate_runtime_args(args, kwargs)
        return self._backend.execute_function(self.name,
                                              *self.signature.order_args(args, kwargs))


def compile_function(signature: FunctionSignature, result_ast: Value,
                     target: str = DEFAULT_TARGET) -> CompiledFunction:
    from .backend import get_backend
    backend = get_backend()
    if backend is None:
        raise RuntimeError("B200 backend not available for execution")
    if backend.has_function(signature.name):
        return CompiledFunction(signature.name, signature, backend, target)
    backend.set_target(target)
    backend.compile_function_from_ast(signature.name, signature.make_param_list(),
                                      signature.return_type, result_ast)
    return CompiledFunction(signature.name, signature, backend, target)


class MLFunction:
    """A user function compiled per input-shape variant and run on B200."""

    _next_id = 0

    def __init__(self, func: Callable, target: str = DEFAULT_TARGET):
        self.func = func
        self._target = target
        self._func_id = MLFunction._next_id
        MLFunction._next_id += 1
        self.signature = FunctionSignature.from_callable(func)
        self.signature.name = f"{func.__name__}_{self._func_id}"
        self._compiled_variants: Dict[Tuple, CompiledFunction] = {}

    def __call__(self, *args, **kwargs):
        if in_symbolic_context():
            # Inline the callee: its body is traced on the caller's values.
            ordered = self.signature.order_args(args, kwargs)
            return self.func(*ordered)
        return self._execute(args, kwargs)

    def _execute(self, args: tuple, kwargs: dict):
        self.signature.validate_runtime_args(args, kwargs)
        ordered = self.signature.order_args(args, kwargs)
        concrete = {}
        for name, val in zip(self.signature.param_names, ordered):
            t = self.signature.param_types[name]
            if t.is_aggregate() and t.is_dynamic:
                concrete[name] = tuple(val.shape)
        key = tuple(concrete[n] for n in self.signature.param_names if n in concrete)
        if key not in self._compiled_variants:
            spec = self.signature.specialize(concrete)
            ast, inferred = validate_function_body(self.func, spec)
            ret = spec.return_type
            if ret.is_aggregate() and ret.is_dynamic:
                if inferred.is_dynamic:
                    raise TypeError(
                        f"Cannot determine return shape for DYN return type in "
                        f"'{self.func.__name__}': abstract evaluation produced dynamic shape. "
                        "Output shape must be deterministic from input shapes.")
                spec = FunctionSignature(spec.name, spec.param_names, spec.param_types, inferred)
            self._compiled_variants[key] = compile_function(spec, ast, target=self._target)
        variant = self._compiled_variants[key]
        return variant.execute(args, kwargs)


def ml_function(func: Callable = None, *, target: str = DEFAULT_TARGET):
    """Decorator: @ml_function or @ml_function(target="b200")."""
    if func is not None:
        return MLFunction(func, target=DEFAULT_TARGET)

    def decorator(f: Callable) -> MLFunction:
        return MLFunction(f, target=target)

    return decorator
