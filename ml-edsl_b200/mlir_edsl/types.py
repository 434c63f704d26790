"""Type system of the dense-layer path: scalar and tensor types, Tensor[...].

Mirrors the reference's mlir_edsl/types.py for the types the path uses
(ScalarType i32/f32/i1 at :80-170, DYN at :172, TensorType at :326-453, the
Tensor[...] subscript syntax at :524-573, runtime argument validation at
:649-705 and return-type matching at :710-751), with the same names, checks
and exception types. No protobuf: types are plain Python objects.
"""
from typing import Any, Tuple

DYN = -1


class Type:
    """Base class of all types."""

    def is_scalar(self) -> bool:
        raise NotImplementedError

    def is_aggregate(self) -> bool:
        raise NotImplementedError

    def is_numeric(self) -> bool:
        raise NotImplementedError

    def is_integer(self) -> bool:
        raise NotImplementedError

    def is_float(self) -> bool:
        raise NotImplementedError

    def is_boolean(self) -> bool:
        raise NotImplementedError


class ScalarType(Type):
    """Scalar element type: i32, f32 or i1."""

    I32, F32, I1 = 0, 1, 2
    _KIND_TO_NAME = {I32: "i32", F32: "f32", I1: "i1"}

    def __init__(self, kind: int):
        if kind not in self._KIND_TO_NAME:
            raise ValueError(f"Unknown scalar kind: {kind}")
        self.kind = kind

    @property
    def name(self) -> str:
        return self._KIND_TO_NAME[self.kind]

    def is_scalar(self):
        return True

    def is_aggregate(self):
        return False

    def is_numeric(self):
        return self.kind in (self.I32, self.F32)

    def is_integer(self):
        return self.kind == self.I32

    def is_float(self):
        return self.kind == self.F32

    def is_boolean(self):
        return self.kind == self.I1

    def __eq__(self, other):
        return isinstance(other, ScalarType) and other.kind == self.kind

    def __hash__(self):
        return hash(("scalar", self.kind))

    def __repr__(self):
        return self.name


i32 = ScalarType(ScalarType.I32)
f32 = ScalarType(ScalarType.F32)
i1 = ScalarType(ScalarType.I1)

PYTHON_TO_MLIR = {int: i32, float: f32, bool: i1}
TYPE_HINT_NAMESPACE = {"i32": i32, "f32": f32, "i1": i1}


class TensorType(Type):
    """Value-semantic tensor type of rank 1-3 (tensor<MxNxT>)."""

    def __init__(self, shape, element_type: ScalarType):
        if isinstance(shape, int):
            self.shape = (shape,)
        elif isinstance(shape, tuple):
            self.shape = tuple(shape)
        else:
            raise TypeError(f"Tensor shape must be int or tuple, got {type(shape).__name__}")
        if not all(isinstance(d, int) and (d > 0 or d == DYN) for d in self.shape):
            raise TypeError(f"All dimensions must be positive integers or DYN, got {self.shape}")
        if len(self.shape) == 0 or len(self.shape) > 3:
            raise TypeError(f"Only 1D, 2D, and 3D tensors supported, got {len(self.shape)}D")
        if not isinstance(element_type, ScalarType):
            raise TypeError(f"element_type must be ScalarType (i32, f32, i1), got {element_type}")
        self.element_type = element_type

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def is_dynamic(self) -> bool:
        return DYN in self.shape

    @property
    def total_elements(self) -> int:
        if self.is_dynamic:
            raise ValueError("Cannot compute total_elements for dynamic tensor")
        n = 1
        for d in self.shape:
            n *= d
        return n

    def is_scalar(self):
        return False

    def is_aggregate(self):
        return True

    def is_numeric(self):
        return self.element_type.is_numeric()

    def is_integer(self):
        return self.element_type.is_integer()

    def is_float(self):
        return self.element_type.is_float()

    def is_boolean(self):
        return self.element_type.is_boolean()

    def to_mlir_string(self) -> str:
        dims = "x".join("?" if d == DYN else str(d) for d in self.shape)
        return f"tensor<{dims}x{self.element_type.name}>"

    def __eq__(self, other):
        return (isinstance(other, TensorType) and self.shape == other.shape
                and self.element_type == other.element_type)

    def __hash__(self):
        return hash(("tensor", self.shape, self.element_type))

    def __repr__(self):
        dims = ", ".join("DYN" if d == DYN else str(d) for d in self.shape)
        return f"Tensor[{self.element_type.name}, {dims}]"


class TensorMeta(type):
    """Enables the Tensor[dtype, d0, ...] subscript syntax."""

    def __getitem__(cls, params):
        if not isinstance(params, tuple):
            raise TypeError("Tensor requires parameters: Tensor[dtype, size] or "
                            "Tensor[dtype, M, N]. Example: Tensor[f32, 4]")
        if len(params) < 2:
            raise TypeError(f"Tensor requires at least 2 parameters (dtype + dimensions), "
                            f"got {len(params)}")
        dtype, dims = params[0], params[1:]
        if not isinstance(dtype, ScalarType):
            raise TypeError(f"First parameter must be element type (i32, f32, i1), got {dtype!r}")
        if len(dims) > 3:
            raise TypeError(f"Only 1D, 2D, and 3D tensors supported, got {len(dims)}D")
        for i, d in enumerate(dims):
            if not isinstance(d, int) or (d <= 0 and d != DYN):
                raise TypeError(f"Dimension {i} must be positive integer or DYN, got {d!r}")
        return TensorType(dims[0] if len(dims) == 1 else tuple(dims), dtype)


class Tensor(metaclass=TensorMeta):
    """Tensor[dtype, dims...] type constructor for @ml_function signatures."""


SCALAR_TO_NUMPY = {ScalarType.F32: "float32", ScalarType.I32: "int32", ScalarType.I1: "bool"}


class TypeSystem:
    """Type-hint parsing and runtime validation (same checks and exception
    types as the reference's TypeSystem)."""

    @classmethod
    def parse_type_hint(cls, hint, context: str = "parameter") -> Type:
        if isinstance(hint, Type):
            return hint
        if hint in PYTHON_TO_MLIR:
            return PYTHON_TO_MLIR[hint]
        raise TypeError(f"Invalid type hint for {context}: {hint}")

    @classmethod
    def validate_value_matches_type(cls, value: Any, type_spec: Type, param_name: str):
        if isinstance(type_spec, TensorType):
            if not (hasattr(value, "shape") and hasattr(value, "dtype")):
                raise TypeError(f"Parameter '{param_name}': expected ndarray for {type_spec}, "
                                f"got {type(value).__name__}")
            if len(value.shape) != len(type_spec.shape):
                raise ValueError(f"Parameter '{param_name}': expected {len(type_spec.shape)}D "
                                 f"tensor, got {len(value.shape)}D")
            if not type_spec.is_dynamic and tuple(value.shape) != tuple(type_spec.shape):
                raise ValueError(f"Parameter '{param_name}': expected shape {type_spec.shape}, "
                                 f"got {tuple(value.shape)}")
            return
        if type_spec.is_boolean():
            if not isinstance(value, bool):
                raise TypeError(f"Parameter '{param_name}' expects bool/i1 but got "
                                f"{type(value).__name__}")
        elif type_spec.is_integer():
            if not isinstance(value, (int, bool)):
                raise TypeError(f"Parameter '{param_name}' expects int/i32 but got "
                                f"{type(value).__name__}")
        elif type_spec.is_float():
            if not isinstance(value, (int, float, bool)):
                raise TypeError(f"Parameter '{param_name}' expects float/f32 but got "
                                f"{type(value).__name__}")
        else:
            raise TypeError(f"Parameter '{param_name}': unknown scalar type {type_spec}")

    @classmethod
    def types_match(cls, inferred: Type, declared: Type) -> Tuple[bool, str]:
        if inferred == declared:
            return True, ""
        if inferred.is_scalar() != declared.is_scalar():
            return False, (f"Type category mismatch:\n  Declared: {declared}\n"
                           f"  Inferred: {inferred}\n  Hint: Cannot mix scalar and array types")
        if inferred.is_scalar():
            return False, (f"Type mismatch:\n  Declared: {declared}\n  Inferred: {inferred}\n"
                           f"  Hint: Change return type or add explicit cast")
        if (type(inferred) == type(declared)
                and inferred.element_type == declared.element_type
                and len(inferred.shape) == len(declared.shape)
                and all(d == DYN or d == i for d, i in zip(declared.shape, inferred.shape))):
            return True, ""
        return False, (f"Array type mismatch:\n  Declared: {declared}\n  Inferred: {inferred}\n"
                       f"  Hint: Ensure array shapes and element types match")
