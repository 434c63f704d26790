"""Seeded synthetic inputs of the benchmark configurations.

Generator: np.random.default_rng(seed); arrays drawn in the listed order; f32
arrays as rng.uniform(lo, hi, shape).astype(float32), i32 arrays as
rng.integers(-8, 9, shape, dtype=int32). Every f32 draw consumes exactly one
64-bit output of the PCG64 stream, so rows [r0, r1) of any f32 array can be
drawn without the rows before them (bit_generator.advance): each rank of a
row-sharded run generates only its own rows, bit-identical to the slice of
the whole array.
"""
from typing import Dict, List, Tuple

import numpy as np

# name -> (seed, lo, hi, [(array, shape), ...], kind)
CONFIGS: Dict[str, Tuple[int, float, float, List[Tuple[str, tuple]], str]] = {
    "matmul_256": (0, -1.0, 1.0, [("A", (256, 256)), ("B", (256, 256))], "f32"),
    "dense_1024": (1, -1.0, 1.0, [("X", (1024, 1024)), ("W", (1024, 1024)), ("b", (1024,))],
                   "f32"),
    "matmul_4096": (2, -1.0, 1.0, [("A", (4096, 4096)), ("B", (4096, 4096))], "f32"),
    "matmul_8192": (2, -1.0, 1.0, [("A", (8192, 8192)), ("B", (8192, 8192))], "f32"),
    # the 8192^3 dense layer: matmul_8192's A and B, then a bias from the same stream
    "dense_8192": (2, -1.0, 1.0, [("A", (8192, 8192)), ("B", (8192, 8192)), ("b", (8192,))],
                   "f32"),
    "matmul_i32_2048": (2, -8, 8, [("A", (2048, 2048)), ("B", (2048, 2048))], "i32"),
    "dense_65536": (3, -0.5, 0.5, [("X", (65536, 4096)), ("W", (4096, 4096)), ("b", (4096,))],
                    "f32"),
    "dense_ragged": (4, -1.0, 1.0, [("X", (1000, 1001)), ("W", (1001, 999)), ("b", (999,))],
                     "f32"),
    "mlp_2layer": (4, -1.0, 1.0, [("X", (512, 4096)), ("W1", (4096, 11008)), ("b1", (11008,)),
                                  ("W2", (11008, 4096)), ("b2", (4096,))], "f32"),
}


def config_inputs(name: str) -> Dict[str, np.ndarray]:
    """Every array of configuration `name`."""
    seed, lo, hi, arrays, kind = CONFIGS[name]
    rng = np.random.default_rng(seed)
    out = {}
    for a, shape in arrays:
        if kind == "i32":
            out[a] = rng.integers(-8, 9, shape, dtype=np.int32)
        else:
            out[a] = rng.uniform(lo, hi, shape).astype(np.float32)
    return out


def _offset(name: str, array: str) -> int:
    _, _, _, arrays, _ = CONFIGS[name]
    off = 0
    for a, shape in arrays:
        if a == array:
            return off
        off += int(np.prod(shape))
    raise KeyError(array)


def config_rows(name: str, array: str, r0: int, r1: int) -> np.ndarray:
    """Rows [r0, r1) of f32 array `array` of configuration `name` (the first
    axis for a 1-D array), drawn on their own."""
    seed, lo, hi, arrays, kind = CONFIGS[name]
    if kind != "f32":
        raise ValueError("row-wise generation is for f32 configurations")
    shape = dict(arrays)[array]
    if not 0 <= r0 <= r1 <= shape[0]:
        raise ValueError(f"rows [{r0}, {r1}) outside {shape}")
    per_row = int(np.prod(shape[1:]))
    rng = np.random.default_rng(seed)
    rng.bit_generator.advance(_offset(name, array) + r0 * per_row)
    return rng.uniform(lo, hi, (r1 - r0,) + tuple(shape[1:])).astype(np.float32)


def config_array(name: str, array: str) -> np.ndarray:
    """The whole f32 array `array` of configuration `name`, alone."""
    shape = dict(CONFIGS[name][3])[array]
    return config_rows(name, array, 0, shape[0])
