"""Generates tests/golden/known_answers.json: the known-answer cases that the
reference's own tests hold for the dense-layer path, restated as data.

Each case records the reference test it restates (file:line in ml-edsl), the
inputs that test builds, the answer it asserts (a literal where the test
writes one, else the NumPy expression the test compares against, evaluated
here in float64) and the test's tolerance. Run: python tests/golden/make_golden.py
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def case(name, source, op, inputs, expected, rtol=0.0, atol=0.0, alpha=0.0):
    return {"name": name, "source": source, "op": op, "alpha": alpha,
            "inputs": {k: {"dtype": str(np.asarray(v).dtype), "data": np.asarray(v).tolist()}
                       for k, v in inputs.items()},
            "expected": np.asarray(expected).tolist(), "rtol": rtol, "atol": atol}


def main():
    f = np.float32
    A22 = np.array([[1.0, 2.0], [3.0, 4.0]], f)
    B22 = np.array([[5.0, 6.0], [7.0, 8.0]], f)
    rng = np.random.default_rng(42)
    S16a = rng.random((16, 16), dtype=f)
    S16b = rng.random((16, 16), dtype=f)
    X24 = np.array([[1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0]], f)
    b4 = np.array([0.1, 0.2, 0.3, 0.4], f)
    Xr = np.array([[-1.0, 2.0, -3.0, 4.0], [5.0, -6.0, 7.0, -8.0]], f)
    Xd = np.array([[1.0, 0.0, 0.0, 0.0], [0.0, 1.0, 0.0, 0.0]], f)
    Wd = np.ones((4, 3), f)
    bd = np.array([0.1, 0.2, 0.3], f)
    f64 = lambda a: np.asarray(a, np.float64)
    cases = [
        case("matmul_identity_2x2", "tests/linalg/test_matmul_execution.py:20-30", "matmul",
             {"A": A22, "B": np.eye(2, dtype=f)}, A22, rtol=1e-4),
        case("matmul_known_2x2", "tests/linalg/test_matmul_execution.py:32-42", "matmul",
             {"A": A22, "B": B22}, [[19.0, 22.0], [43.0, 50.0]], rtol=1e-3),
        case("matmul_ones_8", "tests/linalg/test_matmul_execution.py:44-54", "matmul",
             {"A": np.ones((8, 8), f), "B": np.ones((8, 8), f)}, np.full((8, 8), 8.0), atol=1e-5),
        case("matmul_ones_16", "tests/linalg/test_matmul_execution.py:56-66", "matmul",
             {"A": np.ones((16, 16), f), "B": np.ones((16, 16), f)}, np.full((16, 16), 16.0),
             atol=1e-4),
        case("matmul_seeded_16", "tests/linalg/test_matmul_execution.py:68-79", "matmul",
             {"A": S16a, "B": S16b}, f64(S16a) @ f64(S16b), rtol=1e-4, atol=1e-4),
        case("matmul_zeros", "tests/linalg/test_matmul_execution.py:81-91", "matmul",
             {"A": A22, "B": np.zeros((2, 2), f)}, np.zeros((2, 2)), atol=1e-5),
        case("matmul_i32_identity", "tests/linalg/test_matmul_execution.py:93-103", "matmul_i32",
             {"A": np.eye(2, dtype=np.int32), "B": B22.astype(np.int32)}, [[5, 6], [7, 8]]),
        case("matmul_rect_ones", "tests/linalg/test_binary_op_execution.py:176-186", "matmul",
             {"A": np.ones((2, 3), f), "B": np.ones((3, 4), f)}, np.full((2, 4), 3.0),
             rtol=1e-5),
        case("bias_add_2x4", "tests/linalg/test_binary_op_execution.py:114-124", "bias_add",
             {"X": X24, "b": b4}, f64(X24) + f64(b4), rtol=1e-5),
        case("bias_add_left", "tests/linalg/test_binary_op_execution.py:126-135", "bias_add",
             {"X": np.zeros((2, 4), f), "b": np.array([1.0, 2.0, 3.0, 4.0], f)},
             [[1.0, 2.0, 3.0, 4.0], [1.0, 2.0, 3.0, 4.0]], rtol=1e-5),
        case("bias_add_zero", "tests/linalg/test_binary_op_execution.py:137-145", "bias_add",
             {"X": np.arange(9, dtype=f).reshape(3, 3), "b": np.zeros(3, f)},
             np.arange(9, dtype=np.float64).reshape(3, 3), rtol=1e-5),
        case("dense_no_activation", "tests/linalg/test_binary_op_execution.py:193-208", "dense",
             {"X": Xd, "W": Wd, "b": bd}, f64(Xd) @ f64(Wd) + f64(bd), rtol=1e-4),
        case("relu_1d_mixed", "tests/linalg/test_map_execution.py:74-82", "relu",
             {"X": np.array([-1.0, 2.0, -3.0, 4.0], f)}, [0.0, 2.0, 0.0, 4.0], atol=1e-5),
        case("relu_1d_negative", "tests/linalg/test_map_execution.py:64-72", "relu",
             {"X": np.array([-1.0, -2.0, -3.0, -4.0], f)}, [0.0, 0.0, 0.0, 0.0], atol=1e-5),
        case("leaky_relu_1d_negative", "tests/linalg/test_map_execution.py:94-103", "leaky_relu",
             {"X": np.array([-1.0, -2.0, -10.0, -0.5], f)}, [-0.1, -0.2, -1.0, -0.05],
             atol=1e-5, alpha=0.1),
        case("relu_2d_mixed", "tests/linalg/test_map_execution.py:120-129", "relu",
             {"X": Xr}, np.maximum(f64(Xr), 0.0), rtol=1e-5),
        case("leaky_relu_2d", "tests/linalg/test_map_execution.py:151-161", "leaky_relu",
             {"X": Xr}, np.where(Xr > 0, f64(Xr), f64(Xr) * 0.1), rtol=1e-4, alpha=0.1),
        # linalg.dot / reduce (scalar results)
        case("dot_all_ones", "tests/linalg/test_dot_execution.py:18-26", "dot",
             {"a": np.ones(4, f), "b": np.ones(4, f)}, 4.0, atol=1e-5),
        case("dot_known", "tests/linalg/test_dot_execution.py:28-36", "dot",
             {"a": np.array([1, 2, 3, 4], f), "b": np.ones(4, f)}, 10.0, atol=1e-5),
        case("dot_squares", "tests/linalg/test_dot_execution.py:38-46", "dot",
             {"a": np.array([1, 2, 3], f), "b": np.array([1, 2, 3], f)}, 14.0, atol=1e-5),
        case("dot_i32", "tests/linalg/test_dot_execution.py:48-56", "dot_i32",
             {"a": np.array([1, 2, 3, 4], np.int32), "b": np.array([4, 3, 2, 1], np.int32)}, 20),
        case("dot_zeros", "tests/linalg/test_dot_execution.py:58-66", "dot",
             {"a": np.array([1, 2, 3], f), "b": np.zeros(3, f)}, 0.0, atol=1e-5),
        case("dot_single", "tests/linalg/test_dot_execution.py:68-76", "dot",
             {"a": np.array([3.0], f), "b": np.array([7.0], f)}, 21.0, atol=1e-5),
        case("sum_positive", "tests/linalg/test_reduce_execution.py:21-27", "sum",
             {"a": np.array([1, 2, 3, 4], f)}, 10.0, atol=1e-5),
        case("sum_negatives", "tests/linalg/test_reduce_execution.py:29-35", "sum",
             {"a": np.array([-1, 2, -3, 4], f)}, 2.0, atol=1e-5),
        case("sum_single", "tests/linalg/test_reduce_execution.py:45-51", "sum",
             {"a": np.array([42.0], f)}, 42.0, atol=1e-5),
        case("sum_8", "tests/linalg/test_reduce_execution.py:53-59", "sum",
             {"a": np.arange(1, 9, dtype=f)}, 36.0, atol=1e-4),
        case("max_positive", "tests/linalg/test_reduce_execution.py:67-73", "max",
             {"a": np.array([1, 4, 2, 3], f)}, 4.0, atol=1e-5),
        case("max_negatives", "tests/linalg/test_reduce_execution.py:75-81", "max",
             {"a": np.array([-1, -4, -2, -3], f)}, -1.0, atol=1e-5),
        case("max_last", "tests/linalg/test_reduce_execution.py:91-97", "max",
             {"a": np.array([1, 2, 3, 9], f)}, 9.0, atol=1e-5),
        case("min_positive", "tests/linalg/test_reduce_execution.py:105-111", "min",
             {"a": np.array([3, 1, 4, 2], f)}, 1.0, atol=1e-5),
        case("min_negatives", "tests/linalg/test_reduce_execution.py:113-119", "min",
             {"a": np.array([1, -2, 3, -4], f)}, -4.0, atol=1e-5),
        case("min_first", "tests/linalg/test_reduce_execution.py:129-135", "min",
             {"a": np.array([-9, 2, 3, 4], f)}, -9.0, atol=1e-5),
        case("product", "tests/linalg/test_reduce_execution.py:151-157", "prod",
             {"a": np.array([1, 2, 3, 4], f)}, 24.0, atol=1e-4),
    ]
    with open(os.path.join(HERE, "known_answers.json"), "w") as fh:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": cases}, fh, indent=1)
    print(f"wrote {len(cases)} cases")


if __name__ == "__main__":
    main()
