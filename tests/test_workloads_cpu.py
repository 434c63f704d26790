"""The benchmark's seeded inputs (mlir_edsl.workloads) are the oracle's
(oracle.gen_config_inputs), and rows drawn on their own equal the slice of
the whole array: a row-sharded bench rank times exactly the rows the parity
tests check."""
import numpy as np
import pytest

import oracle
from mlir_edsl import workloads

SMALL = ["matmul_256", "dense_1024", "dense_ragged", "matmul_i32_2048"]


@pytest.mark.parametrize("name", SMALL)
def test_inputs_match_oracle_generator(name):
    a, b = workloads.config_inputs(name), oracle.gen_config_inputs(name)
    assert a.keys() == b.keys()
    for k in a:
        np.testing.assert_array_equal(a[k], b[k])


@pytest.mark.parametrize("name,array,r0,r1", [
    ("dense_1024", "X", 0, 1024), ("dense_1024", "X", 333, 334), ("dense_1024", "W", 5, 700),
    ("dense_1024", "b", 0, 1024), ("dense_ragged", "W", 999, 1001), ("dense_ragged", "b", 17, 18),
    ("matmul_256", "B", 100, 256)])
def test_rows_on_their_own_equal_the_slice(name, array, r0, r1):
    full = oracle.gen_config_inputs(name)[array]
    np.testing.assert_array_equal(workloads.config_rows(name, array, r0, r1), full[r0:r1])


def test_mlp_weights_alone():
    full = workloads.config_inputs("mlp_2layer")
    np.testing.assert_array_equal(workloads.config_array("mlp_2layer", "b2"), full["b2"])
    np.testing.assert_array_equal(workloads.config_rows("mlp_2layer", "W2", 11000, 11008),
                                  full["W2"][11000:])


def test_row_range_checked():
    with pytest.raises(ValueError):
        workloads.config_rows("dense_1024", "X", 10, 2000)
    with pytest.raises(ValueError):
        workloads.config_rows("matmul_i32_2048", "A", 0, 1)
