"""CPU oracle for the dense-layer hot path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, as the checker; the product path never imports it.
"""
from .oracle import (  # noqa: F401
    build, dense_f32, matmul_i32, bias_act_f32, fma_mode, gen_config_inputs, f32_bound,
    reduce_f32, reduce_i32, dot_f32, dot_i32, sum_bound,
    REDUCE_SUM, REDUCE_PROD, REDUCE_MAX, REDUCE_MIN, REDUCE_INIT,
    ACT_NONE, ACT_RELU, ACT_LEAKY_RELU, MODE_AUTO, MODE_FMA, MODE_MULADD,
)
