"""CPU oracle for Kernix's dense matmul path -- test infrastructure only.

Imported by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
as the checker; the product never imports it.
"""
from .oracle import *  # noqa: F401,F403
from .oracle import (THREADS, OracleError, View, broadcast_shape, build, conv2d_dot2, conv2d_reference,  # noqa: F401
                     conv_shape, dense_matmul, gemm_dot2, gemm_ordered_par, lib, matmul_reference, matmul_shape,
                     softmax_temperature, splitmix_next, uniform, validate_dims)
