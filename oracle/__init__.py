"""CPU oracle for the complex Conv2d forward (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
use this package, as the checker.  The product package never imports it.
"""

from .oracle import (  # noqa: F401
    ConvCase,
    backward_autograd_fp64,
    backward_formula_fp64,
    build_c_oracle,
    direct_c,
    four_conv,
    im2col_numpy,
    make_inputs,
    oracle_fp64,
    planar_nhwc_to_complex_nchw,
    rel_frobenius,
    time_cpu_four_conv,
)
from .configs import BASELINE_CASES, CPU_CASE  # noqa: F401
