"""CPU oracle for the quantized-Linear hot path (test infrastructure only).

This package restates, in numpy on the CPU, the reference algorithms of
piR2's quantized Linear path so the CUDA kernels can be checked against them.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import it, and only as the checker or the timed CPU baseline; the product
path (pir2_b200) never imports it.

Pinning: tests/golden/ holds vectors produced by running the reference's own
Triton kernels (integer.py `_prepare`, modulation.py producers, producers.py
`_rms_tail_pack`, thor/packing.py NVFP4 producers and `prepare_fp8`) under
Triton's CPU interpreter, the reference's CPU-runnable `channel_scales`, and
the explicit torch formula of the reference's bitwise Linear test;
tests/test_oracle_golden.py checks this oracle against them.
"""

from .quant import *  # noqa: F401,F403
