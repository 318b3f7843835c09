"""Tactic and swap-AB invariance, the counterparts of piR2's
tests/gpu/test_shape_tactics_gpu.py (a tactic selects a kernel, never the
bytes) and tests/gpu/test_fp4_swap_ab_gpu.py (the swap-AB FP4 GEMM agrees
with the baseline).  On B200 the tcgen05 GEMM plans its tiles per call and
has no separate swap-AB variant, so both must hold bit for bit."""

import pytest
import torch

from pir2_b200 import _lib, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("m", [17, 544])
def test_integer_gemm_is_the_same_for_every_tactic(bits, m):
    torch.manual_seed(bits * 1000 + m)
    x = torch.randn(m, 1536, device="cuda", dtype=torch.bfloat16)
    w = torch.randint(-127, 128, (1536, 1536 if bits == 8 else 768), device="cuda", dtype=torch.int8)
    if bits == 4:
        w = w.view(torch.uint8)
    sw = torch.rand(1536, device="cuda") * 1e-3
    bias = (torch.randn(1536, device="cuda") * 0.01).to(torch.bfloat16)
    qa, sa = ops.quant_rows(x, bits)
    outs = [ops.gemm(qa, sa, w, sw, bias, bits, n_store=1536, tactic=t) for t in range(8)]
    for out in outs[1:]:
        assert torch.equal(out, outs[0])
    assert _lib.device_status() == 0


def test_fp4_swap_ab_equals_the_baseline_linear():
    from pir2_b200.floating import FloatingLinear

    torch.manual_seed(6)
    linear = torch.nn.Linear(1536, 640, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(2, 17, 1536, device="cuda", dtype=torch.bfloat16)
    base = FloatingLinear(linear, "l", "fp4")
    swapped = FloatingLinear(linear, "l", "fp4", fp4_swap_ab=True)
    assert torch.equal(swapped(x), base(x))
    assert _lib.device_status() == 0
