"""Host-side checks of the floating producers and the packs that take their
row maxima from a GEMM: wrong inputs are refused with a ValueError before
anything reaches the library (no GPU needed), and the configuration rules
of the floating fusions follow piR2's (coexecution/optimization/config.py:
74-83)."""

import pytest
import torch

from pir2_b200 import ops
from pir2_b200.config import OptimizationConfig
from pir2_b200.floating import (
    aligned_for,
    prepare_fp8,
    prepare_gelu_packed,
    prepare_norm,
    prepare_rmsnorm_packed,
    prepare_smoothed,
    prepare_swiglu,
)


@pytest.mark.parametrize(
    "kwargs,match",
    [
        ({"precision": "w8a8", "fp_swiglu": True}, "Floating fusion"),
        ({"precision": "w8a8", "fp_grouped": True}, "Floating fusion"),
        ({"precision": "w4a4", "fp_gelu": True}, "Floating producers"),
        ({"precision": "w8a8", "fp_rmsnorm": True}, "Floating producers"),
        ({"precision": "w8a8", "fp_shared_inputs": True}, "Shared floating inputs"),
        ({"precision": "fp4", "fp8_fast_quant": True}, "Fast FP8"),
    ],
)
def test_floating_fusions_need_a_floating_precision(kwargs, match):
    with pytest.raises(ValueError, match=match):
        OptimizationConfig(**kwargs)


def test_floating_fusion_flags_are_accepted_for_fp8_and_fp4():
    for precision in ("fp8", "fp4"):
        config = OptimizationConfig(
            precision=precision, scope="all", fp_grouped=True, fp_swiglu=True, fp_gelu=True, fp_rmsnorm=True,
            fusion=True, norm_modulation_quant=True, residual_norm_quant=True,
        )
        assert config.enabled


def test_floating_alignment_rules():
    # FP8: K % 128 (the E4M3 GEMM's K block), N % 16; NVFP4: K % 256, N % 32.
    assert aligned_for("fp8", 1536, 6144) and not aligned_for("fp8", 1560, 6144)
    assert not aligned_for("fp8", 1536, 6152)
    assert aligned_for("fp4", 2048, 4096) and not aligned_for("fp4", 1920, 4096)
    assert not aligned_for("fp4", 2048, 4112)


def test_fp8_value_slices():
    # One partial maximum per row and 1024-value slice of the first pass.
    assert [ops.fp8_value_slices(k) for k in (16, 1024, 1025, 1536, 6144, 8192)] == [1, 1, 2, 2, 6, 8]


def test_producers_refuse_host_tensors():
    x = torch.zeros(17, 1536, dtype=torch.bfloat16)
    lut = torch.zeros(65536, dtype=torch.bfloat16)
    for precision in ("fp8", "fp4"):
        with pytest.raises(ValueError, match="Floating producer"):
            prepare_swiglu(x, x, lut, precision)
        with pytest.raises(ValueError, match="Floating producer"):
            prepare_gelu_packed(x, lut, precision)
        with pytest.raises(ValueError, match="Floating producer"):
            prepare_rmsnorm_packed(x, torch.ones(1536, dtype=torch.bfloat16), precision, eps=1e-6)
        with pytest.raises(ValueError, match="Floating producer"):
            prepare_norm(x.reshape(1, 17, 1536), precision, eps=1e-6)
        with pytest.raises(ValueError):
            prepare_smoothed(x, precision, torch.ones(1536))
    with pytest.raises(ValueError, match="FP8 packing"):
        prepare_fp8(x)


def test_producers_refuse_other_precisions_and_widths():
    # The producers serve fp8 / fp4 only, and need K % 16 (fp8) or % 32
    # (fp4) and at most 8192 values per row; checked before any launch.
    x = torch.zeros(4, 1536, dtype=torch.bfloat16)
    lut = torch.zeros(65536, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Floating producer"):
        prepare_gelu_packed(x, lut, "w8a8")
    with pytest.raises(ValueError, match="Floating producer"):
        prepare_gelu_packed(torch.zeros(4, 1544, dtype=torch.bfloat16), lut, "fp4")


def test_given_maxima_pack_and_fp8_cast_refuse_host_tensors():
    x = torch.zeros(17, 6144, dtype=torch.bfloat16)
    maxima = torch.zeros(17, 384)
    with pytest.raises(ValueError, match="CUDA BF16"):
        ops.quant_rows_max(x, maxima, 8)
    with pytest.raises(ValueError, match="fp8_cast"):
        ops.fp8_cast(x, maxima.reshape(-1))
    with pytest.raises(ValueError, match="CUDA BF16"):
        ops.floating_rows(x, 32)
