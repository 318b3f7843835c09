"""The oracle's FP8 (E4M3, per-tensor) quantizer, checked on the CPU against
torch's own float8_e4m3fn conversion (an independent round-to-nearest-even
implementation) and against the reference's scale formulas.  The
reference's FP8 kernels are CUDA/CUTLASS (and a Triton variant) that cannot
run here, so this pins the restatement, not the reference binary."""

import numpy as np
import torch

import oracle


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_default_variant_matches_torch_e4m3_cast():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(37, 256, generator=g) * 3.0
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-6, -1e-6, 448.0, -1e4, float("inf"), float("nan")])
    xb = x.to(torch.bfloat16)
    codes, scale = oracle.quant_fp8(_bits(xb))
    f = xb.float()
    amax = torch.where(torch.isfinite(f.abs()), f.abs(), torch.zeros_like(f)).max()
    want_scale = torch.clamp(amax / 448.0, min=1e-12)
    assert np.float32(want_scale.item()) == scale
    inv = (torch.tensor(1.0) / want_scale).float()
    y = torch.nan_to_num(f * inv, nan=-448.0).clamp(-448.0, 448.0)
    want = y.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(codes, want)


def test_fast_variant_uses_the_division_formula():
    g = torch.Generator().manual_seed(1)
    xb = (torch.randn(5, 128, generator=g) * 0.01).to(torch.bfloat16)
    codes, scale = oracle.quant_fp8(_bits(xb), fast=True)
    f = xb.float()
    want_scale = torch.clamp(f.abs().max() * np.float32(1.0 / 448.0), min=1e-12)
    assert np.float32(want_scale.item()) == scale
    want = (f / want_scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(codes, want)


def test_decode_round_trip_and_gemm_reference():
    codes = np.arange(256, dtype=np.uint8)
    codes = codes[(codes & 0x7F) != 0x7F]   # skip NaN
    v = oracle.e4m3_decode(codes)
    t = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(v.astype(np.float32), t)
    qa = np.array([[0x38, 0xB8]], dtype=np.uint8)   # +1, -1
    qw = np.array([[0x40, 0x38]], dtype=np.uint8)   # +2, +1
    assert oracle.fp8_gemm(qa, 0.5, qw, 2.0)[0, 0] == (2.0 - 1.0) * 0.5 * 2.0
