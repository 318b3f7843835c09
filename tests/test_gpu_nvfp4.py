"""NVFP4 GEMM (tcgen05 kind::mxf4nvf4, block16 UE4M3) against the oracle's
fp64 sum of dequantized products.  The reference pins its FP4 GEMM only by
self-consistency tolerances (tests/gpu/test_fp4_swap_ab_gpu.py: rtol 0.008,
atol 0.001); here the bar is one bf16 rounding step of the exact product
(rtol 2^-7) plus atol 1e-3 for fp32 accumulation order."""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import ops

pytestmark = pytest.mark.gpu


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


# Split K over a cluster: (17, 1536, 1536) over 4 ranks with ragged slices
# of 1-2 K blocks, (64, 2048, 4096) over 4, (17, 4096, 608) over 8 with a
# ragged last channel tile, (5, 6144, 1536) over 8 with 3 K blocks per rank;
# the others run unsplit.
@pytest.mark.parametrize(
    "m,k,n",
    [(1, 256, 128), (17, 1536, 1536), (64, 2048, 4096), (300, 1536, 640), (544, 2048, 2048),
     (17, 4096, 608), (5, 6144, 1536)],
)
@pytest.mark.parametrize("with_bias", [False, True])
def test_nvfp4_gemm_matches_dequantized_product(m, k, n, with_bias):
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16) if with_bias else None
    pa, sa = ops.pack_nvfp4(x.cuda())
    pw, sw = ops.pack_nvfp4(w.cuda())
    out = ops.gemm_nvfp4(pa, sa, pw, sw, None if bias is None else bias.cuda(), n=n)
    torch.cuda.synchronize()
    ref = oracle.nvfp4_gemm(
        pa.cpu().numpy(), sa.cpu().numpy(), pw.cpu().numpy(), sw.cpu().numpy(), m, n, k,
        None if bias is None else bits_of(bias),
    )
    got = oracle.bf16_bits_to_f32(bits_of(out))
    want = oracle.bf16_bits_to_f32(ref)
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=1e-3)
    assert float(np.mean(got == want)) > 0.9


@torch.inference_mode()
def test_floating_linear_matches_packed_formula_and_smoothing_identity():
    """FloatingLinear equals pack + GEMM of its own operands, and the
    SmoothQuant path equals the explicitly pre-transformed Linear bitwise,
    (x / s) @ (W * s) (piR2 tests/gpu/test_smoothquant_gpu.py:28-54)."""
    from pir2_b200.floating import FloatingLinear

    torch.manual_seed(4)
    linear = torch.nn.Linear(1536, 640, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(3, 17, 1536, device="cuda", dtype=torch.bfloat16)
    q = FloatingLinear(linear, "l", "fp4")
    y = q(x)
    pa, sa = ops.pack_nvfp4(x.reshape(-1, 1536))
    ref = ops.gemm_nvfp4(pa, sa, q.packed_weight, q.weight_scale, linear.bias, n=640).reshape(3, 17, 640)
    assert torch.equal(y, ref)
    s = (torch.rand(1536, device="cuda") * 3 + 0.25).float()
    smoothed = FloatingLinear(linear, "l", "fp4", smoothing_scale=s)
    explicit = torch.nn.Linear(1536, 640, device="cuda", dtype=torch.bfloat16)
    explicit.weight.copy_((linear.weight.float() * s).to(torch.bfloat16))
    explicit.bias.copy_(linear.bias)
    plain = FloatingLinear(explicit, "e", "fp4")
    x_s = (x.float() / s).to(torch.bfloat16)
    assert torch.equal(smoothed(x), plain(x_s))


@pytest.mark.parametrize("modulate", [False, True])
@pytest.mark.parametrize("residual", [False, True])
@torch.inference_mode()
def test_fp4_norm_producer_dequantizes_close_to_torch_norm(modulate, residual):
    from pir2_b200.floating import prepare_norm

    torch.manual_seed(6)
    b, t, k = 2, 17, 1536
    x = torch.randn(b, t, k, device="cuda", dtype=torch.bfloat16)
    y = torch.randn_like(x) if residual else None
    scale = (0.3 * torch.randn(b, k, device="cuda")).to(torch.bfloat16) if modulate else None
    shift = (0.3 * torch.randn(b, k, device="cuda")).to(torch.bfloat16) if modulate else None
    packed, summed = prepare_norm(x, "fp4", eps=1e-6, scale=scale, shift=shift, residual=y)
    base = x if y is None else summed
    if y is not None:
        assert torch.equal(summed, x + y)
    n = torch.nn.functional.layer_norm(base, (k,), eps=1e-6)
    if modulate:
        n = n * (1 + scale[:, None]) + shift[:, None]
    pe, se = ops.pack_nvfp4(n.reshape(-1, k))
    got = oracle.unpack_nvfp4(packed.data.cpu().numpy(), packed.scale.cpu().numpy(), b * t, k)
    want = oracle.unpack_nvfp4(pe.cpu().numpy(), se.cpu().numpy(), b * t, k)
    # Same value grid; the fused LayerNorm reduces in another order, so a code
    # may move by one E2M1 step.
    assert np.mean(got == want) > 0.97
    assert np.allclose(got, want, rtol=0.34, atol=0.05)


@torch.inference_mode()
def test_smoothquant_profile_binds_shared_scales_into_floating_projections(tmp_path):
    from pir2_b200 import smoothquant as sq
    from pir2_b200.floating import FloatingLinear, FloatingProjections

    torch.manual_seed(11)
    model = torch.nn.ModuleDict(
        {"gate": torch.nn.Linear(512, 256), "up": torch.nn.Linear(512, 256), "down": torch.nn.Linear(256, 512)}
    ).to(device="cuda", dtype=torch.bfloat16)
    sites = {n: (m, "Role", "text") for n, m in model.items()}
    groups = [["gate", "up"]]
    x = torch.randn(41, 512, device="cuda", dtype=torch.bfloat16)
    x[:, :5] *= 20                                             # outlier channels
    with sq.ActivationCalibration(sites, max_rows=8) as calibration:
        h = model["gate"](x) * model["up"](x)
        model["down"](h)
    path = tmp_path / "profile.pt"
    sq.write_profile(path, sites, groups, calibration, "fp4")
    scales, evidence = sq.load_profile(path, sites, groups, "fp4")
    assert scales["gate"] is scales["up"] and evidence["unsmoothed_linears"] == []
    expected = FloatingLinear(model["gate"], "gate", "fp4", smoothing_scale=scales["gate"])(x)
    original = model["gate"](x)
    projections = FloatingProjections(model, ["gate", "up", "down"], smoothing=scales)
    projections.set()
    try:
        assert torch.equal(model["gate"](x), expected)
    finally:
        projections.close()
    assert torch.equal(model["gate"](x), original)
