"""Fused floating producers on the B200 kernels (SwiGLU, GELU, SmoothQuant,
RMSNorm, residual + LayerNorm + AdaLN to FP8 and NVFP4), checked against the
oracle, whose FP8 producers are pinned to the reference's own Triton
producers (tests/test_oracle_golden.py).

Reduction-free producers (LUT, SiLU * up, smoothing, modulation) are bitwise
equal to the oracle: bf16 values, row maxima, E4M3 codes and scale, NVFP4
codes and factors.  The norm producers reduce in their own order, so their
values may sit one bf16 step from the oracle's on some elements; their
second pass (scale and cast of the kernel's own values) is bitwise."""

import numpy as np
import pytest
import torch

import oracle
from oracle import quant as oq
from pir2_b200 import _lib, ops
from pir2_b200.fused import prepare_gelu, prepare_silu

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__file__.rsplit("/", 1)[0] + "/golden/golden.npz")


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b, shape):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16).reshape(shape)).view(torch.bfloat16).cuda()


def assert_factors_equal(sf, want, rows, k):
    """NVFP4 factors at the positions of real rows and 16-blocks (the padding
    of the 128-row x 4-factor atoms is left unwritten, as in piR2's
    torch.empty factor buffers)."""
    blocks_k = (k // 16 + 3) // 4
    rr, jj = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    offsets = oracle.nvfp4_sf_offset(rr, jj, blocks_k)
    assert np.array_equal(np.asarray(sf).reshape(-1)[offsets], np.asarray(want).reshape(-1)[offsets])


def assert_fp8_stage(values, row_max, q, scale, rows):
    """The cast stage of the kernel's own values equals the oracle's; `rows`
    is the replicated scale vector fp8_cast wrote."""
    v = oracle.bf16_bits_to_f32(bits_of(values))
    # Partial maxima: one per row and 1024-value slice (norm producers: one per row).
    per_row = row_max.cpu().numpy().reshape(v.shape[0], -1).max(axis=1)
    assert np.array_equal(per_row.view(np.uint32), oracle.row_finite_max(v).view(np.uint32))
    want_q, want_s = oracle.fp8_producer(v)
    assert np.float32(scale.item()) == want_s
    assert torch.equal(rows, torch.full_like(rows, float(want_s)))
    assert np.array_equal(q.cpu().numpy(), want_q)


@pytest.mark.parametrize("name", ["swiglu", "gelu"])
def test_fp8_lut_producers_equal_reference_golden(name):
    """The reference's own `_swiglu_pack` / `_gelu_pack` + `_fp8_scale_and_cast`
    outputs (golden vectors): values, maxima, codes and scale, bit for bit."""
    if name == "swiglu":
        gate = GOLDEN["fp8p_swiglu_gate"]
        rows, k = 17, 256
        x = from_bits(gate, (rows, k))
        up = from_bits(GOLDEN["fp8p_swiglu_up"], (rows, k))
        values, row_max = ops.floating_rows(x, _lib.OUT_FP8_VALUES, lut=prepare_silu(x.device), up=up)
    else:
        rows, k = 9, 384
        x = from_bits(GOLDEN["fp8p_gelu_x"], (rows, k))
        smooth = torch.from_numpy(GOLDEN["fp8p_gelu_smooth"]).cuda()
        lut = prepare_gelu(x.device, torch.bfloat16, "tanh")
        values, row_max = ops.floating_rows(x, _lib.OUT_FP8_VALUES, lut=lut, smooth=smooth)
    q, scale, rep = ops.fp8_cast(values, row_max)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(values), GOLDEN[f"fp8p_{name}_values"].reshape(rows, k))
    per_row = row_max.cpu().numpy().reshape(rows, -1).max(axis=1)
    assert np.array_equal(per_row.view(np.uint32), GOLDEN[f"fp8p_{name}_rowmax"].view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), GOLDEN[f"fp8p_{name}_q"].reshape(rows, k))
    assert np.float32(scale.item()).view(np.uint32) == GOLDEN[f"fp8p_{name}_s"].view(np.uint32)
    assert torch.equal(rep, torch.full_like(rep, scale.item()))
    assert _lib.device_status() == 0


@pytest.mark.parametrize("mode", ["plain", "gelu", "swiglu"])
@pytest.mark.parametrize("smooth", [False, True])
@pytest.mark.parametrize("rows,k", [(1, 1536), (17, 6144), (544, 2048), (40, 8192)])
def test_floating_rows_fp8_and_nvfp4_equal_oracle(mode, smooth, rows, k):
    """Both floating outputs of the LUT / gated / plain producer, with and
    without SmoothQuant: FP8 values, maxima, codes and scale, and NVFP4 codes
    and factors, bitwise equal to the oracle (gate rows strided, as merged
    gate|up projection views are)."""
    g = torch.Generator().manual_seed(rows * 31 + k + len(mode) + smooth)
    merged = (torch.randn(rows, 2 * k, generator=g) * 3).to(torch.bfloat16).cuda()
    x = merged[:, :k] if mode == "swiglu" else merged[:, :k].contiguous()
    up = merged[:, k:] if mode == "swiglu" else None
    lut = None
    if mode == "gelu":
        lut = prepare_gelu(x.device, torch.bfloat16, "tanh")
    elif mode == "swiglu":
        lut = prepare_silu(x.device)
    s = (0.25 + 2 * torch.rand(k, generator=g)).float().cuda() if smooth else None
    want = oracle.floating_values(
        bits_of(x), lut_bits=None if lut is None else bits_of(lut), up_bits=None if up is None else bits_of(up),
        smooth=None if s is None else s.cpu().numpy(),
    )
    values, row_max = ops.floating_rows(x, _lib.OUT_FP8_VALUES, lut=lut, up=up, smooth=s)
    q, scale, rep = ops.fp8_cast(values, row_max)
    data, sf = ops.floating_rows(x, _lib.OUT_NVFP4, lut=lut, up=up, smooth=s)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(values), oracle.f32_to_bf16_bits(want))
    assert_fp8_stage(values, row_max, q, scale, rep)
    packed, factors = oracle.pack_nvfp4(want)
    assert np.array_equal(data.cpu().numpy(), packed)
    assert_factors_equal(sf.cpu().numpy(), factors, rows, k)
    assert _lib.device_status() == 0


def test_fp8_modulation_producer_equals_oracle_and_norms_cast_bitwise():
    """AdaLN modulation without a norm (no reduction) to FP8 values is
    bitwise the oracle's; RMSNorm and residual + LayerNorm + AdaLN values sit
    within one bf16 step of the reference's golden values (another reduction
    order) and their cast stage is bitwise."""
    g = torch.Generator().manual_seed(5)
    b, t, d = 2, 17, 1536
    x = torch.randn(b * t, d, generator=g).to(torch.bfloat16).cuda()
    scale = (torch.randn(b, d, generator=g) * 0.5).to(torch.bfloat16).cuda()
    shift = (torch.randn(b, d, generator=g) * 0.5).to(torch.bfloat16).cuda()
    values, row_max, _ = ops.norm_quant_rows(x, _lib.OUT_FP8_VALUES, scale=scale, shift=shift, tokens=t)
    want = oq.modulate_values(oracle.bf16_bits_to_f32(bits_of(x)), bits_of(scale), bits_of(shift), t)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(values), oracle.f32_to_bf16_bits(want))
    q, s, rep = ops.fp8_cast(values, row_max)
    assert_fp8_stage(values, row_max, q, s, rep)

    # RMSNorm on the golden input.
    xr = from_bits(GOLDEN["fp8p_rms_x"], (6, 2048))
    gamma = from_bits(GOLDEN["fp8p_rms_gamma"], (2048,))
    values, row_max, _ = ops.norm_quant_rows(xr, _lib.OUT_FP8_VALUES, norm=_lib.NORM_RMS, eps=1e-6, gamma=gamma)
    got = oracle.bf16_bits_to_f32(bits_of(values))
    ref = oracle.bf16_bits_to_f32(GOLDEN["fp8p_rms_values"].reshape(6, 2048))
    assert np.mean(got == ref) > 0.99
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=0)
    q, s, rep = ops.fp8_cast(values, row_max)
    assert_fp8_stage(values, row_max, q, s, rep)

    # Residual + LayerNorm + AdaLN on the golden input; the residual sum is exact.
    xl = from_bits(GOLDEN["fp8p_ln_x"], (b * t, d))
    yl = from_bits(GOLDEN["fp8p_ln_y"], (b * t, d))
    sc = from_bits(GOLDEN["fp8p_ln_scale"], (b, d))
    sh = from_bits(GOLDEN["fp8p_ln_shift"], (b, d))
    values, row_max, summed = ops.norm_quant_rows(
        xl, _lib.OUT_FP8_VALUES, norm=_lib.NORM_LN, eps=1e-6, scale=sc, shift=sh, tokens=t, y=yl
    )
    assert np.array_equal(bits_of(summed), GOLDEN["fp8p_ln_summed"].reshape(b * t, d))
    got = oracle.bf16_bits_to_f32(bits_of(values))
    ref = oracle.bf16_bits_to_f32(GOLDEN["fp8p_ln_values"].reshape(b * t, d))
    assert np.mean(got == ref) > 0.99
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=2 ** -7)
    q, s, rep = ops.fp8_cast(values, row_max)
    assert_fp8_stage(values, row_max, q, s, rep)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("precision", ["fp8", "fp4"])
@torch.inference_mode()
def test_prepare_producers_feed_their_consumer(precision):
    """The floating.py producers (piR2's thor/packing.py API) return a
    FloatingPacked that FloatingLinear consumes: SwiGLU into the down
    projection equals packing the bf16 SwiGLU output through the same
    consumer; GELU likewise; the SmoothQuant producer equals the smoothed
    layer's own pack."""
    from pir2_b200.floating import FloatingLinear, prepare_gelu_packed, prepare_smoothed, prepare_swiglu

    torch.manual_seed(3)
    with torch.device("cuda"):
        down = torch.nn.Linear(1536, 512, bias=True).to(torch.bfloat16)
    layer = FloatingLinear(down, "down", precision)
    gate = torch.randn(2, 17, 1536, device="cuda", dtype=torch.bfloat16)
    up = torch.randn_like(gate)
    silu = prepare_silu(gate.device)
    packed = prepare_swiglu(gate, up, silu, precision)
    h = (silu[gate.view(torch.int16).long() & 0xFFFF].float() * up.float()).to(torch.bfloat16)
    if precision == "fp8":
        # The producer packs with prepare_fp8's arithmetic.
        q, s = ops.quant_fp8(h.reshape(-1, 1536), fast=True)[:2]
        assert torch.equal(packed.data, q) and torch.equal(packed.scale.reshape(1), s)
    else:
        pe, se = ops.pack_nvfp4(h.reshape(-1, 1536))
        assert torch.equal(packed.data, pe)
        assert_factors_equal(packed.scale.cpu().numpy(), se.cpu().numpy(), 34, 1536)
    y = layer(packed)
    assert y.shape == (2, 17, 512)
    assert torch.equal(y, layer.forward_packed(*layer.pack_input(packed), (2, 17)))
    gelu = prepare_gelu(gate.device, torch.bfloat16, "tanh")
    gp = prepare_gelu_packed(gate, gelu, precision)
    hg = gelu[gate.view(torch.int16).long() & 0xFFFF]
    if precision == "fp8":
        assert torch.equal(gp.data, ops.quant_fp8(hg.reshape(-1, 1536), fast=True)[0])
    else:
        assert torch.equal(gp.data, ops.pack_nvfp4(hg.reshape(-1, 1536))[0])
    s = (torch.rand(1536, device="cuda") * 3 + 0.25).float()
    smoothed = FloatingLinear(down, "down", precision, smoothing_scale=s)
    sp = prepare_smoothed(gate.reshape(-1, 1536), precision, s)
    assert torch.equal(smoothed(gate).reshape(-1, 512), smoothed(sp))
    assert _lib.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(17, 1536, 6144), (1, 256, 640), (32, 2048, 1024)])
def test_fp8_gemm_table_and_finite_maxima_feed_the_cast(m, k, n):
    """The E4M3 GEMM with an activation table and per-16-column maxima: the
    maxima count finite values only (a table that sends negative results to
    +inf), and casting the output with them gives the oracle producer's
    codes and scale."""
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    qa, _, sa = ops.quant_fp8(x)
    qw, _, sw = ops.quant_fp8(w, replicate=n, weights=True)
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    table = torch.where(bits < 0, torch.tensor(0x7F80, dtype=torch.int16), bits).view(torch.bfloat16).cuda()
    plain = ops.gemm_fp8(qa, sa, qw, sw, bias, n=n)
    maxima = torch.full((m, n // 16), -1.0, device="cuda")
    y = ops.gemm_fp8(qa, sa, qw, sw, bias, n=n, out_lut=table, max_out=maxima)
    torch.cuda.synchronize()
    want_y = table[plain.view(torch.int16).long() & 0xFFFF]
    assert torch.equal(y.view(torch.int16), want_y.view(torch.int16))
    finite = torch.where(torch.isinf(y.float()), 0.0, y.float().abs())
    assert torch.equal(maxima, finite.reshape(m, n // 16, 16).amax(dim=2))
    q, s, rep = ops.fp8_cast(y, maxima)
    want_q, want_s = oracle.fp8_producer(oracle.bf16_bits_to_f32(bits_of(y)))
    assert np.float32(s.item()) == want_s and np.array_equal(q.cpu().numpy(), want_q)
    assert _lib.device_status() == 0


@torch.inference_mode()
def test_fp8_gelu_from_the_gemm_epilogue_equals_the_producer():
    """The DiT GELU module on the FP8 path: the up projection's epilogue
    applies the GELU table and writes the partial maxima, and the cast packs
    it; the same codes, scale and row scales as the GEMM followed by the
    GELU producer."""
    from pir2_b200.floating import FloatingLinear, _fp8_gelu_from_gemm, prepare_gelu_packed
    from pir2_b200.harness import GELU

    torch.manual_seed(9)
    with torch.device("cuda"):
        module = GELU(1536, 6144, "tanh").to(torch.bfloat16)
    lin = FloatingLinear(module.proj, "proj", "fp8")
    lut = prepare_gelu(torch.device("cuda"), torch.bfloat16, "tanh")
    # Token rows of one robot's DiT (17) and the 32-row limit of the path.
    for rows in (17, 32, 17):
        x = torch.randn(1, rows, 1536, device="cuda", dtype=torch.bfloat16)
        fused = _fp8_gelu_from_gemm(module, lin, lut, x)
        ref = prepare_gelu_packed(lin(x).contiguous(), lut, "fp8")
        assert fused.shape == ref.shape == (1, rows, 6144)
        assert torch.equal(fused.data, ref.data)
        assert torch.equal(fused.scale, ref.scale) and torch.equal(fused.row_scales, ref.row_scales)
    assert _lib.device_status() == 0
