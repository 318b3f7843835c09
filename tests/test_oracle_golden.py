"""Pins the CPU oracle against vectors produced by the piR2 reference itself
(tests/golden/make_golden.py runs the reference's own Triton kernels under
the CPU interpreter, integer, NVFP4 and FP8 producers alike, its
channel_scales and its bitwise-test torch formula).
"""

import os

import numpy as np
import pytest

import oracle

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))

PLAIN = ["k130", "k258", "k1", "k127", "outlier2048", "zeros", "mixed384"]


@pytest.mark.parametrize("name", PLAIN)
@pytest.mark.parametrize("bits", [8, 4])
def test_plain_quant_matches_reference(name, bits):
    q, s = oracle.quant_rows(GOLDEN[f"x_{name}"], bits)
    assert np.array_equal(s.view(np.uint32), GOLDEN[f"s_plain_{name}_b{bits}"].view(np.uint32))
    assert np.array_equal(q.view(np.uint8), GOLDEN[f"q_plain_{name}_b{bits}"].view(np.uint8))
    if bits == 4:
        # Both int4 branches of the reference (pack_reuse True/False) agree.
        assert np.array_equal(q.view(np.uint8), GOLDEN[f"q_plain_{name}_b4_noreuse"].view(np.uint8))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("kind", ["gelu", "gelu_up", "silu_up"])
def test_lut_modes_match_reference(bits, kind):
    lut = GOLDEN["lut_silu" if kind.startswith("silu") else "lut_gelu_tanh"]
    up = GOLDEN["up_k258"] if kind.endswith("_up") else None
    q, s = oracle.quant_rows(GOLDEN["x_k258"], bits, lut_bits=lut, up_bits=up)
    assert np.array_equal(s.view(np.uint32), GOLDEN[f"s_{kind}_k258_b{bits}"].view(np.uint32))
    assert np.array_equal(q.view(np.uint8), GOLDEN[f"q_{kind}_k258_b{bits}"].view(np.uint8))


@pytest.mark.parametrize("bits", [8, 4])
def test_modulation_pack_matches_reference(bits):
    x = GOLDEN["mod_x"].reshape(6, 64)
    q, s = oracle.modulation_pack(x, GOLDEN["mod_scale"].reshape(2, 64), GOLDEN["mod_shift"].reshape(2, 64), 3, bits)
    assert np.array_equal(s.view(np.uint32), GOLDEN[f"mod_s_b{bits}"].view(np.uint32))
    assert np.array_equal(q.view(np.uint8), GOLDEN[f"mod_q_b{bits}"].view(np.uint8))


def _codes(q, bits):
    return oracle.unpack_int4(q).astype(np.int32) if bits == 4 else q.astype(np.int32)


@pytest.mark.parametrize("bits", [8, 4])
def test_norm_modulation_pack_within_one_step(bits):
    # Reduction order is unspecified in the reference (tolerance contract).
    x = GOLDEN["mod_x"].reshape(6, 64)
    q, s = oracle.modulation_pack(
        x, GOLDEN["mod_scale"].reshape(2, 64), GOLDEN["mod_shift"].reshape(2, 64), 3, bits, eps=1e-6
    )
    ref_q = GOLDEN[f"norm_q_b{bits}"]
    assert np.allclose(s, GOLDEN[f"norm_s_b{bits}"], rtol=2 ** -7, atol=0)
    assert np.abs(_codes(q, bits) - _codes(ref_q, bits)).max() <= 1


@pytest.mark.parametrize("bits", [8, 4])
def test_residual_norm_modulation_matches_reference(bits):
    x = GOLDEN["mod_x"].reshape(6, 64)
    q, s, r = oracle.residual_norm_modulation_pack(
        x, GOLDEN["mod_y"].reshape(6, 64), GOLDEN["mod_gate"].reshape(2, 64),
        GOLDEN["mod_scale"].reshape(2, 64), GOLDEN["mod_shift"].reshape(2, 64), 3, bits, 1e-6,
    )
    # The residual is exact BF16 arithmetic: bitwise.
    assert np.array_equal(r, GOLDEN[f"res_r_b{bits}"].reshape(6, 64))
    assert np.allclose(s, GOLDEN[f"res_s_b{bits}"], rtol=2 ** -7, atol=0)
    assert np.abs(_codes(q, bits) - _codes(GOLDEN[f"res_q_b{bits}"], bits)).max() <= 1


@pytest.mark.parametrize("bits", [8, 4])
def test_rms_tail_matches_reference(bits):
    # Given the reference's own variance, the tail is exact.
    x = GOLDEN["rms_x"]
    xf = oracle.bf16_bits_to_f32(x)
    inv = (np.float32(1.0) / np.sqrt((GOLDEN["rms_var"] + np.float32(1e-6)).astype(np.float64))).astype(np.float32)
    n = oracle.bf16_round((xf * inv[:, None]).astype(np.float32))
    v = oracle.bf16_round((n * oracle.bf16_bits_to_f32(GOLDEN["rms_gamma"])[None, :]).astype(np.float32))
    q, s = oracle.quant_rows(oracle.f32_to_bf16_bits(v), bits)
    assert np.array_equal(s.view(np.uint32), GOLDEN[f"rms_s_b{bits}"].view(np.uint32))
    assert np.array_equal(q.view(np.uint8), GOLDEN[f"rms_q_b{bits}"].view(np.uint8))
    # And the oracle's own variance stays within one code.
    q2, _ = oracle.rms_norm_pack(x, GOLDEN["rms_gamma"], 1e-6, bits)
    assert np.abs(_codes(q2, bits) - _codes(q, bits)).max() <= 1


def test_channel_scales_match_reference():
    s = oracle.channel_scales(GOLDEN["sq_amax"], [GOLDEN["sq_w"]], 0.5)
    # pow() of torch (vectorised) and numpy (libm) differ by a few ulp; the
    # scales are an fp32 install-time quantity: relative tolerance 1e-6.
    np.testing.assert_allclose(s, GOLDEN["sq_scales_a05"], rtol=1e-6, atol=0)
    s2 = oracle.channel_scales(GOLDEN["sq_amax"], [GOLDEN["sq_w"], GOLDEN["sq_w2"]], 0.8)
    np.testing.assert_allclose(s2, GOLDEN["sq_scales_group_a08"], rtol=1e-6, atol=0)


@pytest.mark.parametrize("bits", [8, 4])
def test_weight_quant_matches_reference_formula(bits):
    # The golden formula ran on CPU torch, which divides by L.
    w = oracle.bf16_bits_to_f32(GOLDEN["lin_w"])
    q, s = oracle.quantize_weight(w, bits, scale_rule="divide")
    codes = oracle.unpack_int4(q) if bits == 4 else q
    assert np.array_equal(codes[:64, :130], GOLDEN[f"lin_qw_b{bits}"])
    assert np.array_equal(s[:64].view(np.uint32), GOLDEN[f"lin_ws_b{bits}"].view(np.uint32))
    assert np.all(codes[:, 130:] == 0)


@pytest.mark.parametrize("bits", [8, 4])
def test_linear_matches_reference_bitwise_formula(bits):
    """The reference pins its integer Linear bitwise against an explicit torch
    formula (tests/gpu/test_quantization_gpu.py:28-52).  That formula divides
    the activation max by L, where the reference kernels multiply by the fp32
    constant 1/L (integer.py:71, integer_dispatch.cu:237; pinned bitwise by
    the Triton vectors above).  The two scales can differ by one ulp, so the
    formula is compared on the rows where they coincide, which must then be
    bitwise equal; every differing row must be one of the others.  (The
    formula ran on CPU torch, where `tensor / scalar` divides; on CUDA torch
    it multiplies by the reciprocal, which makes the formula and the kernels
    agree on every row there.)"""
    w = oracle.bf16_bits_to_f32(GOLDEN["lin_w"])
    y = oracle.linear_w8a8(GOLDEN["lin_x"], w, GOLDEN["lin_b"], bits, scale_rule="divide")
    ref = GOLDEN[f"lin_y_b{bits}"]
    x = oracle.bf16_bits_to_f32(GOLDEN["lin_x"])
    limit = np.float32(2 ** (bits - 1) - 1)
    m = np.abs(x).max(axis=1).astype(np.float32)
    same = (m / limit).astype(np.float32) == (m * (np.float32(1) / limit)).astype(np.float32)
    assert same.sum() >= 10
    assert np.array_equal(y[same], ref[same])
    assert not np.any((y != ref)[same])


@pytest.mark.parametrize("name", ["r130_k96", "r9_k256"])
def test_nvfp4_pack_matches_reference(name):
    """`_smooth_pack` with FP4 (thor/packing.py:24-54, :314-349): bf16(x / s)
    then E2M1 codes and swizzled UE4M3 block factors, byte for byte (zero
    row, factors that underflow E4M3, a partly used factor group, two
    128-row factor blocks)."""
    x = oracle.bf16_bits_to_f32(GOLDEN[f"fp4_x_{name}"])
    smooth = GOLDEN[f"fp4_smooth_{name}"]
    values = oracle.bf16_round((x / smooth[None, :]).astype(np.float32))
    packed, sf = oracle.pack_nvfp4(values)
    assert np.array_equal(packed, GOLDEN[f"fp4_packed_{name}"])
    assert np.array_equal(sf, GOLDEN[f"fp4_sf_{name}"])


@pytest.mark.parametrize("name", ["r17_k96", "r100_k128", "inf_r33_k130"])
def test_fp8_prepare_matches_reference(name):
    """`prepare_fp8` (thor/packing.py:451-519): per-tensor scale from the
    finite amax and E4M3 codes of the clamped quotients (+-inf left out of
    the amax and clamped to +-448)."""
    q, scale = oracle.quant_fp8(GOLDEN[f"fp8_x_{name}"], fast=True)
    assert np.float32(scale).view(np.uint32) == GOLDEN[f"fp8_s_{name}"].view(np.uint32)
    assert np.array_equal(q, GOLDEN[f"fp8_q_{name}"].reshape(q.shape))


def test_fused_nvfp4_producers_match_reference():
    """`_rmsnorm_pack` and `_norm_modulation_pack` (LayerNorm + residual add
    + per-batch AdaLN) to NVFP4 (thor/packing.py:109-150, :395-415): codes,
    swizzled factors and the bf16 residual sum equal the oracle's
    composition byte for byte on these vectors.  The variance sums differ in
    order (fp32 in the interpreter, fp64 in the oracle), so other inputs may
    land one bf16 step apart, as the reference notes for its own norms."""
    from oracle import quant as oq

    v = oq.rms_norm_values(GOLDEN["fp4rms_x"], GOLDEN["fp4rms_gamma"], 1e-6)
    packed, sf = oq.pack_nvfp4(v)
    assert np.array_equal(packed, GOLDEN["fp4rms_packed"]) and np.array_equal(sf, GOLDEN["fp4rms_sf"])

    tokens, d = 17, 1536
    x = oq.bf16_bits_to_f32(GOLDEN["fp4ln_x"].reshape(-1, d))
    y = oq.bf16_bits_to_f32(GOLDEN["fp4ln_y"].reshape(-1, d))
    r = oq.bf16_round((x + y).astype(np.float32))
    assert np.array_equal(oq.f32_to_bf16_bits(r), GOLDEN["fp4ln_summed"].reshape(-1, d))
    v = oq.modulate_values(oq.layer_norm_values(r, 1e-6), GOLDEN["fp4ln_scale"], GOLDEN["fp4ln_shift"], tokens)
    packed, sf = oq.pack_nvfp4(v)
    assert np.array_equal(packed, GOLDEN["fp4ln_packed"]) and np.array_equal(sf, GOLDEN["fp4ln_sf"])


def _check_fp8_producer(name, values):
    """Values, row maxima, E4M3 codes and scale of one FP8 producer case."""
    assert np.array_equal(oracle.f32_to_bf16_bits(values), GOLDEN[f"fp8p_{name}_values"].reshape(values.shape))
    rowmax = oracle.row_finite_max(values)
    assert np.array_equal(rowmax.view(np.uint32), GOLDEN[f"fp8p_{name}_rowmax"].view(np.uint32))
    q, scale = oracle.fp8_producer(values)
    assert np.float32(scale).view(np.uint32) == GOLDEN[f"fp8p_{name}_s"].view(np.uint32)
    assert np.array_equal(q, GOLDEN[f"fp8p_{name}_q"].reshape(q.shape))


def test_fp8_lut_producers_match_reference():
    """`_swiglu_pack` (one +inf gate: left out of the row maxima, clamped to
    448 in the codes) and `_gelu_pack` with SmoothQuant division, to FP8
    (thor/packing.py:84-107, :352-369, then `_fp8_scale_and_cast` over the
    row maxima, :180-199): the oracle's values, maxima, codes and scale equal
    the reference's bit for bit."""
    v = oracle.floating_values(GOLDEN["fp8p_swiglu_gate"], lut_bits=GOLDEN["lut_silu"],
                               up_bits=GOLDEN["fp8p_swiglu_up"])
    _check_fp8_producer("swiglu", v)
    v = oracle.floating_values(GOLDEN["fp8p_gelu_x"], lut_bits=GOLDEN["lut_gelu_tanh"],
                               smooth=GOLDEN["fp8p_gelu_smooth"])
    _check_fp8_producer("gelu", v)


def test_fp8_norm_producers_match_reference():
    """`_rmsnorm_pack` and `_norm_modulation_pack` (residual add + LayerNorm
    + per-batch AdaLN) to FP8: the oracle's composition equals the
    reference's values, maxima, codes, scale and residual sum on these
    vectors (the variance sums differ in order, fp32 in the interpreter and
    fp64 in the oracle; these inputs round alike)."""
    from oracle import quant as oq

    _check_fp8_producer("rms", oq.rms_norm_values(GOLDEN["fp8p_rms_x"], GOLDEN["fp8p_rms_gamma"], 1e-6))
    tokens, d = 17, 1536
    x = oq.bf16_bits_to_f32(GOLDEN["fp8p_ln_x"].reshape(-1, d))
    y = oq.bf16_bits_to_f32(GOLDEN["fp8p_ln_y"].reshape(-1, d))
    r = oq.bf16_round((x + y).astype(np.float32))
    assert np.array_equal(oq.f32_to_bf16_bits(r), GOLDEN["fp8p_ln_summed"].reshape(-1, d))
    v = oq.modulate_values(oq.layer_norm_values(r, 1e-6), GOLDEN["fp8p_ln_scale"], GOLDEN["fp8p_ln_shift"], tokens)
    _check_fp8_producer("ln", v)
