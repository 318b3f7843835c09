"""The native op schemas registered by pir2_b200.torch_ops, called through
torch.ops exactly as piR2's Python code calls its own extensions, checked
against the oracle:

* pir2_integer::gemm / gemm_biasless (integer_gemm.cu:185-195), including
  the +0 versus -0 split for a null bias;
* pir2_integer_dispatch::linear / prepare (integer_dispatch.cu:127-136);
* pir2_integer_epilogue::gemm (residual) and group_gemm (segments)
  (integer_epilogue.cu:189-341);
* pir2_cutlass_fp4 pack / forward / tactic / swap-AB / policy ops
  (fp4_cutlass_linear.cu:2968-3065, fp4_linear.py:8-15);
and the reference's error behaviour (RuntimeError with its messages).
"""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import torch_ops  # noqa: F401  (registers the schemas)

pytestmark = pytest.mark.gpu


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def randn_bf16(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def problem(g, m, k, n, bits):
    x = randn_bf16(g, m, k)
    w = randn_bf16(g, n, k, scale=0.02)
    b = randn_bf16(g, n, scale=0.01)
    qa, sa = oracle.quant_rows(bits_of(x), bits)
    qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), bits)
    return x, w, b, qa, sa, qw, sw


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def unpacked(q, bits):
    return oracle.unpack_int4(q) if bits == 4 else q


@pytest.mark.parametrize("bits", [8, 4])
def test_integer_gemm_and_biasless_signed_zero(bits):
    """A null bias: `gemm` adds +0 (so -0 becomes +0), `gemm_biasless` keeps
    the sign of an underflowed product."""
    g = torch.Generator().manual_seed(3 + bits)
    m, k, n = 17, 256, 64
    _, _, _, qa, sa, qw, sw = problem(g, m, k, n, bits)
    # Tiny scales make negative products underflow to -0.
    sa_t = np.full_like(sa, 1e-30)
    sw_t = np.full_like(sw, 1e-30)
    acc = oracle.int_matmul(unpacked(qa, bits), unpacked(qw, bits))
    assert (acc < 0).any()
    for op, mode in ((torch.ops.pir2_integer.gemm, 1), (torch.ops.pir2_integer.gemm_biasless, 0)):
        out = op(dev(qa), dev(sa_t), dev(qw), dev(sw_t), None, bits, 3)
        ref = oracle.gemm_epilogue(acc, sa_t, sw_t, None, mode)
        assert out.shape == (m, qw.shape[0])
        assert np.array_equal(bits_of(out), ref)
    plus = bits_of(torch.ops.pir2_integer.gemm(dev(qa), dev(sa_t), dev(qw), dev(sw_t), None, bits, 0))
    minus = bits_of(torch.ops.pir2_integer.gemm_biasless(dev(qa), dev(sa_t), dev(qw), dev(sw_t), None, bits, 0))
    assert (plus == 0x0000).any() and (minus == 0x8000).any() and not np.array_equal(plus, minus)


@pytest.mark.parametrize("bits", [8, 4])
def test_integer_gemm_with_bias_every_tactic(bits):
    g = torch.Generator().manual_seed(11 + bits)
    _, _, b, qa, sa, qw, sw = problem(g, 40, 512, 200, bits)
    ref = oracle.gemm_epilogue(oracle.int_matmul(unpacked(qa, bits), unpacked(qw, bits)), sa, sw, bits_of(b), 2)
    for tactic in range(8):
        out = torch.ops.pir2_integer.gemm(dev(qa), dev(sa), dev(qw), dev(sw), b.cuda(), bits, tactic)
        assert np.array_equal(bits_of(out), ref)


def test_integer_gemm_errors():
    q = torch.zeros(4, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(4, device="cuda")
    w = torch.zeros(8, 128, dtype=torch.int8, device="cuda")
    sw = torch.ones(8, device="cuda")
    with pytest.raises(RuntimeError, match="Unknown integer GEMM tactic"):
        torch.ops.pir2_integer.gemm(q, s, w, sw, None, 8, 8)
    with pytest.raises(RuntimeError, match="bits must be 4 or 8"):
        torch.ops.pir2_integer.gemm(q, s, w, sw, None, 6, 0)
    with pytest.raises(RuntimeError, match="K%128=0, N%8=0"):
        torch.ops.pir2_integer.gemm(q, s, w[:6], sw[:6], None, 8, 0)
    with pytest.raises(RuntimeError, match="Invalid integer storage dtype"):
        torch.ops.pir2_integer.gemm(q.view(torch.uint8), s, w, sw, None, 8, 0)


@pytest.mark.parametrize("bits", [8, 4])
def test_dispatch_prepare_and_linear(bits):
    g = torch.Generator().manual_seed(21 + bits)
    x, w, b, _, _, qw, sw = problem(g, 33, 1000, 96, bits)
    q, s = torch.ops.pir2_integer_dispatch.prepare(x.cuda(), None, None, bits)
    rq, rs = oracle.quant_rows(bits_of(x), bits)
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    # linear = prepare + gemm_biasless (integer_dispatch.cu:110-125).
    y = torch.ops.pir2_integer_dispatch.linear(x.cuda(), dev(qw), dev(sw), b.cuda(), None, None, bits, 0)
    ref = oracle.gemm_epilogue(oracle.int_matmul(unpacked(rq, bits), unpacked(qw, bits)), rs, sw, bits_of(b), 2)
    assert np.array_equal(bits_of(y), ref)
    y0 = torch.ops.pir2_integer_dispatch.linear(x.cuda(), dev(qw), dev(sw), None, None, None, bits, 0)
    ref0 = oracle.gemm_epilogue(oracle.int_matmul(unpacked(rq, bits), unpacked(qw, bits)), rs, sw, None, 0)
    assert np.array_equal(bits_of(y0), ref0)


def test_dispatch_prepare_gated_and_lut_modes():
    g = torch.Generator().manual_seed(8)
    x, up = randn_bf16(g, 9, 384), randn_bf16(g, 9, 384)
    values = torch.arange(65536, device="cuda", dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    lut = torch.nn.functional.silu(values)
    q, s = torch.ops.pir2_integer_dispatch.prepare(x.cuda(), lut, up.cuda(), 8)
    rq, rs = oracle.quant_rows(bits_of(x), 8, lut_bits=bits_of(lut), up_bits=bits_of(up))
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    q, s = torch.ops.pir2_integer_dispatch.prepare(x.cuda(), lut, None, 4)
    rq, rs = oracle.quant_rows(bits_of(x), 4, lut_bits=bits_of(lut))
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    with pytest.raises(RuntimeError, match="multiplier needs a lookup table"):
        torch.ops.pir2_integer_dispatch.prepare(x.cuda(), None, up.cuda(), 8)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("biasless,with_bias", [(False, True), (False, False), (True, False)])
def test_epilogue_residual_gemm(bits, biasless, with_bias):
    g = torch.Generator().manual_seed(31 + bits)
    m, k, n = 17, 1536, 1536
    _, _, b, qa, sa, qw, sw = problem(g, m, k, n, bits)
    residual = randn_bf16(g, m, n)
    bias = b.cuda() if with_bias else None
    out = torch.ops.pir2_integer_epilogue.gemm(
        dev(qa), dev(sa), dev(qw), dev(sw), bias, bits, 7, biasless, residual.cuda()
    )
    mode = 2 if with_bias else (0 if biasless else 1)
    y = oracle.gemm_epilogue(
        oracle.int_matmul(unpacked(qa, bits), unpacked(qw, bits)), sa, sw, bits_of(b) if with_bias else None, mode
    )
    ref = oracle.f32_to_bf16_bits(
        (oracle.bf16_bits_to_f32(y) + oracle.bf16_bits_to_f32(bits_of(residual))).astype(np.float32)
    )
    assert np.array_equal(bits_of(out), ref)


def test_epilogue_residual_gemm_errors():
    q = torch.zeros(65, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(65, device="cuda")
    w = torch.zeros(8, 128, dtype=torch.int8, device="cuda")
    sw = torch.ones(8, device="cuda")
    r = torch.zeros(65, 8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="Residual epilogue requires M<=64"):
        torch.ops.pir2_integer_epilogue.gemm(q, s, w, sw, None, 8, 0, False, r)
    with pytest.raises(RuntimeError, match="tactic must be 0, 2 or 7"):
        torch.ops.pir2_integer_epilogue.gemm(q[:4], s[:4], w, sw, None, 8, 1, False, r[:4])
    with pytest.raises(RuntimeError, match="residual"):
        torch.ops.pir2_integer_epilogue.gemm(q[:4], s[:4], w, sw, None, 8, 0, False, r[:3])


@pytest.mark.parametrize("bits", [8, 4])
def test_epilogue_group_gemm_segments(bits):
    """Segment s of the flat output is the [M, sizes[s]] block of columns
    [offset_s, offset_s + sizes[s]) of the full GEMM."""
    g = torch.Generator().manual_seed(51 + bits)
    m, k = 33, 1536
    sizes = [1536, 512, 512]
    n = sum(sizes)
    _, _, b, qa, sa, qw, sw = problem(g, m, k, n, bits)
    out = torch.ops.pir2_integer_epilogue.group_gemm(dev(qa), dev(sa), dev(qw), dev(sw), b.cuda(), bits, 0, False, sizes)
    full = oracle.gemm_epilogue(oracle.int_matmul(unpacked(qa, bits), unpacked(qw, bits)), sa, sw, bits_of(b), 2)
    got = bits_of(out)
    assert got.shape == (m * n,)
    offset = 0
    for width in sizes:
        seg = got[m * offset : m * (offset + width)].reshape(m, width)
        assert np.array_equal(seg, full[:, offset : offset + width])
        offset += width
    with pytest.raises(RuntimeError, match="widths must cover physical N"):
        torch.ops.pir2_integer_epilogue.group_gemm(dev(qa), dev(sa), dev(qw), dev(sw), None, bits, 0, False, [8, 8])


def _fp4_reference(x, w, b):
    pa, sfa = oracle.pack_nvfp4(x.float().numpy())
    pw, sfw = oracle.pack_nvfp4(w.float().numpy())
    m, k = x.shape
    n = w.shape[0]
    return oracle.nvfp4_gemm(pa, sfa, pw, sfw, m, n, k, None if b is None else bits_of(b))


@pytest.mark.parametrize("m", [1, 17, 130])
def test_fp4_pack_and_forward(m):
    g = torch.Generator().manual_seed(60 + m)
    k, n = 1536, 512
    x, w, b = randn_bf16(g, m, k), randn_bf16(g, n, k, scale=0.02), randn_bf16(g, n, scale=0.01)
    packed_w, scale_w, meta = torch.ops.pir2_cutlass_fp4.pack_linear_weight_gemm_bf16(w.cuda(), "q", "blocks.0")
    assert meta.device.type == "cpu" and meta.tolist() == [n, k]
    pw, sfw = oracle.pack_nvfp4(w.float().numpy())
    assert np.array_equal(packed_w.cpu().numpy(), pw)
    assert np.array_equal(scale_w.cpu().numpy().reshape(-1), sfw.reshape(-1))
    packed_x, scale_x = torch.ops.pir2_cutlass_fp4.pack_activation_gemm_bf16(x.cuda())
    pa, _ = oracle.pack_nvfp4(x.float().numpy())
    assert np.array_equal(packed_x.cpu().numpy(), pa)
    ref = oracle.bf16_bits_to_f32(_fp4_reference(x, w, b))
    outs = [
        torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16(
            packed_x, scale_x, packed_w, scale_w, meta, b.cuda(), "q", "blocks.0")
    ]
    for tactic in range(4):
        outs.append(torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16_tactic(
            packed_x, scale_x, packed_w, scale_w, meta, b.cuda(), "q", "blocks.0", tactic))
    for out in outs:
        assert out.shape == (m, n)
        # NVFP4 GEMM tolerance (the reference pins its FP4 GEMM only to
        # rtol 0.008 / atol 0.001 self-consistency, tests/gpu/test_fp4_swap_ab_gpu.py).
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=2 ** -7, atol=1e-3)
        assert torch.equal(out, outs[0])


def test_fp4_swap_ab_equals_forward_and_policy():
    g = torch.Generator().manual_seed(77)
    m, k, n = 41, 1536, 1536
    x, w, b = randn_bf16(g, m, k), randn_bf16(g, n, k, scale=0.02), randn_bf16(g, n, scale=0.01)
    pw, sw, meta = torch.ops.pir2_cutlass_fp4.pack_linear_weight_gemm_bf16(w.cuda(), "o", "t")
    px, sx = torch.ops.pir2_cutlass_fp4.pack_activation_gemm_bf16(x.cuda())
    y = torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16_swap_ab(px, sx, pw, sw, b.cuda())
    z = torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16(px, sx, pw, sw, meta, b.cuda(), "o", "t")
    assert torch.equal(y, z)
    assert torch.ops.pir2_cutlass_fp4.supports_device(100)
    torch.ops.pir2_cutlass_fp4.set_decode_policy(3)
    assert torch.ops.pir2_cutlass_fp4.get_decode_policy() == 3
    torch.ops.pir2_cutlass_fp4.set_decode_policy(0)
    with pytest.raises(RuntimeError, match="decode policy must be"):
        torch.ops.pir2_cutlass_fp4.set_decode_policy(4)
    with pytest.raises(RuntimeError, match="unknown CUTLASS FP4 GEMM tactic"):
        torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16_tactic(px, sx, pw, sw, meta, None, "o", "t", 5)
    with pytest.raises(RuntimeError, match="Swap-AB supports only"):
        torch.ops.pir2_cutlass_fp4.linear_forward_packed_gemm_bf16_swap_ab(px[:40], sx, pw, sw, b.cuda())
    with pytest.raises(RuntimeError, match="out_features divisible by 32"):
        torch.ops.pir2_cutlass_fp4.pack_linear_weight_gemm_bf16(w[:48].cuda(), "o", "t")
