"""BASELINE configurations 2 and 3 as bitwise parity cases: the fused
RMSNorm (eps 1e-6, gamma ~N(1, 0.1)) + per-token pack, then the W8A8 / W4A4
GEMM, over the full cross product M in {1, 16, 64, 256, 1024} x the decoder
projections K -> N in {2048 -> 4096 (q|k|v), 2048 -> 2048 (o), 2048 -> 12288
(gate|up, int8 through the SwiGLU epilogue), 6144 -> 2048 (down)}; inputs
bf16 ~N(0, 1) with 1 % of the channels x20, weights ~N(0, 0.02).

Every integer stage is compared bit for bit: the RMSNorm pack against the
oracle's tail on the device's own variance (torch's row mean, the
reference's B200 statistics) and rsqrt, the weight codes against the
oracle's quantization, and the GEMM output against the oracle's exact int32
product and dequant epilogue (producers.py:19-53, integer.py:211-256,
integer_gemm.cu:37-59)."""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops
from pir2_b200.fused import prepare_silu

pytestmark = pytest.mark.gpu

SHAPES = [(2048, 4096, False), (2048, 2048, False), (2048, 12288, True), (6144, 2048, False)]


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def outlier_rows(g, m, k):
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20.0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("k,n,swiglu", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 64, 256, 1024])
def test_rmsnorm_pack_and_gemm_bitwise(m, k, n, swiglu, bits):
    g = torch.Generator().manual_seed(m * 31 + k + n + bits)
    x = outlier_rows(g, m, k)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)

    # RMSNorm + pack on the device vs the oracle tail on torch's statistics.
    xd = x.cuda()
    q, s, _ = ops.norm_quant_rows(xd, bits, norm=_lib.NORM_RMS, eps=1e-6, gamma=gamma.cuda())
    var = (xd.float() * xd.float()).mean(-1)
    inv = torch.rsqrt(var + 1e-6)
    rq, rs = oracle.rms_norm_tail_pack(bits_of(x), bits_of(gamma), var.cpu().numpy(), inv.cpu().numpy(), bits)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(q.cpu().numpy(), rq)

    qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), bits)
    ua = oracle.unpack_int4(rq) if bits == 4 else rq
    uw = oracle.unpack_int4(qw) if bits == 4 else qw
    acc = oracle.int_matmul(ua, uw)
    if swiglu and bits == 8:
        half = n // 2
        y = oracle.gemm_epilogue(acc, rs, sw, None, 0)
        lut = prepare_silu(torch.device("cuda"))
        silu = oracle.bf16_bits_to_f32(bits_of(lut.cpu())[y[:, :half]])
        up = oracle.bf16_bits_to_f32(y[:, half:n])
        ref = oracle.f32_to_bf16_bits((silu * up).astype(np.float32))
        cat = lambda t: ops.interleave_gate_up(t, half)   # noqa: E731
        out = ops.gemm_swiglu(q, s, cat(torch.from_numpy(qw).cuda()), cat(torch.from_numpy(sw).cuda()), None,
                              lut, half_n=half)
    else:
        ref = oracle.gemm_epilogue(acc, rs, sw, None, 1)[:, :n]
        out = ops.gemm(q, s, torch.from_numpy(qw).cuda(), torch.from_numpy(sw).cuda(), None, bits, n_store=n)
    got = bits_of(out)
    mismatch = np.argwhere(got != ref)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    assert _lib.device_status() == 0
