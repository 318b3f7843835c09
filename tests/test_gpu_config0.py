"""The reference's CPU-runnable case, a single SmoothQuant W8A8 Linear:
X [256, 2048] ~N(0,1) with 1 % of the channels x20, W [6144, 2048] ~N(0,0.02),
bias ~N(0,0.01), alpha 0.5 from the per-channel |X| maxima, seed 0.  The
smoothing composes the reference's pieces (channel_scales,
coexecution/optimization/backends/thor/smoothquant.py:27-45; W*s to bf16,
thor/linear.py:64-78; bf16(x / s) in the activation pack, thor/packing.py:
69-73) with the symmetric-row-v1 quantizer and GEMM.  The activations enter
as bf16, the dtype of the patched model's Linear inputs.  The B200 path
(smoothed pack kernel, install-time weight quantization on the device,
tcgen05 GEMM) must equal the oracle bit for bit."""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops
from pir2_b200.integer import quantize_weight
from pir2_b200.smoothquant import channel_scales

pytestmark = pytest.mark.gpu


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def test_smoothquant_w8a8_linear_of_the_reference_cpu_case():
    g = torch.Generator().manual_seed(0)
    m, k, n = 256, 2048, 6144
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20.0
    x = x.to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)

    # One set of channel scales for both sides (computed on the host).
    s = channel_scales(x.float().abs().amax(0), [w], 0.5)
    w_s = (w.float() * s).to(torch.bfloat16)

    qa, sa = ops.quant_rows(x.cuda(), 8, smooth=s.cuda())
    qw, sw = quantize_weight(w_s.cuda(), 8)
    out = ops.gemm(qa, sa, qw, sw, bias.cuda(), 8, n_store=n)

    ref = oracle.linear_w8a8(bits_of(x), oracle.bf16_bits_to_f32(bits_of(w_s)), bits_of(bias), 8, smooth=s.numpy())
    got = bits_of(out)
    mismatch = np.argwhere(got != ref)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    assert _lib.device_status() == 0
