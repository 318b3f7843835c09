"""Bounded device waits end with a status the host reads, and the CUDA
context stays usable afterwards (failure detection without a GPU fault:
the wait runs out on an mbarrier that nothing arrives at)."""

import time

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_expired_wait_sets_the_status_word_and_the_context_survives():
    assert _lib.device_status() == 0
    result = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _lib.wait_probe(result)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert result.item() == 0            # the wait gave up
    assert 0.2 < elapsed < 30.0          # after its clock budget (~1 s)
    assert _lib.device_status() == _lib.STATUS_TIMEOUT_PROBE
    assert _lib.device_status() == 0     # read-and-clear

    # The context is still usable: a quantized Linear, bitwise vs the oracle.
    torch.manual_seed(0)
    x = torch.randn(17, 256, dtype=torch.bfloat16)
    w = (torch.randn(128, 256) * 0.02).to(torch.bfloat16)

    def bits(t):
        return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)

    qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits(w)), 8)
    qa, sa = ops.quant_rows(x.cuda(), 8)
    out = ops.gemm(qa, sa, torch.from_numpy(qw).cuda(), torch.from_numpy(sw).cuda(), None, 8, n_store=128)
    ref = oracle.linear_w8a8(bits(x), oracle.bf16_bits_to_f32(bits(w)), None, 8)
    assert np.array_equal(bits(out), ref)
    assert _lib.device_status() == 0
