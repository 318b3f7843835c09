"""pir2b_dit_ffn_static: the one-launch DiT FFN with its scratch in a static
device array (no allocation).  Collected last on purpose: it must give the
same results as the workspace entry point whether it runs alone or after
every other test has used the library."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops


def _call_static(qa, sa, up, down, lut, residual, out):
    m, d = qa.shape
    f = up.out_features
    status = _lib.lib().pir2b_dit_ffn_static(
        qa.data_ptr(), sa.data_ptr(), up.packed_weight.data_ptr(), up.weight_scale.data_ptr(),
        up.bias.data_ptr(), _lib.BIAS_ADD, lut.data_ptr(), down.packed_weight.data_ptr(),
        down.weight_scale.data_ptr(), down.bias.data_ptr(), _lib.BIAS_ADD, residual.data_ptr(),
        residual.stride(0), m, d, f, out.data_ptr(), out.stride(0),
        torch.cuda.current_stream().cuda_stream,
    )
    _lib.check(status, "pir2b_dit_ffn_static")
    return out


def test_static_entry_rejects_sizes_beyond_its_array():
    lib = _lib.lib()
    # m = 65 and f = 16384 exceed the static scratch; checked before any device call.
    for m, f in ((65, 6144), (17, 16384)):
        status = lib.pir2b_dit_ffn_static(
            None, None, None, None, None, 0, None, None, None, None, 0, None, 1536, m, 1536, f,
            None, 1536, None,
        )
        assert status == _lib.EINVAL
        assert b"static" in lib.pir2b_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("m,d,f", [(17, 1536, 6144), (3, 256, 2048)])
def test_static_entry_equals_workspace_entry_on_two_calls(m, d, f):
    g = torch.Generator().manual_seed(7 * m + d)
    x = (torch.randn(m, d, generator=g)).to(torch.bfloat16)
    qa, sa = oracle.quant_rows(x.view(torch.int16).numpy().view(np.uint16), 8)

    def linear(n, k):
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        q, s = oracle.quantize_weight(w.float().numpy(), 8)
        return SimpleNamespace(
            packed_weight=torch.from_numpy(q).cuda(), weight_scale=torch.from_numpy(s).cuda(),
            bias=(torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda(),
            out_features=n, in_features=k, _bias_mode=lambda: _lib.BIAS_ADD,
        )

    up, down = linear(f, d), linear(d, f)
    values = torch.arange(65536, device="cuda", dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    lut = torch.nn.functional.gelu(values, approximate="tanh")
    residual = torch.randn(m, d, generator=g).to(torch.bfloat16).cuda()
    qa_d, sa_d = torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda()
    expected = ops.dit_ffn(qa_d, sa_d, up, down, lut, residual)
    first = _call_static(qa_d, sa_d, up, down, lut, residual, torch.empty_like(expected))
    second = _call_static(qa_d, sa_d, up, down, lut, residual, torch.empty_like(expected))
    torch.cuda.synchronize()
    assert torch.equal(first, expected)
    assert torch.equal(second, expected)
    assert _lib.device_status() == 0
