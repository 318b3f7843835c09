"""Activation lookup tables built by torch on the device.

`prepare_gelu` mirrors coexecution/kernels/common/fused.py:74-83 and the SiLU
table mirrors coexecution/optimization/groot/integer.py:47-53: the table maps
every bf16 bit pattern to torch's own bf16 activation of it, computed on the
GPU, so the packed values match the unfused torch activation exactly.
"""

import torch

_LUTS = {}


def _all_bf16(device, dtype):
    return torch.arange(65536, device=device, dtype=torch.int32).to(torch.int16).view(dtype)


def prepare_gelu(device, dtype, approximate="tanh"):
    key = (torch.device(device), dtype, "gelu", approximate)
    if key not in _LUTS:
        _LUTS[key] = torch.nn.functional.gelu(_all_bf16(device, dtype), approximate=approximate)
    return _LUTS[key]


def prepare_silu(device, dtype=torch.bfloat16):
    key = (torch.device(device), dtype, "silu", None)
    if key not in _LUTS:
        _LUTS[key] = torch.nn.functional.silu(_all_bf16(device, dtype))
    return _LUTS[key]
