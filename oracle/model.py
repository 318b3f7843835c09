"""Oracle-quantized GR00T-shaped policy (test infrastructure only).

Every bf16 nn.Linear of a policy gets the oracle's quantized Linear as its
forward: for W8A8 / W4A4 the symmetric-row-v1 activation pack (quant.py
`quant_rows`, following coexecution/kernels/ampere_ada/integer.py:27-94),
the per-channel weight quantization (`quantize_weight`, integer.py:211-256),
the exact int32 product and the epilogue of integer_gemm.cu:37-59; for fp4
the NVFP4 pack of both operands (thor/packing.py:24-54) and the fp64
dequantized product; for fp8 the per-tensor E4M3 quantization of both
operands (fp8_cutlass_linear.cu:61-120, `quant_fp8`) and the fp64 product
times scale_a * scale_b plus bias.  Everything between the Linears (norms, attention,
activations) stays plain torch on whatever device the policy lives on; the
Linears compute on the host and return to that device.  Linears the fp4 path cannot
take (K % 256 or N % 32) stay bf16, as on the GPU; for fp8 that is K % 128 or N % 16.
"""

import numpy as np
import torch

from . import quant as oq


def _bits_of(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _from_bits(y, lead, n, device):
    t = torch.from_numpy(np.ascontiguousarray(y).view(np.int16)).view(torch.bfloat16).reshape(*lead, n)
    return t.to(device)


def _integer_forward(module, bits):
    w = module.weight.detach().float().cpu().numpy()
    qw, sw = oq.quantize_weight(w, bits)
    uw = oq.unpack_int4(qw) if bits == 4 else qw
    n = w.shape[0]
    bias = None
    if module.bias is not None:
        bias = np.zeros(uw.shape[0], dtype=np.uint16)
        bias[:n] = _bits_of(module.bias)

    def forward(x):
        lead = x.shape[:-1]
        rows = _bits_of(x.reshape(-1, x.shape[-1]))
        qa, sa = oq.quant_rows(rows, bits)
        ua = oq.unpack_int4(qa) if bits == 4 else qa
        acc = oq.int_matmul(ua, uw)
        y = oq.gemm_epilogue(acc, sa, sw, bias, 2 if bias is not None else 1)[:, :n]
        return _from_bits(y, lead, n, x.device)

    return forward


def _nvfp4_forward(module):
    pw, sw = oq.pack_nvfp4(module.weight.detach().float().cpu().numpy())
    bias = None if module.bias is None else _bits_of(module.bias)
    n, k = module.out_features, module.in_features

    def forward(x):
        lead = x.shape[:-1]
        rows = x.reshape(-1, k).float().cpu().numpy()
        pa, sa = oq.pack_nvfp4(rows)
        y = oq.nvfp4_gemm(pa, sa, pw, sw, rows.shape[0], n, k, bias)
        return _from_bits(y, lead, n, x.device)

    return forward


def _fp8_forward(module, fast=False):
    qw, sw = oq.quant_fp8(_bits_of(module.weight))
    bias = None if module.bias is None else _bits_of(module.bias)
    n, k = module.out_features, module.in_features

    def forward(x):
        lead = x.shape[:-1]
        qa, sa = oq.quant_fp8(_bits_of(x.reshape(-1, k)), fast=fast)
        y = oq.fp8_gemm(qa, sa, qw, sw, bias)
        return _from_bits(oq.f32_to_bf16_bits(y.astype(np.float32)), lead, n, x.device)

    return forward


def install_oracle_linears(policy, precision):
    """Replace every bf16 Linear's forward (instance attribute) in place."""
    for module in policy.modules():
        if not isinstance(module, torch.nn.Linear):
            continue
        if precision == "fp4":
            if module.in_features % 256 or module.out_features % 32:
                continue
            module.forward = _nvfp4_forward(module)
        elif precision == "fp8":
            if module.in_features % 128 or module.out_features % 16:
                continue
            module.forward = _fp8_forward(module)
        else:
            module.forward = _integer_forward(module, {"w8a8": 8, "w4a4": 4}[precision])
    return policy
