"""Exact output epilogues of the packed integer GEMM.

Mirrors coexecution/kernels/ampere_ada/epilogue.py: `residual_gemm`
(:360-398) returns the bf16 GEMM result plus a bf16 residual, added in fp32
and rounded to bf16 again, in one tcgen05 kernel (the reference restricts
its native path to M <= 64 and falls back to GEMM + add otherwise; here
every shape is native).  `group_gemm` writes grouped q|k|v outputs as
contiguous segments.
"""

import torch

from . import ops
from .integer import FORMAT_VERSION


def _validate_pack(packed, q):
    if packed.logical_k != q.in_features or packed.bits != q.bits or packed.format_version != FORMAT_VERSION:
        raise ValueError("Incompatible activation pack")


def residual_gemm(packed, q, residual):
    """Padded, contiguous bf16 [M, Npad] after exact residual addition."""
    _validate_pack(packed, q)
    rows = packed.data.shape[0]
    npad = q.packed_weight.shape[0]
    if rows == 0:
        return torch.empty((0, npad), device=packed.data.device, dtype=torch.bfloat16)
    if residual.ndim == 2 and tuple(residual.shape) == (rows, npad):
        matrix = residual
    else:
        matrix = torch.nn.functional.pad(residual.reshape(rows, q.out_features), (0, npad - q.out_features))
    return ops.gemm(
        packed.data, packed.scales, q.packed_weight, q.weight_scale, q.bias, q.bits,
        bias_mode=q._bias_mode(), residual=matrix, n_store=npad, tactic=q.tactic,
    )


def group_gemm(packed, group):
    """One GEMM for a projection group, each member written as its own
    contiguous [M, size] segment (integer_epilogue.cu `group_gemm`)."""
    q = group.linear
    _validate_pack(packed, q)
    out = ops.gemm(
        packed.data, packed.scales, q.packed_weight, q.weight_scale, q.bias, q.bits,
        bias_mode=q._bias_mode(), n_store=q.out_features, tactic=q.tactic,
    )
    return [out.narrow(1, o, s).contiguous() for o, s in zip(group.offsets, group.sizes)]
