"""AdaLN modulation producers that emit packed integer activations.

Mirrors coexecution/kernels/ampere_ada/modulation.py:222-338:
`prepare_modulation` (x already normalized), `prepare_norm_modulation`
(non-affine LayerNorm fused), `prepare_residual_norm_modulation` (gated
residual + LayerNorm, returning the exact bf16 residual) and the
`PackedActivations` carrier.  One fused sm_100a kernel per call.
"""

import math
from dataclasses import dataclass, replace

import torch

from . import _lib, ops
from .integer import PackedActivation


def prepare_modulation(x, scale, shift, bits):
    return _prepare(x, scale, shift, bits)


def prepare_norm_modulation(x, scale, shift, bits, *, eps):
    """Fuse non-affine LayerNorm into packing; FP32 reduction order may differ."""
    if eps is None:
        raise ValueError("LayerNorm epsilon must be finite and positive")
    return _prepare(x, scale, shift, bits, eps=eps)


def prepare_residual_norm_modulation(x, y, gate, scale, shift, bits, *, eps):
    """Return the exact BF16 residual and its fused normalized integer pack."""
    if eps is None:
        raise ValueError("LayerNorm epsilon must be finite and positive")
    return _prepare(x, scale, shift, bits, eps=eps, residual=(y, gate))


def _prepare(x, scale, shift, bits, *, eps=None, residual=None):
    if eps is not None:
        if not isinstance(eps, (int, float)) or not math.isfinite(eps) or eps <= 0:
            raise ValueError("LayerNorm epsilon must be finite and positive")
        eps = float(eps)
    if bits not in (4, 8) or x.ndim != 3 or not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("Modulation packing requires contiguous CUDA BF16 B,T,D and bits=4 or 8")
    b, tokens, k = x.shape
    if min(b, tokens, k) < 1 or k > 8192:
        raise ValueError("Unsupported modulation dimensions")
    for value in (scale, shift):
        if value.shape != (b, 1, k) or value.dtype != x.dtype or value.device != x.device:
            raise ValueError("Modulation scale and shift must match B,1,D, dtype and device")
    scale, shift = scale.reshape(b, k).contiguous(), shift.reshape(b, k).contiguous()
    y = gate = None
    if residual is not None:
        y, gate = residual
        if (
            y.shape != x.shape
            or y.dtype != x.dtype
            or y.device != x.device
            or not y.is_contiguous()
            or gate.shape != (b, 1, k)
            or gate.dtype != x.dtype
            or gate.device != x.device
        ):
            raise ValueError("Residual operands must match BF16 input and B,1,D gate")
        gate = gate.reshape(b, k).contiguous()
        y = y.reshape(b * tokens, k)
    data, scales, res = ops.norm_quant_rows(
        x.reshape(b * tokens, k),
        bits,
        norm=_lib.NORM_NONE if eps is None else _lib.NORM_LN,
        eps=eps or 0.0,
        scale=scale,
        shift=shift,
        tokens=tokens,
        y=y,
        gate=gate,
    )
    packed = PackedActivation(data, scales, (b, tokens), k, bits)
    return packed if residual is None else (res.reshape(b, tokens, k), packed)


@dataclass
class PackedActivations:
    """Internal model boundary carrying only the requested integer formats."""

    packs: dict
    _robotics_packed_input = True

    def for_bits(self, bits):
        if bits not in self.packs:
            raise ValueError("A consumer requested an unprepared integer format")
        return self.packs[bits]

    def with_leading_shape(self, shape):
        shape = tuple(shape)
        if not shape or min(shape) < 1 or any(math.prod(shape) != p.data.shape[0] for p in self.packs.values()):
            raise ValueError("Packed leading shape must preserve the row count")
        return PackedActivations({bits: replace(p, shape=shape) for bits, p in self.packs.items()})
