"""RMSNorm and final-modulation producers that emit packed activations.

Mirrors coexecution/kernels/ampere_ada/producers.py:19-115.  The reference
computes the RMS variance with torch's reduction and packs in a second
kernel; here one fused sm_100a kernel computes the variance (fp32, its own
reduction order: the tolerance contract of the reference, whose fused norm
packs are likewise not bitwise equal to torch), normalizes with the bf16
boundaries bf16(bf16(x * rsqrt(var + eps)) * gamma) and packs.
"""

import math

import torch

from . import _lib, ops
from .integer import PackedActivation
from .modulation import PackedActivations, prepare_modulation


def prepare_rmsnorm(x, weight, eps, bits, *, residual=None):
    """RMSNorm + pack; with `residual`, normalizes bf16(x + residual) and
    also returns that sum (the decoder's residual stream)."""
    if not (
        type(bits) is int
        and bits in (4, 8)
        and x.is_cuda
        and x.device == weight.device
        and x.dtype == weight.dtype == torch.bfloat16
        and x.ndim >= 2
        and x.is_contiguous()
        and weight.is_contiguous()
        and not x.requires_grad
        and not weight.requires_grad
        and 0 < x.shape[-1] <= 8192
        and weight.numel() == x.shape[-1]
        and math.isfinite(eps)
        and eps > 0
    ):
        raise ValueError("RMS producer requires contiguous CUDA BF16 rows and weights")
    k = x.shape[-1]
    rows = x.numel() // k
    y = None if residual is None else residual.reshape(rows, k)
    data, scales, summed = ops.norm_quant_rows(
        x.reshape(rows, k), bits, norm=_lib.NORM_RMS, eps=eps, gamma=weight, y=y
    )
    packed = PackedActivation(data, scales, tuple(x.shape[:-1]), k, bits)
    if residual is None:
        return packed
    return summed.reshape(x.shape), packed


def prepare_final_modulation(x, scale, shift, bits):
    """Input is already normalized; the final DiT's shift/scale order stays."""
    if x.ndim != 3 or scale.shape != shift.shape:
        raise ValueError("Final modulation requires B,T,D and matched scale/shift")
    if scale.ndim == 2:
        if scale.shape != (x.shape[0], x.shape[-1]):
            raise ValueError("Shared condition shape does not match final modulation")
        packed = prepare_modulation(x, scale[:, None], shift[:, None], bits)
    elif scale.ndim == 3 and scale.shape == (x.shape[0], 1, x.shape[-1]):
        packed = prepare_modulation(x, scale, shift, bits)
    elif scale.ndim == 3 and scale.shape == x.shape:
        width = x.shape[-1]
        packed = prepare_modulation(
            x.reshape(-1, 1, width), scale.reshape(-1, 1, width), shift.reshape(-1, 1, width), bits
        )
    else:
        raise ValueError("Unsupported final conditioning shape")
    result = PackedActivations({bits: packed}).with_leading_shape(x.shape[:-1])
    result.shape = x.shape
    return result


class QuantizationProducers:
    """Reversible RMSNorm producers for complete integer consumer groups.

    Mirrors coexecution/optimization/groot/producers.py:13-76: a decoder
    layer's input_layernorm (before q|k|v) and post_attention_layernorm
    (before gate|up) return packed activations when every consumer of that
    norm is quantized.
    """

    def __init__(self, policy, controller):
        quantized = {id(site[0]) for site in controller.sites.values()}
        self.norms = []
        for name, layer in policy.named_modules():
            if type(layer).__name__ != "Qwen3VLTextDecoderLayer":
                continue
            if all(id(getattr(layer.self_attn, a)) in quantized for a in ("q_proj", "k_proj", "v_proj")):
                self.norms.append((name + ".input_layernorm", layer.input_layernorm))
            if all(id(getattr(layer.mlp, a)) in quantized for a in ("gate_proj", "up_proj")):
                self.norms.append((name + ".post_attention_layernorm", layer.post_attention_layernorm))
        self.saved = []
        self.installed_norms = []
        self.bits = None

    def set(self, bits=None):
        self.close()
        if bits is None:
            return
        if bits not in (4, 8):
            raise ValueError("Producer precision must be 4 or 8")
        if not self.norms:
            raise ValueError("Producer fusion selected no complete integer consumers")
        self.saved = [(m, m.forward, "forward" in m.__dict__) for _, m in self.norms]
        try:
            for _, norm in self.norms:

                def forward(x, module=norm, bits=bits):
                    packed = prepare_rmsnorm(x, module.weight, module.variance_epsilon, bits)
                    result = PackedActivations({bits: packed})
                    result.shape = x.shape
                    return result

                norm.forward = forward
            self.installed_norms = list(self.norms)
            self.bits = bits
        except BaseException:
            self.close()
            raise

    def evidence(self):
        return {"rmsnorm": [name for name, _ in self.installed_norms], "bits": self.bits}

    def close(self):
        for module, forward, had in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []
        self.installed_norms = []
        self.bits = None
