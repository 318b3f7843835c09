"""NVFP4 and FP8 (E4M3) Linear layers and NVFP4 producers on the B200 kernels.

Mirrors coexecution/optimization/backends/thor/linear.py
(`FloatingLinear`, :30-190) and packing.py (`FloatingPacked`, the fused
norm/smoothing producers, :15-448): weights are packed once as E2M1 with
UE4M3 factors per 16 elements (the CUTLASS 128x4 swizzled factor layout,
`sfa_offset`), activations are packed per call (optionally fused with
LayerNorm / RMSNorm / AdaLN / residual / SmoothQuant division), and the GEMM
runs on tcgen05 kind::mxf4nvf4 with fp32 accumulation and bf16 output.

FP8 layers (precision "fp8") quantize weights and activations per tensor
to E4M3 (`ops.quant_fp8`: the quantize_bf16 arithmetic, or prepare_fp8's
with `fast_fp8`) and run the tcgen05 kind::f8f6f4 GEMM with fp32
accumulation; FP8 in_features must be a multiple of 128 (piR2: 16).  An
NVFP4 K block of the B200 kernel is 256 values, so fp4 in_features must be
a multiple of 256 (piR2 requires 32); out_features must be a multiple of 32
(fp4) or 16 (fp8) as in piR2.  The fused producers are fp4 only.
"""

import math
from dataclasses import dataclass

import torch

from . import _lib, ops


@dataclass
class FloatingPacked:
    data: torch.Tensor
    scale: torch.Tensor
    shape: tuple
    precision: str
    smoothing_scale: torch.Tensor | None = None


def _check_smoothing_metadata(scale, value):
    if scale is not None and (
        scale.shape != (value.shape[-1],)
        or scale.dtype != torch.float32
        or scale.device != value.device
        or not scale.is_contiguous()
        or scale.requires_grad
    ):
        raise ValueError("SmoothQuant requires contiguous immutable FP32 channel scales")


def _require_fp4(precision):
    if precision != "fp4":
        raise ValueError("This B200 build implements the fp4 floating precision only")


def _producer_rows(x):
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.numel() == 0 or x.requires_grad:
        raise ValueError("Floating producer requires nonempty CUDA BF16 inference")
    k = x.shape[-1]
    if k % 32 or k > 8192:
        raise ValueError("Floating producer requires K % 32 == 0 and K <= 8192")
    return x.reshape(-1, k).contiguous(), k


def prepare_smoothed(matrix, precision, smoothing_scale):
    """bf16(x / s) fused into the FP4 pack (packing.py:314-349)."""
    _require_fp4(precision)
    _check_smoothing_metadata(smoothing_scale, matrix)
    if smoothing_scale is None or matrix.ndim != 2 or not matrix.is_contiguous():
        raise ValueError("Smoothed packing needs a contiguous matrix and channel scales")
    rows, _ = _producer_rows(matrix)
    data, scale, _ = ops.norm_quant_rows(rows, _lib.OUT_NVFP4, smooth=smoothing_scale)
    return FloatingPacked(data, scale, tuple(matrix.shape), precision, smoothing_scale)


def prepare_rmsnorm_packed(x, weight, precision, *, eps, smoothing_scale=None):
    """RMSNorm [+ SmoothQuant] to FP4 (packing.py:395-448)."""
    _require_fp4(precision)
    _check_smoothing_metadata(smoothing_scale, x)
    if not x.is_contiguous() or weight.shape != (x.shape[-1],) or not math.isfinite(eps) or eps <= 0:
        raise ValueError("RMSNorm packing requires contiguous BF16 and positive epsilon")
    rows, _ = _producer_rows(x)
    data, scale, _ = ops.norm_quant_rows(
        rows, _lib.OUT_NVFP4, norm=_lib.NORM_RMS, eps=eps, gamma=weight, smooth=smoothing_scale
    )
    return FloatingPacked(data, scale, tuple(x.shape), precision, smoothing_scale)


def prepare_norm(x, precision, *, eps, scale=None, shift=None, residual=None, smoothing_scale=None):
    """LayerNorm [+ AdaLN] [+ residual] [+ SmoothQuant] to FP4
    (packing.py:234-297).  Returns (packed, bf16 residual sum or None)."""
    _require_fp4(precision)
    _check_smoothing_metadata(smoothing_scale, x)
    if x.ndim != 3 or not x.is_contiguous() or not math.isfinite(eps) or eps <= 0:
        raise ValueError("Norm packing requires contiguous B,T,D and positive epsilon")
    if (scale is None) != (shift is None):
        raise ValueError("Modulation requires both scale and shift")
    b, t, k = x.shape
    tokens = 1
    if scale is not None:
        if scale.shape != shift.shape or scale.shape not in (x.shape, (b, k)):
            raise ValueError("Modulation must match BF16 B,D or per-token B,T,D")
        tokens = t if scale.ndim == 2 else 1
        scale, shift = scale.reshape(-1, k).contiguous(), shift.reshape(-1, k).contiguous()
    y = None
    if residual is not None:
        if residual.shape != x.shape or not residual.is_contiguous():
            raise ValueError("Residual must match contiguous BF16 input")
        y = residual.reshape(-1, k)
    rows, _ = _producer_rows(x)
    data, sf, summed = ops.norm_quant_rows(
        rows, _lib.OUT_NVFP4, norm=_lib.NORM_LN, eps=eps, scale=scale, shift=shift, tokens=tokens,
        y=y, smooth=smoothing_scale,
    )
    packed = FloatingPacked(data, sf, tuple(x.shape), precision, smoothing_scale)
    return packed, (None if summed is None else summed.reshape(x.shape))


def aligned_for(precision, in_features, out_features):
    """Whether a Linear meets the B200 kernels' alignment for `precision`."""
    if precision == "fp8":
        return in_features % 128 == 0 and out_features % 16 == 0
    return in_features % 256 == 0 and out_features % 32 == 0


class FloatingLinear(torch.nn.Module):
    """E4M3 or block-scaled E2M1 GEMM with packed weights (thor/linear.py:30-190)."""

    def __init__(self, linear, name, precision="fp4", *, fast_fp8=False, fp4_swap_ab=False, smoothing_scale=None):
        super().__init__()
        if precision not in ("fp8", "fp4"):
            raise ValueError("Floating precision must be fp8 or fp4")
        if fast_fp8 and precision != "fp8":
            raise ValueError("Fast FP8 quantization requires precision=fp8")
        if fp4_swap_ab and precision != "fp4":
            raise ValueError("FP4 Swap-AB requires precision=fp4")
        if (
            not linear.weight.is_cuda
            or linear.weight.dtype != torch.bfloat16
            or not aligned_for(precision, linear.in_features, linear.out_features)
        ):
            raise ValueError(f"{precision} requires aligned CUDA BF16 Linear weights")
        if torch.cuda.get_device_capability(linear.weight.device) != (10, 0):
            raise ValueError("The B200 floating adapter runs on sm_100 devices")
        if precision == "fp8" and smoothing_scale is not None:
            raise ValueError("SmoothQuant with fp8 is not implemented in this build")
        self.fast_fp8 = fast_fp8
        self.name = name
        self.precision = precision
        self.fp4_swap_ab = fp4_swap_ab   # the tcgen05 kernel has no separate swap-AB variant
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        weight_input = linear.weight.detach().contiguous()
        if smoothing_scale is not None:
            _check_smoothing_metadata(smoothing_scale, weight_input)
            if not torch.isfinite(smoothing_scale).all() or not (smoothing_scale > 0).all():
                raise ValueError("SmoothQuant scales must be finite and positive")
            weight_input = (weight_input.float() * smoothing_scale).to(torch.bfloat16)
            if not torch.isfinite(weight_input).all():
                raise ValueError("SmoothQuant overflowed BF16 weights")
        self.register_buffer("smoothing_scale", smoothing_scale)
        if precision == "fp8":
            # Per-tensor E4M3 weights (pack_linear_weight, fp8_cutlass_linear.cu:
            # 1011-1024); the scale is kept as piR2's scalar and replicated
            # per output channel for the GEMM epilogue.
            packed, scale, columns = ops.quant_fp8(weight_input, replicate=self.out_features, weights=True)
            scale = scale.reshape(())
            self.register_buffer("weight_scale_columns", columns)
        else:
            packed, scale = ops.pack_nvfp4(weight_input)
        self.register_buffer("packed_weight", packed)
        self.register_buffer("weight_scale", scale)
        self.register_buffer(
            "metadata", torch.tensor([self.out_features, self.in_features], dtype=torch.int64)
        )
        self.register_buffer("bias", None if linear.bias is None else linear.bias.detach())

    def pack_input(self, value):
        if isinstance(value, FloatingPacked):
            if (
                value.precision != self.precision
                or value.shape[-1] != self.in_features
                or value.data.device != self.packed_weight.device
                or value.smoothing_scale is not self.smoothing_scale
            ):
                raise ValueError("Floating packed input does not match its consumer")
            return value.data, value.scale
        if (
            value.dtype != torch.bfloat16
            or value.device != self.packed_weight.device
            or value.ndim < 1
            or value.shape[-1] != self.in_features
            or value.numel() == 0
            or value.requires_grad
        ):
            raise ValueError("Floating quantization requires nonempty CUDA BF16 inference activations")
        matrix = value.reshape(-1, self.in_features).contiguous()
        if self.precision == "fp8":
            # Activation scale replicated per row for the GEMM epilogue.
            q, _, rows = ops.quant_fp8(matrix, fast=self.fast_fp8)
            return q, rows
        if self.smoothing_scale is not None:
            packed = prepare_smoothed(matrix, self.precision, self.smoothing_scale)
            return packed.data, packed.scale
        return ops.pack_nvfp4(matrix)

    def forward_packed(self, packed, scale, leading_shape):
        if self.precision == "fp8":
            result = ops.gemm_fp8(
                packed, scale, self.packed_weight, self.weight_scale_columns, self.bias, n=self.out_features
            )
        else:
            result = ops.gemm_nvfp4(
                packed, scale, self.packed_weight, self.weight_scale, self.bias, n=self.out_features
            )
        return result.reshape(*leading_shape, self.out_features)

    def forward(self, value):
        packed, scale = self.pack_input(value)
        shape = value.shape[:-1] if not isinstance(value, FloatingPacked) else value.shape[:-1]
        return self.forward_packed(packed, scale, shape)


class FloatingInputGroup:
    """One activation pack per owner call for sibling projections of the
    same input (q|k|v, k|v, gate|up): thor/linear.py:193-229.  GEMMs, weight
    scales and layers stay independent; the cache lives only inside one
    owner invocation and is keyed on the identical input tensor; a direct
    projection call outside an owner call never reuses it.  Serial
    inference only, like the reference."""

    def __init__(self, linears):
        if any(q.smoothing_scale is not linears[0].smoothing_scale for q in linears):
            raise ValueError("Shared packing requires identical SmoothQuant scales")
        self.linears = linears
        self.active = False
        self.cache = None

    def run(self, forward, *args, **kwargs):
        previous = self.active, self.cache
        self.active, self.cache = True, None
        try:
            return forward(*args, **kwargs)
        finally:
            self.active, self.cache = previous

    def project(self, value, index):
        linear = self.linears[index]
        if not self.active:
            return linear(value)
        if self.cache is None or self.cache[0] is not value or index in self.cache[3]:
            packed, scale = linear.pack_input(value)
            self.cache = (value, packed, scale, set())
        _, packed, scale, used = self.cache
        result = linear.forward_packed(packed, scale, value.shape[:-1])
        used.add(index)
        if len(used) == len(self.linears):
            self.cache = None
        return result


class FloatingProjections:
    """Reversible installation of FloatingLinear on the executed sites that
    meet the FP4 alignment (others stay bf16, as piR2's alignment checks
    exclude them)."""

    def __init__(self, model, executed, *, smoothing=None, precision="fp4", fast_fp8=False, shared_inputs=False,
                 groups=()):
        self.sites = {}
        self.skipped = []
        self.groups = []
        modules = dict(model.named_modules())
        for name in executed:
            module = modules[name]
            if not aligned_for(precision, module.in_features, module.out_features):
                self.skipped.append(name)
                continue
            scale = None if smoothing is None else smoothing.get(name)
            self.sites[name] = (
                module,
                FloatingLinear(module, name, precision, fast_fp8=fast_fp8, smoothing_scale=scale),
            )
        if shared_inputs:
            # Sibling projections of one owner module (the same input tensor).
            for names in groups:
                if not all(n in self.sites for n in names):
                    continue
                owner = names[0].rpartition(".")[0]
                if any(n.rpartition(".")[0] != owner for n in names):
                    continue
                group = FloatingInputGroup([self.sites[n][1] for n in names])
                self.groups.append((modules[owner], [self.sites[n][0] for n in names], group))
        self.saved = []

    def set(self):
        self.close()
        for module, linear in self.sites.values():
            self.saved.append((module, "forward" in module.__dict__, module.__dict__.get("forward")))
            module.forward = linear.forward
        for owner, members, group in self.groups:
            self.saved.append((owner, "forward" in owner.__dict__, owner.__dict__.get("forward")))
            original = owner.forward
            owner.forward = lambda *args, g=group, f=original, **kw: g.run(f, *args, **kw)
            for index, member in enumerate(members):
                member.forward = lambda x, g=group, i=index: g.project(x, i)

    def close(self):
        for module, had, forward in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []
