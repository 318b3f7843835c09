"""NVFP4 and FP8 (E4M3) Linear layers and their fused producers on the B200
kernels.

Mirrors coexecution/optimization/backends/thor/linear.py
(`FloatingLinear`, `FloatingInputGroup`, `FloatingProjectionGroup`,
:30-309), packing.py (`FloatingPacked` and the fused producers, :15-519)
and coexecution/optimization/groot/floating.py (`FloatingProjections`, the
SwiGLU / GELU / RMSNorm producer installation, :17-372).

NVFP4 weights are packed once as E2M1 with UE4M3 factors per 16 elements
(the CUTLASS 128x4 swizzled factor layout, `sfa_offset`); activations are
packed per call, fused with the producing operation where configured, and
the GEMM runs on tcgen05 kind::mxf4nvf4 with fp32 accumulation and bf16
output.  FP8 layers quantize weights and activations per tensor to E4M3
(`ops.quant_fp8`: quantize_bf16's arithmetic, or prepare_fp8's with
`fast_fp8`) and run the E4M3 GEMM (tcgen05 kind::f8f6f4, or warp-level e4m3
MMAs for at most 32 token rows) with fp32 accumulation.  The fused FP8
producers keep piR2's two passes (packing.py:1-4: a per-tensor scale needs
the global maximum): the producer writes bf16 values and row maxima, then
`ops.fp8_cast` scales and casts with prepare_fp8's arithmetic.

FP8 in_features must be a multiple of 128 (piR2: 16); an NVFP4 K block of
the B200 kernel is 256 values, so fp4 in_features must be a multiple of 256
(piR2: 32); out_features must be a multiple of 32 (fp4) or 16 (fp8) as in
piR2.  Producers accept rows of at most 8192 values (piR2: 65536).
"""

import math
from dataclasses import dataclass

import torch

from . import _lib, ops


@dataclass
class FloatingPacked:
    """A packed activation (packing.py:15-21).  For fp8, `scale` is the 0-d
    per-tensor scale and `row_scales` the same scale replicated per row, the
    operand the E4M3 GEMM reads."""

    data: torch.Tensor
    scale: torch.Tensor
    shape: tuple
    precision: str
    smoothing_scale: torch.Tensor | None = None
    row_scales: torch.Tensor | None = None


_FORMATS = {"fp4": _lib.OUT_NVFP4, "fp8": _lib.OUT_FP8_VALUES}


def _check_smoothing_metadata(scale, value):
    if scale is not None and (
        scale.shape != (value.shape[-1],)
        or scale.dtype != torch.float32
        or scale.device != value.device
        or not scale.is_contiguous()
        or scale.requires_grad
    ):
        raise ValueError("SmoothQuant requires contiguous immutable FP32 channel scales")


def _producer_rows(x, precision):
    """packing.py:152-177 (_producer_buffers): checks; the rows as a
    contiguous [rows, k] matrix."""
    if (
        precision not in _FORMATS
        or not x.is_cuda
        or x.dtype != torch.bfloat16
        or x.numel() == 0
        or x.requires_grad
        or x.shape[-1] % (16 if precision == "fp8" else 32)
        or x.shape[-1] > 8192
    ):
        raise ValueError("Floating producer requires nonempty aligned CUDA BF16 inference")
    k = x.shape[-1]
    return x.reshape(-1, k).contiguous(), k


def _finish_producer(data, auxiliary, shape, precision, smoothing_scale=None):
    """packing.py:180-199: NVFP4 is complete; the FP8 first pass (bf16 values,
    row maxima) is scaled and cast to E4M3."""
    if precision == "fp4":
        return FloatingPacked(data, auxiliary, tuple(shape), precision, smoothing_scale)
    packed, scale, rows = ops.fp8_cast(data, auxiliary)
    return FloatingPacked(packed, scale.reshape(()), tuple(shape), precision, smoothing_scale, rows)


def prepare_fp8(matrix):
    """packing.py:485-519: fresh E4M3 codes and one fp32 scale with the
    two-pass arithmetic (scale = max(amax * (1/448), 1e-12), v / scale)."""
    if (
        not matrix.is_cuda
        or matrix.dtype != torch.bfloat16
        or not matrix.is_contiguous()
        or matrix.ndim != 2
        or matrix.numel() == 0
    ):
        raise ValueError("FP8 packing requires a nonempty contiguous CUDA BF16 matrix")
    packed, scale, _ = ops.quant_fp8(matrix, fast=True)
    return packed.view(torch.float8_e4m3fn), scale.reshape(())


def prepare_smoothed(matrix, precision, smoothing_scale):
    """bf16(x / s) fused into the pack (packing.py:314-349)."""
    _check_smoothing_metadata(smoothing_scale, matrix)
    if smoothing_scale is None or matrix.ndim != 2 or not matrix.is_contiguous():
        raise ValueError("Smoothed packing needs a contiguous matrix and channel scales")
    rows, _ = _producer_rows(matrix, precision)
    data, aux = ops.floating_rows(rows, _FORMATS[precision], smooth=smoothing_scale)
    return _finish_producer(data, aux, matrix.shape, precision, smoothing_scale)


def prepare_swiglu(gate, up, lut, precision, *, smoothing_scale=None):
    """Native BF16 SiLU lookup, multiply and floating packing in one pass
    (packing.py:84-107, :201-231): v = bf16(f32(lut[gate]) * f32(up))."""
    shape = tuple(gate.shape)
    _producer_rows(gate, precision)
    _check_smoothing_metadata(smoothing_scale, gate)
    if up.shape != gate.shape or up.device != gate.device or up.dtype != gate.dtype:
        raise ValueError("SwiGLU operands must have identical shape, device and dtype")
    if lut.shape != (65536,) or lut.device != gate.device or lut.dtype != gate.dtype:
        raise ValueError("SwiGLU requires the native BF16 SiLU lookup table")
    k = shape[-1]
    # Merged gate/up views have a contiguous last dimension but strided rows.
    gate, up = gate.reshape(-1, k), up.reshape(-1, k)
    if gate.stride(1) != 1 or up.stride(1) != 1:
        raise ValueError("SwiGLU producer requires contiguous columns")
    data, aux = ops.floating_rows(gate, _FORMATS[precision], lut=lut, up=up, smooth=smoothing_scale)
    return _finish_producer(data, aux, shape, precision, smoothing_scale)


def prepare_gelu_packed(x, lut, precision, *, smoothing_scale=None):
    """Native BF16 GELU lookup, channel balancing and packing in one pass
    (packing.py:352-392)."""
    _check_smoothing_metadata(smoothing_scale, x)
    if not x.is_contiguous():
        raise ValueError("GELU packing requires contiguous activations")
    if lut.shape != (65536,) or lut.device != x.device or lut.dtype != x.dtype:
        raise ValueError("GELU packing requires a native BF16 lookup table")
    rows, _ = _producer_rows(x, precision)
    data, aux = ops.floating_rows(rows, _FORMATS[precision], lut=lut, smooth=smoothing_scale)
    return _finish_producer(data, aux, x.shape, precision, smoothing_scale)


def prepare_rmsnorm_packed(x, weight, precision, *, eps, smoothing_scale=None):
    """RMSNorm [+ SmoothQuant] to packed input, preserving BF16 stages
    (packing.py:395-448): n = bf16(x * rsqrt(sum(x^2) / k + eps)),
    v = bf16(n * weight)."""
    _check_smoothing_metadata(smoothing_scale, x)
    if (
        not x.is_contiguous()
        or weight.shape != (x.shape[-1],)
        or weight.device != x.device
        or weight.dtype != x.dtype
        or not weight.is_contiguous()
        or not math.isfinite(eps)
        or eps <= 0
    ):
        raise ValueError("RMSNorm packing requires contiguous BF16 and positive epsilon")
    rows, _ = _producer_rows(x, precision)
    data, aux, _ = ops.norm_quant_rows(
        rows, _FORMATS[precision], norm=_lib.NORM_RMS, eps=eps, gamma=weight, smooth=smoothing_scale
    )
    return _finish_producer(data, aux, x.shape, precision, smoothing_scale)


def prepare_norm(x, precision, *, eps, scale=None, shift=None, residual=None, smoothing_scale=None):
    """LayerNorm [+ AdaLN] [+ residual] [+ SmoothQuant] directly to packed
    input (packing.py:234-297).  Returns (packed, bf16 x + residual or None)."""
    _producer_rows(x, precision)
    _check_smoothing_metadata(smoothing_scale, x)
    if x.ndim != 3 or not x.is_contiguous() or not math.isfinite(eps) or eps <= 0:
        raise ValueError("Norm packing requires contiguous B,T,D and positive epsilon")
    if (scale is None) != (shift is None):
        raise ValueError("Modulation requires both scale and shift")
    b, t, k = x.shape
    tokens = 1
    if scale is not None:
        for value in (scale, shift):
            if (
                value.dtype != x.dtype
                or value.device != x.device
                or value.shape not in (x.shape, (b, k))
                or value.stride(-1) != 1
            ):
                raise ValueError("Modulation must match BF16 B,D or per-token B,T,D")
        if scale.shape != shift.shape:
            raise ValueError("Modulation shapes must match")
        tokens = t if scale.ndim == 2 else 1
        scale, shift = scale.reshape(-1, k), shift.reshape(-1, k)
        if scale.stride(0) != shift.stride(0):
            scale, shift = scale.contiguous(), shift.contiguous()
    y = None
    if residual is not None:
        if (
            residual.shape != x.shape
            or residual.dtype != x.dtype
            or residual.device != x.device
            or not residual.is_contiguous()
        ):
            raise ValueError("Residual must match contiguous BF16 input")
        y = residual.reshape(-1, k)
    data, aux, summed = ops.norm_quant_rows(
        x.reshape(-1, k), _FORMATS[precision], norm=_lib.NORM_LN, eps=eps, scale=scale, shift=shift,
        tokens=tokens, y=y, smooth=smoothing_scale,
    )
    packed = _finish_producer(data, aux, x.shape, precision, smoothing_scale)
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
            if self.precision == "fp8":
                rows = value.row_scales
                if rows is None:
                    # A carrier built elsewhere holds the scalar scale only.
                    rows = value.scale.reshape(1).float().expand(value.data.shape[0]).contiguous()
                return value.data.view(torch.uint8), rows
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
        if self.smoothing_scale is not None:
            # thor/linear.py:128-132: smoothed sites pack with the fused
            # division (for fp8 with prepare_fp8's arithmetic).
            packed = prepare_smoothed(matrix, self.precision, self.smoothing_scale)
            return packed.data, (packed.row_scales if self.precision == "fp8" else packed.scale)
        if self.precision == "fp8":
            # Activation scale replicated per row for the GEMM epilogue.
            q, _, rows = ops.quant_fp8(matrix, fast=self.fast_fp8)
            return q, rows
        return ops.pack_nvfp4(matrix)

    def forward_packed(self, packed, scale, leading_shape, residual=None):
        """The GEMM of packed input; `residual` (bf16, the output's shape) is
        added as bf16(y + residual) in fp32, in the E4M3 GEMM's epilogue (the
        NVFP4 GEMM has none: a separate add, the same arithmetic)."""
        if self.precision == "fp8":
            res = None if residual is None else residual.reshape(-1, self.out_features)
            if res is not None and res.stride(-1) != 1:
                res = res.contiguous()
            result = ops.gemm_fp8(
                packed, scale, self.packed_weight, self.weight_scale_columns, self.bias, n=self.out_features,
                residual=res,
            )
            return result.reshape(*leading_shape, self.out_features)
        result = ops.gemm_nvfp4(
            packed, scale, self.packed_weight, self.weight_scale, self.bias, n=self.out_features
        ).reshape(*leading_shape, self.out_features)
        return result if residual is None else result + residual

    def forward(self, value, residual=None):
        packed, scale = self.pack_input(value)
        return self.forward_packed(packed, scale, value.shape[:-1], residual)


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


class FloatingProjectionGroup:
    """One concatenated GEMM per same-input owner invocation
    (thor/linear.py:232-309).  FP8 requantizes the concatenated weights with
    one shared per-tensor scale; FP4 keeps each row's block-16 factors (its
    packed rows equal the members' own).  A missing member bias is zeros."""

    def __init__(self, modules, name, precision, fast_fp8, contiguous=False, *, fp4_swap_ab=False,
                 smoothing_scale=None):
        self.sizes = [m.out_features for m in modules]
        merged = torch.nn.Linear(modules[0].in_features, sum(self.sizes), bias=False, device="meta",
                                 dtype=torch.bfloat16)
        merged.weight = torch.nn.Parameter(torch.cat([m.weight.detach() for m in modules]), requires_grad=False)
        if any(m.bias is not None for m in modules):
            merged.bias = torch.nn.Parameter(
                torch.cat([m.bias.detach() if m.bias is not None else m.weight.new_zeros(m.out_features)
                           for m in modules]),
                requires_grad=False,
            )
        self.linear = FloatingLinear(merged, name, precision, fast_fp8=fast_fp8, fp4_swap_ab=fp4_swap_ab,
                                     smoothing_scale=smoothing_scale)
        self.contiguous = contiguous
        self.active, self.cache = False, None

    run = FloatingInputGroup.run

    def project(self, value, index):
        if not self.active or self.cache is None or self.cache[0] is not value or index in self.cache[2]:
            parts = self.linear(value).split(self.sizes, dim=-1)
            if self.contiguous:
                parts = tuple(p.contiguous() for p in parts)
            if not self.active:
                return parts[index]
            self.cache = (value, parts, set())
        _, parts, used = self.cache
        result = parts[index]
        used.add(index)
        if len(used) == len(self.sizes):
            self.cache = None
        return result


class _Patches:
    """Instance-level method replacements, restored last-in first-out."""

    def __init__(self):
        self.saved = []

    def replace(self, module, attr, value):
        self.saved.append((module, attr, attr in module.__dict__, module.__dict__.get(attr)))
        setattr(module, attr, value)

    def restore(self):
        for module, attr, had, value in reversed(self.saved):
            if had:
                setattr(module, attr, value)
            elif attr in module.__dict__:
                delattr(module, attr)
        self.saved = []


# FP8 DiT FFN: the GELU producer's table and partial maxima come from the up
# projection's epilogue (`_fp8_gelu_from_gemm`); False keeps the separate
# producer pass.  Both give the same codes.
FP8_GELU_FROM_GEMM = True


def _fp8_gelu_from_gemm(module, linear, lut, x):
    """gelu(proj(x)) packed to E4M3 with the table and the partial maxima
    written by the E4M3 GEMM's epilogue (at most 32 token rows), else the
    module's GEMM followed by the GELU producer."""
    packed, scale = linear.pack_input(x)
    rows = packed.shape[0]
    if rows > 32 or linear.packed_weight.shape[0] % 16:
        return module.gelu(module.proj(x))
    maxima = torch.empty((rows, linear.packed_weight.shape[0] // 16), device=packed.device, dtype=torch.float32)
    y = ops.gemm_fp8(packed, scale, linear.packed_weight, linear.weight_scale_columns, linear.bias,
                     n=linear.out_features, out_lut=lut, max_out=maxima)
    q, s, rep = ops.fp8_cast(y, maxima)
    shape = tuple(x.shape[:-1]) + (linear.out_features,)
    return FloatingPacked(q, s.reshape(()), shape, "fp8", None, rep)


class FloatingProjections:
    """Reversible installation of the floating Linear layers and producers
    (coexecution/optimization/groot/floating.py:17-372): every executed site
    that meets the alignment becomes a FloatingLinear (others stay bf16 and
    are listed in `skipped`); with `shared_inputs`, sibling projections of
    one owner call share one activation pack; with `grouped`, they run as
    one concatenated GEMM; `swiglu`, `gelu` and `rmsnorm` install the fused
    producers in front of the text MLP's down projection, the DiT FFN's down
    projection and the text MLP's gate|up input."""

    def __init__(self, model, executed, *, smoothing=None, precision="fp4", fast_fp8=False, shared_inputs=False,
                 grouped=False, swiglu=False, gelu=False, rmsnorm=False, groups=None):
        from .projections import inventory

        self.model = model
        self.precision = precision
        self.smoothing = {} if smoothing is None else dict(smoothing)
        self.sites = {}
        self.skipped = []
        self.groups = []
        self.coverage = {"swiglu_producers": [], "gelu_producers": [], "rmsnorm_producers": [],
                         "merged_projection_groups": [], "shared_input_groups": []}
        _, found_groups, self.activations, self.text = inventory(model, expanded=True)
        groups = found_groups if groups is None else groups
        modules = dict(model.named_modules())
        for name in executed:
            module = modules[name]
            if not aligned_for(precision, module.in_features, module.out_features):
                self.skipped.append(name)
                continue
            self.sites[name] = (
                module,
                FloatingLinear(module, name, precision, fast_fp8=fast_fp8,
                               smoothing_scale=self.smoothing.get(name)),
            )
        if shared_inputs or grouped:
            roles = {n: (r, sc) for n, (_, r, sc) in inventory(model, expanded=True)[0].items()}
            # Sibling projections of one owner module (the same input tensor).
            for names in groups:
                if not all(n in self.sites for n in names):
                    continue
                owner = names[0].rpartition(".")[0]
                if any(n.rpartition(".")[0] != owner for n in names):
                    continue
                members = [self.sites[n][0] for n in names]
                if grouped:
                    group = FloatingProjectionGroup(
                        members, owner, precision, fast_fp8,
                        contiguous=roles.get(names[0]) == ("AttnQ", "text"),
                        smoothing_scale=self.smoothing.get(names[0]),
                    )
                    self.coverage["merged_projection_groups"].append(
                        {"owner": owner, "members": list(names),
                         "weight_scale": "one tensor per merged group" if precision == "fp8"
                         else "unchanged block-16 row scales"})
                else:
                    group = FloatingInputGroup([self.sites[n][1] for n in names])
                    self.coverage["shared_input_groups"].append({"owner": owner, "members": list(names)})
                self.groups.append((modules[owner], members, group))
        self.options = {"swiglu": swiglu, "gelu": gelu, "rmsnorm": rmsnorm}
        self._patches = _Patches()

    def linear_of(self, module):
        """The FloatingLinear installed on `module` (None if it has none)."""
        for site, linear in self.sites.values():
            if site is module:
                return linear
        return None

    def input_smoothing(self, module):
        """The SmoothQuant scale of a quantized site (None if unsmoothed)."""
        for name, (site, _) in self.sites.items():
            if site is module:
                return self.smoothing.get(name)
        return None

    def _quantized(self, *modules):
        ids = {id(m) for m, _ in self.sites.values()}
        return all(id(m) in ids for m in modules)

    def set(self):
        from .fused import prepare_gelu, prepare_silu

        self.close()
        patches = self._patches
        modules = dict(self.model.named_modules())
        names = {id(m): n for n, m in modules.items()}
        for module, linear in self.sites.values():
            patches.replace(module, "forward", linear.forward)
        precision = self.precision
        # The SwiGLU producer replaces the text MLP's forward before the
        # gate|up group wraps it (floating.py:162-197), so one owner call
        # still shares one pack or runs one merged GEMM.
        if self.options["swiglu"]:
            for mlp, down in self.text:
                if not self._quantized(mlp.gate_proj, mlp.up_proj, mlp.down_proj):
                    continue
                lut = prepare_silu(mlp.down_proj.weight.device)
                smooth = self.input_smoothing(mlp.down_proj)

                def forward(x, mlp=mlp, lut=lut, smooth=smooth):
                    packed = prepare_swiglu(mlp.gate_proj(x), mlp.up_proj(x), lut, precision, smoothing_scale=smooth)
                    return mlp.down_proj(packed)

                patches.replace(mlp, "forward", forward)
                self.coverage["swiglu_producers"].append(down)
        for owner, members, group in self.groups:
            original = owner.forward
            patches.replace(owner, "forward", lambda *args, g=group, f=original, **kw: g.run(f, *args, **kw))
            for index, member in enumerate(members):
                patches.replace(member, "forward", lambda x, g=group, i=index: g.project(x, i))
        if self.options["gelu"]:
            for module, attr, down, approximate in self.activations:
                if down not in self.sites:
                    continue
                weight = modules[down].weight
                lut = prepare_gelu(weight.device, weight.dtype, approximate)
                smooth = self.input_smoothing(modules[down])
                patches.replace(module, attr, lambda x, lut=lut, smooth=smooth: prepare_gelu_packed(
                    x.contiguous(), lut, precision, smoothing_scale=smooth))
                self.coverage["gelu_producers"].append(down)
                proj = getattr(module, "proj", None)
                proj_linear = None if proj is None else self.linear_of(proj)
                if (FP8_GELU_FROM_GEMM and precision == "fp8" and attr == "gelu" and smooth is None
                        and proj_linear is not None):
                    # FP8: the GELU table and the producer's partial maxima in
                    # the up projection's epilogue (few-token launches), so
                    # only the cast remains (the same values, maxima, codes).
                    patches.replace(module, "forward", lambda x, module=module, lin=proj_linear, lut=lut: (
                        _fp8_gelu_from_gemm(module, lin, lut, x)))
                if attr == "gelu":
                    # The eval Dropout between the DiT FFN's GELU and its down
                    # projection passes the packed carrier through.
                    parents = [m for m in self.model.modules()
                               if hasattr(m, "net") and len(m.net) >= 3 and m.net[0] is module]
                    if len(parents) != 1:
                        raise ValueError("GELU producer requires a unique FFN owner")
                    dropout = parents[0].net[1]
                    if not isinstance(dropout, torch.nn.Dropout) or dropout.training:
                        raise ValueError("GELU producer requires eval Dropout")
                    original_dropout = dropout.forward
                    patches.replace(dropout, "forward", lambda x, original=original_dropout: (
                        x if isinstance(x, FloatingPacked) else original(x)))
        if self.options["rmsnorm"]:
            for layer in self.model.modules():
                if type(layer).__name__ != "Qwen3VLTextDecoderLayer":
                    continue
                if not self._quantized(layer.mlp.gate_proj, layer.mlp.up_proj):
                    continue
                norm = layer.post_attention_layernorm
                if type(norm).__name__ != "Qwen3VLTextRMSNorm":
                    raise ValueError("RMSNorm producer requires Qwen3VLTextRMSNorm")
                smooth = self.input_smoothing(layer.mlp.gate_proj)
                patches.replace(norm, "forward", lambda x, norm=norm, smooth=smooth: prepare_rmsnorm_packed(
                    x.contiguous(), norm.weight, precision, eps=norm.variance_epsilon, smoothing_scale=smooth))
                self.coverage["rmsnorm_producers"].append(names[id(layer.mlp.gate_proj)])

    def close(self):
        self._patches.restore()
        for key in ("swiglu_producers", "gelu_producers", "rmsnorm_producers"):
            self.coverage[key] = []


class FloatingConnections:
    """DiT normalization / residual producers for the floating projections
    (coexecution/optimization/groot/floating_connections.py:12-133): AdaLN
    `norm1` modules whose attention inputs are all quantized return packed
    input from the LayerNorm + modulation producer; with `residual`, the
    block's attention residual add, `norm3` and the FFN input pack run as one
    producer (`prepare_norm` with a residual)."""

    def __init__(self, model, floating, *, residual=False):
        self.floating = floating
        self.norms, self.blocks = [], []
        precision = floating.precision
        blocks = model.action_head.model.transformer_blocks
        for block in blocks:
            names = ("to_q",) if block.attn1.is_cross_attention else ("to_q", "to_k", "to_v")
            if floating._quantized(*(getattr(block.attn1, n) for n in names)):
                if block.norm_type != "ada_norm":
                    raise ValueError("Floating norm fusion requires AdaLayerNorm")
                if block.pos_embed is not None:
                    raise ValueError("Floating norm fusion requires no position embeddings")
                self.norms.append((block.norm1, floating.input_smoothing(block.attn1.to_q)))
            if residual and floating._quantized(block.ff.net[0].proj):
                if block.pos_embed is not None:
                    raise ValueError("Floating residual fusion requires no position embeddings")
                self.blocks.append((block, floating.input_smoothing(block.ff.net[0].proj),
                                    floating.linear_of(block.ff.net[2])))
        if not self.norms or (residual and not self.blocks):
            raise ValueError("Floating norm fusion selected no compatible DiT projections")
        for norm in [*(n.norm for n, _ in self.norms), *(b.norm3 for b, _, _ in self.blocks)]:
            if not isinstance(norm, torch.nn.LayerNorm) or norm.elementwise_affine:
                raise ValueError("Floating norm fusion requires non-affine LayerNorm")
        self.precision = precision
        self._patches = _Patches()

    def set(self):
        self.close()
        precision = self.precision
        for norm, smooth in self.norms:

            def forward(x, temb=None, norm=norm, smooth=smooth):
                scale, shift = norm.linear(norm.silu(temb)).chunk(2, dim=-1)
                packed, _ = prepare_norm(x, precision, eps=norm.norm.eps, scale=scale, shift=shift,
                                         smoothing_scale=smooth)
                return packed

            self._patches.replace(norm, "forward", forward)
        for block, smooth, down in self.blocks:

            def forward(hidden_states, attention_mask=None, encoder_hidden_states=None,
                        encoder_attention_mask=None, temb=None, block=block, smooth=smooth, down=down):
                x = hidden_states
                normalized = block.norm1(x, temb) if block.norm_type == "ada_norm" else block.norm1(x)
                mask = encoder_attention_mask if encoder_hidden_states is not None else attention_mask
                attention = block.attn1(normalized, encoder_hidden_states=encoder_hidden_states, attention_mask=mask)
                if block.final_dropout is not None:
                    attention = block.final_dropout(attention)
                packed, summed = prepare_norm(x, precision, eps=block.norm3.eps, residual=attention.contiguous(),
                                              smoothing_scale=smooth)
                if down is None or len(block.ff.net) != 3:
                    return summed + block.ff(packed)
                # summed + ff(packed), the add in the down projection's
                # epilogue: bf16(y + summed) in fp32, as torch's bf16 add.
                h = block.ff.net[1](block.ff.net[0](packed))
                return down(h, residual=summed)

            self._patches.replace(block, "forward", forward)

    def close(self):
        self._patches.restore()


class FloatingTextFusion:
    """Text decoder attention on the floating path with merged q|k|v
    projections (fp_grouped): the input RMSNorm packs straight to the
    floating format (the RMSNorm producer, as piR2's fp_rmsnorm does for the
    MLP input), the merged q|k|v GEMM runs once, and one kernel applies
    q_norm / k_norm, the rotary embedding and the [B, H, T, D] relayout
    (`ops.qk_norm_rope`, the BF16 fusion piR2's operator fusion performs
    with its own kernels, coexecution/fused_ops.py).  Layers whose q|k|v are
    not one merged group keep their forward."""

    def __init__(self, model, floating):
        self.targets = []
        by_q = {}
        for _, members, group in floating.groups:
            if isinstance(group, FloatingProjectionGroup) and len(members) == 3:
                by_q[id(members[0])] = group
        for layer in model.modules():
            if type(layer).__name__ != "Qwen3VLTextDecoderLayer":
                continue
            attn = layer.self_attn
            group = by_q.get(id(attn.q_proj))
            if group is None or attn.head_dim != 128 or group.sizes != [
                attn.heads * attn.head_dim, attn.kv_heads * attn.head_dim, attn.kv_heads * attn.head_dim
            ]:
                continue
            if type(layer.input_layernorm).__name__ != "Qwen3VLTextRMSNorm":
                continue
            self.targets.append((layer, group, floating.input_smoothing(attn.q_proj)))
        self.precision = floating.precision
        self._patches = _Patches()

    def set(self):
        self.close()
        precision = self.precision
        for layer, group, smooth in self.targets:
            norm, attn = layer.input_layernorm, layer.self_attn
            self._patches.replace(norm, "forward", lambda x, norm=norm, smooth=smooth: prepare_rmsnorm_packed(
                x.contiguous(), norm.weight, precision, eps=norm.variance_epsilon, smoothing_scale=smooth))

            def forward(x, cos, sin, attn=attn, group=group):
                b, t = x.shape[0], x.shape[1]
                qkv = group.linear(x)
                q, k, v = ops.qk_norm_rope(
                    qkv.reshape(b * t, qkv.shape[-1]), attn.q_norm.weight, attn.k_norm.weight, cos, sin,
                    tokens=t, hq=attn.heads, hk=attn.kv_heads, eps=attn.q_norm.variance_epsilon,
                )
                y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
                return attn.o_proj(y.transpose(1, 2).reshape(b, t, attn.heads * attn.head_dim))

            self._patches.replace(attn, "forward", forward)

    def close(self):
        self._patches.restore()
