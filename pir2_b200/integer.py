"""symmetric-row-v1 integer Linear layers (W8A8 / W4A4) on the B200 kernels.

Mirrors the reference module coexecution/kernels/ampere_ada/integer.py:
`PackedActivation` (:97-104), `prepare_activation` (:107-173),
`IntegerLinear` (:176-301), `IntegerProjectionGroup` (:304-377) and
`IntegerProjectionSlice` (:380-397), with the same names, arguments, packed
formats and error behaviour.  Weight packing happens once at construction;
every forward runs two sm_100a kernels of libpir2b.so (activation pack and
tcgen05 GEMM with the fused dequant epilogue).
"""

import weakref
from dataclasses import dataclass

import torch

from . import _lib, ops

FORMAT_VERSION = "symmetric-row-v1"


def load_integer_extension():
    """Loads libpir2b.so (raises when it is missing; no fallback)."""
    return _lib.lib()


# W4A4 GEMMs over more token rows than this run on the int8 kernel over
# unpacked codes (same int32 sums, so bitwise the same output): past the
# small-M regime the GEMM is bound by MMA issue rather than weight bytes, and
# the int8 kernel reads its operands by TMA with no in-kernel unpack.
WIDE_INT4_ROWS = 64

# W8A8 layers given plain bf16 rows can pack them inside the GEMM (one
# launch instead of pack + GEMM, bitwise the same output) up to
# FUSED_PACK_ROWS rows and, when each GEMM CTA stages whole rows,
# FUSED_PACK_BYTES of them.  Off by default (0 rows): inside the control
# step the in-CTA pack (row copy, row maxima and divisions run by four warps
# of every CTA) costs more than the separate pack launch it removes (action
# head 4.05 vs 3.15 ms on one box).
FUSED_PACK_ROWS = 0
FUSED_PACK_BYTES = 96 * 1024


@dataclass
class PackedActivation:
    data: torch.Tensor
    scales: torch.Tensor
    shape: tuple
    logical_k: int
    bits: int
    format_version: str = FORMAT_VERSION


def prepare_activation(x, bits, *, up=None, gelu=None, pack_reuse=False, smooth=None):
    """Per-token symmetric quantization of BF16 rows (integer.py:107-173).

    gelu selects the GELU lookup table ("tanh" or "none"); with `up` the
    packed value is bf16(gelu(x) * up).  `pack_reuse` is accepted for API
    parity: both reference int4 packings produce identical bytes.  `smooth`
    (fp32 [K]) fuses the SmoothQuant division bf16(x / s) into the pack.
    """
    del pack_reuse
    if (
        bits not in (4, 8)
        or not x.is_cuda
        or x.dtype != torch.bfloat16
        or x.stride(-1) != 1
        or x.ndim < 2
    ):
        raise ValueError("Expected CUDA BF16 rows with unit feature stride and bits=4 or 8")
    lut = None
    if gelu is not None:
        if gelu not in ("tanh", "none"):
            raise ValueError("Unsupported GELU approximation")
        from .fused import prepare_gelu

        lut = prepare_gelu(x.device, x.dtype, gelu)
    if up is not None and (
        gelu is None
        or up.shape != x.shape
        or up.device != x.device
        or up.dtype != x.dtype
        or up.stride(-1) != 1
    ):
        raise ValueError("Invalid gated activation input")
    k = x.shape[-1]
    if k < 1 or k > 65536:
        raise ValueError("Unsupported activation dimensions")
    if x.numel() // k < 1:
        raise ValueError("Unsupported activation dimensions")
    data, scales = ops.quant_rows(x, bits, lut=lut, up=up, smooth=smooth)
    return PackedActivation(data, scales, tuple(x.shape[:-1]), k, bits)


class IntegerLinear(torch.nn.Module):
    """Packed integer Linear; `backend` names the B200 kernel family."""

    def __init__(
        self,
        packed,
        scales,
        bias,
        in_features,
        out_features,
        bits,
        tactic=0,
        pack_reuse=False,
        biasless_epilogue=False,
    ):
        super().__init__()
        self.register_buffer("packed_weight", packed)
        self.register_buffer("weight_scale", scales)
        self.register_buffer("bias", bias)
        self.register_buffer(
            "_weight_descriptor",
            torch.empty(0, device=packed.device, dtype=torch.bfloat16),
            persistent=False,
        )
        self.in_features = in_features
        self.out_features = out_features
        self.bits = bits
        self.tactic = tactic
        self.pack_reuse = pack_reuse
        self.biasless_epilogue = biasless_epilogue
        self.backend = f"pir2b_tcgen05_int{bits}_s32_bf16"
        self._ops = load_integer_extension()

    @property
    def weight(self):
        return self._weight_descriptor

    @classmethod
    def from_linear(cls, linear, *, bits=8, tactic=0, pack_reuse=False, biasless_epilogue=False):
        """Per-output-channel weight quantization (integer.py:211-256)."""
        if bits not in (4, 8) or not linear.weight.is_cuda or linear.weight.dtype != torch.bfloat16:
            raise ValueError("IntegerLinear requires CUDA BF16 weights and bits=4 or 8")
        load_integer_extension()
        packed, scales = quantize_weight(linear.weight, bits)
        n = linear.weight.shape[0]
        bias = None
        if linear.bias is not None:
            bias = torch.nn.functional.pad(linear.bias.detach().to(torch.bfloat16), (0, ops.npad(n) - n))
        return cls(
            packed,
            scales,
            bias,
            linear.weight.shape[1],
            n,
            bits,
            tactic,
            pack_reuse,
            biasless_epilogue,
        )

    def pack_input(self, x):
        if getattr(x, "_robotics_packed_input", False):
            packed = x.for_bits(self.bits)
            if packed.logical_k != self.in_features:
                raise ValueError("Wrong prepared input feature count")
            return packed
        if x.shape[-1] != self.in_features:
            raise ValueError("Wrong input feature count")
        return prepare_activation(x, self.bits, pack_reuse=self.pack_reuse)

    def _bias_mode(self):
        if self.bias is not None:
            return _lib.BIAS_ADD
        return _lib.BIAS_NONE if self.biasless_epilogue else _lib.BIAS_ZERO

    def forward_packed(self, packed, out_lut=None, residual=None, max_out=None):
        """GEMM of a pack with this layer's weights.  `residual` (bf16, same
        leading shape, `out_features` wide) is added in the epilogue: the
        bf16 result plus the residual in fp32, rounded to bf16 again.  A
        residual can also be staged with `pending_residual` by a fusion
        installer that keeps the model's own forward code."""
        if (
            packed.logical_k != self.in_features
            or packed.bits != self.bits
            or packed.format_version != FORMAT_VERSION
        ):
            raise ValueError("Incompatible activation pack")
        if residual is None:
            residual = self.__dict__.pop("_pending_residual", None)
        data, weight, bits = packed.data, self.packed_weight, self.bits
        if bits == 4 and data.shape[0] > WIDE_INT4_ROWS:
            data, weight, bits = ops.unpack_int4(data), self.wide_weight(), 8
        out = ops.gemm(
            data,
            packed.scales,
            weight,
            self.weight_scale,
            self.bias,
            bits,
            bias_mode=self._bias_mode(),
            out_lut=out_lut,
            residual=residual,
            n_store=self.out_features,
            tactic=self.tactic,
            max_out=max_out,
        )
        return out.reshape(*packed.shape, self.out_features)

    def fused_pack_ok(self, x, *, with_max=False):
        """Whether `forward_rows` takes these bf16 rows (with_max: the row
        maxima come from x_max, so only K slices are staged)."""
        if (
            self.bits != 8
            or not isinstance(x, torch.Tensor)
            or x.dtype != torch.bfloat16
            or not x.is_cuda
            or x.dim() < 2
            or x.stride(-1) != 1
            or x.shape[-1] != self.in_features
            or self.in_features % 8
        ):
            return False
        rows = x.numel() // x.shape[-1]
        return 1 <= rows <= FUSED_PACK_ROWS and (with_max or rows * x.shape[-1] * 2 <= FUSED_PACK_BYTES)

    def forward_rows(self, x, x_max=None, out_lut=None, max_out=None):
        """GEMM of bf16 rows with the plain activation pack fused into the
        GEMM kernel: bitwise `forward_packed(prepare_activation(x, 8))`.
        `x_max` (fp32 [rows, parts]) may carry the rows' |x| maxima, e.g. the
        `max_out` of the layer that produced x."""
        rows = x.reshape(-1, x.shape[-1])
        residual = self.__dict__.pop("_pending_residual", None)
        out = ops.gemm_rows(
            rows,
            self.packed_weight,
            self.weight_scale,
            self.bias,
            x_max=x_max,
            bias_mode=self._bias_mode(),
            out_lut=out_lut,
            residual=residual,
            n_store=self.out_features,
            max_out=max_out,
        )
        return out.reshape(*x.shape[:-1], self.out_features)

    def wide_weight(self):
        """The int4 weights unpacked to int8 containers, made once per
        weight tensor (kept outside the module's state)."""
        key = (self.packed_weight.data_ptr(), self.packed_weight.device)
        cached = self.__dict__.get("_wide_weight")
        if cached is None or cached[0] != key:
            cached = (key, ops.unpack_int4(self.packed_weight))
            self.__dict__["_wide_weight"] = cached
        return cached[1]

    def pending_residual(self, residual):
        """Stages a residual for the next forward of this layer only."""
        self.__dict__["_pending_residual"] = residual

    def forward_gelu(self, x, up=None, *, approximate="tanh"):
        if x.shape[-1] != self.in_features:
            raise ValueError("Wrong input feature count")
        return self.forward_packed(
            prepare_activation(x, self.bits, up=up, gelu=approximate, pack_reuse=self.pack_reuse)
        )

    def forward(self, x):
        return self.forward_packed(self.pack_input(x))


def quantize_weight(weight, bits):
    """Install-time per-output-channel quantization (integer.py:222-238):
    s = max|w| / L (1 for an all-zero row), q = clamp(round(w / s)), K padded
    to a multiple of 128 and N to a multiple of 8, int4 low-nibble first."""
    w = weight.detach().float()
    if not torch.isfinite(w).all():
        raise ValueError("Weights must be finite")
    limit = 2 ** (bits - 1) - 1
    maximum = w.abs().amax(dim=1)
    scales = torch.where(maximum > 0, maximum / limit, torch.ones_like(maximum))
    values = torch.round(w / scales[:, None]).clamp(-limit, limit).to(torch.int8)
    n, k = w.shape
    values = torch.nn.functional.pad(values, (0, ops.kpad(k) - k, 0, ops.npad(n) - n))
    scales = torch.nn.functional.pad(scales, (0, ops.npad(n) - n), value=1.0)
    if bits == 4:
        values = ((values[:, 0::2].to(torch.int32) & 15) | ((values[:, 1::2].to(torch.int32) & 15) << 4)).to(
            torch.uint8
        )
    return values.contiguous(), scales.contiguous()


class IntegerProjectionGroup(torch.nn.Module):
    """Init-time packed concatenation; one GEMM per homogeneous sibling group
    (integer.py:304-377)."""

    def __init__(self, linears, *, contiguous_outputs=True):
        super().__init__()
        if len(linears) < 2 or any(not isinstance(m, IntegerLinear) for m in linears):
            raise ValueError("At least two integer projections are required")
        first = linears[0]
        key = lambda m: (  # noqa: E731
            m.in_features,
            m.bits,
            m.tactic,
            m.pack_reuse,
            m.biasless_epilogue,
            m.packed_weight.device,
        )
        if any(key(m) != key(first) for m in linears):
            raise ValueError("Projection format, input width, tactic and device must match")
        self.sizes = tuple(m.out_features for m in linears)
        self.contiguous_outputs = contiguous_outputs
        physical = [m.packed_weight.shape[0] for m in linears]
        self.offsets = tuple(sum(physical[:i]) for i in range(len(linears)))
        bias = None
        if any(m.bias is not None for m in linears):
            bias = torch.cat(
                [
                    m.bias
                    if m.bias is not None
                    else torch.zeros(m.packed_weight.shape[0], device=m.packed_weight.device, dtype=torch.bfloat16)
                    for m in linears
                ]
            )
        self.linear = IntegerLinear(
            torch.cat([m.packed_weight for m in linears]),
            torch.cat([m.weight_scale for m in linears]),
            bias,
            first.in_features,
            sum(physical),
            first.bits,
            first.tactic,
            first.pack_reuse,
            first.biasless_epilogue,
        )
        self._input = self._output = None
        self._remaining = set()

    def forget(self):
        """Drops the cached group output (the next project() recomputes)."""
        self._input = self._output = None
        self._remaining = set()

    def project(self, x, index):
        if self._input is not x or index not in self._remaining:
            self._input = x
            self._output = self.linear(x)
            self._remaining = set(range(len(self.sizes)))
        output = self._output.narrow(-1, self.offsets[index], self.sizes[index])
        if self.contiguous_outputs:
            output = output.contiguous()
        self._remaining.remove(index)
        if not self._remaining:
            self._input = self._output = None
        return output


class IntegerProjectionSlice(torch.nn.Module):
    def __init__(self, group, index):
        super().__init__()
        object.__setattr__(self, "_group", weakref.ref(group))
        self.index = index
        self.in_features = group.linear.in_features
        self.out_features = group.sizes[index]

    @property
    def weight(self):
        return self._group().linear.weight

    @property
    def bits(self):
        return self._group().linear.bits

    def forward(self, x):
        return self._group().project(x, self.index)
