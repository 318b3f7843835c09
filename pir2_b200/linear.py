"""Cached activation preparation and PreparedLinear.

Mirrors coexecution/optimization/backends/integer/linear.py: `selected_tactic`
and `install_shape_tactics` (:23-48), `prepare` (:51-90), `pack_swiglu`
(:93-94) and `PreparedLinear` (:97-106).  Tactic ids are accepted and kept
for API parity; the B200 GEMM picks its tile shape per call from M, N, K.
"""

from types import SimpleNamespace

from .fused import prepare_gelu
from .integer import IntegerLinear, PackedActivation
from . import ops


def selected_tactic(q, rows):
    return getattr(q, "shape_tactics", {}).get(rows, q.tactic)


def install_shape_tactics(q, choices):
    """Binds per-row-count tactic choices to a projection (no repacking)."""
    q.shape_tactics = {
        rows: tactic
        for (bits, rows, k, n, bias), tactic in choices.items()
        if (bits, k, n, bias) == (q.bits, q.in_features, q.out_features, q.bias is not None)
    }
    original = getattr(q, "_reference_ops", q._ops)
    q._reference_ops = original
    q._ops = SimpleNamespace(shape_tactics=q.shape_tactics, library=original)


def prepare(x, bits, lut=None, up=None):
    """Activation pack with an optional LUT (GELU/SiLU) and gate multiplier."""
    k = x.shape[-1]
    data, scales = ops.quant_rows(x, bits, lut=lut, up=up)
    return PackedActivation(data, scales, tuple(x.shape[:-1]), k, bits)


def pack_swiglu(gate, up, lut, bits):
    return prepare(gate, bits, lut, up)


class PreparedLinear(IntegerLinear):
    def pack_input(self, x):
        if getattr(x, "_robotics_packed_input", False):
            return x.for_bits(self.bits)
        return prepare(x, self.bits)

    def forward_gelu(self, x, up=None, *, approximate="tanh"):
        return self.forward_packed(prepare(x, self.bits, prepare_gelu(x.device, x.dtype, approximate), up))
