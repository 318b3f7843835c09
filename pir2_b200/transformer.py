"""Reversible installation of integer projections into a GR00T-shaped model.

Mirrors `TransformerINT` (coexecution/optimization/groot/integer.py:16-175):
every executed site gets 8- and 4-bit `PreparedLinear`s built once; sibling
groups (q|k|v, k|v, gate|up) share one concatenated GEMM; GELU activations
become identity with the GELU fused into the down-projection's pack; text
MLPs pack bf16(SiLU(gate) * up) straight into the down projection.
`set("bf16" | "w8a8" | "w4a4")` swaps instance `forward`s; `close()`
restores the model exactly.
"""

from .fused import prepare_gelu, prepare_silu
from .integer import IntegerProjectionGroup
from .linear import PreparedLinear, prepare
from .projections import inventory


class TransformerINT:
    def __init__(self, model, executed, native=False, expanded=False, condition_group=False, packed=None):
        sites, groups, activations, text = inventory(model, expanded)
        if condition_group:
            dit = model.action_head.model
            names = {id(module): name for name, module in model.named_modules()}
            # Every block's AdaLN projection and the output modulation consume
            # the same activated condition: one group, one GEMM.
            groups.append(
                [names[id(block.norm1.linear)] for block in dit.transformer_blocks] + [names[id(dit.proj_out_1)]]
            )
        self.sites = {n: s for n, s in sites.items() if n in executed}
        self.groups = [g for g in groups if all(n in self.sites for n in g)]
        self.activations = [a for a in activations if a[2] in self.sites]
        self.text = [(m, n) for m, n in text if n in self.sites]
        # `packed` ({site: {bits: (packed_weight, weight_scale, bias)}}, from
        # weight_cache.load) skips install-time quantization.
        self.quant = {
            bits: {
                n: (
                    PreparedLinear(*packed[n][bits], m.in_features, m.out_features, bits, 0, True, True)
                    if packed is not None
                    else PreparedLinear.from_linear(m, bits=bits, pack_reuse=True, biasless_epilogue=True)
                )
                for n, (m, _, _) in self.sites.items()
            }
            for bits in (8, 4)
        }
        entries = [(m, "forward") for m, _, _ in self.sites.values()]
        entries += [(m, attr) for m, attr, _, _ in self.activations]
        entries += [(m, "forward") for m, _ in self.text]
        self.saved = [(m, a, a in m.__dict__, getattr(m, a)) for m, a in entries]
        device = next(model.parameters()).device
        self.silu_lut = prepare_silu(device)
        self.grouped = {bits: [] for bits in (8, 4)}
        for bits in (8, 4):
            for names in self.groups:
                # Text Q/K RMSNorm needs contiguous inputs; other consumers
                # accept row-strided views of the grouped output.
                contiguous = self.sites[names[0]][1] == "AttnQ" and self.sites[names[0]][2] == "text"
                group = IntegerProjectionGroup([self.quant[bits][n] for n in names], contiguous_outputs=contiguous)
                group.linear.pack_input = lambda x, bits=bits: (
                    x.for_bits(bits) if getattr(x, "_robotics_packed_input", False) else prepare(x, bits)
                )
                self.grouped[bits].append((names, group))
        self.native = native
        self.candidates = None
        if native:
            for bits in (8, 4):
                for q in list(self.quant[bits].values()) + [g.linear for _, g in self.grouped[bits]]:
                    q.forward = lambda x, q=q: self.dispatch(q, x)
                    q.forward_gelu = lambda x, up=None, approximate="tanh", q=q: self.dispatch(
                        q, x, prepare_gelu(x.device, x.dtype, approximate), up
                    )
        self.mode = "bf16"

    def dispatch(self, q, x, lut=None, up=None):
        """Candidate override, then packed input, then pack + GEMM."""
        if self.candidates is not None:
            result = self.candidates.dispatch(q, x, lut, up)
            if result is not None:
                return result
        if getattr(x, "_robotics_packed_input", False):
            return q.forward_packed(x.for_bits(q.bits))
        if lut is None and up is None and q.fused_pack_ok(x):
            # Few W8A8 rows: the plain pack runs inside the GEMM.
            return q.forward_rows(x)
        return q.forward_packed(prepare(x, q.bits, lut, up))

    def _pack_dispatch_input(self, q, x, lut=None, up=None):
        if self.candidates is not None:
            return self.candidates.pack_input(q, x, lut, up)
        if getattr(x, "_robotics_packed_input", False):
            return x.for_bits(q.bits)
        return prepare(x, q.bits, lut, up)

    def install_candidates(self, candidates):
        self.candidates = candidates
        if candidates.implementation == "reference":
            return
        for bits in (8, 4):
            for q in list(self.quant[bits].values()) + [g.linear for _, g in self.grouped[bits]]:
                q.forward = lambda x, q=q: self.dispatch(q, x)
                q.forward_gelu = lambda x, up=None, approximate="tanh", q=q: self.dispatch(
                    q, x, prepare_gelu(x.device, x.dtype, approximate), up
                )

    def clear_projection_cache(self):
        for groups in self.grouped.values():
            for _, group in groups:
                group._input = group._output = None
                group._remaining.clear()

    def set(self, mode):
        self.clear_projection_cache()
        for m, attr, had, original in self.saved:
            if had:
                setattr(m, attr, original)
            elif attr in m.__dict__:
                delattr(m, attr)
        self.mode = mode
        if mode == "bf16":
            return
        bits = {"w8a8": 8, "w4a4": 4}[mode]
        linears = self.quant[bits]
        for name, (m, _, _) in self.sites.items():
            m.forward = linears[name].forward
        for names, group in self.grouped[bits]:
            for i, name in enumerate(names):
                self.sites[name][0].forward = lambda x, g=group, i=i: g.project(x, i)
        for activation, attr, down, approximate in self.activations:
            setattr(activation, attr, lambda x: x)
            self.sites[down][0].forward = lambda x, q=linears[down], a=approximate: q.forward_gelu(x, approximate=a)
        for mlp, down in self.text:

            def forward(x, m=mlp, q=linears[down]):
                gate, up = m.gate_proj(x), m.up_proj(x)
                return self.dispatch(q, gate, self.silu_lut, up)

            mlp.forward = forward

    def close(self):
        self.set("bf16")
