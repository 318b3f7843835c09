"""Reversible installation of integer projections into a GR00T-shaped model.

Provides the plugin surface of piR2's `TransformerINT`
(coexecution/optimization/groot/integer.py:16-175): the constructor
arguments, `set("bf16" | "w8a8" | "w4a4")`, `close()`, `dispatch(q, x, lut,
up)`, `install_candidates`, `clear_projection_cache`, and the `sites`,
`groups`, `activations`, `text`, `quant[bits][name]` and `grouped[bits]`
tables the other installers read.  How it does so is this package's own:

* `ForwardPatches` is a ledger of replaced instance attributes: the first
  replacement of an (object, attribute) pair records whether the instance
  had its own value, and `restore()` puts every pair back exactly;
* the projections of both precisions are built once (`_site_linears`),
  from the bf16 weights or from a packed-weight cache, and sibling groups
  (q|k|v, k|v, gate|up, the DiT condition group) share one concatenated
  GEMM (`IntegerProjectionGroup`);
* what a precision changes in the model is a list of patches
  (`_mode_patches`): site forwards, group members reading their slice of
  the shared output, GELU modules that become identities while their down
  projection packs through the GELU table, and text MLPs that pack
  bf16(SiLU(gate) * up) straight into the down projection.  `set` undoes
  the previous list and applies the new one.
"""

from .fused import prepare_gelu, prepare_silu
from .integer import IntegerProjectionGroup
from .linear import PreparedLinear, prepare
from .projections import inventory

_MODE_BITS = {"w8a8": 8, "w4a4": 4}


class ForwardPatches:
    """Ledger of instance attributes replaced on model objects."""

    def __init__(self):
        self._first = {}

    def replace(self, obj, attr, value):
        key = (id(obj), attr)
        if key not in self._first:
            own = obj.__dict__
            self._first[key] = (obj, attr, attr in own, own.get(attr))
        setattr(obj, attr, value)

    def restore(self):
        for obj, attr, had_own, value in self._first.values():
            if had_own:
                setattr(obj, attr, value)
            else:
                obj.__dict__.pop(attr, None)
        self._first.clear()


def _is_packed(x):
    return getattr(x, "_robotics_packed_input", False)


def _condition_group(model):
    """Every DiT block's AdaLN projection and the output modulation read the
    same activated condition, so they form one GEMM."""
    dit = model.action_head.model
    names = {id(module): name for name, module in model.named_modules()}
    return [names[id(block.norm1.linear)] for block in dit.transformer_blocks] + [names[id(dit.proj_out_1)]]


def _site_linears(sites, bits, packed):
    """{name: PreparedLinear} for one precision: quantized from the module's
    weights, or rebuilt from `packed` ({name: {bits: (weight, scale,
    bias)}}, see weight_cache.load) without quantizing again."""
    table = {}
    for name, (module, _, _) in sites.items():
        if packed is None:
            table[name] = PreparedLinear.from_linear(module, bits=bits, pack_reuse=True, biasless_epilogue=True)
        else:
            weight, scale, bias = packed[name][bits]
            table[name] = PreparedLinear(
                weight, scale, bias, module.in_features, module.out_features, bits, 0, True, True
            )
    return table


class TransformerINT:
    def __init__(self, model, executed, native=False, expanded=False, condition_group=False, packed=None):
        sites, groups, activations, text = inventory(model, expanded)
        if condition_group:
            groups = [*groups, _condition_group(model)]
        self.sites = {name: site for name, site in sites.items() if name in executed}
        self.groups = [names for names in groups if set(names) <= self.sites.keys()]
        self.activations = [entry for entry in activations if entry[2] in self.sites]
        self.text = [(mlp, down) for mlp, down in text if down in self.sites]
        self.quant = {bits: _site_linears(self.sites, bits, packed) for bits in (8, 4)}
        self.grouped = {bits: [(names, self._group(names, bits)) for names in self.groups] for bits in (8, 4)}
        self.silu_lut = prepare_silu(next(model.parameters()).device)
        self.native = native
        self.candidates = None
        self.mode = "bf16"
        self._patches = ForwardPatches()
        if native:
            self._route_through_dispatch()

    # ------------------------------------------------------------ building
    def _group(self, names, bits):
        _, role, component = self.sites[names[0]]
        # The text q/k RMSNorm reads contiguous rows; every other consumer
        # takes row-strided views of the shared output.
        group = IntegerProjectionGroup(
            [self.quant[bits][name] for name in names],
            contiguous_outputs=(role, component) == ("AttnQ", "text"),
        )
        group.linear.pack_input = lambda x, bits=bits: x.for_bits(bits) if _is_packed(x) else prepare(x, bits)
        return group

    def _all_linears(self, bits):
        return [*self.quant[bits].values(), *(group.linear for _, group in self.grouped[bits])]

    def _route_through_dispatch(self):
        """Every projection's forward and forward_gelu go through dispatch()
        (candidate override, packed input, fused pack, pack + GEMM)."""
        for bits in (8, 4):
            for q in self._all_linears(bits):
                q.forward = lambda x, q=q: self.dispatch(q, x)
                q.forward_gelu = lambda x, up=None, approximate="tanh", q=q: self.dispatch(
                    q, x, prepare_gelu(x.device, x.dtype, approximate), up
                )

    def _mode_patches(self, bits):
        linears = self.quant[bits]
        for name, (module, _, _) in self.sites.items():
            yield module, "forward", linears[name].forward
        for names, group in self.grouped[bits]:
            for index, name in enumerate(names):
                yield self.sites[name][0], "forward", lambda x, group=group, index=index: group.project(x, index)
        for module, attr, down, approximate in self.activations:
            yield module, attr, lambda x: x
            yield self.sites[down][0], "forward", lambda x, q=linears[down], a=approximate: q.forward_gelu(
                x, approximate=a
            )
        for mlp, down in self.text:
            yield mlp, "forward", lambda x, mlp=mlp, q=linears[down]: self.dispatch(
                q, mlp.gate_proj(x), self.silu_lut, mlp.up_proj(x)
            )

    # ------------------------------------------------------------ calls
    def dispatch(self, q, x, lut=None, up=None):
        """One quantized projection call: a candidate kernel if one claims
        it, else the packed input as given, else (plain rows, few W8A8
        tokens) the pack fused into the GEMM, else pack then GEMM."""
        if self.candidates is not None:
            result = self.candidates.dispatch(q, x, lut, up)
            if result is not None:
                return result
        if _is_packed(x):
            return q.forward_packed(x.for_bits(q.bits))
        if lut is None and up is None and q.fused_pack_ok(x):
            return q.forward_rows(x)
        return q.forward_packed(prepare(x, q.bits, lut, up))

    def _pack_dispatch_input(self, q, x, lut=None, up=None):
        if self.candidates is not None:
            return self.candidates.pack_input(q, x, lut, up)
        return x.for_bits(q.bits) if _is_packed(x) else prepare(x, q.bits, lut, up)

    def install_candidates(self, candidates):
        self.candidates = candidates
        if candidates.implementation != "reference":
            self._route_through_dispatch()

    def clear_projection_cache(self):
        for grouped in self.grouped.values():
            for _, group in grouped:
                group.forget()

    # ------------------------------------------------------------ modes
    def set(self, mode):
        self.clear_projection_cache()
        self._patches.restore()
        self.mode = mode
        if mode == "bf16":
            return
        for obj, attr, value in self._mode_patches(_MODE_BITS[mode]):
            self._patches.replace(obj, attr, value)

    def close(self):
        self.set("bf16")
