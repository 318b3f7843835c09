"""GR00T DiT connections to the packed producers.

Provides piR2's `AdditionalConnections` and `packed_input`
(coexecution/optimization/groot/integer_connections.py:21-226: the same
constructor, `set(mode, expanded=, fuse=, norm_quant=, residual_quant=)`
options, validation messages and `close()`), built on this package's
`ForwardPatches` ledger.  What `set` installs:

* fixed-category projections (`W[category]`, `b[category]` of a
  category-indexed module) become a quantized Linear, guarded on every call
  to batch 1 and the one category id they were built for;
* AdaLN `norm1` modules whose attention inputs are all quantized return
  packed activations straight from the fused modulation producer (or, with
  `norm_quant`, the LayerNorm + modulation producer);
* with `residual_quant`, a block's ungated attention residual, `norm3` and
  the FFN input pack run as the residual + LayerNorm + modulation producer
  with a unit gate and zero modulation.
"""

import torch

from .linear import PreparedLinear
from .modulation import (
    PackedActivations,
    prepare_modulation,
    prepare_norm_modulation,
    prepare_residual_norm_modulation,
)
from .transformer import ForwardPatches

__all__ = ["AdditionalConnections", "packed_input"]

_MODE_BITS = {"w8a8": 8, "w4a4": 4}


def packed_input(packed, shape):
    """A packed activation that looks like the bf16 tensor it replaces: the
    attention reads the batch size from `.shape` before the q projection."""
    result = PackedActivations({packed.bits: packed}).with_leading_shape(shape[:-1])
    result.shape = shape
    return result


def _attention_inputs(block):
    return ("to_q",) if block.attn1.is_cross_attention else ("to_q", "to_k", "to_v")


def _category_linear(name, module, category):
    """The category's slice of a category-indexed projection as a bf16
    Linear (weight W[category]^T, bias b[category])."""
    W, b = module.W, module.b
    if W.ndim != 3 or b.shape != (W.shape[0], W.shape[2]) or not isinstance(category, int) or not 0 <= category < W.shape[0]:
        raise ValueError(f"Invalid fixed category projection: {name}")
    linear = torch.nn.Linear(W.shape[1], W.shape[2], device="meta", dtype=torch.bfloat16)
    linear.weight = torch.nn.Parameter(W[category].t().contiguous(), requires_grad=False)
    linear.bias = torch.nn.Parameter(b[category], requires_grad=False)
    return linear


def _category_forward(controller, q, category):
    def forward(x, cat_ids):
        # One explicit batch-1 embodiment: checked on every call.
        if x.shape[0] != 1 or cat_ids.numel() != 1 or cat_ids.dtype not in (torch.int32, torch.int64):
            raise ValueError("Fixed category quantization requires B1 and one integer category ID")
        torch._assert_async(cat_ids.reshape(-1)[0] == category, f"Fixed category quantization requires category {category}")
        return controller.dispatch(q, x)

    return forward


def _norm_forward(norm, bits, with_layernorm):
    """AdaLN norm1 -> packed input.  Without `with_layernorm` the module's
    own LayerNorm runs first and the producer only modulates and packs."""
    producer = prepare_norm_modulation if with_layernorm else prepare_modulation
    options = {"eps": norm.norm.eps} if with_layernorm else {}

    def forward(x, temb=None):
        scale, shift = norm.linear(norm.silu(temb)).chunk(2, dim=-1)
        values = x if with_layernorm else norm.norm(x)
        if scale.ndim == 3:
            # Per-token modulation: one modulation row per token.
            width = x.shape[-1]
            rows = lambda t: t.reshape(-1, 1, width)  # noqa: E731
            packed = producer(rows(values), rows(scale), rows(shift), bits, **options)
        else:
            packed = producer(values, scale[:, None], shift[:, None], bits, **options)
        return packed_input(packed, x.shape)

    return forward


def _residual_block_forward(block, bits):
    """x + ff(pack(LN(x + attn(norm1(x))))) with the residual add, norm3 and
    pack as one producer (unit gate, zero modulation)."""
    weight = block.ff.net[0].proj.weight
    zero = torch.zeros((1, 1, block.dim), device=weight.device, dtype=weight.dtype)
    one = torch.ones_like(zero)

    def forward(hidden_states, attention_mask=None, encoder_hidden_states=None, encoder_attention_mask=None, temb=None):
        x = hidden_states
        normalized = block.norm1(x, temb) if block.norm_type == "ada_norm" else block.norm1(x)
        mask = encoder_attention_mask if encoder_hidden_states is not None else attention_mask
        attention = block.attn1(normalized, encoder_hidden_states=encoder_hidden_states, attention_mask=mask)
        rows = (x.shape[0], 1, x.shape[-1])
        residual, packed = prepare_residual_norm_modulation(
            x, attention.contiguous(), one.expand(rows), zero.expand(rows), zero.expand(rows), bits, eps=block.norm3.eps
        )
        return residual + block.ff(packed_input(packed, x.shape))

    return forward


def _is_plain_layernorm(norm):
    return isinstance(norm, torch.nn.LayerNorm) and not norm.elementwise_affine


class AdditionalConnections:
    def __init__(self, policy, controller, categories):
        self.controller = controller
        self.categories = categories
        self.all_blocks = policy.model.action_head.model.transformer_blocks
        if controller is None:
            self.norms = [block.norm1 for block in self.all_blocks]
        else:
            quantized = {id(module) for module, _, _ in controller.sites.values()}
            self.norms = [
                block.norm1
                for block in self.all_blocks
                if all(id(getattr(block.attn1, name)) in quantized for name in _attention_inputs(block))
            ]
        self.blocks = []
        self.linears = {name: _category_linear(name, module, category) for name, (module, category) in categories.items()}
        self.quant = {
            bits: {
                name: PreparedLinear.from_linear(linear, bits=bits, pack_reuse=True, biasless_epilogue=True)
                for name, linear in self.linears.items()
            }
            for bits in (8, 4)
        }
        self._patches = ForwardPatches()

    def _residual_targets(self):
        quantized = {id(module) for module, _, _ in self.controller.sites.values()}
        return [block for block in self.all_blocks if id(block.ff.net[0].proj) in quantized]

    def _validate(self, mode, fuse, norm_quant, residual_quant):
        if (norm_quant or residual_quant) and (not fuse or mode == "bf16"):
            raise ValueError("Norm quantization fusion requires fusion and integer precision")
        if residual_quant and not norm_quant:
            raise ValueError("Residual fusion requires norm quantization fusion")
        if mode == "bf16":
            return []
        blocks = self._residual_targets() if residual_quant else []
        if norm_quant:
            if not self.norms:
                raise ValueError("Norm fusion selected no fully quantized attention input")
            layer_norms = [n.norm for n in self.norms] + [b.norm3 for b in blocks]
            if not all(_is_plain_layernorm(n) for n in layer_norms):
                raise ValueError("Norm fusion requires non-affine LayerNorm")
        if residual_quant and (not blocks or any(getattr(b, "pos_embed", None) is not None for b in blocks)):
            raise ValueError("Residual fusion requires quantized FFN inputs without position embeddings")
        return blocks

    def set(self, mode, *, expanded=True, fuse=True, norm_quant=False, residual_quant=False):
        self.close()
        blocks = self._validate(mode, fuse, norm_quant, residual_quant)
        if mode == "bf16":
            return
        bits = _MODE_BITS[mode]
        if expanded:
            for name, (module, category) in self.categories.items():
                self._patches.replace(module, "forward", _category_forward(self.controller, self.quant[bits][name], category))
        if fuse:
            for norm in self.norms:
                self._patches.replace(norm, "forward", _norm_forward(norm, bits, norm_quant))
        self.blocks = blocks
        for block in blocks:
            self._patches.replace(block, "forward", _residual_block_forward(block, bits))

    def close(self):
        self._patches.restore()
        self.blocks = []
