"""Residual-add fusion for the GR00T decoder layers and DiT blocks.

piR2 runs the residual epilogue as an operator candidate (residual writer of
coexecution/kernels/ampere_ada/epilogue.py) and fuses the DiT attention
residual with norm3 + pack (AdditionalConnections residual_quant).  This
installer applies the residual epilogue where the residual stream meets a
quantized projection, keeping the model's own forward code:

* `Qwen3VLTextDecoderLayer`: h + o_proj(...) and h + down_proj(...) become
  o_proj / down_proj GEMMs whose epilogue adds h;
* DiT `BasicTransformerBlock`: x + to_out(...) and x + ff(...) likewise, and
  norm3 (non-affine LayerNorm) + pack of the FFN input becomes the fused
  LayerNorm producer (zero AdaLN modulation, which leaves the normalized
  bf16 values unchanged, as piR2's residual fusion does);
* with `ffn_kernel=True` (W8A8, <= 32 tokens) the FFN (up GEMM, GELU,
  pack, down GEMM, residual) runs as one launch (`ops.dit_ffn`, bitwise the
  same values);
* otherwise the FFN's GELU moves from the down projection's pack (piR2's
  `forward_gelu`, a LUT applied while packing) into the up projection's GEMM
  epilogue (the same torch-built LUT applied to its bf16 output), so the down
  projection packs plain values: the codes are identical, and the LUT
  gathers run once per output element inside a kernel that is already
  running; the up GEMM also writes the per-16-channel maxima of its output,
  from which the down projection's pack takes its row scales
  (`ops.quant_rows_max`: no second reduction over the 6144-wide rows, the
  same codes);
* with the fused pack enabled (`integer.FUSED_PACK_ROWS`, off by default)
  and few W8A8 rows, the up GEMM also writes the per-16-channel maxima of
  its output and the down GEMM packs that output inside itself from them
  (`IntegerLinear.forward_rows`): one launch fewer, the same codes.

Results are bitwise those of the unfused quantized model: the epilogue adds
the residual to the bf16 GEMM output in fp32 and rounds once, exactly as
torch's bf16 addition does.
"""

import torch

from . import integer, ops
from .connections import packed_input
from .fused import prepare_gelu, prepare_silu
from .linear import prepare
from .modulation import prepare_norm_modulation

# The down projections' packs (DiT FFN, text MLP) take their row maxima
# from the producing GEMM's epilogue (per-16-channel maxima of gelu(up(x))
# or of silu(gate) * up) instead of reducing the 6144-wide rows again
# (`ops.quant_rows_max`, the same bytes), for at most PACK_FROM_GEMM_MAX_ROWS
# rows: every CTA of a row re-reads the row's maxima (384 floats for 6144
# columns), which costs more than the row reduction it saves at batched
# sizes (34816 rows: ~320 MB of extra reads).
PACK_FROM_GEMM_MAX = True
PACK_FROM_GEMM_MAX_ROWS = 2048


class ResidualFusion:
    def __init__(self, model, controller, *, ffn_kernel=False):
        self.controller = controller
        self.ffn_kernel = ffn_kernel
        self.saved = []
        self.layers, self.blocks = [], []
        for name, module in model.named_modules():
            kind = type(module).__name__
            if kind == "Qwen3VLTextDecoderLayer" and self._quantized(module.self_attn.o_proj, module.mlp.down_proj):
                self.layers.append(module)
            elif kind == "BasicTransformerBlock" and self._quantized(module.attn1.to_out[0], module.ff.net[2]):
                self.blocks.append(module)

    def _quantized(self, *modules):
        sites = {id(m): n for n, (m, _, _) in self.controller.sites.items()}
        return all(id(m) in sites for m in modules)

    @staticmethod
    def _ffn_fits(up_q, down_q):
        d, f = up_q.in_features, up_q.out_features
        if d % 128 or f % 1024 or down_q.in_features != f or down_q.out_features != d:
            return False
        device = up_q.packed_weight.device
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        return f // 128 + 8 * (d // 128) <= sms and up_q.packed_weight.shape == (f, d)

    def _q(self, module, bits):
        sites = {id(m): n for n, (m, _, _) in self.controller.sites.items()}
        return self.controller.quant[bits][sites[id(module)]]

    def set(self, bits, *, norm_pack=True):
        self.close()
        for layer in self.layers:
            self.saved.append((layer, "forward" in layer.__dict__, layer.__dict__.get("forward")))
            o_q, down_q = self._q(layer.self_attn.o_proj, bits), self._q(layer.mlp.down_proj, bits)

            def forward(h, cos, sin, layer=layer, o_q=o_q, down_q=down_q):
                o_q.pending_residual(h)
                h = layer.self_attn(layer.input_layernorm(h), cos, sin)
                down_q.pending_residual(h)
                return layer.mlp(layer.post_attention_layernorm(h))

            layer.forward = forward
        for block in self.blocks:
            self.saved.append((block, "forward" in block.__dict__, block.__dict__.get("forward")))
            out_q, down_q = self._q(block.attn1.to_out[0], bits), self._q(block.ff.net[2], bits)
            zero = torch.zeros((1, 1, block.dim), device=block.ff.net[2].weight.device, dtype=torch.bfloat16)
            fuse_norm = (
                norm_pack
                and isinstance(block.norm3, torch.nn.LayerNorm)
                and not block.norm3.elementwise_affine
                and self._quantized(block.ff.net[0].proj)
            )
            act = block.ff.net[0]
            gelu_epilogue = (
                type(act).__name__ == "GELU"
                and self._quantized(act.proj)
                and len(block.ff.net) == 3
                and isinstance(block.ff.net[1], torch.nn.Dropout)
            )
            up_q = self._q(act.proj, bits) if gelu_epilogue else None
            lut = prepare_gelu(down_q.packed_weight.device, torch.bfloat16, act.approximate) if gelu_epilogue else None
            # The one-launch FFN (`ops.dit_ffn`, up + GELU + pack + down +
            # residual) is exact but measured slower inside the step (3.34 vs
            # 3.06 ms for the action head: its epilogue phases run on one
            # CTA's 128 threads per channel tile), so it is only installed
            # when asked for.
            ffn_kernel = self.ffn_kernel and gelu_epilogue and bits == 8 and self._ffn_fits(up_q, down_q)

            def forward(
                hidden_states,
                attention_mask=None,
                encoder_hidden_states=None,
                encoder_attention_mask=None,
                temb=None,
                block=block,
                out_q=out_q,
                down_q=down_q,
                zero=zero,
                fuse_norm=fuse_norm,
                bits=bits,
                up_q=up_q,
                lut=lut,
                ffn_kernel=ffn_kernel,
            ):
                x = hidden_states
                normalized = block.norm1(x, temb) if block.norm_type == "ada_norm" else block.norm1(x)
                out_q.pending_residual(x)
                x = block.attn1(
                    normalized,
                    encoder_hidden_states=encoder_hidden_states,
                    attention_mask=encoder_attention_mask if encoder_hidden_states is not None else attention_mask,
                )
                if fuse_norm:
                    shape = (x.shape[0], 1, x.shape[-1])
                    packed = prepare_norm_modulation(
                        x, zero.expand(shape), zero.expand(shape), bits, eps=block.norm3.eps
                    )
                    ff_in = packed_input(packed, x.shape)
                else:
                    ff_in = block.norm3(x)
                down_q.pending_residual(x)
                if up_q is None:
                    return block.ff(ff_in)
                packed = ff_in.for_bits(bits) if getattr(ff_in, "_robotics_packed_input", False) else prepare(ff_in, bits)
                if ffn_kernel and packed.data.shape[0] <= 32:
                    residual = down_q.__dict__.pop("_pending_residual")
                    out = ops.dit_ffn(packed.data, packed.scales, up_q, down_q, lut, residual)
                    return out.reshape(x.shape)
                if (
                    bits == 8
                    and integer.FUSED_PACK_ROWS > 0
                    and self.controller.candidates is None
                    and up_q.packed_weight.shape[0] % 16 == 0
                ):
                    maxes = torch.empty(
                        (packed.data.shape[0], up_q.packed_weight.shape[0] // 16),
                        device=packed.data.device, dtype=torch.float32,
                    )
                    hidden = up_q.forward_packed(packed, out_lut=lut, max_out=maxes)
                    if down_q.fused_pack_ok(hidden, with_max=True):
                        # The down projection packs gelu(up(x)) inside its
                        # GEMM from the up GEMM's per-16-channel maxima.
                        return down_q.forward_rows(hidden, x_max=maxes)
                    return self.controller.dispatch(down_q, hidden)
                if (
                    PACK_FROM_GEMM_MAX
                    and self.controller.candidates is None
                    and up_q.packed_weight.shape[0] % 16 == 0
                    and packed.data.shape[0] <= PACK_FROM_GEMM_MAX_ROWS
                ):
                    rows = packed.data.shape[0]
                    maxes = torch.empty(
                        (rows, up_q.packed_weight.shape[0] // 16), device=packed.data.device, dtype=torch.float32
                    )
                    hidden = up_q.forward_packed(packed, out_lut=lut, max_out=maxes)
                    k = hidden.shape[-1]
                    data, scales = ops.quant_rows_max(hidden.reshape(rows, k), maxes, bits)
                    return down_q.forward_packed(
                        integer.PackedActivation(data, scales, tuple(hidden.shape[:-1]), k, bits)
                    )
                hidden = up_q.forward_packed(packed, out_lut=lut)      # gelu(up(x)), bf16
                return self.controller.dispatch(down_q, hidden)

            block.forward = forward

    def close(self):
        for module, had, forward in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []


class SwiGLUFusion:
    """gate|up GEMM with the SwiGLU epilogue for the Qwen3 text MLPs (W8A8).

    TransformerINT runs a text MLP as one gate|up group GEMM followed by the
    down projection's gated pack bf16(SiLU(gate) * up) (piR2's
    coexecution/optimization/groot/integer.py:166-172).  Here the gate|up
    GEMM itself writes bf16(SiLU(gate) * up) (the same torch-built SiLU
    table, the same rounding), half as many output bytes, and the down
    projection packs it plainly: activation codes, and so the results, are
    bitwise those of the unfused path.  The group's weights, scales and bias
    are copied once into the kernel's interleaved layout (128-channel gate
    and up blocks side by side).
    """

    def __init__(self, model, controller):
        self.controller = controller
        self.saved = []
        self.sites = []
        names = {id(m): n for n, (m, _, _) in controller.sites.items()}
        groups = {tuple(n): g for n, g in controller.grouped[8]}
        for mlp, down in controller.text:
            key = (names.get(id(mlp.gate_proj)), names.get(id(mlp.up_proj)))
            group = groups.get(key)
            if group is None or group.sizes[0] != group.sizes[1] or group.sizes[0] % 128:
                continue
            half = group.sizes[0]
            linear = group.linear
            weight = ops.interleave_gate_up(linear.packed_weight[: 2 * half], half)
            scale = ops.interleave_gate_up(linear.weight_scale[: 2 * half], half)
            bias = None if linear.bias is None else ops.interleave_gate_up(linear.bias[: 2 * half], half)
            self.sites.append((mlp, controller.quant[8][down], half, weight, scale, bias, linear._bias_mode()))
        device = next(model.parameters()).device
        self.silu = prepare_silu(device)

    def set(self):
        self.close()
        for mlp, down_q, half, weight, scale, bias, bias_mode in self.sites:
            self.saved.append((mlp, "forward" in mlp.__dict__, mlp.__dict__.get("forward")))

            def forward(x, down_q=down_q, half=half, weight=weight, scale=scale, bias=bias, bias_mode=bias_mode):
                packed = x.for_bits(8) if getattr(x, "_robotics_packed_input", False) else prepare(x, 8)
                if (
                    PACK_FROM_GEMM_MAX
                    and self.controller.candidates is None
                    and packed.data.shape[0] <= PACK_FROM_GEMM_MAX_ROWS
                ):
                    # The down projection's pack from the SwiGLU epilogue's
                    # per-16-column maxima (the same codes as packing h).
                    rows = packed.data.shape[0]
                    maxes = torch.empty((rows, half // 16), device=packed.data.device, dtype=torch.float32)
                    hidden = ops.gemm_swiglu(
                        packed.data, packed.scales, weight, scale, bias, self.silu, half_n=half,
                        bias_mode=bias_mode, max_out=maxes,
                    )
                    data, scales = ops.quant_rows_max(hidden, maxes, 8)
                    return down_q.forward_packed(integer.PackedActivation(data, scales, tuple(packed.shape), half, 8))
                hidden = ops.gemm_swiglu(
                    packed.data, packed.scales, weight, scale, bias, self.silu, half_n=half, bias_mode=bias_mode
                )
                return self.controller.dispatch(down_q, hidden.reshape(*packed.shape, half))

            mlp.forward = forward

    def close(self):
        for module, had, forward in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []
