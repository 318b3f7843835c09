"""BF16 pointwise fusion around the quantized text-attention projections.

piR2 fuses Qwen3's rotary embedding and RMSNorm with Triton kernels
(coexecution/fused_ops.py, fusion modes "rope", "rmsnorm", "rope_rms",
"all").  `TextAttentionFusion` does the same next to the quantized path: the
grouped q|k|v GEMM runs once, then one sm_100a kernel applies the per-head
q_norm / k_norm, the rotary embedding and the [B, H, T, D] relayout of q, k
and v (replacing three contiguous copies, two torch RMSNorms and two torch
RoPE chains).  With `causal_kernel=True` causal attention runs on
`ops.attention_causal`, which writes the o_proj input rows directly
(replacing torch SDPA and the [B, H, T, D] -> [B, T, H*D] transpose copy);
the default keeps torch SDPA, measured faster at the GR00T shape.  The RoPE arithmetic is bitwise torch's; the per-head mean of
squares is reduced in a different order than torch's (tolerance-level, like
piR2's own fused norms), and so is the attention softmax.
"""

import torch.nn.functional as F

from . import ops


class TextAttentionFusion:
    def __init__(self, model, controller, *, causal_kernel=False):
        self.controller = controller
        self.causal_kernel = causal_kernel
        self.saved = []
        names = {id(m): n for n, m in model.named_modules()}
        self.targets = []
        for module in model.modules():
            if type(module).__name__ != "Qwen3VLTextAttention":
                continue
            if module.head_dim != 128:
                continue
            q_name = names.get(id(module.q_proj))
            self.targets.append((module, q_name))

    def _group(self, bits, q_name):
        for names, group in self.controller.grouped[bits]:
            if names[0] == q_name and len(names) == 3:
                return group
        return None

    def set(self, bits):
        self.close()
        for attn, q_name in self.targets:
            group = self._group(bits, q_name)
            if group is None:
                continue
            self.saved.append((attn, "forward" in attn.__dict__, attn.__dict__.get("forward")))

            def forward(x, cos, sin, attn=attn, group=group):
                b, t = x.shape[0], x.shape[1]
                qkv = group.linear(x)
                q, k, v = ops.qk_norm_rope(
                    qkv.reshape(b * t, qkv.shape[-1]),
                    attn.q_norm.weight,
                    attn.k_norm.weight,
                    cos,
                    sin,
                    tokens=t,
                    hq=attn.heads,
                    hk=attn.kv_heads,
                    eps=attn.q_norm.variance_epsilon,
                )
                if self.causal_kernel:
                    y = ops.attention_causal(q, k, v)
                    return attn.o_proj(y.view(b, t, attn.heads * attn.head_dim))
                y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
                return attn.o_proj(y.transpose(1, 2).reshape(b, t, attn.heads * attn.head_dim))

            attn.forward = forward

    def close(self):
        for module, had, forward in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []


class DiTAttentionFusion:
    """DiT attention on the row attention kernel.

    piR2's `PreparedAttention.attend` (coexecution/groot_pointwise.py:58-92)
    projects q, k and v, views them as [B, H, T, D], runs torch SDPA and
    transposes the result back to [B, T, H*D] for the output projection.
    Here the same projections feed `ops.attention_rows`, which reads the
    projection rows in place (grouped q|k|v output, or the cached context
    k/v) and writes [B*T, H*D] rows; masked calls keep the original forward.
    """

    # Head dimensions the kernel is instantiated for.
    HEAD_DIMS = (32, 48, 64, 96, 128)

    def __init__(self, model, *, cross_only=True):
        self.saved = []
        # At the DiT shapes the kernel wins on cross-attention (17 x 544
        # keys: 6.6 vs 8.4 us for cuDNN SDPA + transpose) and loses slightly
        # on 17 x 17 self-attention (2.9 vs 2.6 us), so by default only
        # cross-attention blocks are routed through it.
        self.targets = [
            m
            for m in model.modules()
            if type(m).__name__ == "Attention"
            and m.head_dim in self.HEAD_DIMS
            and (m.is_cross_attention or not cross_only)
        ]

    @staticmethod
    def _context_rows(kv, b):
        # [B, H, S, D] head views of [B, S, H*D] projection rows.
        s = kv.shape[2]
        return kv.transpose(1, 2).reshape(b * s, kv.shape[1] * kv.shape[3])

    def set(self):
        self.close()
        for attn in self.targets:
            self.saved.append((attn, "forward" in attn.__dict__, attn.__dict__.get("forward")))
            original = type(attn).forward

            def forward(x, encoder_hidden_states=None, attention_mask=None, attn=attn, original=original):
                if attention_mask is not None:
                    return original(attn, x, encoder_hidden_states, attention_mask)
                b, t = x.shape[0], x.shape[1]
                width = attn.heads * attn.head_dim
                q = attn.to_q(x)
                if attn.is_cross_attention and attn.kv_cache is not None:
                    k, v = (self._context_rows(z, b) for z in attn.kv_cache)
                else:
                    context = x if encoder_hidden_states is None else encoder_hidden_states
                    k, v = attn.to_k(context), attn.to_v(context)
                    k, v = k.reshape(-1, width), v.reshape(-1, width)
                y = ops.attention_rows(
                    q.reshape(b * t, width), k, v, batch=b, heads=attn.heads, head_dim=attn.head_dim
                )
                return attn.to_out[1](attn.to_out[0](y.view(b, t, width)))

            attn.forward = forward

    def close(self):
        for module, had, forward in self.saved:
            if had:
                module.forward = forward
            elif "forward" in module.__dict__:
                del module.forward
        self.saved = []
