"""GR00T-shaped synthetic model used by the benchmark and the tests.

The GR00T model code is upstream of piR2 and absent here, so this module
builds, in plain torch with random-init bf16 weights, the shapes piR2's
quantized Linear path runs on, with the module class names its inventory
recognises (coexecution/optimization/groot/projections.py:6-72):

* a Qwen3-1.7B-shaped text decoder truncated to 16 layers
  (`Qwen3VLTextDecoderLayer` with `Qwen3VLTextAttention`: GQA 16 q / 8 kv
  heads of 128, per-head q/k RMSNorm, RoPE theta 1e6, causal SDPA;
  `Qwen3VLTextMLP`: SwiGLU 6144; RMSNorm eps 1e-6), fed 2 x 256 visual
  embeddings plus 32 text tokens (vocab 151936) and returning the layer-16
  features [B, 544, 2048];
* a flow-matching DiT action head (`BasicTransformerBlock` x 16, hidden 1536
  = 32 heads x 48, AdaLN timestep conditioning with non-affine LayerNorm,
  even blocks cross-attend to the VLM features, GELU(tanh) FFN 6144,
  1 state token (dim 64) + 16 action tokens (dim 32)), integrated with 4
  Euler steps from N(0, 1) actions.  Cross-attention K/V of the context are
  computed once per control step and reused by the 4 steps, as piR2's action
  K/V reuse does (coexecution/optimization/groot/kv_reuse.py:1-10).

Nothing here is the quantized path itself: TransformerINT swaps the Linear
layers of this model for the B200 kernels.
"""

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class VLMConfig:
    hidden: int = 2048
    layers: int = 16
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 6144
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    visual_tokens: int = 512
    text_tokens: int = 32
    hidden_act: str = "silu"


@dataclass
class DiTConfig:
    hidden: int = 1536
    layers: int = 16
    heads: int = 32
    head_dim: int = 48
    ff: int = 6144
    context: int = 2048
    state_dim: int = 64
    action_dim: int = 32
    action_horizon: int = 16
    steps: int = 4
    timestep_channels: int = 256
    eps: float = 1e-5


def _linear(i, o, bias, std=0.02):
    layer = nn.Linear(i, o, bias=bias)
    with torch.no_grad():
        layer.weight.normal_(0.0, std)
        if bias:
            layer.bias.normal_(0.0, 0.01)
    return layer


# ------------------------------------------------------------------ VLM
class Qwen3VLTextRMSNorm(nn.Module):
    def __init__(self, width, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.variance_epsilon = eps

    def forward(self, x):
        dtype = x.dtype
        h = x.float()
        variance = h.pow(2).mean(-1, keepdim=True)
        h = h * torch.rsqrt(variance + self.variance_epsilon)
        return self.weight * h.to(dtype)


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class Qwen3VLTextAttention(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.heads, self.kv_heads, self.head_dim = c.heads, c.kv_heads, c.head_dim
        self.q_proj = _linear(c.hidden, c.heads * c.head_dim, False)
        self.k_proj = _linear(c.hidden, c.kv_heads * c.head_dim, False)
        self.v_proj = _linear(c.hidden, c.kv_heads * c.head_dim, False)
        self.o_proj = _linear(c.heads * c.head_dim, c.hidden, False)
        self.q_norm = Qwen3VLTextRMSNorm(c.head_dim, c.eps)
        self.k_norm = Qwen3VLTextRMSNorm(c.head_dim, c.eps)

    def forward(self, x, cos, sin):
        b, t = x.shape[0], x.shape[1]
        q = self.q_norm(self.q_proj(x).view(b, t, self.heads, self.head_dim)).transpose(1, 2)
        k = self.k_norm(self.k_proj(x).view(b, t, self.kv_heads, self.head_dim)).transpose(1, 2)
        v = self.v_proj(x).view(b, t, self.kv_heads, self.head_dim).transpose(1, 2)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        return self.o_proj(y.transpose(1, 2).reshape(b, t, self.heads * self.head_dim))


class Qwen3VLTextMLP(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.config = SimpleNamespace(hidden_act=c.hidden_act)
        self.gate_proj = _linear(c.hidden, c.intermediate, False)
        self.up_proj = _linear(c.hidden, c.intermediate, False)
        self.down_proj = _linear(c.intermediate, c.hidden, False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class Qwen3VLTextDecoderLayer(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.input_layernorm = Qwen3VLTextRMSNorm(c.hidden, c.eps)
        self.self_attn = Qwen3VLTextAttention(c)
        self.post_attention_layernorm = Qwen3VLTextRMSNorm(c.hidden, c.eps)
        self.mlp = Qwen3VLTextMLP(c)

    def forward(self, h, cos, sin):
        h = h + self.self_attn(self.input_layernorm(h), cos, sin)
        return h + self.mlp(self.post_attention_layernorm(h))


class Backbone(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.config = c
        self.embed_tokens = nn.Embedding(c.vocab, c.hidden)
        with torch.no_grad():
            self.embed_tokens.weight.normal_(0.0, 0.02)
        self.layers = nn.ModuleList(Qwen3VLTextDecoderLayer(c) for _ in range(c.layers))
        self._rope = None

    def rope(self, t, device, dtype):
        key = (t, device, dtype)
        if self._rope is None or self._rope[0] != key:
            c = self.config
            inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=device, dtype=torch.float32) / c.head_dim))
            freqs = torch.outer(torch.arange(t, device=device, dtype=torch.float32), inv)
            emb = torch.cat((freqs, freqs), dim=-1)
            self._rope = (key, emb.cos().to(dtype), emb.sin().to(dtype))
        return self._rope[1], self._rope[2]

    def forward(self, visual, input_ids):
        h = torch.cat((visual, self.embed_tokens(input_ids)), dim=1)
        cos, sin = self.rope(h.shape[1], h.device, h.dtype)
        for layer in self.layers:
            h = layer(h, cos, sin)
        return h


# ------------------------------------------------------------------ DiT
class SharedSiLU(nn.Module):
    """SiLU of the timestep condition, computed once per DiT forward.

    Every block's AdaLN and the output modulation receive the same activated
    condition tensor (as piR2's pointwise DiT fusion arranges,
    coexecution/groot_pointwise.py:171-258), so a grouped condition GEMM is
    computed once per step rather than once per block.
    """

    def __init__(self):
        super().__init__()
        self._temb = None
        self._value = None

    def forward(self, temb):
        if temb is not self._temb:
            self._temb, self._value = temb, F.silu(temb)
        return self._value

    def reset(self):
        self._temb = self._value = None


class AdaLayerNorm(nn.Module):
    def __init__(self, dim, eps, silu):
        super().__init__()
        self.silu = silu
        self.linear = _linear(dim, 2 * dim, True)
        self.norm = nn.LayerNorm(dim, eps=eps, elementwise_affine=False)

    def forward(self, x, temb):
        scale, shift = self.linear(self.silu(temb)).chunk(2, dim=-1)
        if scale.ndim == 2:
            scale, shift = scale[:, None], shift[:, None]
        return self.norm(x) * (1 + scale) + shift


class Attention(nn.Module):
    def __init__(self, dim, heads, head_dim, cross_dim=None):
        super().__init__()
        self.heads, self.head_dim = heads, head_dim
        self.is_cross_attention = cross_dim is not None
        self.to_q = _linear(dim, heads * head_dim, True)
        self.to_k = _linear(cross_dim or dim, heads * head_dim, True)
        self.to_v = _linear(cross_dim or dim, heads * head_dim, True)
        self.to_out = nn.ModuleList([_linear(heads * head_dim, dim, True), nn.Dropout(0.0)])
        self.kv_cache = None

    def kv(self, context):
        b, s = context.shape[0], context.shape[1]
        k = self.to_k(context).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        v = self.to_v(context).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        return k, v

    def forward(self, x, encoder_hidden_states=None, attention_mask=None):
        shape = x.shape
        b, t = shape[0], shape[1]
        q = self.to_q(x).view(b, t, self.heads, self.head_dim).transpose(1, 2)
        if self.is_cross_attention and self.kv_cache is not None:
            k, v = self.kv_cache
        else:
            k, v = self.kv(x if encoder_hidden_states is None else encoder_hidden_states)
        y = F.scaled_dot_product_attention(q, k, v, attn_mask=attention_mask)
        y = y.transpose(1, 2).reshape(b, t, self.heads * self.head_dim)
        return self.to_out[1](self.to_out[0](y))


class GELU(nn.Module):
    """diffusers-style GELU projection: forward = gelu(proj(x))."""

    def __init__(self, dim_in, dim_out, approximate="tanh"):
        super().__init__()
        self.proj = _linear(dim_in, dim_out, True)
        self.approximate = approximate

    def gelu(self, gate):
        return F.gelu(gate, approximate=self.approximate)

    def forward(self, x):
        return self.gelu(self.proj(x))


class FeedForward(nn.Module):
    def __init__(self, dim, inner):
        super().__init__()
        self.net = nn.ModuleList([GELU(dim, inner, "tanh"), nn.Dropout(0.0), _linear(inner, dim, True)])

    def forward(self, x):
        for module in self.net:
            x = module(x)
        return x


class BasicTransformerBlock(nn.Module):
    def __init__(self, c, cross, silu):
        super().__init__()
        self.dim = c.hidden
        self.norm_type = "ada_norm"
        self.pos_embed = None
        self.final_dropout = None
        self.norm1 = AdaLayerNorm(c.hidden, c.eps, silu)
        self.attn1 = Attention(c.hidden, c.heads, c.head_dim, c.context if cross else None)
        self.norm3 = nn.LayerNorm(c.hidden, eps=c.eps, elementwise_affine=False)
        self.ff = FeedForward(c.hidden, c.ff)

    def forward(self, hidden_states, attention_mask=None, encoder_hidden_states=None, encoder_attention_mask=None, temb=None):
        x = hidden_states
        attention = self.attn1(
            self.norm1(x, temb),
            encoder_hidden_states=encoder_hidden_states,
            attention_mask=encoder_attention_mask if encoder_hidden_states is not None else attention_mask,
        )
        x = attention + x
        return self.ff(self.norm3(x)) + x


class TimestepEmbedder(nn.Module):
    def __init__(self, channels, dim):
        super().__init__()
        self.linear_1 = _linear(channels, dim, True)
        self.act = nn.SiLU()
        self.linear_2 = _linear(dim, dim, True)

    def forward(self, x):
        return self.linear_2(self.act(self.linear_1(x)))


class TimestepEncoder(nn.Module):
    def __init__(self, channels, dim):
        super().__init__()
        self.channels = channels
        self.timestep_embedder = TimestepEmbedder(channels, dim)

    def forward(self, t, dtype):
        half = self.channels // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        args = t.float()[:, None] * 1000.0 * freqs[None]
        emb = torch.cat((torch.cos(args), torch.sin(args)), dim=-1).to(dtype)
        return self.timestep_embedder(emb)


class DiT(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.config = c
        self.timestep_encoder = TimestepEncoder(c.timestep_channels, c.hidden)
        self.condition_silu = SharedSiLU()
        self.transformer_blocks = nn.ModuleList(
            BasicTransformerBlock(c, cross=(i % 2 == 0), silu=self.condition_silu) for i in range(c.layers)
        )
        self.norm_out = nn.LayerNorm(c.hidden, eps=1e-6, elementwise_affine=False)
        self.proj_out_1 = _linear(c.hidden, 2 * c.hidden, True)
        self.proj_out_2 = _linear(c.hidden, c.hidden, True)

    def cache_context(self, context):
        for block in self.transformer_blocks:
            if block.attn1.is_cross_attention:
                block.attn1.kv_cache = block.attn1.kv(context)

    def clear_context(self):
        for block in self.transformer_blocks:
            block.attn1.kv_cache = None

    def forward(self, x, context, timestep):
        temb = self.timestep_encoder(timestep, x.dtype)
        for block in self.transformer_blocks:
            ctx = context if block.attn1.is_cross_attention else None
            x = block(x, encoder_hidden_states=ctx, temb=temb)
        shift, scale = self.proj_out_1(self.condition_silu(temb)).chunk(2, dim=-1)
        self.condition_silu.reset()
        x = self.norm_out(x) * (1 + scale[:, None]) + shift[:, None]
        return self.proj_out_2(x)


class ActionHead(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.config = c
        self.model = DiT(c)
        self.state_encoder = _linear(c.state_dim, c.hidden, True)
        self.action_encoder = _linear(c.action_dim, c.hidden, True)
        self.action_decoder = _linear(c.hidden, c.action_dim, True)
        self.position_embedding = nn.Parameter(torch.randn(1 + c.action_horizon, c.hidden) * 0.02)

    def velocity(self, state_tokens, actions, features, t):
        x = torch.cat((state_tokens, self.action_encoder(actions)), dim=1) + self.position_embedding
        y = self.model(x, features, t)
        # Decode the whole sequence, then keep the action tokens (as GR00T
        # slices the decoder's output), so the decoder reads whole rows.
        return self.action_decoder(y)[:, 1:]

    def get_action(self, features, state, noise):
        """4-step Euler integration of the flow from N(0, 1) actions."""
        c = self.config
        self.model.cache_context(features)
        try:
            state_tokens = self.state_encoder(state)
            actions = noise
            dt = 1.0 / c.steps
            b = noise.shape[0]
            for step in range(c.steps):
                t = torch.full((b,), step * dt, device=noise.device, dtype=torch.float32)
                actions = actions + dt * self.velocity(state_tokens, actions, features, t)
            return actions
        finally:
            self.model.clear_context()


class GR00TPolicy(nn.Module):
    """VLM prefill + DiT flow-matching action head."""

    def __init__(self, vlm=None, dit=None):
        super().__init__()
        self.backbone = Backbone(vlm or VLMConfig())
        self.action_head = ActionHead(dit or DiTConfig())

    def forward(self, visual, input_ids, state, noise):
        features = self.backbone(visual, input_ids)
        return self.action_head.get_action(features, state, noise)


def build_policy(device="cuda", *, vlm=None, dit=None, seed=0):
    """Random-init bf16 policy on `device` (weights ~N(0, 0.02))."""
    torch.manual_seed(seed)
    with torch.device(device):
        policy = GR00TPolicy(vlm, dit)
    return policy.to(torch.bfloat16).eval().requires_grad_(False)


def synthetic_inputs(batch, device="cuda", *, vlm=None, dit=None, seed=1):
    """Seeded synthetic inputs: 2 views x 256 visual embeddings ~N(0, 1),
    32 text token ids, a state vector and N(0, 1) initial actions."""
    vlm, dit = vlm or VLMConfig(), dit or DiTConfig()
    g = torch.Generator(device="cpu").manual_seed(seed)
    visual = torch.randn(batch, vlm.visual_tokens, vlm.hidden, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, vlm.vocab, (batch, vlm.text_tokens), generator=g)
    state = torch.randn(batch, 1, dit.state_dim, generator=g).to(torch.bfloat16)
    noise = torch.randn(batch, dit.action_horizon, dit.action_dim, generator=g).to(torch.bfloat16)
    return [t.to(device) for t in (visual, ids, state, noise)]
