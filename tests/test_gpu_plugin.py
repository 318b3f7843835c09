"""GPU contract tests of the plugin API, ported from piR2's own GPU tests
(tests/gpu/test_quantization_gpu.py, test_shape_tactics_gpu.py): the
installed quantized Linear matches the explicit quantized formula bitwise
and restores the model; grouped projections dispatch once; fused packs equal
their unfused counterparts; graph replay equals eager.
"""

from types import SimpleNamespace
from unittest.mock import patch

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops
from pir2_b200.connections import AdditionalConnections
from pir2_b200.fused import prepare_gelu
from pir2_b200.integer import prepare_activation
from pir2_b200.linear import prepare
from pir2_b200.projections import inventory
from pir2_b200.transformer import TransformerINT

pytestmark = pytest.mark.gpu


def equal(actual, expected):
    assert actual.shape == expected.shape and actual.dtype == expected.dtype
    assert torch.equal(actual.contiguous().view(torch.uint8), expected.contiguous().view(torch.uint8))


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(device)


class Norm(torch.nn.Module):
    """AdaLN fixture of piR2's tests (tests/helpers/projection_models.py:18-33)."""

    def __init__(self, width):
        super().__init__()
        self.norm = torch.nn.LayerNorm(width, elementwise_affine=False, device="cuda", dtype=torch.bfloat16)
        self.silu = torch.nn.SiLU()
        self.linear = torch.nn.Linear(width, 2 * width, device="cuda", dtype=torch.bfloat16)

    def forward(self, x, temb):
        scale, shift = self.linear(self.silu(temb)).chunk(2, dim=-1)
        if scale.ndim == 2:
            scale, shift = scale[:, None], shift[:, None]
        return self.norm(x) * (1 + scale) + shift


def policy_for(blocks):
    return SimpleNamespace(model=SimpleNamespace(action_head=SimpleNamespace(model=SimpleNamespace(transformer_blocks=blocks))))


def torch_quantized_linear(x, weight, bias, bits):
    """The reference's explicit formula (test_quantization_gpu.py:37-44),
    evaluated with CUDA torch (where `tensor / scalar` multiplies by the
    fp32 reciprocal, as the reference kernels do)."""
    limit = 2 ** (bits - 1) - 1
    xs = x.float().abs().amax(dim=-1) / limit
    ws = weight.float().abs().amax(dim=-1) / limit
    qx = torch.round(x.float() / xs[:, None]).clamp(-limit, limit)
    qw = torch.round(weight.float() / ws[:, None]).clamp(-limit, limit)
    acc = (qx.double() @ qw.double().t()).float()   # exact integers
    y = acc * xs[:, None] * ws[None, :]
    if bias is not None:
        y = y + bias.float()
    return y.to(torch.bfloat16)


def test_cuda_scalar_division_is_a_reciprocal_multiply():
    """Pins the torch behaviour the reference's weight scales rely on."""
    g = torch.Generator(device="cuda").manual_seed(0)
    m = torch.rand(1 << 20, device="cuda", generator=g) * 10
    for limit in (127, 7):
        via_div = m / limit
        via_mul = m * (torch.tensor(1.0, device="cuda") / limit)
        assert torch.equal(via_div, via_mul)
        true_div = m / torch.full_like(m, limit)
        assert not torch.equal(via_div, true_div)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("native", [False, True])
@torch.inference_mode()
def test_integer_linear_matches_quantized_reference_and_restores(bits, native):
    torch.manual_seed(195)
    linear = torch.nn.Linear(130, 64, device="cuda", dtype=torch.bfloat16).eval()
    model = torch.nn.Sequential(linear)
    x = torch.randn(17, 130, device="cuda", dtype=torch.bfloat16)
    original = model(x)
    expected = torch_quantized_linear(x, linear.weight, linear.bias, bits)
    adapter = TransformerINT(model, {"0"}, native=native, expanded=True)
    try:
        adapter.set(f"w{bits}a{bits}")
        equal(model(x), expected)
        # And the CPU oracle agrees bitwise.
        ref = oracle.linear_w8a8(bits_of(x), linear.weight.float().cpu().numpy(), bits_of(linear.bias), bits)
        assert np.array_equal(bits_of(model(x)), ref)
    finally:
        adapter.close()
    assert "forward" not in linear.__dict__
    equal(model(x), original)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("tokens", [1, 41])
@torch.inference_mode()
def test_condition_group_reuses_pack_and_gemm_and_releases_inputs(bits, tokens):
    dit = torch.nn.Module()
    blocks = [torch.nn.Module(), torch.nn.Module()]
    for block in blocks:
        block.norm1 = Norm(64)
    dit.transformer_blocks = torch.nn.ModuleList(blocks)
    dit.proj_out_1 = torch.nn.Linear(64, 128, device="cuda", dtype=torch.bfloat16)
    model = torch.nn.Module()
    model.action_head = torch.nn.Module()
    model.action_head.model = dit
    sites = inventory(model, expanded=True)[0]
    modules = [site[0] for site in sites.values()]
    condition = torch.randn((1, 64) if tokens == 1 else (1, tokens, 64), device="cuda", dtype=torch.bfloat16)
    adapter = TransformerINT(model, sites, native=True, expanded=True, condition_group=True)
    try:
        for _ in range(2):
            expected = [adapter.quant[bits][name](condition) for name in sites]
            adapter.set(f"w{bits}a{bits}")
            with patch.object(adapter, "dispatch", wraps=adapter.dispatch) as dispatch:
                actual = [module(condition) for module in modules]
                assert dispatch.call_count == 1
            for value, reference in zip(actual, expected):
                equal(value, reference)
            group = adapter.grouped[bits][0][1]
            assert group._input is None and group._output is None
            condition.add_(0.25)
        modules[0](condition)
        assert group._input is condition
    finally:
        adapter.close()
    assert group._input is None and group._output is None
    assert not group._remaining
    assert all("forward" not in module.__dict__ for module in modules)


@pytest.mark.parametrize("bits", [8, 4])
@torch.inference_mode()
def test_fused_activation_pack_matches_reference(bits):
    x = torch.randn(17, 258, device="cuda", dtype=torch.bfloat16)
    up = torch.randn_like(x)
    lut = prepare_gelu(x.device, x.dtype, "tanh")
    actual = prepare(x, bits, lut, up)
    expected = prepare_activation(x, bits, up=up, gelu="tanh", pack_reuse=True)
    equal(actual.data, expected.data)
    equal(actual.scales, expected.scales)
    # ... and both equal the pack of the materialized bf16(gelu(x) * up).
    plain = prepare_activation((torch.nn.functional.gelu(x, approximate="tanh") * up), bits)
    equal(actual.data, plain.data)
    equal(actual.scales, plain.scales)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("per_token", [False, True])
@torch.inference_mode()
def test_modulation_pack_preserves_shared_and_per_token_inputs(bits, per_token):
    norm = Norm(64)
    x = torch.randn(2, 3, 64, device="cuda", dtype=torch.bfloat16)
    temb = torch.randn((2, 3, 64) if per_token else (2, 64), device="cuda", dtype=torch.bfloat16)
    expected = prepare_activation(norm(x, temb), bits, pack_reuse=True)
    adapter = AdditionalConnections(policy_for([SimpleNamespace(norm1=norm)]), None, {})
    try:
        adapter.set(f"w{bits}a{bits}")
        actual = norm(x, temb).for_bits(bits)
        equal(actual.data, expected.data)
        equal(actual.scales, expected.scales)
        assert actual.shape == expected.shape
    finally:
        adapter.close()
    assert "forward" not in norm.__dict__


@pytest.mark.parametrize("bits", [8, 4])
@torch.inference_mode()
def test_graph_replay_equals_eager(bits):
    torch.manual_seed(3)
    linear = torch.nn.Linear(1536, 6144, device="cuda", dtype=torch.bfloat16).eval()
    model = torch.nn.Sequential(linear)
    adapter = TransformerINT(model, {"0"}, native=True, expanded=True)
    try:
        adapter.set(f"w{bits}a{bits}")
        for rows in (41, 153, 17):
            x = torch.randn(rows, 1536, device="cuda", dtype=torch.bfloat16)
            eager = model(x)
            graph = torch.cuda.CUDAGraph()
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    out = model(x)
            eager2 = model(x)
            graph.replay()
            torch.cuda.synchronize()
            equal(out, eager)
            equal(eager2, eager)
            x.add_(0.5)
            graph.replay()
            torch.cuda.synchronize()
            equal(out, model(x))
    finally:
        adapter.close()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("cross", [False, True])
@torch.inference_mode()
def test_dit_attention_fusion_matches_sdpa_forward_and_restores(cross):
    from pir2_b200.harness import Attention
    from pir2_b200.pointwise import DiTAttentionFusion

    torch.manual_seed(7)
    with torch.device("cuda"):
        attn = Attention(1536, 32, 48, 2048 if cross else None).to(torch.bfloat16).eval()
    x = torch.randn(2, 17, 1536, device="cuda", dtype=torch.bfloat16)
    context = torch.randn(2, 544, 2048, device="cuda", dtype=torch.bfloat16) if cross else None
    if cross:
        attn.kv_cache = attn.kv(context)
    reference = attn(x, encoder_hidden_states=context)
    fusion = DiTAttentionFusion(torch.nn.Sequential(attn), cross_only=False)
    assert fusion.targets == [attn]
    fusion.set()
    try:
        fused = attn(x, encoder_hidden_states=context)
    finally:
        fusion.close()
    assert "forward" not in attn.__dict__
    # Both paths run the same bf16 projections; the attention core differs
    # only in summation order and bf16 rounding of its output.
    torch.testing.assert_close(fused.float(), reference.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("bits,ffn_kernel,fused_pack", [(8, False, False), (8, True, False), (4, False, False), (8, False, True)])
@torch.inference_mode()
def test_residual_and_gelu_epilogue_fusion_is_bitwise(bits, ffn_kernel, fused_pack, monkeypatch):
    """Residual adds in the o-proj / down-proj epilogues and the FFN GELU in
    the up-projection epilogue give bitwise the unfused quantized blocks;
    so does the opt-in in-GEMM activation pack (o-proj from whole rows,
    down-proj from the up GEMM's per-16-channel maxima)."""
    from pir2_b200 import integer
    from pir2_b200.fusion import ResidualFusion
    from pir2_b200.harness import DiTConfig, VLMConfig, build_policy

    dit = DiTConfig(layers=2)
    policy = build_policy("cuda", dit=dit, vlm=VLMConfig(layers=1, vocab=2048))
    model = policy.action_head.model
    names, _, _, _ = inventory(policy)
    executed = {n for n in names if n.startswith("action_head.model.transformer_blocks")}
    adapter = TransformerINT(policy, executed, native=True, expanded=True)
    fusion = ResidualFusion(policy, adapter, ffn_kernel=ffn_kernel)
    assert len(fusion.blocks) == 2
    torch.manual_seed(5)
    x = torch.randn(2, 17, dit.hidden, device="cuda", dtype=torch.bfloat16)
    temb = torch.randn(2, dit.hidden, device="cuda", dtype=torch.bfloat16)
    context = torch.randn(2, 544, dit.context, device="cuda", dtype=torch.bfloat16)
    try:
        adapter.set(f"w{bits}a{bits}")
        outs = []
        for block in model.transformer_blocks:
            ctx = context if block.attn1.is_cross_attention else None
            outs.append(block(x, encoder_hidden_states=ctx, temb=temb))
        fusion.set(bits, norm_pack=False)
        if fused_pack:
            monkeypatch.setattr(integer, "FUSED_PACK_ROWS", 64)
            monkeypatch.setattr(integer, "FUSED_PACK_BYTES", 128 * 1024)   # 34 rows of 1536
            calls = []
            original = ops.gemm_rows
            monkeypatch.setattr(ops, "gemm_rows", lambda *a, **k: calls.append(k.get("x_max") is not None) or original(*a, **k))
        for block, ref in zip(model.transformer_blocks, outs):
            ctx = context if block.attn1.is_cross_attention else None
            equal(block(x, encoder_hidden_states=ctx, temb=temb), ref)
        if fused_pack:
            assert True in calls and False in calls   # down-proj from maxima, o-proj from whole rows
    finally:
        fusion.close()
        adapter.close()


@torch.inference_mode()
def test_swiglu_epilogue_fusion_is_bitwise():
    """Text MLP through the SwiGLU GEMM epilogue == the unfused W8A8 MLP
    (group GEMM + gated SiLU pack), bit for bit, and restores."""
    from pir2_b200.fusion import SwiGLUFusion
    from pir2_b200.harness import DiTConfig, VLMConfig, build_policy

    policy = build_policy("cuda", dit=DiTConfig(layers=2), vlm=VLMConfig(layers=2, vocab=2048))
    names = inventory(policy)[0]
    executed = {n for n in names if n.startswith("backbone.layers")}
    adapter = TransformerINT(policy, executed, native=True, expanded=True)
    fusion = SwiGLUFusion(policy, adapter)
    assert len(fusion.sites) == 2
    torch.manual_seed(9)
    x = torch.randn(1, 544, 2048, device="cuda", dtype=torch.bfloat16)
    try:
        adapter.set("w8a8")
        mlps = [layer.mlp for layer in policy.backbone.layers]
        refs = [mlp(x) for mlp in mlps]
        fusion.set()
        for mlp, ref in zip(mlps, refs):
            equal(mlp(x), ref)
        fusion.close()
        equal(mlps[0](x), refs[0])
    finally:
        fusion.close()
        adapter.close()


@torch.inference_mode()
def test_text_attention_causal_kernel_matches_sdpa_path_and_restores():
    """Quantized text attention with the causal row kernel == the same fused
    layer on torch SDPA + transpose, to bf16 tolerance: the attention core
    differs only in summation order, which may move a few o_proj input codes
    by one step, so the check is on the relative error of the whole output."""
    from pir2_b200.harness import DiTConfig, VLMConfig, build_policy
    from pir2_b200.pointwise import TextAttentionFusion

    policy = build_policy("cuda", dit=DiTConfig(layers=2), vlm=VLMConfig(layers=2, vocab=2048))
    names = inventory(policy)[0]
    executed = {n for n in names if n.startswith("backbone.layers")}
    adapter = TransformerINT(policy, executed, native=True, expanded=True)
    torch.manual_seed(11)
    x = torch.randn(1, 544, 2048, device="cuda", dtype=torch.bfloat16)
    cos, sin = policy.backbone.rope(544, x.device, x.dtype)
    attns = [layer.self_attn for layer in policy.backbone.layers]
    sdpa = TextAttentionFusion(policy, adapter, causal_kernel=False)
    kernel = TextAttentionFusion(policy, adapter, causal_kernel=True)
    try:
        adapter.set("w8a8")
        sdpa.set(8)
        refs = [attn(x, cos, sin) for attn in attns]
        sdpa.close()
        kernel.set(8)
        assert all("forward" in attn.__dict__ for attn in attns)
        for attn, ref in zip(attns, refs):
            out = attn(x, cos, sin).float()
            err = (out - ref.float()).norm() / ref.float().norm()
            assert err < 1e-2, float(err)
        kernel.close()
        assert all("forward" not in attn.__dict__ for attn in attns)
    finally:
        sdpa.close()
        kernel.close()
        adapter.close()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("precision", ["fp8", "fp4"])
@pytest.mark.parametrize("grouped", [False, True])
@torch.inference_mode()
def test_floating_session_installs_producers(precision, grouped):
    """The floating session with every producer piR2 wires for fp8 / fp4
    (coexecution/optimization/groot/floating.py:162-346 and
    floating_connections.py): shared-input or merged (grouped) projections,
    SwiGLU, GELU and RMSNorm producers, the DiT LayerNorm + AdaLN and
    residual + LayerNorm producers.  Every site is covered, the actions stay
    close to the unfused floating session's, and closing restores every
    module."""
    from pir2_b200.config import OptimizationConfig
    from pir2_b200.harness import DiTConfig, VLMConfig, build_policy, synthetic_inputs
    from pir2_b200.session import GrootOptimizations

    vlm, dit = VLMConfig(layers=2, vocab=2048), DiTConfig(layers=2)
    policy = build_policy("cuda", dit=dit, vlm=vlm)
    inputs = synthetic_inputs(1, "cuda", vlm=vlm, dit=dit)
    bf16_actions = policy(*inputs)
    with GrootOptimizations(SimpleNamespace(model=policy), OptimizationConfig(precision=precision, scope="all")):
        plain = policy(*inputs)
    config = OptimizationConfig(
        precision=precision, scope="all", fp_shared_inputs=not grouped, fp_grouped=grouped, fp_swiglu=True,
        fp_gelu=True, fp_rmsnorm=True, fusion=True, norm_modulation_quant=True, residual_norm_quant=True,
    )
    with GrootOptimizations(SimpleNamespace(model=policy), config) as session:
        coverage = session.coverage["floating"]
        assert len(coverage["swiglu_producers"]) == vlm.layers
        assert len(coverage["rmsnorm_producers"]) == vlm.layers
        assert len(coverage["gelu_producers"]) >= dit.layers
        merged = coverage["merged_projection_groups" if grouped else "shared_input_groups"]
        assert len(merged) >= 2 * vlm.layers
        assert session.coverage["norm_quantization_fusion"]["attention_producers"] > 0
        assert session.coverage["norm_quantization_fusion"]["residual_ffn_producers"] == dit.layers
        # Merged q|k|v: RMSNorm producer + fused q/k norm and RoPE on every text layer.
        assert session.coverage["text_attention_fusion"] == (vlm.layers if grouped else 0)
        fused = policy(*inputs)
    assert torch.equal(policy(*inputs), bf16_actions)
    assert all("forward" not in m.__dict__ for m in policy.modules())
    assert all("gelu" not in m.__dict__ for m in policy.modules())
    assert torch.isfinite(fused).all()
    rel = ((fused.float() - plain.float()).norm() / plain.float().norm()).item()
    print(f"{precision} grouped={grouped}: fused producers vs unfused floating {rel:.3e}")
    assert rel < (0.05 if precision == "fp8" else 0.15)
    assert _lib.device_status() == 0
