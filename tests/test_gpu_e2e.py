"""End-to-end parity of a reduced GR00T-shaped policy (2 VLM layers, 2 DiT
blocks, full widths, 4 Euler steps) on the B200 path.

The oracle policy is the same policy with every Linear replaced by the
oracle's quantized Linear (computed on the host, returned to the GPU);
everything between the Linears runs the same torch GPU code.  So:

- with the plugin's unfused installation (TransformerINT only) the
  actions must be bitwise identical to the oracle policy's: every integer
  stage is exact and the activations (GELU, SiLU·up) are applied through
  torch-built LUTs that equal torch's own results;
- with the fused installation (norm/modulation/residual producers, q/k
  RMSNorm + RoPE, row attention) the producers round in a different order
  (activation codes may move by one), so actions are compared by relative L2;
- against the unquantized bf16 policy the quantization error itself is
  bounded (relative L2).

piR2 pins no end-to-end actions; this build pins them here.  Comparing
with a CPU oracle policy instead is not informative: CPU and GPU torch
attention differ by ~0.4 % relative, which moves activation codes across
rounding boundaries and changes quantized outputs by about the
quantization noise itself.
"""

import copy
from types import SimpleNamespace

import pytest
import torch

from oracle.model import install_oracle_linears
from pir2_b200 import harness
from pir2_b200.config import OptimizationConfig
from pir2_b200.session import GrootOptimizations

pytestmark = pytest.mark.gpu

VLM = harness.VLMConfig(layers=2, vocab=2048)
DIT = harness.DiTConfig(layers=2)

# Relative-L2 bounds on the actions: (fused vs oracle policy, vs bf16).
# W4A4: about twice the measured fused-vs-oracle distance (0.14).
TOLERANCE = {"w8a8": (0.05, 0.10), "w4a4": (0.28, 0.80), "fp4": (0.10, 0.60), "fp8": (0.05, 0.30)}


def _rel_l2(a, b):
    a, b = a.detach().float(), b.detach().float()
    return (a - b).norm().item() / b.norm().item()


def _fused(precision):
    if precision in ("fp4", "fp8"):
        # Every floating producer (SwiGLU, GELU, RMSNorm, DiT norm/residual),
        # shared packs: the configuration bench.py times.
        return OptimizationConfig(
            precision=precision, scope="all", fp_shared_inputs=True, fp_swiglu=True, fp_gelu=True,
            fp_rmsnorm=True, fusion=True, norm_modulation_quant=True, residual_norm_quant=True,
        )
    return OptimizationConfig(
        precision=precision, fusion=True, scope="all", group_conditioning=True,
        norm_modulation_quant=True, residual_norm_quant=True,
    )


@pytest.fixture(scope="module")
def policies():
    with torch.inference_mode():
        policy = harness.build_policy("cuda", vlm=VLM, dit=DIT)
        inputs = harness.synthetic_inputs(1, "cuda", vlm=VLM, dit=DIT)
        bf16_actions = policy(*inputs)
    return policy, inputs, bf16_actions


@pytest.mark.parametrize("precision", ["w8a8", "w4a4"])
@torch.inference_mode()
def test_unfused_actions_equal_oracle_policy_bitwise(policies, precision):
    policy, inputs, bf16_actions = policies
    oracle_policy = install_oracle_linears(copy.deepcopy(policy), precision)
    with GrootOptimizations(SimpleNamespace(model=policy), OptimizationConfig(precision=precision, scope="all")):
        actions = policy(*inputs)
    assert torch.equal(policy(*inputs), bf16_actions)     # restored
    assert torch.equal(actions, oracle_policy(*inputs))


@pytest.mark.parametrize("precision", ["w8a8", "w4a4", "fp4", "fp8"])
@torch.inference_mode()
def test_fused_actions_match_oracle_policy(policies, precision):
    policy, inputs, bf16_actions = policies
    oracle_policy = install_oracle_linears(copy.deepcopy(policy), precision)
    with GrootOptimizations(SimpleNamespace(model=policy), _fused(precision)):
        actions = policy(*inputs)
    assert torch.equal(policy(*inputs), bf16_actions)     # restored
    assert torch.isfinite(actions).all()
    oracle_actions = oracle_policy(*inputs)
    rel_oracle = _rel_l2(actions, oracle_actions)
    rel_bf16 = _rel_l2(actions, bf16_actions)
    print(f"{precision}: fused vs oracle policy {rel_oracle:.3e}, vs bf16 {rel_bf16:.3e}, "
          f"oracle vs bf16 {_rel_l2(oracle_actions, bf16_actions):.3e}")
    tol_oracle, tol_bf16 = TOLERANCE[precision]
    assert rel_oracle <= tol_oracle
    assert rel_bf16 <= tol_bf16
