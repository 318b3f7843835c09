"""End-to-end action parity of a reduced GR00T-shaped policy (2 VLM layers,
2 DiT blocks, full widths): the fused B200 path against (a) the same
policy with every Linear replaced by the oracle's quantized Linear on the
CPU, and (b) the unquantized bf16 policy.

piR2 pins no end-to-end actions; this build pins them here.  Tolerances
(relative L2 over all actions, and max-abs) are stated per precision; the
oracle comparison differs only by rounding in the torch parts (norms,
attention) between CPU and GPU and in the fused producers' reduction order,
which can move individual activation codes by one.
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

# Relative L2 bounds: (VLM features vs oracle, actions vs oracle, actions vs
# bf16).  The flow integration amplifies single-code differences, so the
# action bounds are looser than the feature bounds; int4 codes are 18x
# coarser than int8 codes.
TOLERANCE = {"w8a8": (0.02, 0.03, 0.10), "w4a4": (0.10, 0.40, 0.80), "fp4": (0.10, 0.40, 0.80)}


def _rel_l2(a, b):
    a, b = a.detach().cpu().float(), b.detach().cpu().float()
    return (a - b).norm().item() / b.norm().item()


def _config(precision):
    if precision == "fp4":
        return OptimizationConfig(precision="fp4", scope="all")
    return OptimizationConfig(
        precision=precision, fusion=True, scope="all", group_conditioning=True,
        norm_modulation_quant=True, residual_norm_quant=True,
    )


@pytest.mark.parametrize("precision", ["w8a8", "w4a4", "fp4"])
@torch.inference_mode()
def test_actions_match_oracle_quantized_policy(precision):
    policy = harness.build_policy("cuda", vlm=VLM, dit=DIT)
    cpu_policy = copy.deepcopy(policy).to("cpu")
    inputs = harness.synthetic_inputs(1, "cuda", vlm=VLM, dit=DIT)
    cpu_inputs = [t.cpu() for t in inputs]
    bf16_actions = policy(*inputs)
    with GrootOptimizations(SimpleNamespace(model=policy), _config(precision)):
        features = policy.backbone(*inputs[:2])
        actions = policy(*inputs)
    restored = policy(*inputs)
    platform = _rel_l2(bf16_actions, cpu_policy(*cpu_inputs))   # bf16 GPU vs bf16 CPU
    install_oracle_linears(cpu_policy, precision)
    oracle_features = cpu_policy.backbone(*cpu_inputs[:2])
    oracle_actions = cpu_policy(*cpu_inputs)

    assert torch.equal(restored, bf16_actions)          # the session restored the model
    assert torch.isfinite(actions).all()
    rel_features = _rel_l2(features, oracle_features)
    rel_oracle = _rel_l2(actions, oracle_actions)
    rel_bf16 = _rel_l2(actions, bf16_actions)
    print(
        f"{precision}: features vs oracle {rel_features:.3e}; actions vs oracle {rel_oracle:.3e}, "
        f"vs bf16 {rel_bf16:.3e}; bf16 GPU vs CPU {platform:.3e}"
    )
    tol_features, tol_actions, tol_bf16 = TOLERANCE[precision]
    assert rel_features <= tol_features
    assert rel_oracle <= tol_actions
    assert rel_bf16 <= tol_bf16
