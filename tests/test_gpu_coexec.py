"""VLM / action-head co-execution (piR2's S1/S2, coexecution/run.py:33-105)
on the W8A8 fused path: the co-executed steps, replayed from their two CUDA
graphs, must produce exactly the actions of the serial computation on the
previous observation's features, and publish exactly the features of the
current observation (the two streams change no arithmetic)."""

from types import SimpleNamespace

import pytest
import torch

from pir2_b200 import harness
from pir2_b200.config import OptimizationConfig
from pir2_b200.engine import CoExecutionStep, ControlStep
from pir2_b200.session import GrootOptimizations

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 3])
def test_coexecuted_steps_equal_the_serial_computation(batch):
    vlm, dit = harness.VLMConfig(layers=2, vocab=2048), harness.DiTConfig(layers=2)
    policy = harness.build_policy("cuda", vlm=vlm, dit=dit)
    config = OptimizationConfig(
        precision="w8a8", fusion=True, scope="all", group_conditioning=True,
        norm_modulation_quant=True, residual_norm_quant=True,
    )
    observations = [harness.synthetic_inputs(batch, "cuda", vlm=vlm, dit=dit, seed=10 + k) for k in range(4)]
    with GrootOptimizations(SimpleNamespace(model=policy), config), torch.inference_mode():
        engine = CoExecutionStep(policy, batch)
        engine.prime(observations[0])
        engine.capture()
        # capture() ran each graph's step once eagerly: publish observation 0 again.
        engine.prime(observations[0])
        got = [engine.step(obs).clone() for obs in observations[1:]]
        features = [policy.backbone(obs[0], obs[1]) for obs in observations]
        want = [
            policy.action_head.get_action(features[k - 1], observations[k][2], observations[k][3]).cpu()
            for k in range(1, len(observations))
        ]
        slot = engine.slots[engine.parity]
        assert torch.equal(slot, features[-1])
        for a, b in zip(got, want):
            assert torch.equal(a, b)
        # The serial graph (headline engine) agrees with the eager policy too.
        serial = ControlStep(policy, batch)
        serial.load(observations[1])
        serial.capture()
        eager = policy(*observations[1])
        assert torch.equal(serial.step([t.cpu() for t in observations[1]]), eager.cpu())
        engine.release()
        serial.release()
