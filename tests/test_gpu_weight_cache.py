"""Packed-weight cache through the session: the first installation writes
the cache, a second one (fresh policy, same weights) loads it without
quantizing and gives bitwise the same actions; changed weights are refused
and leave the model restored."""

from types import SimpleNamespace

import pytest
import torch

from pir2_b200 import harness, weight_cache
from pir2_b200.config import OptimizationConfig
from pir2_b200.session import GrootOptimizations

pytestmark = pytest.mark.gpu

VLM = harness.VLMConfig(layers=1, vocab=2048)
DIT = harness.DiTConfig(layers=2)


@pytest.mark.parametrize("precision", ["w8a8", "w4a4"])
@torch.inference_mode()
def test_session_writes_then_loads_the_packed_weight_cache(tmp_path, precision, monkeypatch):
    path = tmp_path / "packed.pt"
    config = OptimizationConfig(precision=precision, scope="all", packed_weights=path)
    policy = harness.build_policy("cuda", vlm=VLM, dit=DIT)
    inputs = harness.synthetic_inputs(1, "cuda", vlm=VLM, dit=DIT)
    with GrootOptimizations(SimpleNamespace(model=policy), config) as session:
        first = policy(*inputs)
        assert session.evidence()["coverage"]["packed_weights"]["written"]
    assert path.exists()

    # A second policy with the same weights: the cache is used, nothing is quantized.
    again = harness.build_policy("cuda", vlm=VLM, dit=DIT)
    from pir2_b200 import integer

    def refuse(*args, **kwargs):
        raise AssertionError("install-time quantization ran despite the cache")

    monkeypatch.setattr(integer, "quantize_weight", refuse)
    with GrootOptimizations(SimpleNamespace(model=again), config) as session:
        second = again(*inputs)
        assert session.evidence()["coverage"]["packed_weights"]["loaded"]
    assert torch.equal(first, second)

    # Changed weights: refused before anything is swapped in.
    with torch.no_grad():
        next(m for m in again.modules() if isinstance(m, torch.nn.Linear)).weight.add_(0.01)
    reference = again(*inputs)
    with pytest.raises(ValueError, match="stale|shape|entry"):
        with GrootOptimizations(SimpleNamespace(model=again), config):
            pass
    assert torch.equal(again(*inputs), reference)
    assert weight_cache.CACHE_VERSION == 1
