"""Packed-weight cache (pir2_b200/weight_cache.py): file format, validation
and rejection of stale or foreign caches, on the CPU (no kernels run)."""

from types import SimpleNamespace

import pytest
import torch

from pir2_b200 import weight_cache
from pir2_b200.config import OptimizationConfig


def fake_controller(seed=0):
    g = torch.Generator().manual_seed(seed)
    modules, quant = {}, {8: {}, 4: {}}
    for name, (n, k, bias) in {"a.q": (64, 256, False), "a.o": (256, 64, True)}.items():
        lin = torch.nn.Linear(k, n, bias=bias).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, generator=g))
        modules[name] = lin
        for bits in (8, 4):
            cols = k if bits == 8 else k // 2
            quant[bits][name] = SimpleNamespace(
                packed_weight=torch.randint(0, 255, (n, cols), generator=g, dtype=torch.uint8),
                weight_scale=torch.rand(n, generator=g),
                bias=torch.randn(n, generator=g).to(torch.bfloat16) if bias else None,
            )
    sites = {name: (m, "kind", "dit") for name, m in modules.items()}
    return SimpleNamespace(sites=sites, quant=quant), modules


def test_round_trip_returns_the_saved_tensors(tmp_path):
    controller, modules = fake_controller()
    path = tmp_path / "packed.pt"
    weight_cache.save(controller, path)
    loaded = weight_cache.load(path, modules, "cpu")
    for name in modules:
        for bits in (8, 4):
            q = controller.quant[bits][name]
            w, s, b = loaded[name][bits]
            assert torch.equal(w, q.packed_weight) and torch.equal(s, q.weight_scale)
            assert (b is None and q.bias is None) or torch.equal(b, q.bias)


def test_changed_weights_missing_sites_and_foreign_files_are_rejected(tmp_path):
    controller, modules = fake_controller()
    path = tmp_path / "packed.pt"
    weight_cache.save(controller, path)
    with torch.no_grad():
        modules["a.q"].weight[3, 5] += 1.0
    with pytest.raises(ValueError, match="stale"):
        weight_cache.load(path, modules, "cpu")
    _, fresh = fake_controller()
    fresh["a.extra"] = torch.nn.Linear(64, 64).to(torch.bfloat16)
    with pytest.raises(ValueError, match="no entry"):
        weight_cache.load(path, fresh, "cpu")
    other = tmp_path / "other.pt"
    torch.save({"format": "something else"}, other)
    with pytest.raises(ValueError, match="Not a packed-weight cache"):
        weight_cache.load(other, fresh, "cpu")
    payload = torch.load(path, weights_only=True)
    payload["version"] = 0
    torch.save(payload, other)
    with pytest.raises(ValueError, match="version"):
        weight_cache.load(other, fake_controller()[1], "cpu")


def test_fingerprint_is_exact_and_position_sensitive():
    w = torch.randn(8, 16).to(torch.bfloat16)
    assert weight_cache.fingerprint(w) == weight_cache.fingerprint(w.clone())
    swapped = w.clone()
    swapped[[0, 1]] = swapped[[1, 0]]
    if not torch.equal(swapped, w):
        assert weight_cache.fingerprint(swapped) != weight_cache.fingerprint(w)


def test_config_accepts_the_cache_only_for_integer_precision(tmp_path):
    OptimizationConfig(precision="w8a8", packed_weights=tmp_path / "p.pt")
    with pytest.raises(ValueError, match="packed-weight cache"):
        OptimizationConfig(precision="bf16", packed_weights=tmp_path / "p.pt")
