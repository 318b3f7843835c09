"""SmoothQuant host logic (CPU): channel scales pinned to the reference's
own outputs, shared-input grouping, calibration hooks and the
pir2.thor.smoothquant.v1 profile validation."""

import os

import numpy as np
import pytest
import torch

from pir2_b200 import smoothquant as sq

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def test_channel_scales_equal_reference_outputs():
    amax = torch.from_numpy(GOLDEN["sq_amax"])
    w = torch.from_numpy(GOLDEN["sq_w"])
    w2 = torch.from_numpy(GOLDEN["sq_w2"])
    # Same torch expression as the reference on the same device: bitwise.
    assert np.array_equal(sq.channel_scales(amax, [w], 0.5).numpy(), GOLDEN["sq_scales_a05"])
    assert np.array_equal(sq.channel_scales(amax, [w, w2], 0.8).numpy(), GOLDEN["sq_scales_group_a08"])


@pytest.mark.parametrize("alpha", [-0.1, 1.5, float("nan"), True])
def test_channel_scales_reject_bad_alpha(alpha):
    with pytest.raises(ValueError, match="alpha"):
        sq.channel_scales(torch.ones(4), [torch.ones(2, 4)], alpha)


def test_channel_scales_reject_bad_statistics():
    with pytest.raises(ValueError, match="statistics"):
        sq.channel_scales(torch.tensor([1.0, -1.0]), [torch.ones(2, 2)], 0.5)
    with pytest.raises(ValueError, match="channel count"):
        sq.channel_scales(torch.ones(3), [torch.ones(2, 4)], 0.5)
    with pytest.raises(ValueError, match="at least one"):
        sq.channel_scales(torch.ones(3), [], 0.5)


def test_projection_groups_partition():
    sites = {"q": 0, "k": 0, "v": 0, "o": 0, "up": 0}
    assert sq.projection_groups(sites, [["q", "k", "v"], ["gate", "up"]]) == [["q", "k", "v"], ["up"], ["o"]]


def _model():
    torch.manual_seed(0)
    model = torch.nn.ModuleDict(
        {"q": torch.nn.Linear(32, 16), "k": torch.nn.Linear(32, 16), "o": torch.nn.Linear(16, 32)}
    ).to(torch.bfloat16)
    sites = {n: (m, "Role", "text") for n, m in model.items()}
    return model, sites, [["q", "k"]]


def test_calibration_profile_round_trip_and_validation(tmp_path):
    model, sites, groups = _model()
    x = torch.randn(3, 5, 32, dtype=torch.bfloat16)
    rng = torch.get_rng_state().clone()
    with sq.ActivationCalibration(sites, rows_per_call=4, max_rows=6) as calibration:
        for factor in (1, 2, 3):
            h = x * factor
            model["q"](h), model["k"](h)
            model["o"](model["q"](h))
    assert torch.equal(rng, torch.get_rng_state())          # private generator
    assert all(not m._forward_hooks for m in model.values())
    assert calibration.calls == {"q": 6, "k": 3, "o": 3}
    assert all(s.shape[0] <= 6 for s in calibration.samples.values())
    assert torch.equal(calibration.maxima["q"], (x * 3).float().abs().reshape(-1, 32).amax(0))

    path = tmp_path / "profile.pt"
    sq.write_profile(path, sites, groups, calibration, "fp4")
    scales, evidence = sq.load_profile(path, sites, groups, "fp4")
    assert scales["q"] is scales["k"]                       # one bound tensor per group
    assert evidence["smoothed_linears"] == ["k", "o", "q"] and evidence["unsmoothed_linears"] == []
    with pytest.raises(ValueError, match="schema or precision"):
        sq.load_profile(path, sites, groups, "fp8")

    profile = torch.load(path, weights_only=True)
    profile["linears"]["k"]["weight_sha256"] = "wrong"
    torch.save(profile, path)
    with pytest.raises(ValueError, match="weight mismatch"):
        sq.load_profile(path, sites, groups, "fp4")

    profile = torch.load(path, weights_only=True)
    del profile["linears"]["k"]
    torch.save(profile, path)
    with pytest.raises(ValueError, match="partial"):
        sq.load_profile(path, sites, groups, "fp4")

    profile = torch.load(path, weights_only=True)
    profile["linears"]["k"] = dict(profile["linears"]["q"], scale=profile["linears"]["q"]["scale"] * 2)
    profile["linears"]["k"]["weight_sha256"] = sq.weight_digest(model["k"].weight)
    torch.save(profile, path)
    with pytest.raises(ValueError, match="different scales"):
        sq.load_profile(path, sites, groups, "fp4")

    profile["linears"]["k"]["scale"] = profile["linears"]["q"]["scale"]
    profile["upstream_revision"] = "other"
    torch.save(profile, path)
    with pytest.raises(ValueError, match="revision"):
        sq.load_profile(path, sites, groups, "fp4")
