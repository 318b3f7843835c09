"""SmoothQuant channel balancing for the B200 quantized Linear path.

Mirrors coexecution/optimization/backends/thor/smoothquant.py (piR2):

- `channel_scales` (:27-45): s_c = clamp(amax_c^alpha /
  clamp(max over the group's weights of |W_nc|, 1e-5)^(1 - alpha), 1e-5),
  all in fp32 on the weights' device;
- `projection_groups` (:48-57): consumers of one input (q|k|v, k|v,
  gate|up) share one scale vector;
- `ActivationCalibration` (:60-121): eager forward hooks collecting
  per-input-channel maxima and a bounded deterministic row sample from a
  private generator;
- `load_profile` (:124-176): the `pir2.thor.smoothquant.v1` profile file
  (torch.save of a dict), validated against the installed weights by
  SHA-256 and bound once per group on the device.

The weights are multiplied by s when packed (`FloatingLinear`), the
activations are divided by s inside the pack kernels (`smooth` argument of
`pir2b_quant_rows` / `pir2b_norm_quant_rows`).  Profiles written for piR2
load here unchanged and vice versa (same schema string, same upstream
revision tag, same record keys).
"""

import hashlib
import math
from contextlib import ExitStack
from pathlib import Path

import torch

PROFILE_SCHEMA = "pir2.thor.smoothquant.v1"
# Revision tag piR2 stamps into its profiles (the upstream SmoothQuant
# commit its formula follows); kept identical so profiles interoperate.
UPSTREAM_REVISION = "c61476d728e42ae0d8a35e7e78494edcac3237b5"


def weight_digest(weight):
    """SHA-256 of the weight's raw bytes (host copy)."""
    data = weight.detach().contiguous().view(torch.uint8).cpu().numpy()
    return hashlib.sha256(data.tobytes()).hexdigest()


@torch.no_grad()
def channel_scales(activation_absmax, weights, alpha):
    """Per-input-channel balancing scales shared by every weight in `weights`."""
    if isinstance(alpha, bool) or not math.isfinite(alpha) or not 0 <= alpha <= 1:
        raise ValueError("SmoothQuant alpha must be finite and in [0,1]")
    if not weights:
        raise ValueError("SmoothQuant needs at least one weight")
    device = weights[0].device
    amax = activation_absmax.detach().to(device=device, dtype=torch.float32)
    if amax.ndim != 1 or not torch.isfinite(amax).all() or (amax < 0).any():
        raise ValueError("Invalid activation channel statistics")
    if any(w.ndim != 2 or w.shape[1] != amax.numel() for w in weights):
        raise ValueError("SmoothQuant channel count differs from weight inputs")
    per_weight = [w.detach().float().abs().amax(0) for w in weights]
    wmax = torch.stack(per_weight).amax(0).clamp(min=1e-5)
    scales = (amax.pow(alpha) / wmax.pow(1 - alpha)).clamp(min=1e-5)
    if not torch.isfinite(scales).all():
        raise ValueError("Nonfinite SmoothQuant scales")
    return scales.contiguous()


def projection_groups(sites, groups):
    """Partition `sites` into shared-input groups (in `groups` order), then
    singletons for the rest."""
    grouped, seen = [], set()
    for group in groups:
        members = [name for name in group if name in sites]
        if members:
            grouped.append(members)
            seen.update(members)
    return grouped + [[name] for name in sites if name not in seen]


def rows_on_gpu(x):
    return x.is_cuda and torch.cuda.is_available()


class ActivationCalibration:
    """Context manager recording, per site, the running per-channel |x| max
    and up to `max_rows` sampled input rows (`rows_per_call` per call).

    Sampling draws from a private generator seeded with `seed`, so the
    model's global RNG state never moves.  Hooks raise under CUDA-graph
    capture: calibration is eager only.
    """

    def __init__(self, sites, *, rows_per_call=4, max_rows=128, seed=1000):
        if rows_per_call < 1 or max_rows < 1:
            raise ValueError("Calibration sample bounds must be positive")
        self.sites = sites
        self.rows_per_call, self.max_rows, self.seed = rows_per_call, max_rows, seed
        self.maxima, self.samples, self.calls = {}, {}, {}
        self.stack = ExitStack()
        self.generator = None

    def _observe(self, name, module, x):
        if rows_on_gpu(x) and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("SmoothQuant calibration requires eager inference")
        rows = x.detach().reshape(-1, module.in_features)
        amax = rows.float().abs().amax(0)
        if not torch.isfinite(amax).all():
            raise ValueError(f"Nonfinite calibration activation: {name}")
        previous = self.maxima.get(name)
        self.maxima[name] = amax if previous is None else torch.maximum(previous, amax)
        self.calls[name] = self.calls.get(name, 0) + 1
        pick = torch.randperm(rows.shape[0], device=rows.device, generator=self.generator)
        sample = rows[pick[: self.rows_per_call]].clone()
        if name in self.samples:
            sample = torch.cat((self.samples[name], sample))
        if sample.shape[0] > self.max_rows:
            keep = torch.randperm(sample.shape[0], device=rows.device, generator=self.generator)
            sample = sample[keep[: self.max_rows]].contiguous()
        self.samples[name] = sample

    def __enter__(self):
        device = next(iter(self.sites.values()))[0].weight.device
        self.generator = torch.Generator(device=device).manual_seed(self.seed)
        try:
            for name, (module, _, _) in self.sites.items():
                handle = module.register_forward_hook(
                    lambda m, inputs, _out, name=name: self._observe(name, m, inputs[0])
                )
                self.stack.callback(handle.remove)
        except BaseException:
            self.stack.close()
            raise
        return self

    def __exit__(self, *exception):
        self.stack.close()


def _check_scale(name, scale, module):
    if (
        not isinstance(scale, torch.Tensor)
        or scale.dtype != torch.float32
        or scale.shape != (module.in_features,)
        or scale.requires_grad
        or not torch.isfinite(scale).all()
        or not (scale > 0).all()
    ):
        raise ValueError(f"Invalid SmoothQuant channel scale: {name}")


def load_profile(path, sites, groups, precision):
    """Read and validate a profile; returns ({site: scale on device}, evidence).

    Every member of a shared-input group gets the same bound tensor (the
    pack kernels and FloatingLinear check identity, not just equality)."""
    profile = torch.load(path, map_location="cpu", weights_only=True)
    if profile.get("schema") != PROFILE_SCHEMA or profile.get("precision") != precision:
        raise ValueError("SmoothQuant profile schema or precision mismatch")
    if profile.get("upstream_revision") != UPSTREAM_REVISION:
        raise ValueError("SmoothQuant profile uses an unrecognized source revision")
    records = profile.get("linears", {})
    if not records or records.keys() - sites.keys():
        raise ValueError("SmoothQuant profile has no sites or unsupported projection names")
    bound = {}
    for names in projection_groups(sites, groups):
        present = [n for n in names if n in records]
        if not present:
            continue
        if len(present) != len(names):
            raise ValueError("SmoothQuant shared-input group has partial scales")
        shared = records[names[0]]["scale"]
        for name in names:
            module = sites[name][0]
            record = records[name]
            _check_scale(name, record["scale"], module)
            if not torch.equal(record["scale"], shared):
                raise ValueError("SmoothQuant shared-input consumers have different scales")
            if record.get("weight_sha256") != weight_digest(module.weight):
                raise ValueError(f"SmoothQuant profile weight mismatch: {name}")
        on_device = shared.to(device=sites[names[0]][0].weight.device).contiguous()
        for name in names:
            bound[name] = on_device
    evidence = {
        "schema": PROFILE_SCHEMA,
        "upstream_revision": UPSTREAM_REVISION,
        "profile_sha256": hashlib.sha256(Path(path).read_bytes()).hexdigest(),
        "smoothed_linears": sorted(bound),
        "unsmoothed_linears": sorted(sites.keys() - bound.keys()),
        "calibration": profile.get("calibration", {}),
        "method": "FP32 channel balancing; BF16 rounding; divide fused into packing",
        "original_weights_modified": False,
        "task_quality_acceptance": "not_assessed",
    }
    return bound, evidence


def write_profile(path, sites, groups, calibration, precision, alpha=0.5):
    """Build a profile from an `ActivationCalibration`: one `channel_scales`
    per shared-input group (maxima of the group's first member, as piR2's
    tooling does), weight digests per site."""
    records = {}
    for names in projection_groups(sites, groups):
        if any(n not in calibration.maxima for n in names):
            continue
        scale = channel_scales(
            calibration.maxima[names[0]], [sites[n][0].weight for n in names], alpha
        ).cpu()
        for name in names:
            records[name] = {"scale": scale, "weight_sha256": weight_digest(sites[name][0].weight)}
    profile = {
        "schema": PROFILE_SCHEMA,
        "upstream_revision": UPSTREAM_REVISION,
        "precision": precision,
        "linears": records,
        "calibration": {"alpha": alpha, "calls": dict(calibration.calls)},
    }
    torch.save(profile, path)
    return profile
