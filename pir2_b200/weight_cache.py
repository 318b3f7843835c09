"""Versioned on-disk cache of packed symmetric-row-v1 weights.

Installation quantizes every executed projection twice (8 and 4 bits,
`quantize_weight`, the install-time step of coexecution/kernels/ampere_ada/
integer.py:211-256).  `save` writes those packed tensors, keyed by site
name, to one `torch.save` file; `load` reads them back for a model whose
projection weights are unchanged, so `TransformerINT(..., packed=...)`
builds its layers without quantizing.  The cache is rejected (ValueError)
when the format, the library's format version, a site's shape or a site's
weight fingerprint does not match: a stale cache can never be used silently.

File layout (a dict):
  format: "pir2b.packed-weights"; version: 1; weight_format: "symmetric-row-v1"
  sites: {name: {"in_features", "out_features", "bias": bool,
                 "fingerprint": [int, int, int],
                 "8": {"packed_weight", "weight_scale", "bias"},
                 "4": {...}}}
Tensors are stored on the CPU; `load` moves them to the requested device.
"""

from pathlib import Path

import torch

from .integer import FORMAT_VERSION

CACHE_FORMAT = "pir2b.packed-weights"
CACHE_VERSION = 1


def fingerprint(weight):
    """Exact integer digest of a bf16 weight tensor computed on its device:
    [element count, sum of the 16-bit patterns, position-weighted sum]."""
    bits = weight.detach().contiguous().view(torch.int16).reshape(-1).to(torch.int64)
    position = torch.arange(bits.numel(), device=bits.device, dtype=torch.int64) % 65521 + 1
    return [int(bits.numel()), int(bits.sum().item()), int((bits * position).sum().item())]


def save(controller, path):
    """Writes the packed 8- and 4-bit weights of a TransformerINT."""
    sites = {}
    for name, (module, _, _) in controller.sites.items():
        entry = {
            "in_features": module.in_features,
            "out_features": module.out_features,
            "bias": module.bias is not None,
            "fingerprint": fingerprint(module.weight),
        }
        for bits in (8, 4):
            q = controller.quant[bits][name]
            entry[str(bits)] = {
                "packed_weight": q.packed_weight.detach().cpu(),
                "weight_scale": q.weight_scale.detach().cpu(),
                "bias": None if q.bias is None else q.bias.detach().cpu(),
            }
        sites[name] = entry
    payload = {
        "format": CACHE_FORMAT,
        "version": CACHE_VERSION,
        "weight_format": FORMAT_VERSION,
        "sites": sites,
    }
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    torch.save(payload, tmp)
    tmp.replace(path)


def load(path, modules, device):
    """Reads a cache written by `save` for the given {site name: Linear}.

    Returns {site name: {bits: (packed_weight, weight_scale, bias)}} on
    `device`.  Raises ValueError when the cache does not belong to these
    weights (format, version, missing site, shape or fingerprint)."""
    payload = torch.load(Path(path), map_location="cpu", weights_only=True)
    if not isinstance(payload, dict) or payload.get("format") != CACHE_FORMAT:
        raise ValueError("Not a packed-weight cache")
    if payload.get("version") != CACHE_VERSION or payload.get("weight_format") != FORMAT_VERSION:
        raise ValueError("Packed-weight cache version does not match this library")
    sites = payload.get("sites", {})
    out = {}
    for name, module in modules.items():
        entry = sites.get(name)
        if entry is None:
            raise ValueError(f"Packed-weight cache has no entry for {name}")
        if (
            entry["in_features"] != module.in_features
            or entry["out_features"] != module.out_features
            or entry["bias"] != (module.bias is not None)
        ):
            raise ValueError(f"Packed-weight cache shape mismatch for {name}")
        if entry["fingerprint"] != fingerprint(module.weight):
            raise ValueError(f"Packed-weight cache is stale for {name} (weights changed)")
        out[name] = {
            bits: tuple(
                None if entry[str(bits)][key] is None else entry[str(bits)][key].to(device)
                for key in ("packed_weight", "weight_scale", "bias")
            )
            for bits in (8, 4)
        }
    return out
