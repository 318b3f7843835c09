"""Integer tactic files (configs/quantization/**) and their assignment.

Loads the reference's three tactic formats (coexecution/optimization/
tactics.py:8-121) with the same validation errors:

* site tactics: {"8": {site: id}, "4": {...}};
* group tactics: rows {"bits", "members", "tactic"}, or legacy rows
  {"bits", "shape", "tactic"} matched by the group's [rows, K, N, bias]
  signature from the coverage file;
* shape tactics: a row list [{"bits", "shape": [M, K, N, bias], "tactic"}],
  or a schema_version-1 profile that must match the running backend.

On B200 a tactic id is validated and recorded on its projection
(`.tactic`, `.shape_tactics`), but the tcgen05 GEMM plans its tiles from
M, N and K on every call, so no tactic changes a result; piR2 has the same
rule (a tactic selects a kernel, never the bytes).
"""

import json
import math
from pathlib import Path

_PROFILE_FIELDS = ("backend_id", "backend_revision", "device_arch", "quant_format")
_PROFILE_BITS = {"w8a8-symmetric-row-v1": 8, "w4a4-symmetric-row-v1": 4}


def read_json(path, default):
    """The parsed file, or `default` when no path is configured."""
    if path is None:
        return default
    return json.loads(Path(path).read_text())


def checked_tactic(value):
    if type(value) is int and 0 <= value <= 7:
        return value
    raise ValueError("Integer tactic must be an integer in [0, 7]")


def _profile_rows(profile, backend_evidence):
    """Validates a shape-tactic profile against the running backend and
    returns (its rows, the bits its quant_format implies)."""
    if profile.get("schema_version") != 1 or type(profile.get("schema_version")) is not int:
        raise ValueError("Shape tactic profile schema_version must be 1")
    if not all(isinstance(profile.get(field), str) and profile[field] for field in _PROFILE_FIELDS):
        raise ValueError("Shape tactic profile requires backend/revision/architecture/format metadata")
    if backend_evidence is None:
        raise ValueError("Shape tactic profiles require runtime backend evidence")
    for field in _PROFILE_FIELDS:
        running = backend_evidence.get(field)
        if running in (None, "unknown") or running != profile[field]:
            raise ValueError(f"Shape tactic profile {field} does not match the runtime backend")
    if profile["backend_id"] != "pir2_integer":
        raise ValueError("Integer shape tactics require the pir2_integer backend")
    bits = _PROFILE_BITS.get(profile["quant_format"])
    if bits is None:
        raise ValueError("Unsupported integer shape tactic quant_format")
    return profile.get("rows"), bits


def _shape_key(row):
    """(bits, M, K, N, bias) of one shape-tactic row, validated."""
    bits, shape = row["bits"], row["shape"]
    valid = (
        type(bits) is int
        and bits in (4, 8)
        and isinstance(shape, list)
        and len(shape) == 4
        and all(type(size) is int and size > 0 for size in shape[:3])
        and type(shape[3]) is bool
    )
    if not valid:
        raise ValueError("Expected bits 4/8 and shape [positive M, K, N, bool bias]")
    return (bits, *shape)


def read_shape_tactics(path, *, backend_evidence=None):
    """{(bits, M, K, N, bias): tactic} from a shape-tactic file."""
    content = read_json(path, [])
    rows, profile_bits = content, None
    if isinstance(content, dict):
        rows, profile_bits = _profile_rows(content, backend_evidence)
    if not isinstance(rows, list):
        raise TypeError("Shape tactics must contain a JSON row list")
    table = {}
    for row in rows:
        key = _shape_key(row)
        if profile_bits is not None and key[0] != profile_bits:
            raise ValueError("Shape tactic bits do not match the profile quant_format")
        if key in table:
            raise ValueError("Duplicate integer shape tactic")
        table[key] = checked_tactic(row["tactic"])
    return table


def _group_tactic(rows, bits, names, linear, coverage):
    """The tactic of one projection group: rows naming its members, else
    legacy rows matching its [rows, K, N, bias] signature; 0 when none."""
    chosen = {checked_tactic(r["tactic"]) for r in rows if r["bits"] == bits and r.get("members") == list(names)}
    if not chosen:
        legacy = [r for r in rows if r["bits"] == bits and "shape" in r]
        if legacy and names[0] in coverage:
            lead = coverage[names[0]]["shape"][:-1]
            signature = [math.prod(lead), linear.in_features, linear.out_features, linear.bias is not None]
            chosen = {checked_tactic(r["tactic"]) for r in legacy if r["shape"] == signature}
    if len(chosen) > 1:
        raise ValueError("Conflicting grouped tactics")
    return chosen.pop() if chosen else 0


def apply_tactics(controller, extra, config, coverage, *, backend_evidence=None):
    """Records the configured tactic ids on the installed projections
    (`controller`: TransformerINT, `extra`: AdditionalConnections)."""
    shapes = None
    if config.shape_tactics is not None:
        shapes = read_shape_tactics(config.shape_tactics, backend_evidence=backend_evidence)
    singles = read_json(config.tactics, {})
    group_rows = read_json(config.group_tactics, [])
    for bits in (8, 4):
        sites = {**controller.quant[bits], **extra.quant[bits]}
        for name, tactic in singles.get(str(bits), {}).items():
            if name in sites:
                sites[name].tactic = checked_tactic(tactic)
        for names, group in controller.grouped[bits]:
            group.linear.tactic = _group_tactic(group_rows, bits, names, group.linear, coverage)
    if shapes is None:
        return
    from .linear import install_shape_tactics

    for bits in (8, 4):
        projections = [*controller.quant[bits].values(), *extra.quant[bits].values()]
        projections += [group.linear for _, group in controller.grouped[bits]]
        for q in projections:
            install_shape_tactics(q, shapes)
