"""GPU-free contract tests of the plugin surface (configuration, tactics,
inventory, session guards, benchmark helpers), in the manner of piR2's
tests/contracts/test_groot_optimization.py."""

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from pir2_b200 import harness
from pir2_b200.config import OptimizationConfig, add_optimization_arguments, optimization_config
from pir2_b200.projections import inventory
from pir2_b200.session import GrootOptimizations, selected_component
from pir2_b200.tactics import apply_tactics, read_shape_tactics

ROOT = Path(__file__).resolve().parents[1]
# A checkout of the piR2 repository, for the test that loads its shipped
# configuration presets (skipped when the variable is unset).
REFERENCE = Path(os.environ["PIR2_REFERENCE"]) if os.environ.get("PIR2_REFERENCE") else None


# ----------------------------------------------------------------- config
def test_default_config_is_disabled():
    assert not OptimizationConfig().enabled
    assert OptimizationConfig(precision="w8a8").enabled


@pytest.mark.parametrize(
    "kwargs,match",
    [
        ({"precision": "int3"}, "Precision"),
        ({"action_kv_reuse": True}, "action-cuda-graph"),
        ({"fp_smoothquant": Path("x.pt"), "precision": "w8a8"}, "SmoothQuant"),
        ({"fp4_swap_ab": True, "precision": "w8a8"}, "Swap-AB"),
        ({"group_conditioning": True, "precision": "w8a8"}, "Condition grouping"),
        ({"norm_modulation_quant": True, "precision": "w8a8"}, "Norm quantization"),
        ({"residual_norm_quant": True}, "Residual fusion"),
        ({"category_id": 1, "scope": "transformer"}, "scope=all"),
        ({"precision": "fp4", "group_conditioning": True, "fusion": True, "scope": "all"}, "Floating precision"),
        ({"fusion_mode": "rope"}, "Selective mode"),
        ({"scope": "everything"}, "scope"),
        ({"component": "vlm", "category_id": 0, "scope": "all"}, "DiT component"),
    ],
)
def test_invalid_configurations_are_rejected(kwargs, match):
    with pytest.raises(ValueError, match=match):
        OptimizationConfig(**kwargs)


def test_cli_flags_round_trip():
    parser = argparse.ArgumentParser()
    add_optimization_arguments(parser)
    args = parser.parse_args(
        [
            "--inference-precision", "w4a4", "--operator-fusion", "--quantization-scope", "all",
            "--group-conditioning", "--norm-modulation-quant", "--residual-norm-quant",
        ]
    )
    config = optimization_config(args)
    assert config.precision == "w4a4" and config.group_conditioning and config.residual_norm_quant


def test_selected_component():
    assert selected_component("backbone.layers.0.mlp.up_proj", "vlm")
    assert not selected_component("action_head.model.proj_out_1", "vlm")
    assert selected_component("action_head.model.proj_out_1", "dit")
    with pytest.raises(ValueError):
        selected_component("x", "both")


# ----------------------------------------------------------------- tactics
def test_explicit_tactics_and_group_defaults(tmp_path):
    linears, groups = tmp_path / "tactics.json", tmp_path / "groups.json"
    linears.write_text(json.dumps({"8": {"q": 3}, "4": {"q": 6}}))
    groups.write_text(json.dumps([{"bits": 8, "members": ["q", "k", "v"], "tactic": 2}]))
    quant = {bits: {"q": SimpleNamespace(tactic=0)} for bits in (8, 4)}
    grouped = {bits: [(["q", "k", "v"], SimpleNamespace(linear=SimpleNamespace(tactic=7)))] for bits in (8, 4)}
    controller = SimpleNamespace(quant=quant, grouped=grouped)
    extra = SimpleNamespace(quant={8: {}, 4: {}})
    config = OptimizationConfig(tactics=linears, group_tactics=groups)
    apply_tactics(controller, extra, config, {})
    assert [quant[b]["q"].tactic for b in (8, 4)] == [3, 6]
    assert [grouped[b][0][1].linear.tactic for b in (8, 4)] == [2, 0]
    groups.write_text(json.dumps([{"bits": 8, "members": ["q", "k", "v"], "tactic": 8}]))
    with pytest.raises(ValueError, match="tactic"):
        apply_tactics(controller, extra, config, {})


@pytest.mark.parametrize(
    "row",
    [
        {"bits": True, "shape": [41, 130, 64, True], "tactic": 2},
        {"bits": 8, "shape": [True, 130, 64, True], "tactic": 2},
        {"bits": 8, "shape": [41, 0, 64, True], "tactic": 2},
        {"bits": 8, "shape": [41, 130, 64, 1], "tactic": 2},
        {"bits": 8, "shape": [41, 130, 64, True], "tactic": 8},
    ],
)
def test_shape_tactics_reject_invalid_signatures(tmp_path, row):
    path = tmp_path / "shapes.json"
    path.write_text(json.dumps([row]))
    with pytest.raises(ValueError):
        read_shape_tactics(path)


def test_shape_tactics_reject_duplicates_and_unbound_profiles(tmp_path):
    path = tmp_path / "shapes.json"
    row = {"bits": 8, "shape": [41, 130, 64, True], "tactic": 2}
    path.write_text(json.dumps([row, row]))
    with pytest.raises(ValueError, match="Duplicate"):
        read_shape_tactics(path)
    profile = {
        "schema_version": 1, "backend_id": "pir2_integer", "backend_revision": "abc",
        "device_arch": "sm_100a", "quant_format": "w8a8-symmetric-row-v1", "rows": [row],
    }
    path.write_text(json.dumps(profile))
    with pytest.raises(ValueError, match="evidence"):
        read_shape_tactics(path)
    evidence = {k: profile[k] for k in ("backend_id", "backend_revision", "device_arch", "quant_format")}
    assert read_shape_tactics(path, backend_evidence=evidence) == {(8, 41, 130, 64, True): 2}


@pytest.mark.skipif(REFERENCE is None or not REFERENCE.exists(), reason="PIR2_REFERENCE not set")
def test_reference_presets_load_through_the_public_tactic_interface():
    preset = REFERENCE / "configs/quantization/groot-libero10-ada"
    coverage = json.loads((preset / "coverage.json").read_text())["linears"]
    singles = json.loads((preset / "tactics.json").read_text())
    controller = SimpleNamespace(
        quant={bits: {name: SimpleNamespace(tactic=-1) for name in coverage} for bits in (8, 4)},
        grouped={8: [], 4: []},
    )
    extra = SimpleNamespace(quant={8: {}, 4: {}})
    config = OptimizationConfig(tactics=preset / "tactics.json", group_tactics=preset / "group-tactics.json")
    apply_tactics(controller, extra, config, coverage)
    assert all(q.tactic in range(8) for q in controller.quant[8].values() if q.tactic != -1)
    assert set(coverage) <= set(singles["8"])
    spatial = REFERENCE / "configs/quantization/groot-libero-spatial-ada/w8-shape-tactics.json"
    assert len(read_shape_tactics(spatial)) > 0


# ----------------------------------------------------------------- inventory / session
def tiny_policy():
    return harness.build_policy(
        "cpu", vlm=harness.VLMConfig(layers=2, vocab=256), dit=harness.DiTConfig(layers=2)
    )


def test_inventory_roles_groups_and_scopes():
    policy = tiny_policy()
    sites, groups, activations, text = inventory(policy, expanded=False)
    roles = {name: role for name, (_, role, _) in sites.items()}
    assert roles["backbone.layers.0.self_attn.q_proj"] == "AttnQ"
    assert roles["backbone.layers.1.mlp.down_proj"] == "FFNdown"
    assert roles["action_head.model.transformer_blocks.0.ff.net.2"] == "FFNdown"
    assert sites["action_head.model.transformer_blocks.1.attn1.to_q"][2] == "dit"
    # cross-attention blocks group only k|v; self-attention q|k|v
    assert ["action_head.model.transformer_blocks.0.attn1.to_k", "action_head.model.transformer_blocks.0.attn1.to_v"] in groups
    assert any(len(g) == 3 and g[0].endswith("transformer_blocks.1.attn1.to_q") for g in groups)
    assert len(activations) == 2 and len(text) == 2
    expanded = inventory(policy, expanded=True)[0]
    extra = set(expanded) - set(sites)
    assert "action_head.model.proj_out_1" in extra and "action_head.state_encoder" in extra
    assert all(expanded[n][1] == "AdditionalLinear" for n in extra)


def test_session_rejects_cpu_models_and_restores():
    policy = tiny_policy()
    session = GrootOptimizations(SimpleNamespace(model=policy), OptimizationConfig(precision="w8a8"))
    with pytest.raises(ValueError, match="CUDA"):
        session.__enter__()
    assert not session._active
    assert all("forward" not in m.__dict__ for m in policy.modules())


def test_disabled_session_is_a_no_op_and_evidence_hashes_files(tmp_path):
    path = tmp_path / "tactics.json"
    path.write_text(json.dumps({"8": {}, "4": {}}))
    config = OptimizationConfig(tactics=path)
    with GrootOptimizations(object(), config) as session:
        evidence = session.evidence()
    assert len(evidence["config"]["tactics"]["sha256"]) == 64


# ----------------------------------------------------------------- benchmark helpers
def _gloo_worker(rank, world, port, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, str(ROOT))
    import bench

    bench.barrier(world)
    value = bench.max_over_ranks(float(rank + 1) * 1.5, world)
    queue.put((rank, value))
    dist.destroy_process_group()


def test_bench_rank_reduction_over_gloo():
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: 3.0, 1: 3.0}


def test_bench_reference_arm_prints_the_contract_line():
    # OMP_NUM_THREADS=1 as torchrun sets it: the arm still uses every core.
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--cpu-sample-seconds", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT, env={**os.environ, "OMP_NUM_THREADS": "1"},
    )
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "impl", "cpu_baseline", "e2e", "higher_is_better", "config"):
        assert key in line
    assert line["impl"] == "reference" and line["higher_is_better"] is False
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_bench_reference_arm_under_torchrun_prints_one_line():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = subprocess.run(
        [
            sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
            "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
            "--impl", "reference", "--gpus", "2", "--steps", "1", "--cpu-sample-seconds", "1",
        ],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(s) for s in out.stdout.splitlines() if s.startswith("{")]
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2
    assert lines[0]["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))


def test_bench_algorithmic_bytes_per_gemm():
    sys.path.insert(0, str(ROOT))
    import bench

    # M=17 K=1536 N=6144 W8A8: weights, codes, row and channel scales, output.
    s = dict(bits=8, m=17, n=6144, k=1536, npad=6144)
    assert bench.gemm_bytes(s) == 9437184 + 26112 + 68 + 24576 + 208896
    # The residual epilogue also reads a bf16 [m, n] tile.
    assert bench.gemm_bytes(dict(s, residual=True)) == bench.gemm_bytes(s) + 2 * 17 * 6144
    # W4A4: half a byte per operand value.
    assert bench.gemm_bytes(dict(s, bits=4)) == 9437184 // 2 + 26112 // 2 + 68 + 24576 + 208896
    # A bias vector is read once.
    assert bench.gemm_bytes(dict(s, bias=True)) == bench.gemm_bytes(s) + 2 * 6144
    # SwiGLU multiplies gate and up rows but writes half the columns.
    g = dict(bits=8, m=544, n=12288, k=2048, npad=12288, out_n=6144)
    assert bench.gemm_bytes(g) == 12288 * 2048 + 544 * 2048 + 4 * 544 + 4 * 12288 + 2 * 544 * 6144
    # E4M3: one byte per value and replicated fp32 scales, as int8.
    assert bench.gemm_bytes(dict(s, bits="fp8")) == bench.gemm_bytes(s)
    # NVFP4: half a byte per value plus one UE4M3 factor per 16 values.
    f = dict(bits="fp4", m=17, n=6144, k=1536, npad=6144)
    assert bench.gemm_bytes(f) == (6144 + 17) * 1536 // 2 + (6144 + 17) * 1536 // 16 + 2 * 17 * 6144
