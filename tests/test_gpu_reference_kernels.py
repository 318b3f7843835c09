"""Parity with the reference's OWN CUDA kernels, run on the same B200.

oracle/ref_build.py compiles the reference's CUTLASS-free kernels of this
path from their sources (sm_100a, the reference's flags) into oracle/_ref/:
  * `pir2_integer_dispatch::prepare` (coexecution/kernels/ampere_ada/csrc/
    integer_dispatch.cu:11-108), the native per-row activation pack the
    reference dispatches to on a CUDA device;
  * `pir2_int4_gemv::gemv` (int4_gemv.cu:23-126), its exact single-row INT4
    GEMV.
They run in a subprocess (tests/reference_runner.py) because the reference
registers the op namespace `pir2_integer_dispatch`, as pir2_b200.torch_ops
does.  Our kernels are called through the C ABI and compared bit for bit.
"""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBS = [os.path.join(ROOT, "oracle", "_ref", n, n + ".so") for n in ("ref_integer_dispatch", "ref_int4_gemv")]
RUNNER = os.path.join(ROOT, "tests", "reference_runner.py")

if not all(os.path.exists(p) for p in LIBS):
    pytest.skip("reference kernels not built (python -m oracle.ref_build <reference checkout>)",
                allow_module_level=True)


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def run_reference(tmp_path, cases, time_it=False):
    """cases: list of dicts with 'kind' and arrays; returns the runner's
    outputs as a list of dicts (suffixes without the c<i>_ prefix)."""
    flat = {}
    for i, case in enumerate(cases):
        for key, value in case.items():
            flat[f"c{i}_{key}"] = value
    src, dst = str(tmp_path / "cases.npz"), str(tmp_path / "out.npz")
    np.savez(src, **flat)
    args = [sys.executable, RUNNER, src, dst] + (["--time"] if time_it else [])
    proc = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    got = dict(np.load(dst))
    return [{k.split("_", 1)[1]: v for k, v in got.items() if k.startswith(f"c{i}_")} for i in range(len(cases))]


def device_lut(kind):
    values = torch.arange(65536, device="cuda", dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    return torch.nn.functional.silu(values) if kind == "silu" else torch.nn.functional.gelu(values, approximate=kind)


PACK_SHAPES = [(1, 2048), (17, 1536), (17, 6144), (64, 130), (544, 2048), (3, 8192)]


@pytest.mark.parametrize("bits", [8, 4])
def test_pack_bitwise_vs_reference_native_prepare(tmp_path, bits):
    """Plain, GELU-table and SiLU-gated packs of our quant_rows kernels equal
    the reference's native `prepare` (integer_dispatch.cu) byte for byte:
    codes, int4 nibbles and fp32 scales, incl. zero rows and K padding."""
    g = torch.Generator().manual_seed(bits)
    gelu, silu = device_lut("tanh"), device_lut("silu")
    cases, ours = [], []
    for m, k in PACK_SHAPES:
        x = torch.randn(m, k, generator=g)
        x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20.0
        x[0] = 0.0   # an all-zero row: scale 1.0
        x = x.to(torch.bfloat16)
        up = torch.randn(m, k, generator=g).to(torch.bfloat16)
        for mode in ("plain", "lut", "gated"):
            case = {"kind": np.array("prepare"), "x": bits_of(x), "bits": np.int64(bits)}
            lut = None if mode == "plain" else (gelu if mode == "lut" else silu)
            if lut is not None:
                case["lut"] = bits_of(lut)
            if mode == "gated":
                case["up"] = bits_of(up)
            cases.append(case)
            q, s = ops.quant_rows(x.cuda(), bits, lut=lut, up=up.cuda() if mode == "gated" else None)
            ours.append((q.cpu().numpy().view(np.uint8), s.cpu().numpy(), (m, k, mode)))
    refs = run_reference(tmp_path, cases)
    for (q, s, what), ref in zip(ours, refs):
        assert np.array_equal(s.view(np.uint32), ref["s"].view(np.uint32)), what
        assert np.array_equal(q, ref["q"]), what


@pytest.mark.parametrize("bias", [True, False])
def test_int4_single_row_gemm_bitwise_vs_reference_gemv(tmp_path, bias):
    """W4A4 with one token row: our tcgen05 GEMM (int4 kernel) equals the
    reference's exact INT4 GEMV (int4_gemv.cu) bit for bit, with the bias
    (piR2 `gemm`) and without it (`gemm_biasless`)."""
    g = torch.Generator().manual_seed(7 + bias)
    cases, ours = [], []
    for k, n in ((1536, 1536), (1536, 6144), (2048, 4096), (6144, 2048), (1536, 52224)):
        x = torch.randn(1, k, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), 4)
        qa, sa = ops.quant_rows(x.cuda(), 4)
        b = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if bias else None
        case = {"kind": np.array("gemv"), "a": qa.cpu().numpy().view(np.uint8), "sa": sa.cpu().numpy(),
                "b": np.ascontiguousarray(qw), "sb": np.ascontiguousarray(sw)}
        if bias:
            case["bias"] = bits_of(b)
        cases.append(case)
        y = ops.gemm(qa, sa, torch.from_numpy(qw).cuda(), torch.from_numpy(sw).cuda(),
                     b.cuda() if bias else None, 4, bias_mode=None if bias else _lib.BIAS_NONE)
        ours.append((bits_of(y), (k, n)))
    refs = run_reference(tmp_path, cases)
    for (y, what), ref in zip(ours, refs):
        mismatch = np.argwhere(y != ref["y"])
        assert mismatch.size == 0, f"{what}: {len(mismatch)} mismatches, first {mismatch[:4].tolist()}"


def _timed(fn):
    """Device time per launch: 200 launches captured in one CUDA graph,
    median of 5 replays (CUDA events), so host call overhead is excluded."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(200):
            fn()
    times = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / 200)
    return sorted(times)[2]


def test_reference_kernel_timings(tmp_path, capsys):
    """Times our kernels and the reference's own ones on the same inputs
    (200 launches captured in one CUDA graph, median of 5 replays, CUDA
    events: device time, host call overhead excluded) and prints one JSON
    line per case.  Reports only; correctness is pinned by the tests above."""
    import json

    g = torch.Generator().manual_seed(3)
    cases, ours, labels = [], [], []
    for m, k in ((17, 1536), (17, 6144), (544, 2048), (544, 6144)):
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        cases.append({"kind": np.array("prepare"), "x": bits_of(x), "bits": np.int64(8)})
        xd = x.cuda()
        ours.append(_timed(lambda: ops.quant_rows(xd, 8)))   # noqa: B023
        labels.append({"op": "W8 activation pack", "m": m, "k": k})
    for k, n in ((1536, 1536), (1536, 6144), (6144, 1536)):
        x = torch.randn(1, k, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), 4)
        qa, sa = ops.quant_rows(x.cuda(), 4)
        b = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
        cases.append({"kind": np.array("gemv"), "a": qa.cpu().numpy().view(np.uint8), "sa": sa.cpu().numpy(),
                      "b": np.ascontiguousarray(qw), "sb": np.ascontiguousarray(sw), "bias": bits_of(b)})
        wd, swd, bd = torch.from_numpy(qw).cuda(), torch.from_numpy(sw).cuda(), b.cuda()
        ours.append(_timed(lambda: ops.gemm(qa, sa, wd, swd, bd, 4)))   # noqa: B023
        labels.append({"op": "W4A4 GEMM, one token row", "m": 1, "k": k, "n": n})
    refs = run_reference(tmp_path, cases, time_it=True)
    with capsys.disabled():
        for label, us, ref in zip(labels, ours, refs):
            print(json.dumps({**label, "ours_us": round(us, 2), "reference_us": round(float(ref["us"]), 2)}))
