"""Runs the reference's own CUDA kernels (built from its sources for sm_100a
by oracle/ref_build.py into oracle/_ref/) on cases from an .npz file, in a
process of its own: the reference registers the torch op namespace
`pir2_integer_dispatch`, which pir2_b200.torch_ops also registers.  Test
infrastructure only.

usage: python tests/reference_runner.py <cases.npz> <out.npz> [--time]

A case `c<i>_kind` is "prepare" (c<i>_x bf16 bits as uint16 [m, k],
optional c<i>_lut / c<i>_up, c<i>_bits) -> c<i>_q, c<i>_s; or "gemv"
(c<i>_a uint8 [1, k/2], c<i>_sa, c<i>_b uint8 [n, k/2], c<i>_sb, c<i>_bias
bits) -> c<i>_y (bf16 bits).  With --time each case is also launched 200
times back to back inside one CUDA graph and c<i>_us holds the median
per-launch device time of 5 replays (CUDA events)."""

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")


def bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def timed(fn):
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


def main():
    cases, out_path = sys.argv[1], sys.argv[2]
    time_it = "--time" in sys.argv[3:]
    for name in ("ref_integer_dispatch", "ref_int4_gemv"):
        torch.ops.load_library(os.path.join(REF, name, name + ".so"))
    data = dict(np.load(cases))
    out = {}
    i = 0
    while f"c{i}_kind" in data:
        kind = str(data[f"c{i}_kind"])
        if kind == "prepare":
            x = bf16(data[f"c{i}_x"])
            lut = bf16(data[f"c{i}_lut"]) if f"c{i}_lut" in data else None
            up = bf16(data[f"c{i}_up"]) if f"c{i}_up" in data else None
            bits = int(data[f"c{i}_bits"])
            fn = lambda: torch.ops.pir2_integer_dispatch.prepare(x, lut, up, bits)  # noqa: E731
            q, s = fn()
            out[f"c{i}_q"] = q.cpu().numpy().view(np.uint8)
            out[f"c{i}_s"] = s.cpu().numpy()
        elif kind == "gemv":
            a = torch.from_numpy(data[f"c{i}_a"]).cuda()
            sa = torch.from_numpy(data[f"c{i}_sa"]).cuda()
            b = torch.from_numpy(data[f"c{i}_b"]).cuda()
            sb = torch.from_numpy(data[f"c{i}_sb"]).cuda()
            bias = bf16(data[f"c{i}_bias"]) if f"c{i}_bias" in data else None
            fn = lambda: torch.ops.pir2_int4_gemv.gemv(a, sa, b, sb, bias, 4, bias is None)  # noqa: E731
            y = fn()
            out[f"c{i}_y"] = y.cpu().view(torch.int16).numpy().view(np.uint16)
        else:
            raise SystemExit(f"unknown case kind {kind}")
        if time_it:
            out[f"c{i}_us"] = np.float64(timed(fn))
        torch.cuda.synchronize()
        i += 1
    np.savez(out_path, **out)


if __name__ == "__main__":
    main()
