"""Benchmark: GR00T control-step latency (VLM prefill + 4-step DiT) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--precision w8a8|w4a4] [--batch B]

One step = one GR00T-shaped control step per robot: Qwen3-shaped 16-layer VLM
prefill over 544 tokens, then 4 Euler steps of the 16-block DiT, every
Linear layer on the W8A8 (or W4A4) tcgen05 kernels, the whole step replayed
from one CUDA graph.  Synthetic seeded inputs and random-init weights (no
checkpoints or datasets exist here).  With N GPUs each rank runs its own
robot(s) (independent instances, no collective: weak scaling); timing is
CUDA events on the step's stream, max over ranks.  Each step streams about
3.1 GB of packed weights and activations from DRAM (the DiT's weights once
per Euler step), far larger than the 126 MB L2, so no L2 flush is needed
between steps.

`--impl reference` times the reference's quantized-Linear arithmetic on the
host cores instead: piR2 has no CPU implementation of this path (its kernels
reject CPU tensors), so this is the CPU restatement in oracle/ (numpy
quantize + exact int GEMM + dequant epilogue, torch CPU for norms and
attention), over full, unscaled control steps: the whole policy is built on
the host, one untimed step runs, then steps are timed back to back until
--steps are done or --cpu-budget-seconds have passed (at least one); the
line reports the number of steps it actually timed.  The `cpu_baseline` of
our own arm's line is a bounded sample instead (one VLM layer and a
two-block DiT over the 4 Euler steps, scaled by layer counts), so the
default run stays within minutes; its `sample` field says so.
"""

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from types import SimpleNamespace

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "GR00T step latency ms (VLM+4-step DiT) B=1"
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
# int8 dense tensor peak measured on this pool's B200 by the kind::i8
# issue-rate probe (`bench.py --int8-peak`): 8190 MAC/clk/SM x 148 SMs,
# 4513 TOPS from CUDA events (the SMs averaged ~1.86 GHz over the probe;
# 4.76 POPS would need 1965 MHz throughout).
INT8_PEAK_TOPS = 4520.0
FP4_NOMINAL_TOPS = 9000.0
FP8_NOMINAL_TOPS = 4500.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--precision", choices=["w8a8", "w4a4", "fp4", "fp8"], default="w8a8")
    p.add_argument("--batch", type=int, default=1, help="robots per GPU")
    p.add_argument(
        "--robots",
        type=int,
        default=None,
        help="total robots sharded over the GPUs (batched config: B=64 -> 64/N per GPU, strong scaling)",
    )
    p.add_argument(
        "--batched-robots",
        type=int,
        default=64,
        help="robots of the batched record (split over the GPUs, strong scaling); 0 skips it",
    )
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--fp-shared-inputs", action="store_true",
                   help="fp8/fp4: sibling projections share one pack (fp_shared_inputs) instead of running as "
                        "one merged GEMM (fp_grouped, the default: 7.8 vs 8.3 ms fp8, 6.6 vs 6.7 ms fp4)")
    p.add_argument("--cpu-sample-seconds", type=float, default=20.0,
                   help="host time of the CPU baseline sample in our arm's line")
    p.add_argument("--cpu-budget-seconds", type=float, default=60.0,
                   help="--impl reference: timed full CPU steps stop after this long (at least one)")
    p.add_argument(
        "--kernel",
        metavar="M,K,N",
        help="time one quantized GEMM shape alone (for kernel profiling), not the step",
    )
    p.add_argument("--kernel-weights-mb", type=float, default=600.0, help="rotating weight copies for --kernel")
    p.add_argument("--sweep", action="store_true",
                   help="BASELINE configs 2/3: time every (precision, M, K, N) GEMM point against its roofline")
    p.add_argument("--kernel-residual", action="store_true", help="--kernel with the bf16 residual epilogue")
    p.add_argument("--int8-peak", action="store_true",
                   help="measure the int8 tensor-core issue rate (tcgen05 kind::i8 probe) behind INT8_PEAK_TOPS")
    p.add_argument("--step-gemms", action="store_true",
                   help="record the step's GEMM shapes, then launch every small-M (M <= 64) shape twice "
                        "inside the NVTX range pir2b_step_gemms (one-kernel ncu traffic captures)")
    return p.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value, world):
    """Maximum of a per-rank scalar (NCCL on GPUs, gloo on CPU ranks)."""
    if world == 1:
        return value
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks():
    try:
        with open(PEAKS_PATH) as f:
            data = json.load(f)
        return data["hbm_gbs"], "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file,
                stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        self.file.seek(0)
        mhz, max_mhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.file.name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max_mhz, "reasons": sorted(reasons), "samples": len(mhz)}


class GemmTimer:
    """Brackets every pir2b_gemm launch with CUDA events.  Used while
    capturing a separate graph of the step: the events become event-record
    nodes, so a replay times each GEMM on the device with no host gaps."""

    def __init__(self):
        self.records = []
        self._start = None

    def before(self, device):
        self._start = torch.cuda.Event(enable_timing=True, external=True)
        self._start.record(torch.cuda.current_stream(device))

    def after(self, device, **shape):
        end = torch.cuda.Event(enable_timing=True, external=True)
        end.record(torch.cuda.current_stream(device))
        self.records.append((self._start, end, shape))


def gemm_bytes(s):
    """Algorithmic HBM bytes of one recorded GEMM launch: each operand,
    scale vector, bias, residual and output once.  `n` is the weight rows the
    GEMM multiplies (gate and up for SwiGLU), `out_n` the bf16 columns it
    writes (half of them for SwiGLU)."""
    out = 2 * s["m"] * s.get("out_n", s["n"])
    res = 2 * s["m"] * s["n"] if s.get("residual") else 0
    res += 2 * s["npad"] if s.get("bias") else 0
    if s["bits"] == "fp4":
        # E2M1 operands (half a byte per value) + one UE4M3 factor per 16.
        return (s["n"] + s["m"]) * s["k"] * 9 // 16 + out + res
    if s["bits"] == "fp8":
        s = dict(s, bits=8)   # one byte per E4M3 value, like int8
    wb = s["npad"] * s["k"] * s["bits"] // 8
    if s.get("input") == "rows":
        # Fused pack: the GEMM reads the bf16 rows themselves.
        return wb + 2 * s["m"] * s["k_logical"] + 4 * s["npad"] + out + res
    return wb + s["m"] * s["k"] * s["bits"] // 8 + 4 * s["m"] + 4 * s["npad"] + out + res


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# small-M W8A8 GEMM, weighted over the step's 281 small-M launches: one-kernel
# ncu captures of every small-M shape of the step (`bench.py --step-gemms`;
# per-shape figures in profiles/gemm_small_m_step_shapes_traffic.md).
# None for the other precisions.
SMALL_M_TRAFFIC_BYTES = {"w8a8": 7234785}


def roofline(engine, hbm_peak, peak_kind, precision):
    """Times each GEMM launch of one step (a graph captured with event nodes
    around every GEMM, replayed once warm); reports the small-M GEMMs (the
    weight-streaming launches that dominate a B=1 step) against HBM and the
    large-M ones against the int8 tensor peak."""
    from pir2_b200 import ops

    timer = GemmTimer()
    graph = torch.cuda.CUDAGraph()
    ops.launch_recorder = timer
    try:
        with torch.inference_mode():
            with torch.cuda.graph(graph, stream=engine.stream):
                engine.policy(*engine.static)
    finally:
        ops.launch_recorder = None
    timer_records = list(timer.records)
    with torch.cuda.stream(engine.stream):
        graph.replay()
        graph.replay()
    engine.stream.synchronize()
    timer.records = timer_records
    small = {"t": 0.0, "bytes": 0.0, "n": 0}
    large = {"t": 0.0, "ops": 0.0, "n": 0}
    for start, end, s in timer.records:
        ms = start.elapsed_time(end)
        if s["m"] <= 64:
            small["t"] += ms
            small["bytes"] += gemm_bytes(s)
            small["n"] += 1
        else:
            large["t"] += ms
            large["ops"] += 2.0 * s["m"] * s["n"] * s["k"]
            large["n"] += 1
    total = small["t"] + large["t"]
    peak_tops = {"fp4": FP4_NOMINAL_TOPS, "fp8": FP8_NOMINAL_TOPS}.get(precision, INT8_PEAK_TOPS)
    achieved = small["bytes"] / (small["t"] * 1e-3) / 1e9 if small["t"] else 0.0
    tops = large["ops"] / (large["t"] * 1e-3) / 1e12 if large["t"] else 0.0
    in_step = {
        "method": "each GEMM of one step bracketed by CUDA-event nodes in a captured graph of the step "
                  "(the event nodes break programmatic dependent launch: about +5 us per small-M launch)",
        "achieved": round(achieved, 1),
        "frac": round(achieved / hbm_peak, 4),
        "avg_launch_us": round(small["t"] * 1e3 / max(small["n"], 1), 2),
        "large_m_achieved_tops": round(tops, 1),
        "large_m_frac": round(tops / peak_tops, 4),
    }
    if precision in ("w8a8", "w4a4"):
        chain_small, chain_large = chain_roofline([s for _, _, s in timer.records], precision, hbm_peak, peak_tops)
        achieved, small_avg = chain_small["achieved"], chain_small["avg_launch_us"]
        tops = chain_large["achieved_tops"]
        method = ("the step's GEMM shapes, each back to back in a CUDA graph over rotating weight copies "
                  "(weights from DRAM), weighted by launch count; CUDA events around the graph replays")
    else:
        small_avg = round(small["t"] * 1e3 / max(small["n"], 1), 2)
        method = in_step["method"]
    return {
        "_gemm_ms_small": small["t"],
        "kernel": {"fp4": "gemm_fp4_kernel",
                   "fp8": "gemm_few_kernel<9> (M<=32, e4m3 warp MMAs; gemm_i8_kernel<9> kind::f8f6f4 for 33-64 rows)"}.get(
            precision, f"gemm_few_kernel<{precision[1:2]}> (M<=32; gemm_i8_kernel for 33-64 rows)"
        )
        + " small-M (M<=64) launches",
        "bound": "hbm",
        "achieved": round(achieved, 1),
        "peak": hbm_peak,
        "unit": "GB/s",
        "frac": round(achieved / hbm_peak, 4),
        "peak_source": f"{peak_kind} hbm_gbs",
        "traffic": SMALL_M_TRAFFIC_BYTES.get(precision),
        "traffic_unit": "DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, one-kernel capture)",
        "algorithmic_bytes_per_launch": round(small["bytes"] / max(small["n"], 1)),
        "launches": small["n"],
        "avg_launch_us": small_avg,
        "method": method,
        "in_step_event_timed": in_step,
        "share_of_gemm_time": round(small["t"] / total, 3) if total else None,
        "large_m": {
            "kernel": "gemm_pair_kernel (2-SM tiles) where the planner picks them, else gemm_i8_kernel"
            if precision in ("w8a8", "w4a4") else None,
            "bound": "tensor",
            "launches": large["n"],
            "achieved_tops": round(tops, 1),
            "peak_tops": peak_tops,
            "frac": round(tops / peak_tops, 4),
            "peak_source": {
                "fp4": "nominal dense FP4 (no measured FP4 peak)",
                "fp8": "nominal dense FP8 (no measured FP8 peak)",
            }.get(precision, "measured int8 kind::i8 issue-rate probe"),
        },
    }


def chain_roofline(records, precision, hbm_peak, peak_tops, weights_mb=300.0, warmup=3):
    """The step's integer GEMM launches re-timed without event nodes: every
    distinct shape (M, K, N, epilogue) runs back to back in a CUDA graph over
    rotating weight copies (weights streamed from DRAM, as in the step),
    weighted by its launch count in the step.  Returns (small-M: algorithmic
    bytes / time, large-M: 2MNK / time) as dicts."""
    from collections import Counter

    from pir2_b200 import ops

    counts = Counter(
        (s["bits"], s["m"], s["k"], s["npad"], s.get("out_n", s["n"]), s["n"], bool(s.get("residual")),
         bool(s.get("bias")))
        for s in records
        if s["bits"] in (4, 8) and s.get("input") != "rows"
    )
    small = {"t": 0.0, "bytes": 0.0, "n": 0}
    large = {"t": 0.0, "ops": 0.0, "n": 0}
    g = torch.Generator(device="cuda").manual_seed(11)
    for (b, m, k, npad, out_n, n, residual, bias), count in counts.items():
        swiglu = out_n != n
        cols = k if b == 8 else k // 2
        dtype = torch.int8 if b == 8 else torch.uint8
        lo, hi = (-127, 128) if b == 8 else (0, 256)
        copies = max(1, min(32, int(weights_mb * 1e6 // (npad * cols))))
        ws = [torch.randint(lo, hi, (npad, cols), device="cuda", dtype=dtype, generator=g) for _ in range(copies)]
        qa = torch.randint(lo, hi, (m, cols), device="cuda", dtype=dtype, generator=g)
        sa = torch.rand(m, device="cuda", generator=g)
        sw = torch.rand(npad, device="cuda", generator=g)
        bvec = torch.zeros(npad, device="cuda", dtype=torch.bfloat16) if bias else None
        res = torch.zeros(m, out_n, device="cuda", dtype=torch.bfloat16) if residual else None
        out = torch.empty(m, out_n, device="cuda", dtype=torch.bfloat16)
        if swiglu:
            from pir2_b200.fused import prepare_silu

            lut = prepare_silu(torch.device("cuda"))
            launch = lambda i: ops.gemm_swiglu(qa, sa, ws[i % copies], sw, bvec, lut, half_n=out_n, out=out)  # noqa: E731
        else:
            launch = lambda i: ops.gemm(qa, sa, ws[i % copies], sw, bvec, b, n_store=out_n, out=out,  # noqa: E731
                                        residual=res)
        us = _time_graph_launches(launch, max(copies, 16), warmup)
        shape = {"bits": b, "m": m, "k": k, "n": n, "npad": npad, "out_n": out_n, "residual": residual,
                 "bias": bias}
        if m <= 64:
            small["t"] += count * us
            small["bytes"] += count * gemm_bytes(shape)
            small["n"] += count
        else:
            large["t"] += count * us
            large["ops"] += count * 2.0 * m * n * k
            large["n"] += count
        del ws
    torch.cuda.empty_cache()
    gbs = small["bytes"] / (small["t"] * 1e3) if small["t"] else 0.0
    tops = large["ops"] / (large["t"] * 1e6) if large["t"] else 0.0
    return (
        {"achieved": round(gbs, 1), "frac": round(gbs / hbm_peak, 4), "launches": small["n"],
         "avg_launch_us": round(small["t"] / max(small["n"], 1), 3),
         "algorithmic_bytes_per_launch": round(small["bytes"] / max(small["n"], 1))},
        {"achieved_tops": round(tops, 1), "frac": round(tops / peak_tops, 4), "launches": large["n"],
         "avg_launch_us": round(large["t"] / max(large["n"], 1), 3)},
    )


def workload_config(args, world):
    """The workload both arms report, identical between them: the per-GPU
    share of the robots (one control step each) and how they are spread."""
    return {
        "workload": f"GR00T-shaped control step per GPU, {args.batch} robot(s): VLM prefill 544 tokens x 16 layers + DiT 16 blocks x 4 Euler steps",
        "precision": args.precision,
        "batch_per_gpu": args.batch,
        "robots_total": args.batch * world,
        "parallelism": f"independent robots, dp{world}, no collective",
        "l2": "inputs larger than L2: each step streams ~3.1 GB of packed weights and activations (> 126 MB L2); no flush",
    }


# ------------------------------------------------------------------ CPU arm
def cpu_oracle_step(args, budget_s):
    """The reference's quantized-Linear arithmetic on the host cores, on a
    bounded sample: one VLM decoder layer (544 tokens) and a two-block DiT
    (one cross-, one self-attention block) through the 4 Euler steps, scaled
    to 16 layers / 16 blocks.  Returns (ms_per_step, cores, sample text)."""
    from threadpoolctl import threadpool_limits

    from oracle.model import install_oracle_linears
    from pir2_b200 import harness

    # Every host thread this process may run on, for torch and for numpy's
    # BLAS (torchrun starts ranks with OMP_NUM_THREADS=1, which would leave
    # the oracle's products on one thread).
    cores = len(os.sched_getaffinity(0)) or 1
    torch.set_num_threads(cores)
    with threadpool_limits(limits=cores, user_api="blas"):
        return _cpu_oracle_sample(args, budget_s, cores, install_oracle_linears, harness)


def _cpu_oracle_sample(args, budget_s, cores, install_oracle_linears, harness):
    vlm = harness.VLMConfig(layers=1, vocab=2048)
    dit = harness.DiTConfig(layers=2)
    policy = harness.build_policy("cpu", vlm=vlm, dit=dit)

    install_oracle_linears(policy, args.precision)
    visual, ids, state, noise = harness.synthetic_inputs(args.batch, "cpu", vlm=vlm, dit=dit)
    layer = policy.backbone.layers[0]
    with torch.inference_mode():
        h = torch.cat((visual, policy.backbone.embed_tokens(ids)), dim=1)
        cos, sin = policy.backbone.rope(h.shape[1], h.device, h.dtype)
        t_vlm, t_dit, reps = 0.0, 0.0, 0
        start = time.perf_counter()
        while reps == 0 or time.perf_counter() - start < budget_s:
            t0 = time.perf_counter()
            feat = layer(h, cos, sin)
            t1 = time.perf_counter()
            policy.action_head.get_action(feat, state, noise)
            t2 = time.perf_counter()
            t_vlm += t1 - t0
            t_dit += t2 - t1
            reps += 1
    full_ms = 1e3 * (16 * t_vlm / reps + 8 * t_dit / reps)
    sample = (
        f"{reps} x (1 VLM layer over 544 tokens + 2-block DiT x 4 Euler steps), batch {args.batch}, "
        f"oracle {args.precision.upper()} linears + torch CPU norms/attention, scaled x16 VLM layers / x8 DiT block pairs"
    )
    return full_ms, cores, sample


def cpu_full_steps(args, warmup, steps, budget_s):
    """Full, unscaled control steps of the reference's quantized-Linear
    arithmetic on the host cores: the whole policy (16 VLM layers, 16 DiT
    blocks, 4 Euler steps) with every Linear on the oracle, `warmup` untimed
    steps, then timed steps until `steps` are done or `budget_s` has passed
    (at least one).  Returns (ms_per_step, steps_timed, cores, seconds)."""
    from threadpoolctl import threadpool_limits

    from oracle.model import install_oracle_linears
    from pir2_b200 import harness

    cores = len(os.sched_getaffinity(0)) or 1
    torch.set_num_threads(cores)
    with threadpool_limits(limits=cores, user_api="blas"), torch.inference_mode():
        policy = harness.build_policy("cpu")
        install_oracle_linears(policy, args.precision)
        inputs = harness.synthetic_inputs(args.batch, "cpu")
        for _ in range(warmup):
            policy(*inputs)
        done, start = 0, time.perf_counter()
        while done < max(steps, 1):
            policy(*inputs)
            done += 1
            if time.perf_counter() - start >= budget_s:
                break
        elapsed = time.perf_counter() - start
    return 1e3 * elapsed / done, done, cores, elapsed


def run_reference(args, world, rank):
    if rank != 0:
        return
    warmup = min(args.warmup, 1)
    ms, done, cores, elapsed = cpu_full_steps(args, warmup, args.steps, args.cpu_budget_seconds)
    sample = (
        f"{done} full control step(s) timed back to back ({elapsed:.1f} s) after {warmup} untimed, batch "
        f"{args.batch}: the whole policy with every Linear on the oracle's {args.precision.upper()} "
        "arithmetic, torch CPU norms/attention; nothing scaled"
    )
    line = {
        "metric": METRIC,
        "value": round(ms, 3),
        "unit": "ms",
        "impl": "reference",
        "n_gpus": args.gpus,
        "steps": done,
        "warmup": warmup,
        "requested_steps": args.steps,
        "requested_warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "weak" if args.robots is None else "strong",
        "vs_baseline": None,
        "dtype": {"w8a8": "int8", "w4a4": "int4", "fp4": "e2m1", "fp8": "e4m3"}[args.precision],
        "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def build_engine(args, local):
    from pir2_b200 import harness
    from pir2_b200.config import OptimizationConfig
    from pir2_b200.engine import ControlStep
    from pir2_b200.session import GrootOptimizations

    device = torch.device("cuda", local)
    policy = harness.build_policy(device)
    if args.precision in ("fp4", "fp8"):
        # Every floating producer piR2 wires for fp8 / fp4: merged sibling
        # projections (or one pack per shared input), SwiGLU / GELU / RMSNorm
        # producers, the DiT LayerNorm + AdaLN and residual + LayerNorm
        # producers, the cross-attention kernel.
        config = OptimizationConfig(
            precision=args.precision, scope="all", fp_shared_inputs=args.fp_shared_inputs,
            fp_grouped=not args.fp_shared_inputs, fp_swiglu=True, fp_gelu=True, fp_rmsnorm=True, fusion=True,
            norm_modulation_quant=True, residual_norm_quant=True,
        )
    else:
        config = OptimizationConfig(
            precision=args.precision,
            fusion=True,
            scope="all",
            group_conditioning=True,
            norm_modulation_quant=True,
            residual_norm_quant=True,
        )
    session = GrootOptimizations(SimpleNamespace(model=policy), config)
    session.__enter__()
    engine = ControlStep(policy, args.batch, device=device, graph=not args.no_graph)
    inputs = harness.synthetic_inputs(args.batch, device)
    engine.load(inputs)
    engine.capture()
    host_inputs = [t.cpu().pin_memory() for t in harness.synthetic_inputs(args.batch, "cpu", seed=2)]
    return engine, session, host_inputs


def run_ours(args, world, rank, local):
    from pir2_b200 import _lib

    engine, session, host_inputs = build_engine(args, local)
    stream = engine.stream
    for _ in range(args.warmup):
        engine.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # The NVTX range lets a profiler select exactly the timed steps.
        torch.cuda.nvtx.range_push("pir2b_timed")
        e0.record(stream)
        for _ in range(args.steps):
            engine.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    clock_summary = clocks.summary()

    # End to end through the public step call: pinned host inputs -> H2D ->
    # graph -> D2H of the actions, every step.
    for _ in range(2):
        engine.step(host_inputs)
    barrier(world)
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        engine.step(host_inputs)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps, world)

    hbm, kind = peaks()
    roof = roofline(engine, hbm, kind, args.precision)
    status = _lib.device_status()
    roof["share_of_step"] = round(roof.pop("_gemm_ms_small", 0.0) / ms, 3) if ms else None
    cpu = None
    if rank == 0 and world == 1:
        cpu_ms, cores, sample = cpu_oracle_step(args, budget_s=args.cpu_sample_seconds)
        cpu = {"value": round(cpu_ms, 3), "unit": "ms", "cores": cores, "kind": "port", "sample": sample}
    # Kernel launches inside one timed step (graph nodes of this library).
    launches = count_launches(engine)
    phases = phase_breakdown(engine)
    engine.release()
    coexec = coexec_b1_record(engine.policy, args, world, local)
    batched = batched_record(engine.policy, args, world, local) if args.batched_robots else None
    session.close()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(ms, 4),
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": False,
            "scaling": "weak" if args.robots is None else "strong",
            "vs_baseline": None,
            "dtype": {"w8a8": "int8", "w4a4": "int4", "fp4": "e2m1", "fp8": "e4m3"}[args.precision],
            "data": "synthetic",
            "config": workload_config(args, world),
            "graph": not args.no_graph,
            "e2e": {
                "value": round(e2e_ms, 4),
                "unit": "ms",
                "h2d_bytes_per_step": engine.h2d_bytes(),
                "d2h_bytes_per_step": engine.d2h_bytes(),
            },
            "gpu_launches": launches,
            "phases": phases,
            "coexec_b1": coexec,
            "batched": batched,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clock_summary,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)


def _timed_steps(step, stream, steps, warmup, world):
    """Device time per step of `step()` replayed `steps` times on `stream`
    after `warmup` untimed calls, bracketed by a barrier and a device
    synchronize on both sides; the max over ranks."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / steps, world)


def batched_record(policy, args, world, local):
    """BASELINE's batched configuration: `--batched-robots` independent robots
    split evenly over the GPUs (strong scaling, no collective).  Each GPU
    times its share two ways: the serial control step (VLM prefill then the
    4-step DiT, one graph) and the co-executed step (DiT on the previous
    features while the VLM prefills the next observation on a second stream,
    as piR2's S1/S2 run).  Max over ranks; throughput is whole-job robot
    steps per second."""
    from pir2_b200 import harness
    from pir2_b200.engine import CoExecutionStep, ControlStep

    robots = args.batched_robots
    if robots % world:
        raise SystemExit(f"--batched-robots {robots} does not split over {world} GPUs")
    share = robots // world
    device = torch.device("cuda", local)
    steps, warmup = min(args.steps, 20), min(max(args.warmup, 3), 5)
    inputs = harness.synthetic_inputs(share, device, seed=3)
    serial = ControlStep(policy, share, device=device)
    serial.load(inputs)
    serial.capture()
    serial_ms = _timed_steps(serial.replay, serial.stream, steps, warmup, world)
    serial.release()
    del serial
    coexec = CoExecutionStep(policy, share, device=device)
    coexec.prime(inputs)
    coexec.capture()
    coexec_ms = _timed_steps(coexec.replay, coexec.stream, steps, warmup, world)
    coexec.release()
    del coexec
    torch.cuda.empty_cache()
    return {
        "robots_total": robots,
        "robots_per_gpu": share,
        "n_gpus": world,
        "scaling": "strong",
        "steps": steps,
        "warmup": warmup,
        "serial_ms_per_step": round(serial_ms, 4),
        "coexec_ms_per_step": round(coexec_ms, 4),
        "robot_steps_per_s": round(robots / (coexec_ms * 1e-3), 1),
        "robot_steps_per_s_serial": round(robots / (serial_ms * 1e-3), 1),
        "coexec": "VLM prefill of observation k on a second stream while the 4-step DiT acts on observation k-1's features",
        "note": "each GPU holds the full packed weights; no collective; time is the max over ranks",
    }


def coexec_b1_record(policy, args, world, local):
    """The B=1 control loop with VLM and DiT co-executed (S1/S2): per-step
    device time, max over ranks, next to the serial headline."""
    from pir2_b200 import harness
    from pir2_b200.engine import CoExecutionStep

    device = torch.device("cuda", local)
    steps, warmup = min(args.steps, 50), min(max(args.warmup, 3), 5)
    engine = CoExecutionStep(policy, args.batch, device=device)
    engine.prime(harness.synthetic_inputs(args.batch, device))
    engine.capture()
    ms = _timed_steps(engine.replay, engine.stream, steps, warmup, world)
    engine.release()
    return {"ms_per_step": round(ms, 4), "steps": steps, "batch_per_gpu": args.batch,
            "what": "DiT on the previous features while the VLM prefills the next observation on a second stream"}


def phase_breakdown(engine, reps=50):
    """Device time of the VLM prefill and of the 4-step action head, each
    replayed from its own graph (diagnostic split of the step)."""
    policy = engine.policy
    visual, ids, state, noise = engine.static
    results = {}
    with torch.inference_mode():
        features = policy.backbone(visual, ids)
        phases = {
            "vlm_prefill_ms": lambda: policy.backbone(visual, ids),
            "action_head_ms": lambda: policy.action_head.get_action(features, state, noise),
        }
        for name, fn in phases.items():
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(engine.stream):
                fn()
            engine.stream.synchronize()
            with torch.cuda.graph(graph, stream=engine.stream):
                fn()
            with torch.cuda.stream(engine.stream):
                for _ in range(3):
                    graph.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(engine.stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(engine.stream)
            engine.stream.synchronize()
            results[name] = round(e0.elapsed_time(e1) / reps, 4)
            del graph
    return results


def count_launches(engine):
    """Counts this library's kernel launches in one step (packs, norm
    producers, GEMMs, attention, q/k norm + RoPE, NVFP4), by wrapping the
    C-ABI entry points for one eager step (each launches one kernel for the
    shapes of the step)."""
    from pir2_b200 import _lib

    lib = _lib.lib()
    names = [
        "pir2b_quant_rows",
        "pir2b_norm_quant_rows",
        "pir2b_gemm",
        "pir2b_qk_norm_rope",
        "pir2b_attention_rows",
        "pir2b_pack_nvfp4",
        "pir2b_gemm_nvfp4",
    ]
    counts = {n: 0 for n in names}
    originals = {n: getattr(lib, n) for n in names}

    class Counting:
        def __init__(self, name, fn):
            self.name, self.fn = name, fn

        def __call__(self, *a):
            counts[self.name] += 1
            return self.fn(*a)

    try:
        for n in names:
            setattr(lib, n, Counting(n, originals[n]))
        with torch.inference_mode(), torch.cuda.stream(engine.stream):
            engine.policy(*engine.static)
        engine.stream.synchronize()
    finally:
        for n in names:
            setattr(lib, n, originals[n])
    return sum(counts.values())


SWEEP_M = (1, 16, 64, 256, 1024)
SWEEP_SHAPES = ((2048, 4096), (2048, 2048), (2048, 12288), (6144, 2048))


def _time_graph_launches(launch, count, warmup):
    """Median over 5 replays of a CUDA graph of `count` launches, in us per
    launch."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 1)):
            launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(count):
            launch(i)
    for _ in range(max(warmup, 1)):
        graph.replay()
    torch.cuda.synchronize()
    times = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(5):
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / count)
    del graph
    return sorted(times)[2]


def sweep_point(precision, m, k, n, weights_mb, warmup):
    """One (precision, M, K, N) point of BASELINE configs 2 and 3: the GEMM
    alone (activation pack excluded), back to back in a CUDA graph over
    rotating weight copies totalling ~weights_mb so each launch streams its
    weights from DRAM.  Returns the time and both rooflines: algorithmic
    bytes (weights, packed activations, scales, bf16 output) over the
    measured HBM copy bandwidth, and 2MNK over the tensor peak; `bound` is
    the one with the longer ideal time."""
    from pir2_b200 import ops

    hbm, _ = peaks()
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    if precision == "nvfp4":
        wbytes = n * k // 2 + n * k // 16
        copies = max(1, min(64, int(weights_mb * 1e6 // wbytes)))
        ws = [ops.pack_nvfp4((torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16))
              for _ in range(copies)]
        pa, sa = ops.pack_nvfp4(torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16))
        launch = lambda i: ops.gemm_nvfp4(pa, sa, ws[i % copies][0], ws[i % copies][1], n=n, out=out)  # noqa: E731
        algo = wbytes + m * k // 2 + m * k // 16 + 2 * m * n
        peak_tops = FP4_NOMINAL_TOPS
    else:
        bits = 8 if precision == "w8a8" else 4
        kp, npd = ops.kpad(k), ops.npad(n)
        cols = kp if bits == 8 else kp // 2
        dtype = torch.int8 if bits == 8 else torch.uint8
        lo, hi = (-127, 128) if bits == 8 else (0, 256)
        wbytes = npd * cols
        copies = max(1, min(64, int(weights_mb * 1e6 // wbytes)))
        ws = [torch.randint(lo, hi, (npd, cols), device="cuda", dtype=dtype, generator=g) for _ in range(copies)]
        qa = torch.randint(lo, hi, (m, cols), device="cuda", dtype=dtype, generator=g)
        sa = torch.rand(m, device="cuda", generator=g)
        sw = torch.rand(npd, device="cuda", generator=g)
        launch = lambda i: ops.gemm(qa, sa, ws[i % copies], sw, None, bits, n_store=n, out=out)  # noqa: E731
        algo = wbytes + m * cols + 4 * m + 4 * npd + 2 * m * n
        peak_tops = INT8_PEAK_TOPS
    us = _time_graph_launches(launch, max(copies, 20), warmup)
    ops_ = 2.0 * m * n * k
    gbs = algo / us / 1e3
    tops = ops_ / us / 1e6
    bound = "hbm" if algo / (hbm * 1e3) >= ops_ / (peak_tops * 1e6) else "tensor"
    return {
        "precision": precision, "m": m, "k": k, "n": n, "us": round(us, 3),
        "GBs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
        "TOPS": round(tops, 1), "tensor_frac": round(tops / peak_tops, 4),
        "bound": bound, "frac": round(gbs / hbm if bound == "hbm" else tops / peak_tops, 4),
    }


def run_sweep(args):
    """BASELINE configs 2/3: M x (K, N) for W8A8, W4A4 and NVFP4, one JSON
    line per point plus a summary line."""
    rows = []
    for precision in ("w8a8", "w4a4", "nvfp4"):
        for k, n in SWEEP_SHAPES:
            for m in SWEEP_M:
                row = sweep_point(precision, m, k, n, args.kernel_weights_mb, args.warmup)
                rows.append(row)
                print(json.dumps(row), flush=True)
    hbm, kind = peaks()
    print(json.dumps({
        "sweep": "BASELINE configs 2/3 (GEMM alone, back to back, weights streamed from DRAM)",
        "points": len(rows), "hbm_peak_gbs": hbm, "hbm_peak_kind": kind,
        "int8_peak_tops": INT8_PEAK_TOPS, "fp4_peak_tops": FP4_NOMINAL_TOPS,
        "small_m_hbm_frac_median": sorted(r["hbm_frac"] for r in rows if r["bound"] == "hbm")[
            len([r for r in rows if r["bound"] == "hbm"]) // 2] if any(r["bound"] == "hbm" for r in rows) else None,
    }), flush=True)


def run_kernel(args):
    """Times one quantized GEMM shape (activation pack excluded): rotating
    weight copies totalling ~--kernel-weights-mb keep each launch's weights
    out of L2.  Prints one JSON line with the per-launch time and rooflines."""
    from pir2_b200 import ops

    m, k, n = (int(v) for v in args.kernel.split(","))
    if args.precision in ("fp8", "fp4"):
        return run_kernel_floating(args, m, k, n)
    bits = 8 if args.precision == "w8a8" else 4
    kp, npd = ops.kpad(k), ops.npad(n)
    wbytes = npd * kp * bits // 8
    copies = max(1, min(64, int(args.kernel_weights_mb * 1e6 // wbytes)))
    g = torch.Generator(device="cuda").manual_seed(0)
    cols = kp if bits == 8 else kp // 2
    dtype = torch.int8 if bits == 8 else torch.uint8
    lo, hi = (-127, 128) if bits == 8 else (0, 256)
    weights = [torch.randint(lo, hi, (npd, cols), device="cuda", dtype=dtype, generator=g) for _ in range(copies)]
    qa = torch.randint(lo, hi, (m, cols), device="cuda", dtype=dtype, generator=g)
    sa = torch.rand(m, device="cuda", generator=g)
    sw = torch.rand(npd, device="cuda", generator=g)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16) if args.kernel_residual else None
    iters = max(args.steps, copies)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 1)):
            ops.gemm(qa, sa, weights[i % copies], sw, None, bits, n_store=n, out=out, residual=res)
    torch.cuda.synchronize()
    # One CUDA graph of `iters` launches back to back (each a different weight
    # copy), replayed: the launches chain with programmatic dependent launch
    # as they do inside the control step.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(iters):
            ops.gemm(qa, sa, weights[i % copies], sw, None, bits, n_store=n, out=out, residual=res)
    for _ in range(max(args.warmup, 1)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(5):
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / iters)
    us = sorted(times)[2]
    algo = wbytes + m * cols + 4 * m + 4 * npd + 2 * m * n * (2 if res is not None else 1)
    hbm, _ = peaks()
    import ctypes

    from pir2_b200 import _lib

    plan = [ctypes.c_int() for _ in range(4)] + [ctypes.c_int64(), ctypes.c_int(), ctypes.c_int()]
    _lib.lib().pir2b_gemm_plan(bits, m, npd, kp, torch.cuda.get_device_properties(0).multi_processor_count,
                               *[ctypes.byref(v) for v in plan])
    bn, mtiles, splits, stages, _, wt, pair = [v.value for v in plan]
    few = m <= 32   # the planner's few-token rule for packed int8/int4 inputs
    print(json.dumps({
        "kernel": f"gemm_few_kernel<{bits}>" if few else ("gemm_pair_kernel (2-SM)" if pair else f"gemm_i8_kernel<{bits}>"),
        "plan": {"bn": bn, "token_tiles": mtiles, "splits": splits, "stages": stages, "weight_tiles": wt},
        "m": m, "k": k, "n": n, "residual": res is not None,
        "us_per_launch": round(us, 3),
        "algorithmic_bytes": algo, "GBs": round(algo / us / 1e3, 1), "hbm_frac": round(algo / us / 1e3 / hbm, 4),
        "TOPS": round(2 * m * n * k / us / 1e6, 1), "int8_frac": round(2 * m * n * k / us / 1e6 / INT8_PEAK_TOPS, 4),
        "weight_copies": copies, "launches": iters,
        "note": "median of 5 replays of a CUDA graph of back-to-back launches",
    }), flush=True)


def run_kernel_floating(args, m, k, n):
    """--kernel for the E4M3 (fp8) and NVFP4 (fp4) GEMMs: weights and tokens
    are packed once from seeded bf16 by this library's own packs, then timed
    like the integer GEMM (rotating weight copies, one graph of back-to-back
    launches, median of 5 replays)."""
    from pir2_b200 import ops

    fp8 = args.precision == "fp8"
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    if fp8:
        qw, _, sw = ops.quant_fp8(w, replicate=n, weights=True)
        qa, _, sa = ops.quant_fp8(x)
        wbytes = qw.numel() + 4 * n
        abytes = qa.numel() + 4 * m
    else:
        qw, sw = ops.pack_nvfp4(w)
        qa, sa = ops.pack_nvfp4(x)
        wbytes = n * k // 2 + n * k // 16
        abytes = m * k // 2 + m * k // 16
    copies = max(1, min(64, int(args.kernel_weights_mb * 1e6 // wbytes)))
    weights = [(qw.clone(), sw.clone()) for _ in range(copies)]
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16) if args.kernel_residual else None
    if res is not None and not fp8:
        raise SystemExit("--kernel-residual: the NVFP4 GEMM has no residual epilogue")

    def launch(i):
        cw, cs = weights[i % copies]
        if fp8:
            ops.gemm_fp8(qa, sa, cw, cs, None, n=n, residual=res, out=out)
        else:
            ops.gemm_nvfp4(qa, sa, cw, cs, None, n=n, out=out)

    iters = max(args.steps, copies)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 1)):
            launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(iters):
            launch(i)
    for _ in range(max(args.warmup, 1)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(5):
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / iters)
    us = sorted(times)[2]
    algo = wbytes + abytes + 2 * m * n * (2 if res is not None else 1)
    hbm, _ = peaks()
    print(json.dumps({
        "kernel": (("gemm_few_kernel<9>" if m <= 32 else "gemm_i8_kernel<9>") if fp8 else "gemm_fp4_kernel"),
        "precision": args.precision,
        "m": m, "k": k, "n": n, "residual": res is not None,
        "us_per_launch": round(us, 3),
        "algorithmic_bytes": algo, "GBs": round(algo / us / 1e3, 1), "hbm_frac": round(algo / us / 1e3 / hbm, 4),
        "TFLOPS": round(2 * m * n * k / us / 1e6, 1),
        "weight_copies": copies, "launches": iters,
        "note": "median of 5 replays of a CUDA graph of back-to-back launches",
    }), flush=True)


def run_int8_peak(args):
    """INT8_PEAK_TOPS: every SM issues 128 x 256 x 32 kind::i8 MMAs back to
    back into a TMEM accumulator (pir2b_int8_peak_probe); reports MAC per
    clock per SM from the SM cycle counters, TOPS from CUDA events, and the
    SM clocks sampled meanwhile."""
    import ctypes

    from pir2_b200 import _lib

    lib = _lib.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    cycles = torch.zeros(sms, dtype=torch.int64, device="cuda")
    iters = 4096
    stream = torch.cuda.current_stream()

    def launch():
        _lib.check(lib.pir2b_int8_peak_probe(iters, sms, ctypes.c_void_p(cycles.data_ptr()),
                                             ctypes.c_void_p(stream.cuda_stream)), "pir2b_int8_peak_probe")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    times, per_clk = [], []
    with ClockSampler(0) as sampler:
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launch()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) * 1e-3)
            per_clk.append(iters * 4 * 128 * 256 * 32 / float(cycles.max().item()))
    clocks = sampler.summary()
    macs = float(sms) * iters * 4 * 128 * 256 * 32
    mac_clk = sorted(per_clk)[2]
    print(json.dumps({
        "int8_peak_probe": "tcgen05.mma.kind::i8 M=128 N=256 K=32, back to back, operands in shared memory",
        "sms": sms,
        "mac_per_clk_per_sm": round(mac_clk, 1),
        "tops_events": round(2 * macs / sorted(times)[2] / 1e12, 1),
        "tops_at_max_clock": round(2 * mac_clk * sms * (clocks["sm_max_mhz"] or 1965.0) * 1e6 / 1e12, 1),
        "bench_int8_peak_tops": INT8_PEAK_TOPS,
        "clocks": clocks,
        "device_status": _lib.device_status(),
    }), flush=True)


def run_step_gemms(args):
    """Records the GEMM launches of one eager control step (the bench's
    configuration), then launches each distinct small-M packed-input integer
    shape twice with random codes inside the NVTX range `pir2b_step_gemms`,
    printing one JSON line per shape with its launch count in the step."""
    from collections import Counter

    from pir2_b200 import ops

    engine, session, _ = build_engine(args, 0)

    class Recorder:
        def __init__(self):
            self.shapes = []

        def before(self, device):
            pass

        def after(self, device, **shape):
            self.shapes.append(shape)

    rec = Recorder()
    ops.launch_recorder = rec
    try:
        with torch.inference_mode(), torch.cuda.stream(engine.stream):
            engine.policy(*engine.static)
    finally:
        ops.launch_recorder = None
    torch.cuda.synchronize()
    counts = Counter(json.dumps(s, sort_keys=True) for s in rec.shapes)
    g = torch.Generator(device="cuda").manual_seed(3)
    torch.cuda.nvtx.range_push("pir2b_step_gemms")
    for key, count in counts.most_common():
        s = json.loads(key)
        if s["m"] > 64 or s["bits"] not in (4, 8) or s.get("input") == "rows" or s.get("out_n"):
            continue
        b, m, k, npad, n = s["bits"], s["m"], s["k"], s["npad"], s["n"]
        cols = k if b == 8 else k // 2
        dtype = torch.int8 if b == 8 else torch.uint8
        lo, hi = (-127, 128) if b == 8 else (0, 256)
        w = torch.randint(lo, hi, (npad, cols), device="cuda", dtype=dtype, generator=g)
        qa = torch.randint(lo, hi, (m, cols), device="cuda", dtype=dtype, generator=g)
        sa = torch.rand(m, device="cuda", generator=g)
        sw = torch.rand(npad, device="cuda", generator=g)
        bias = torch.zeros(npad, device="cuda", dtype=torch.bfloat16) if s.get("bias") else None
        res = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16) if s.get("residual") else None
        for _ in range(2):
            ops.gemm(qa, sa, w, sw, bias, b, n_store=n, residual=res)
        torch.cuda.synchronize()
        print(json.dumps({"shape": s, "launches_in_step": count, "algorithmic_bytes": gemm_bytes(s)}), flush=True)
    torch.cuda.nvtx.range_pop()
    session.__exit__(None, None, None)


def main():
    args = parse()
    if args.int8_peak:
        torch.cuda.set_device(0)
        run_int8_peak(args)
        return
    if args.step_gemms:
        torch.cuda.set_device(0)
        run_step_gemms(args)
        return
    if args.kernel:
        torch.cuda.set_device(0)
        run_kernel(args)
        return
    if args.sweep:
        torch.cuda.set_device(0)
        run_sweep(args)
        return
    if args.impl == "reference":
        # Rank 0 alone times the host path; no process group is needed.
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if args.robots is not None:
            if args.robots % world:
                raise SystemExit(f"--robots {args.robots} does not split over {world} GPUs")
            args.batch = args.robots // world
        run_reference(args, world, int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup(args)
    if args.robots is not None:
        if args.robots % world:
            raise SystemExit(f"--robots {args.robots} does not split over {world} GPUs")
        args.batch = args.robots // world
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
