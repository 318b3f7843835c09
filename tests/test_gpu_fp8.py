"""FP8 (E4M3, per-tensor) path on the B200 kernels: the quantizer's codes
and scale are bitwise the oracle's (both reference variants), the tcgen05
kind::f8f6f4 GEMM and the few-token e4m3 GEMM (at most 32 rows) match the oracle's fp64 sum of dequantized products to
one bf16 rounding step (rtol 2^-7) plus atol 1e-3 for fp32 accumulation
order, and FloatingLinear(precision="fp8") equals quantizer + GEMM."""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("rows,k", [(1, 128), (17, 1536), (544, 2048), (3000, 256), (7, 1032)])
@pytest.mark.parametrize("fast", [False, True])
def test_quant_fp8_codes_and_scale_equal_oracle(rows, k, fast):
    g = torch.Generator().manual_seed(rows + k)
    x = torch.randn(rows, k, generator=g) * 2.0
    x[0, :6] = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), float("nan"), 1e-30])
    xb = x.to(torch.bfloat16)
    q, scale, rep = ops.quant_fp8(xb.cuda(), fast=fast)
    want_q, want_s = oracle.quant_fp8(bits_of(xb), fast=fast)
    assert np.float32(scale.item()) == want_s
    assert torch.equal(rep, torch.full_like(rep, float(want_s)))
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("rows,k", [(1, 1536), (17, 6144), (544, 2048), (2000, 8192)])
@pytest.mark.parametrize("fast", [False, True])
def test_quant_fp8_two_pass_equals_cluster_quantizer(rows, k, fast):
    """Activations take the two-launch quantizer (row maxima, then scale and
    cast), weights the one-launch cluster kernel: same codes and scale, also
    for rows that are a strided view."""
    g = torch.Generator().manual_seed(rows + k)
    x = (torch.randn(rows, k + 64, generator=g) * 3).to(torch.bfloat16).cuda()
    x[rows // 2, 7] = float("inf")
    view = x[:, :k]
    q1, s1, r1 = ops.quant_fp8(view, fast=fast)
    q2, s2, _ = ops.quant_fp8(view.contiguous(), fast=fast, weights=True)
    assert torch.equal(s1, s2) and torch.equal(q1, q2)
    assert torch.equal(r1, s1.expand(rows))
    want_q, want_s = oracle.quant_fp8(bits_of(view), fast=fast)
    assert np.float32(s1.item()) == want_s and np.array_equal(q1.cpu().numpy(), want_q)
    assert _lib.device_status() == 0


@pytest.mark.parametrize(
    "m,k,n",
    [(1, 2048, 4096), (17, 1536, 1536), (64, 1024, 2048), (300, 1536, 640), (544, 2048, 4096)],
)
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_fp8_matches_dequantized_product(m, k, n, with_bias):
    g = torch.Generator().manual_seed(m * 3 + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16) if with_bias else None
    qa, sa, sa_rows = ops.quant_fp8(x.cuda())
    qw, sw, sw_cols = ops.quant_fp8(w.cuda(), replicate=n, weights=True)
    out = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, None if bias is None else bias.cuda(), n=n)
    torch.cuda.synchronize()
    want = oracle.fp8_gemm(qa.cpu().numpy(), sa.item(), qw.cpu().numpy(), sw.item(),
                           None if bias is None else bits_of(bias))
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=1e-3)
    assert _lib.device_status() == 0


@pytest.fixture
def few_mode():
    """Sets the few-token kernel override for one test and restores it."""
    previous = []

    def set_mode(mode):
        previous.append(_lib.set_few_mode(mode))

    yield set_mode
    if previous:
        _lib.set_few_mode(previous[0])


@pytest.mark.parametrize(
    "m,k,n",
    [(1, 1536, 1536), (5, 128, 1032), (9, 2048, 2048), (17, 1536, 6144), (17, 6144, 1536), (24, 4096, 640),
     (32, 2048, 4096)],
)
@pytest.mark.parametrize("few", [True, False])
def test_gemm_fp8_few_rows_both_kernels(m, k, n, few, few_mode):
    """At most 32 token rows: the few-token kernel (warp-level e4m3 MMAs,
    fp32 partials added in warp order) and the tcgen05 kernel both match the
    fp64 dequantized product within the FP8 tolerance, with bias and the
    residual epilogue; each is deterministic (two launches, equal bits)."""
    few_mode(0 if few else 2)
    g = torch.Generator().manual_seed(m * 7 + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    qa, sa, sa_rows = ops.quant_fp8(x.cuda())
    qw, sw, sw_cols = ops.quant_fp8(w.cuda(), replicate=n, weights=True)
    out = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, bias.cuda(), n=n)
    again = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, bias.cuda(), n=n)
    with_res = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, bias.cuda(), n=n, residual=res.cuda())
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    want = oracle.fp8_gemm(qa.cpu().numpy(), sa.item(), qw.cpu().numpy(), sw.item(), bits_of(bias))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=2 ** -7, atol=1e-3)
    # The residual epilogue adds the bf16 result and the bf16 residual in fp32.
    assert torch.equal(with_res.cpu(), (out.cpu().float() + res.float()).to(torch.bfloat16))
    assert _lib.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(544, 2048, 4096), (544, 6144, 2048), (1088, 2048, 12288), (4352, 2048, 4096)])
@pytest.mark.parametrize("pair", [1, 2])
def test_gemm_fp8_many_rows_on_two_sm_tiles(m, k, n, pair):
    """Many token rows: the 2-SM tile kernel on kind::f8f6f4 (pair mode 1
    forces it where it applies) and the one-SM kernel (mode 2) both match
    the fp64 dequantized product, with bias and the residual epilogue."""
    previous = _lib.set_pair_mode(pair)
    try:
        g = torch.Generator().manual_seed(m + k + n + pair)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
        bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
        res = torch.randn(m, n, generator=g).to(torch.bfloat16)
        qa, sa, sa_rows = ops.quant_fp8(x.cuda())
        qw, sw, sw_cols = ops.quant_fp8(w.cuda(), replicate=n, weights=True)
        out = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, bias.cuda(), n=n)
        with_res = ops.gemm_fp8(qa, sa_rows, qw, sw_cols, bias.cuda(), n=n, residual=res.cuda())
        torch.cuda.synchronize()
        want = oracle.fp8_gemm(qa.cpu().numpy(), sa.item(), qw.cpu().numpy(), sw.item(), bits_of(bias))
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=2 ** -7, atol=1e-3)
        assert torch.equal(with_res.cpu(), (out.cpu().float() + res.float()).to(torch.bfloat16))
    finally:
        _lib.set_pair_mode(previous)
    assert _lib.device_status() == 0


def test_gemm_fp8_residual_and_floating_linear():
    from pir2_b200.floating import FloatingLinear

    g = torch.Generator().manual_seed(3)
    with torch.device("cuda"):
        linear = torch.nn.Linear(1536, 4608, bias=True).to(torch.bfloat16)
    x = torch.randn(2, 17, 1536, generator=g).to(torch.bfloat16).cuda()
    layer = FloatingLinear(linear, "probe", "fp8")
    qa, _, rows = ops.quant_fp8(x.reshape(-1, 1536))
    direct = ops.gemm_fp8(qa, rows, layer.packed_weight, layer.weight_scale_columns, layer.bias, n=4608)
    assert torch.equal(layer(x).reshape(-1, 4608), direct)
    res = torch.randn(34, 4608, generator=g).to(torch.bfloat16).cuda()
    with_res = ops.gemm_fp8(qa, rows, layer.packed_weight, layer.weight_scale_columns, layer.bias, n=4608,
                            residual=res)
    want = (direct.float() + res.float()).to(torch.bfloat16)
    assert torch.equal(with_res, want)
    # The layer's residual form is the GEMM's residual epilogue (as the DiT
    # FFN down projection uses it): exactly bf16(y + residual).
    r3 = res.reshape(2, 17, 4608)
    assert torch.equal(layer(x, residual=r3), (layer(x).float() + r3.float()).to(torch.bfloat16))
    fast = FloatingLinear(linear, "probe", "fp8", fast_fp8=True)
    q2, _, rows2 = ops.quant_fp8(x.reshape(-1, 1536), fast=True)
    assert torch.equal(fast(x).reshape(-1, 4608),
                       ops.gemm_fp8(q2, rows2, fast.packed_weight, fast.weight_scale_columns, fast.bias, n=4608))
    assert _lib.device_status() == 0


@pytest.mark.parametrize("precision", ["fp8", "fp4"])
@torch.inference_mode()
def test_shared_input_packing_is_bitwise_and_packs_once(precision, monkeypatch):
    """fp_shared_inputs: sibling projections of one input (q|k|v, k|v,
    gate|up) pack it once per owner call; actions are bitwise unchanged."""
    from types import SimpleNamespace

    from pir2_b200 import harness
    from pir2_b200.config import OptimizationConfig
    from pir2_b200.session import GrootOptimizations

    vlm, dit = harness.VLMConfig(layers=1, vocab=2048), harness.DiTConfig(layers=2)
    policy = harness.build_policy("cuda", vlm=vlm, dit=dit)
    inputs = harness.synthetic_inputs(1, "cuda", vlm=vlm, dit=dit)
    pack = "quant_fp8" if precision == "fp8" else "pack_nvfp4"
    original = getattr(ops, pack)
    calls = []
    monkeypatch.setattr(ops, pack, lambda *a, **k: calls.append(1) or original(*a, **k))
    results = []
    for shared in (False, True):
        config = OptimizationConfig(precision=precision, scope="all", fp_shared_inputs=shared)
        with GrootOptimizations(SimpleNamespace(model=policy), config) as session:
            calls.clear()   # weight packs happen at install
            actions = policy(*inputs)
            results.append((actions, len(calls), session.coverage["shared_input_groups"]))
    assert torch.equal(results[0][0], results[1][0])
    assert results[1][2] > 0 and results[1][1] < results[0][1]
    assert _lib.device_status() == 0
