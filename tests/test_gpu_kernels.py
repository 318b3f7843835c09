"""Parity of the sm_100a kernels (called through the C ABI) with the oracle.

Integer stages (codes, scales, int32 accumulators through the epilogue) and
packed bytes are compared bitwise; fused norm producers within one
quantization code (their reduction order differs from any reference order);
NVFP4 packs bitwise against the oracle's IEEE-division restatement.
"""

import numpy as np
import pytest
import torch

import oracle
from pir2_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def to_dev(bits, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def device_lut(kind):
    """Activation table built by torch on the device, as the reference does
    (coexecution/kernels/common/fused.py:74-83, groot/integer.py:47-53)."""
    values = torch.arange(65536, device="cuda", dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    if kind == "silu":
        return torch.nn.functional.silu(values)
    return torch.nn.functional.gelu(values, approximate=kind)


def randn_bf16(g, *shape, outliers=False):
    x = torch.randn(*shape, generator=g)
    if outliers:
        cols = torch.randperm(shape[-1], generator=g)[: max(1, shape[-1] // 100)]
        x[..., cols] *= 20.0
    return x.to(torch.bfloat16)


def assert_status_clean():
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize(
    "rows,k",
    [(1, 2048), (17, 130), (5, 1), (3, 127), (64, 6144), (1024, 2048), (7, 12288), (2, 40000), (17, 6144), (1, 4100)],
)
def test_quant_rows_plain_bitwise(bits, rows, k):
    g = torch.Generator().manual_seed(rows * 131 + k)
    x = randn_bf16(g, rows, k, outliers=True)
    q, s = ops.quant_rows(x.cuda(), bits)
    rq, rs = oracle.quant_rows(bits_of(x), bits)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))
    assert_status_clean()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(1, 2048), (17, 6144), (17, 130), (3, 127), (64, 6144), (1088, 6144)])
def test_quant_rows_with_given_maxima_bitwise(bits, rows, k):
    """The pack that takes its row maxima as per-16-column partial maxima
    (from the producing GEMM's epilogue) writes the oracle's codes and
    scales, including zero rows and +-inf values."""
    g = torch.Generator().manual_seed(rows * 7 + k + bits)
    x = randn_bf16(g, rows, k, outliers=True)
    x[0] = 0.0
    if rows > 2:
        x[2, k // 2] = float("inf")
    xc = x.cuda()
    parts = -(-k // 16)
    padded = torch.zeros(rows, parts * 16, dtype=torch.float32)
    padded[:, :k] = x.float().abs()
    maxima = padded.reshape(rows, parts, 16).amax(dim=2).contiguous().cuda()
    q, s = ops.quant_rows_max(xc, maxima, bits)
    rq, rs = oracle.quant_rows(bits_of(x), bits)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))
    # The GEMM epilogue's maxima feed it directly: same bytes as quant_rows.
    q2, s2 = ops.quant_rows(xc, bits)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    assert_status_clean()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("kind", ["tanh", "none", "silu"])
@pytest.mark.parametrize("gated", [False, True])
def test_quant_rows_lut_modes_bitwise(bits, kind, gated):
    g = torch.Generator().manual_seed(7)
    x = randn_bf16(g, 17, 258)
    up = randn_bf16(g, 17, 258)
    lut = device_lut(kind)
    q, s = ops.quant_rows(x.cuda(), bits, lut=lut, up=up.cuda() if gated else None)
    rq, rs = oracle.quant_rows(bits_of(x), bits, lut_bits=bits_of(lut), up_bits=bits_of(up) if gated else None)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))


@pytest.mark.parametrize("bits", [8, 4])
def test_quant_rows_cluster_path_lut_gated_bitwise(bits):
    """Few long rows take the cluster-split kernel; LUT and gate included."""
    g = torch.Generator().manual_seed(8)
    x = randn_bf16(g, 17, 6144)
    up = randn_bf16(g, 17, 6144)
    lut = device_lut("silu")
    q, s = ops.quant_rows(x.cuda(), bits, lut=lut, up=up.cuda())
    rq, rs = oracle.quant_rows(bits_of(x), bits, lut_bits=bits_of(lut), up_bits=bits_of(up))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))


def test_quant_rows_strided_rows_and_zero_rows():
    g = torch.Generator().manual_seed(3)
    base = randn_bf16(g, 6, 4096)
    base[2] = 0
    view = base.cuda()[:, 1024:3072]          # row stride 4096, 16-byte aligned
    q, s = ops.quant_rows(view, 8)
    rq, rs = oracle.quant_rows(bits_of(base[:, 1024:3072]), 8)
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    assert s[2].item() == 1.0
    odd = base.cuda()[:, 3:1003]              # misaligned start: scalar path
    q, s = ops.quant_rows(odd, 4)
    rq, rs = oracle.quant_rows(bits_of(base[:, 3:1003]), 4)
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_quant_rows_smoothing_bitwise():
    g = torch.Generator().manual_seed(11)
    x = randn_bf16(g, 9, 2048, outliers=True)
    smooth = (torch.rand(2048, generator=g) * 4 + 0.25).float()
    q, s = ops.quant_rows(x.cuda(), 8, smooth=smooth.cuda())
    rq, rs = oracle.quant_rows(bits_of(x), 8, smooth=smooth.numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


GEMM_SHAPES = [
    (1, 2048, 4096),
    (16, 2048, 2048),
    (17, 130, 64),
    (33, 1536, 1536),
    (64, 6144, 2048),
    (256, 2048, 4096),
    (300, 1024, 520),
    (544, 2048, 4096),
    (1024, 2048, 2048),
    (1088, 1536, 6144),
    # two weight tiles per CTA: the last CTA's second tile partly or wholly
    # beyond N (47 / 95 / 71 channel tiles)
    (1088, 1536, 6000),
    (544, 256, 12040),
    (700, 512, 9000),
]


def quantized_problem(g, m, k, n, bits, bias=True):
    x = randn_bf16(g, m, k, outliers=True)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if bias else None
    qa, sa = oracle.quant_rows(bits_of(x), bits)
    qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), bits)
    return x, w, b, qa, sa, qw, sw


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
def test_gemm_bitwise(bits, m, k, n):
    g = torch.Generator().manual_seed(m * 7 + k + n)
    x, w, b, qa, sa, qw, sw = quantized_problem(g, m, k, n, bits)
    npad = qw.shape[0]
    bias_full = np.zeros(npad, dtype=np.uint16)
    bias_full[:n] = bits_of(b)
    out = ops.gemm(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
        torch.from_numpy(sw).cuda(), to_dev(bias_full), bits, n_store=n,
    )
    ua = oracle.unpack_int4(qa) if bits == 4 else qa
    uw = oracle.unpack_int4(qw) if bits == 4 else qw
    ref = oracle.gemm_epilogue(oracle.int_matmul(ua, uw), sa, sw, bias_full, 2)[:, :n]
    got = bits_of(out)
    assert got.shape == ref.shape
    mismatch = np.argwhere(got != ref)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    assert_status_clean()


@pytest.mark.parametrize("bias_mode", [_lib.BIAS_NONE, _lib.BIAS_ZERO])
def test_gemm_bias_modes_and_negative_zero(bias_mode):
    g = torch.Generator().manual_seed(5)
    m, k, n = 20, 256, 64
    _, _, _, qa, sa, qw, sw = quantized_problem(g, m, k, n, 8, bias=False)
    qa[3] = 0                                  # exact zero row -> -0 * s stays +-0
    sa_neg = sa.copy()
    sa_neg[4] = -sa_neg[4]                     # negative scale produces -0 for acc == 0
    qa[4, :] = 0
    out = ops.gemm(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa_neg).cuda(), torch.from_numpy(qw).cuda(),
        torch.from_numpy(sw).cuda(), None, 8, bias_mode=bias_mode,
    )
    ref = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa_neg, sw, None, bias_mode)
    assert np.array_equal(bits_of(out), ref)
    row4 = bits_of(out)[4]
    assert np.all(row4 == (0x8000 if bias_mode == _lib.BIAS_NONE else 0))


def test_gemm_output_lut_epilogue():
    g = torch.Generator().manual_seed(9)
    m, k, n = 17, 1536, 6144
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, n, 8)
    lut = device_lut("tanh")
    out = ops.gemm(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
        torch.from_numpy(sw).cuda(), b.cuda(), 8, out_lut=lut,
    )
    ref = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa, sw, bits_of(b), 2, bits_of(lut))
    assert np.array_equal(bits_of(out), ref)


def codes(q, bits):
    q = q.cpu().numpy() if isinstance(q, torch.Tensor) else q
    return oracle.unpack_int4(q).astype(np.int32) if bits == 4 else q.astype(np.int32)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows", [544, 1088, 1, 5, 17])
def test_rmsnorm_producer_bitwise_vs_torch_row_mean(bits, rows):
    """The integer RMSNorm pack is bit-exact against the reference's B200
    path: fp32 squares, torch's row mean on the device (the variance bytes
    of rms_statistics.py:171-190), rsqrt(var + eps) on the device, then the
    `_rms_tail_pack` arithmetic (producers.py:19-53).  The oracle's
    restatement of torch's reduction order is pinned to torch here too."""
    g = torch.Generator().manual_seed(21 + rows)
    x = randn_bf16(g, rows, 2048, outliers=True)
    gamma = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    xd = x.cuda()
    sq = xd.float() * xd.float()
    var = sq.mean(-1)
    inv = torch.rsqrt(var + 1e-6)
    bw, factor = oracle.torch_row_mean_config(rows, 2048)
    assert np.array_equal(oracle.torch_row_mean(sq.cpu().numpy(), bw, factor), var.cpu().numpy())
    q, s, _ = ops.norm_quant_rows(xd, bits, norm=_lib.NORM_RMS, eps=1e-6, gamma=gamma.cuda())
    rq, rs = oracle.rms_norm_tail_pack(bits_of(x), bits_of(gamma), var.cpu().numpy(), inv.cpu().numpy(), bits)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(q.cpu().numpy(), rq)


def test_rmsnorm_residual_producer_bitwise():
    """The decoder's fused residual + RMSNorm pack: r = bf16(x + y) is written
    out and packed exactly as RMSNorm of r."""
    g = torch.Generator().manual_seed(5)
    x, y = randn_bf16(g, 544, 2048), randn_bf16(g, 544, 2048, outliers=True)
    gamma = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    q, s, r = ops.norm_quant_rows(x.cuda(), 8, norm=_lib.NORM_RMS, eps=1e-6, gamma=gamma.cuda(), y=y.cuda())
    rsum = (x.cuda().float() + y.cuda().float()).to(torch.bfloat16)
    assert torch.equal(r, rsum)
    var = (rsum.float() * rsum.float()).mean(-1)
    inv = torch.rsqrt(var + 1e-6)
    rq, rs = oracle.rms_norm_tail_pack(bits_of(rsum.cpu()), bits_of(gamma), var.cpu().numpy(), inv.cpu().numpy(), 8)
    assert np.array_equal(s.cpu().numpy(), rs) and np.array_equal(q.cpu().numpy(), rq)


def test_rmsnorm_pack_refuses_rows_outside_the_reproduced_order():
    x = torch.zeros(32, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="row-mean order"):
        ops.norm_quant_rows(x, 8, norm=_lib.NORM_RMS, eps=1e-6, gamma=torch.ones(64, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("kind", ["mod", "norm", "res"])
def test_adaln_producers(bits, kind):
    g = torch.Generator().manual_seed(33)
    bsz, tokens, k = 4, 17, 1536
    x = randn_bf16(g, bsz * tokens, k)
    scale = (0.5 * torch.randn(bsz, k, generator=g)).to(torch.bfloat16)
    shift = (0.5 * torch.randn(bsz, k, generator=g)).to(torch.bfloat16)
    y = randn_bf16(g, bsz * tokens, k)
    gate = randn_bf16(g, bsz, k)
    kwargs = dict(scale=scale.cuda(), shift=shift.cuda(), tokens=tokens)
    if kind == "mod":
        q, s, _ = ops.norm_quant_rows(x.cuda(), bits, **kwargs)
        rq, rs = oracle.modulation_pack(bits_of(x), bits_of(scale), bits_of(shift), tokens, bits)
        assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
        return
    if kind == "norm":
        q, s, _ = ops.norm_quant_rows(x.cuda(), bits, norm=_lib.NORM_LN, eps=1e-6, **kwargs)
        rq, rs = oracle.modulation_pack(bits_of(x), bits_of(scale), bits_of(shift), tokens, bits, eps=1e-6)
    else:
        q, s, r = ops.norm_quant_rows(
            x.cuda(), bits, norm=_lib.NORM_LN, eps=1e-6, y=y.cuda(), gate=gate.cuda(), **kwargs
        )
        rq, rs, rr = oracle.residual_norm_modulation_pack(
            bits_of(x), bits_of(y), bits_of(gate), bits_of(scale), bits_of(shift), tokens, bits, 1e-6
        )
        assert np.array_equal(bits_of(r), rr)
    assert np.allclose(s.cpu().numpy(), rs, rtol=2 ** -7, atol=0)
    assert np.abs(codes(q, bits) - codes(rq, bits)).max() <= 1


@pytest.mark.parametrize("rows,k", [(1, 2048), (17, 1536), (300, 6144)])
def test_nvfp4_pack_bitwise(rows, k):
    g = torch.Generator().manual_seed(rows + k)
    x = randn_bf16(g, rows, k, outliers=True)
    x[0, :16] = 0
    packed, sf = ops.pack_nvfp4(x.cuda())
    rp, rsf = oracle.pack_nvfp4(oracle.bf16_bits_to_f32(bits_of(x)))
    assert np.array_equal(packed.cpu().numpy(), rp)
    sfg = sf.cpu().numpy()
    blocks_k = (k // 16 + 3) // 4
    rr, jj = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    off = oracle.nvfp4_sf_offset(rr, jj, blocks_k)
    assert np.array_equal(sfg.reshape(-1)[off], rsf.reshape(-1)[off])


def test_qk_norm_rope_matches_torch():
    """Fused q/k RMSNorm + RoPE vs the torch sequence it replaces: RoPE is
    bitwise; the per-head mean of squares is reduced in another order, so a
    rare element may differ by one bf16 ulp."""
    g = torch.Generator().manual_seed(77)
    b, t, hq, hk, d = 1, 544, 16, 8, 128
    qkv = (torch.randn(b * t, (hq + 2 * hk) * d, generator=g) * 2).to(torch.bfloat16).cuda()
    qw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).cuda()
    kw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).cuda()
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = torch.outer(torch.arange(t, dtype=torch.float32), inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16).cuda(), emb.sin().to(torch.bfloat16).cuda()
    q, k, v = ops.qk_norm_rope(qkv, qw, kw, cos, sin, tokens=t, hq=hq, hk=hk, eps=1e-6)

    def rms(x, w):
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
        return w * h.to(torch.bfloat16)

    def rot(x):
        return torch.cat((-x[..., d // 2:], x[..., : d // 2]), dim=-1)

    view = qkv.view(b, t, hq + 2 * hk, d)
    rq = rms(view[:, :, :hq], qw).transpose(1, 2)
    rk = rms(view[:, :, hq : hq + hk], kw).transpose(1, 2)
    rq = rq * cos + rot(rq) * sin
    rk = rk * cos + rot(rk) * sin
    rv = view[:, :, hq + hk :].transpose(1, 2)
    assert torch.equal(v, rv.contiguous())
    for got, ref in ((q, rq), (k, rk)):
        diff = (got.float() - ref.float()).abs()
        ulp = ref.float().abs().clamp_min(1e-3) * 2 ** -7
        assert bool((diff <= ulp).all())
        assert float((got != ref).float().mean()) < 0.01


def test_gemm_residual_epilogue_bitwise():
    g = torch.Generator().manual_seed(41)
    for m, k, n in ((17, 1536, 1536), (544, 2048, 2048), (64, 6144, 2048), (700, 512, 9000)):
        _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, n, 8)
        residual = randn_bf16(g, m, n)
        out = ops.gemm(
            torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
            torch.from_numpy(sw).cuda(), b.cuda(), 8, residual=residual.cuda(), n_store=n,
        )
        y = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa, sw, bits_of(b), 2)[:, :n]
        ref = oracle.f32_to_bf16_bits(
            (oracle.bf16_bits_to_f32(y) + oracle.bf16_bits_to_f32(bits_of(residual))).astype(np.float32)
        )
        assert np.array_equal(bits_of(out), ref)


def _plan_of(m, n, k):
    import ctypes

    lib = _lib.lib()
    out = [ctypes.c_int() for _ in range(4)] + [ctypes.c_int64(), ctypes.c_int(), ctypes.c_int()]
    assert lib.pir2b_gemm_plan(8, m, n, k, 148, *[ctypes.byref(v) for v in out]) == 0
    bn, mt, splits, stages, smem, wt, pair = [v.value for v in out]
    return dict(bn=bn, mt=mt, splits=splits, stages=stages, wt=wt, pair=pair)


# 2-SM tiles (one or two weight tiles per CTA), token tiles of 80-256 rows,
# ragged channel counts (the odd CTA of the last pair partly or wholly past
# N) and ragged last token tiles.
PAIR_SHAPES = [
    (65, 2048, 12288),
    (256, 1536, 6144),
    (544, 2048, 4096),
    (700, 512, 9000),
    (1088, 1536, 6000),
    (2176, 2048, 4096),
    (2100, 384, 1000),
    (5000, 256, 4096),
    (3000, 1024, 8192),
]


@pytest.fixture
def pair_mode():
    """Sets the planner's 2-SM override for one test and restores it."""
    previous = []

    def set_mode(mode):
        previous.append(_lib.set_pair_mode(mode))

    yield set_mode
    if previous:
        _lib.set_pair_mode(previous[0])


@pytest.mark.parametrize("m,k,n", PAIR_SHAPES)
@pytest.mark.parametrize("epilogue", ["bias", "lut", "residual", "max_out"])
def test_gemm_pair_tiles_bitwise(m, k, n, epilogue, pair_mode):
    """The 2-SM kernel (tcgen05.mma.cta_group::2, even CTA issuing for the
    pair) against the oracle's exact product and epilogue, for every
    epilogue variant the one-SM kernel has."""
    pair_mode(1)
    g = torch.Generator().manual_seed(m + k + n)
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, n, 8)
    npad = qw.shape[0]
    plan = _plan_of(m, npad, qw.shape[1])
    assert plan["pair"] == 1, plan
    y = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa, sw, np.pad(bits_of(b), (0, npad - n)), 2,
                             bits_of(device_lut("tanh").cpu()) if epilogue == "lut" else None)[:, :n]
    args = dict(n_store=n)
    if epilogue == "lut":
        args["out_lut"] = device_lut("tanh")
    if epilogue == "residual":
        residual = randn_bf16(g, m, n)
        args["residual"] = residual.cuda()
        y = oracle.f32_to_bf16_bits(
            (oracle.bf16_bits_to_f32(y) + oracle.bf16_bits_to_f32(bits_of(residual))).astype(np.float32))
    if epilogue == "max_out":
        args["max_out"] = torch.full((m, npad // 16), -1.0, device="cuda")
    bias = torch.zeros(npad, dtype=torch.bfloat16)
    bias[:n] = b
    if epilogue == "max_out" and npad % 16:
        # Per-16-channel maxima need whole groups of padded channels.
        with pytest.raises(ValueError, match="npad % 16"):
            ops.gemm(torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
                     torch.from_numpy(sw).cuda(), bias.cuda(), 8, **args)
        return
    out = ops.gemm(torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
                   torch.from_numpy(sw).cuda(), bias.cuda(), 8, **args)
    got = bits_of(out)
    mismatch = np.argwhere(got != y)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    if epilogue == "max_out":
        yf = np.abs(oracle.bf16_bits_to_f32(y))
        groups = n // 16
        want = yf[:, : groups * 16].reshape(m, groups, 16).max(-1)
        assert np.array_equal(args["max_out"][:, :groups].cpu().numpy(), want)
    assert_status_clean()


def rounding_tie_problem(m, n, seed, traps_per_row=8):
    """Int8 codes, scales and bias whose epilogue values sit exactly on bf16
    rounding ties where a fused multiply-add (one rounding of acc*sa*sw + b)
    would round the other way.  Token row r has codes (1, 127) in columns
    (2r, 2r+1), so acc[r, c] = qw[c, 2r] + 127 qw[c, 2r+1] is free per
    element; for `traps_per_row` columns of each row it is searched for such
    a tie, elsewhere it is random.  Returns qa, sa, qw, sw, bias bits, acc,
    the number of planted ties."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    kpad = (2 * m + 127) // 128 * 128
    sa = rng.uniform(0.5, 2.0, m).astype(f32)
    # acc * sa * sw of the order of the bias: ties where the bias cancels most
    # of the product are the ones a fused multiply-add rounds differently.
    sw = rng.uniform(1e-5, 3e-5, n).astype(f32)
    bias = oracle.f32_to_bf16_bits(rng.normal(0.0, 0.05, n).astype(f32))
    bf = oracle.bf16_bits_to_f32(bias)
    acc = rng.integers(-16000, 16001, (m, n)).astype(np.int64)
    cand = np.arange(-16000, 16001)
    planted = 0
    for r in range(m):
        y1 = (cand.astype(f32) * sa[r]).astype(f32)
        for t in range(traps_per_row):
            c = (r * traps_per_row + t) % n
            y3 = ((y1 * sw[c]).astype(f32) + bf[c]).astype(f32)
            tie = (y3.view(np.uint32) & 0xFFFF) == 0x8000
            fused = (y1.astype(np.float64) * np.float64(sw[c]) + np.float64(bf[c])).astype(f32)
            idx = np.flatnonzero(tie & (oracle.f32_to_bf16_bits(fused) != oracle.f32_to_bf16_bits(y3)))
            if idx.size:
                acc[r, c] = cand[idx[rng.integers(idx.size)]]
                planted += 1
    hi = np.rint(acc / 127.0).astype(np.int64)
    lo = acc - 127 * hi
    qa = np.zeros((m, kpad), np.int8)
    qw = np.zeros((n, kpad), np.int8)
    rows = np.arange(m)
    qa[rows, 2 * rows] = 1
    qa[rows, 2 * rows + 1] = 127
    qw[:, 2 * rows] = lo.T
    qw[:, 2 * rows + 1] = hi.T
    return qa, sa, qw, sw, bias, acc.astype(np.int32), planted


@pytest.fixture
def few_mode():
    """Sets the few-token kernel override for one test and restores it."""
    previous = []

    def set_mode(mode):
        previous.append(_lib.set_few_mode(mode))

    yield set_mode
    if previous:
        _lib.set_few_mode(previous[0])


FEW_SHAPES = [(1, 1536, 1536), (17, 1536, 6144), (17, 6144, 1536), (16, 2048, 2048), (32, 2048, 4096),
              (5, 128, 520), (17, 8192, 264)]


@pytest.mark.parametrize("kernel", ["few", "tcgen05"])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("m,k,n", FEW_SHAPES)
@pytest.mark.parametrize("epilogue", ["bias", "lut", "residual", "max_out"])
def test_few_row_gemm_both_kernels_bitwise(m, k, n, bits, epilogue, kernel, few_mode):
    """GEMMs of at most 32 token rows on the few-token kernel (warp-level
    integer MMAs, K split over the CTA's warps) and on the tcgen05 split-K
    kernel, against the oracle's exact product and epilogue: bias, output
    table, residual, per-16-channel maxima; K from 128 to 8192 (1-64 K
    chunks over 8 or 16 warps), ragged channel counts."""
    few_mode(1 if kernel == "few" else 2)
    g = torch.Generator().manual_seed(m * 3 + k + n + bits)
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, n, bits)
    npad = qw.shape[0]
    bias = torch.zeros(npad, dtype=torch.bfloat16)
    bias[:n] = b
    args = dict(n_store=n)
    lut_bits = None
    if epilogue == "lut":
        lut = device_lut("tanh")
        args["out_lut"], lut_bits = lut, bits_of(lut.cpu())
    ua = oracle.unpack_int4(qa) if bits == 4 else qa
    uw = oracle.unpack_int4(qw) if bits == 4 else qw
    y = oracle.gemm_epilogue(oracle.int_matmul(ua, uw), sa, sw, bits_of(bias), 2, lut_bits)[:, :n]
    if epilogue == "residual":
        residual = randn_bf16(g, m, n)
        args["residual"] = residual.cuda()
        y = oracle.f32_to_bf16_bits(
            (oracle.bf16_bits_to_f32(y) + oracle.bf16_bits_to_f32(bits_of(residual))).astype(np.float32))
    if epilogue == "max_out":
        if npad % 16:
            pytest.skip("per-16-channel maxima need npad % 16 == 0")
        args["max_out"] = torch.full((m, npad // 16), -1.0, device="cuda")
    out = ops.gemm(torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
                   torch.from_numpy(sw).cuda(), bias.cuda(), bits, **args)
    got = bits_of(out)
    mismatch = np.argwhere(got != y)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    if epilogue == "max_out":
        groups = n // 16
        want = np.abs(oracle.bf16_bits_to_f32(y))[:, : groups * 16].reshape(m, groups, 16).max(-1)
        assert np.array_equal(args["max_out"][:, :groups].cpu().numpy(), want)
    assert_status_clean()


@pytest.mark.parametrize("m,mode,few", [(16, 0, 1), (16, 0, 2), (32, 0, 1), (64, 0, 0), (100, 1, 0), (100, 2, 0),
                                        (256, 1, 0), (256, 2, 0)])
def test_gemm_epilogue_rounding_ties_bitwise(m, mode, few, pair_mode, few_mode):
    """Planted bf16 rounding ties in the dequant + bias epilogue: every GEMM
    plan (split-K small tiles, one-SM and 2-SM many-token tiles) must round
    acc*sa*sw + bias in the reference's order (two multiplies, then the add,
    each rounded), not as one fused multiply-add."""
    pair_mode(mode)
    few_mode(few)
    n = 512
    qa, sa, qw, sw, bias, acc, planted = rounding_tie_problem(m, n, seed=m)
    assert planted >= m // 2
    assert np.array_equal(oracle.int_matmul(qa, qw), acc)
    ref = oracle.gemm_epilogue(acc, sa, sw, bias, 2)
    out = ops.gemm(torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(qw).cuda(),
                   torch.from_numpy(sw).cuda(), to_dev(bias), 8)
    got = bits_of(out)
    mismatch = np.argwhere(got != ref)
    assert mismatch.size == 0, f"{len(mismatch)} of {planted} planted ties, first at {mismatch[:4].tolist()}"
    assert_status_clean()


@pytest.mark.parametrize("m,mode", [(16, 0), (100, 1), (100, 2), (256, 1), (256, 2)])
def test_gemm_swiglu_rounding_ties_bitwise(m, mode, pair_mode):
    """The same planted ties in the gate and up values of the SwiGLU
    epilogue (gate|up interleaved in 128-row blocks)."""
    from pir2_b200.fused import prepare_silu

    pair_mode(mode)
    half = 256
    qa, sa, qw, sw, bias, acc, planted = rounding_tie_problem(m, 2 * half, seed=1000 + m)
    assert planted >= m // 2
    lut = prepare_silu(torch.device("cuda"))
    y = oracle.gemm_epilogue(acc, sa, sw, bias, 2)
    silu = oracle.bf16_bits_to_f32(bits_of(lut.cpu())[y[:, :half]])
    up = oracle.bf16_bits_to_f32(y[:, half:])
    ref = oracle.f32_to_bf16_bits((silu * up).astype(np.float32))
    cat = lambda t: ops.interleave_gate_up(t, half)   # noqa: E731
    out = ops.gemm_swiglu(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), cat(torch.from_numpy(qw).cuda()),
        cat(torch.from_numpy(sw).cuda()), cat(to_dev(bias)), lut, half_n=half,
    )
    got = bits_of(out)
    mismatch = np.argwhere(got != ref)
    assert mismatch.size == 0, f"{len(mismatch)} mismatches, first at {mismatch[:4].tolist()}"
    assert_status_clean()


@pytest.mark.parametrize("m,k,half", [(544, 2048, 6144), (1088, 1536, 3000), (130, 256, 640), (4400, 512, 1024)])
def test_gemm_swiglu_pair_tiles_bitwise(m, k, half, pair_mode):
    """gate|up on 2-SM tiles: CTA r of pair p holds gate block 2p + r and its
    up block; the value is bf16(silu_lut[gate] * up) of the exact outputs."""
    from pir2_b200.fused import prepare_silu

    pair_mode(1)
    half_pad = (half + 127) // 128 * 128
    g = torch.Generator().manual_seed(m + k + half)
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, 2 * half_pad, 8)
    lut = prepare_silu(torch.device("cuda"))
    y = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa, sw, bits_of(b), 2)
    silu = oracle.bf16_bits_to_f32(bits_of(lut.cpu())[y[:, :half]])
    up = oracle.bf16_bits_to_f32(y[:, half_pad : half_pad + half])
    ref = oracle.f32_to_bf16_bits((silu * up).astype(np.float32))
    cat = lambda t: ops.interleave_gate_up(t, half_pad)   # noqa: E731
    out = ops.gemm_swiglu(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), cat(torch.from_numpy(qw).cuda()),
        cat(torch.from_numpy(sw).cuda()), cat(b.cuda()), lut, half_n=half_pad,
    )[:, :half]
    got = bits_of(out)
    mismatch = np.argwhere(got != ref)
    detail = [(int(r), int(c), hex(got[r, c]), hex(ref[r, c]), hex(y[r, c]), hex(y[r, half_pad + c]))
              for r, c in mismatch[:4]]
    assert mismatch.size == 0, f"{len(mismatch)} mismatches (row, col, got, want, gate, up): {detail}"
    assert_status_clean()


@pytest.mark.parametrize("m,k,half,mode", [(544, 2048, 6144, 1), (544, 2048, 6144, 2), (17, 1536, 1024, 0),
                                           (300, 512, 640, 2)])
def test_gemm_swiglu_max_out_feeds_the_pack_bitwise(m, k, half, mode, pair_mode):
    """The SwiGLU epilogue's per-16-column maxima (2-SM and one-SM plans)
    equal |h|'s, and packing h from them gives the bytes of packing h."""
    from pir2_b200.fused import prepare_silu

    pair_mode(mode)
    g = torch.Generator().manual_seed(m * 3 + k + half)
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, 2 * half, 8)
    lut = prepare_silu(torch.device("cuda"))
    cat = lambda t: ops.interleave_gate_up(t, half)   # noqa: E731
    args = (torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), cat(torch.from_numpy(qw).cuda()),
            cat(torch.from_numpy(sw).cuda()), cat(b.cuda()), lut)
    plain = ops.gemm_swiglu(*args, half_n=half)
    maxes = torch.full((m, half // 16), -1.0, device="cuda")
    out = ops.gemm_swiglu(*args, half_n=half, max_out=maxes)
    assert torch.equal(out, plain)
    want = out.float().abs().reshape(m, half // 16, 16).amax(dim=2)
    assert torch.equal(maxes, want)
    q1, s1 = ops.quant_rows_max(out, maxes, 8)
    q2, s2 = ops.quant_rows(out, 8)
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    assert_status_clean()


def _sdpa_rows(q, k, v, b, heads, d):
    """fp32 torch SDPA over [B*T, H*D] rows, result as rows."""
    t, s = q.shape[0] // b, k.shape[0] // b
    qh = q.float().reshape(b, t, heads, d).transpose(1, 2)
    kh = k.float().reshape(b, s, heads, d).transpose(1, 2)
    vh = v.float().reshape(b, s, heads, d).transpose(1, 2)
    y = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
    return y.transpose(1, 2).reshape(b * t, heads * d)


@pytest.mark.parametrize(
    "b,t,s,heads,d",
    [
        (1, 17, 17, 32, 48),      # DiT self-attention: one CTA per head
        (1, 17, 544, 32, 48),     # DiT cross-attention: 8-CTA cluster per head
        (2, 17, 544, 32, 48),
        (3, 5, 33, 4, 64),
        (1, 9, 130, 2, 128),      # 2 chunks, padded keys
        (1, 70, 300, 4, 48),      # two query tiles of 64 across the cluster combine
        (2, 3, 1500, 2, 32),      # 188 keys per CTA: three online-softmax blocks, ragged
        (1, 33, 96, 3, 96),
    ],
)
def test_attention_rows_matches_fp32_sdpa(b, t, s, heads, d):
    # Tolerance: bf16 output rounding (2^-8 relative) plus fp32 summation
    # order; inputs are exactly representable bf16.
    g = torch.Generator(device="cuda").manual_seed(5)
    w = heads * d
    q = torch.randn(b * t, w, device="cuda", generator=g).to(torch.bfloat16)
    kv = torch.randn(b * s, 2 * w, device="cuda", generator=g).to(torch.bfloat16)
    k, v = kv[:, :w], kv[:, w:]            # row stride 2*w, as a grouped k|v output
    out = ops.attention_rows(q, k, v, batch=b, heads=heads, head_dim=d)
    ref = _sdpa_rows(q, k, v, b, heads, d)
    torch.testing.assert_close(out.float(), ref, atol=4e-3, rtol=8e-3)


def test_attention_rows_strided_query_and_argument_errors():
    heads, d, t = 4, 48, 7
    w = heads * d
    g = torch.Generator(device="cuda").manual_seed(6)
    qkv = torch.randn(t, 3 * w, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = qkv[:, :w], qkv[:, w:2 * w], qkv[:, 2 * w:]
    out = ops.attention_rows(q, k, v, batch=1, heads=heads, head_dim=d)
    torch.testing.assert_close(out.float(), _sdpa_rows(q, k, v, 1, heads, d), atol=4e-3, rtol=8e-3)
    with pytest.raises(ValueError):
        ops.attention_rows(q, k, v, batch=1, heads=heads, head_dim=12)   # unsupported head_dim
    long_kv = torch.zeros(20000, 2 * w, device="cuda", dtype=torch.bfloat16)   # keys exceed shared memory
    with pytest.raises(ValueError):
        ops.attention_rows(q, long_kv[:, :w], long_kv[:, w:], batch=1, heads=heads, head_dim=d)


def _int8_layer(g, n, k, bias=True):
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    qw, sw = oracle.quantize_weight(oracle.bf16_bits_to_f32(bits_of(w)), 8)
    b = None
    if bias:
        b = np.zeros(qw.shape[0], dtype=np.uint16)
        b[:n] = bits_of((torch.randn(n, generator=g) * 0.01).to(torch.bfloat16))
        b = to_dev(b)
    return torch.from_numpy(qw).cuda(), torch.from_numpy(sw).cuda(), b


@pytest.mark.parametrize(
    "m,k,n",
    [
        (17, 1536, 1536),   # DiT o-proj: 8-rank split-K, 1-2 K blocks per rank
        (1, 1536, 1536),
        (32, 1536, 4608),
        (17, 2048, 3072),
        (5, 328, 200),      # ragged K (kpad 384) and channels
        (64, 1024, 1024),
    ],
)
@pytest.mark.parametrize("residual", [False, True])
def test_gemm_rows_fused_pack_equals_pack_then_gemm(m, k, n, residual):
    """The in-GEMM activation pack gives bitwise the pack kernel + GEMM."""
    g = torch.Generator().manual_seed(m * 3 + k + n)
    x = randn_bf16(g, m, k, outliers=True).cuda()
    qw, sw, b = _int8_layer(g, n, k)
    res = randn_bf16(g, m, n).cuda() if residual else None
    qa, sa = ops.quant_rows(x, 8)
    want = ops.gemm(qa, sa, qw, sw, b, 8, n_store=n, residual=res)
    got = ops.gemm_rows(x, qw, sw, b, n_store=n, residual=res)
    assert np.array_equal(bits_of(got), bits_of(want))
    # A strided view of wider rows reads only the first k columns.
    wide = torch.cat([x, randn_bf16(g, m, 64).cuda()], 1)
    got2 = ops.gemm_rows(wide[:, :k], qw, sw, b, n_store=n, residual=res)
    assert np.array_equal(bits_of(got2), bits_of(want))
    assert_status_clean()


@pytest.mark.parametrize("m,d,f", [(17, 1536, 6144), (3, 256, 1024), (32, 512, 2048)])
def test_gemm_max_out_feeds_the_next_fused_pack(m, d, f):
    """up GEMM (GELU table epilogue) writes per-16-channel |y| maxima; the
    down GEMM packs the up output inside itself from those maxima and its own
    K slice: bitwise the pack kernel + GEMM chain."""
    from pir2_b200.fused import prepare_gelu

    g = torch.Generator().manual_seed(m + d + f)
    x = randn_bf16(g, m, d, outliers=True).cuda()
    up_w, up_s, up_b = _int8_layer(g, f, d)
    dn_w, dn_s, dn_b = _int8_layer(g, d, f)
    lut = prepare_gelu(torch.device("cuda"), torch.bfloat16, "tanh")
    res = randn_bf16(g, m, d).cuda()
    qa, sa = ops.quant_rows(x, 8)
    h_ref = ops.gemm(qa, sa, up_w, up_s, up_b, 8, n_store=f, out_lut=lut)
    maxes = torch.full((m, up_w.shape[0] // 16), -1.0, device="cuda")
    h = ops.gemm(qa, sa, up_w, up_s, up_b, 8, n_store=f, out_lut=lut, max_out=maxes)
    assert np.array_equal(bits_of(h), bits_of(h_ref))
    want_max = h_ref.float().abs().reshape(m, -1, 16).amax(-1)
    assert torch.equal(maxes, want_max)
    qh, sh = ops.quant_rows(h_ref, 8)
    want = ops.gemm(qh, sh, dn_w, dn_s, dn_b, 8, n_store=d, residual=res)
    got = ops.gemm_rows(h, dn_w, dn_s, dn_b, x_max=maxes, n_store=d, residual=res)
    assert np.array_equal(bits_of(got), bits_of(want))
    # The fused pack can itself emit maxima for a following one.
    m2 = torch.full((m, dn_w.shape[0] // 16), -1.0, device="cuda")
    got3 = ops.gemm_rows(h, dn_w, dn_s, dn_b, x_max=maxes, n_store=d, residual=res, max_out=m2)
    assert np.array_equal(bits_of(got3), bits_of(want))
    assert torch.equal(m2, want.float().abs().reshape(m, -1, 16).amax(-1))
    assert_status_clean()


def test_gemm_rows_rejects_what_it_cannot_fuse():
    g = torch.Generator().manual_seed(1)
    qw, sw, b = _int8_layer(g, 256, 8192)
    with pytest.raises(ValueError):
        ops.gemm_rows(randn_bf16(g, 65, 8192).cuda(), qw, sw, b)    # more than one token tile
    with pytest.raises(ValueError):
        ops.gemm_rows(randn_bf16(g, 64, 8192).cuda(), qw, sw, b)    # whole rows exceed shared memory
    qw2, sw2, b2 = _int8_layer(g, 256, 100)
    with pytest.raises(ValueError):
        ops.gemm_rows(randn_bf16(g, 4, 100).cuda(), qw2, sw2, b2)   # k % 8 != 0
    assert_status_clean()


@pytest.mark.parametrize("rows,k", [(1, 128), (544, 2048), (37, 6144), (4096, 1536)])
def test_unpack_int4_matches_oracle(rows, k):
    g = np.random.default_rng(rows + k)
    packed = g.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    got = ops.unpack_int4(torch.from_numpy(packed).cuda()).cpu().numpy()
    assert np.array_equal(got, oracle.unpack_int4(packed))
    assert_status_clean()


@pytest.mark.parametrize("m", [65, 300, 1088])
@torch.inference_mode()
def test_w4a4_many_token_layer_on_unpacked_codes_equals_int4_kernel(m):
    """An IntegerLinear(bits=4) over more than WIDE_INT4_ROWS rows runs the
    int8 GEMM on unpacked codes; its output is bitwise the int4 kernel's and
    the oracle's, with and without a residual."""
    from pir2_b200.integer import WIDE_INT4_ROWS, IntegerLinear, prepare_activation

    assert m > WIDE_INT4_ROWS
    torch.manual_seed(m)
    with torch.device("cuda"):
        linear = torch.nn.Linear(1536, 1000, bias=True).to(torch.bfloat16)
    layer = IntegerLinear.from_linear(linear, bits=4)
    x = torch.randn(m, 1536, device="cuda", dtype=torch.bfloat16)
    residual = torch.randn(m, 1000, device="cuda", dtype=torch.bfloat16)
    packed = prepare_activation(x, 4)
    direct = ops.gemm(packed.data, packed.scales, layer.packed_weight, layer.weight_scale, layer.bias, 4,
                      n_store=1000)
    equal = lambda a, b: np.array_equal(bits_of(a), bits_of(b))   # noqa: E731
    assert equal(layer.forward_packed(packed), direct)
    direct_res = ops.gemm(packed.data, packed.scales, layer.packed_weight, layer.weight_scale, layer.bias,
                          4, n_store=1000, residual=residual)
    assert equal(layer.forward_packed(packed, residual=residual), direct_res)
    qa = packed.data.cpu().numpy()
    ref = oracle.gemm_epilogue(
        oracle.int_matmul(oracle.unpack_int4(qa), oracle.unpack_int4(layer.packed_weight.cpu().numpy())),
        packed.scales.cpu().numpy(), layer.weight_scale.cpu().numpy(), bits_of(layer.bias.cpu()), 2,
    )[:, :1000]
    assert np.array_equal(bits_of(direct.cpu()), ref)
    assert_status_clean()


@pytest.mark.parametrize(
    "b,t,hq,hk",
    [
        (1, 544, 16, 8),    # GR00T text layers: 9 query tiles, 9 key blocks
        (2, 544, 16, 8),
        (1, 1, 2, 1),
        (1, 63, 4, 4),      # one ragged query tile, no grouping
        (1, 65, 4, 2),      # second tile holds one query
        (3, 200, 8, 2),     # ragged key block, group of 4
    ],
)
def test_attention_causal_matches_fp32_sdpa(b, t, hq, hk):
    # Tolerance: bf16 output rounding (2^-8 relative) plus fp32 summation
    # order and the bf16 probabilities fed to the P.V MMA; inputs are
    # exactly representable bf16 and the reference runs in fp32.
    g = torch.Generator(device="cuda").manual_seed(t + hq)
    q = torch.randn(b, hq, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(b, hk, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(b, hk, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    out = ops.attention_causal(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(hq // hk, 1), v.float().repeat_interleave(hq // hk, 1),
        is_causal=True,
    )
    ref = ref.transpose(1, 2).reshape(b * t, hq * 128)
    torch.testing.assert_close(out.float(), ref, atol=4e-3, rtol=8e-3)
    assert _lib.device_status() == 0


def test_attention_causal_writes_strided_rows_only():
    """Rows of a wider buffer: columns beyond hq*128 are left untouched."""
    b, t, hq, hk = 1, 100, 4, 2
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(b, hq, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(b, hk, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(b, hk, t, 128, device="cuda", generator=g).to(torch.bfloat16)
    wide = torch.full((b * t, hq * 128 + 64), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.attention_causal(q, k, v, out=wide[:, : hq * 128])
    assert torch.equal(wide[:, hq * 128 :], torch.full_like(wide[:, hq * 128 :], 7.0))
    ref = ops.attention_causal(q, k, v)
    assert torch.equal(wide[:, : hq * 128], ref)
    with pytest.raises(ValueError):
        ops.attention_causal(q, k[:, :, :50].contiguous(), v)


@pytest.mark.parametrize("m,k,half", [(544, 2048, 6144), (17, 1536, 256), (300, 256, 384)])
def test_gemm_swiglu_bitwise(m, k, half):
    """gate|up GEMM with the SwiGLU epilogue == the gated pack's value
    bf16(silu_lut[gate] * up) of the two exact GEMM outputs."""
    from pir2_b200.fused import prepare_silu

    g = torch.Generator().manual_seed(m + k + half)
    _, _, b, qa, sa, qw, sw = quantized_problem(g, m, k, 2 * half, 8)
    lut = prepare_silu(torch.device("cuda"))
    y = oracle.gemm_epilogue(oracle.int_matmul(qa, qw), sa, sw, bits_of(b), 2)[:, : 2 * half]
    gate = oracle.bf16_bits_to_f32(y[:, :half])
    up = oracle.bf16_bits_to_f32(y[:, half:])
    silu = oracle.bf16_bits_to_f32(bits_of(lut.cpu())[y[:, :half]])
    ref = oracle.f32_to_bf16_bits((silu * up).astype(np.float32))
    del gate
    cat = lambda t: ops.interleave_gate_up(t, half)   # noqa: E731
    out = ops.gemm_swiglu(
        torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(), cat(torch.from_numpy(qw).cuda()),
        cat(torch.from_numpy(sw).cuda()), cat(b.cuda()), lut, half_n=half,
    )
    assert np.array_equal(bits_of(out), ref)


@pytest.mark.parametrize("m,d,f", [(17, 1536, 6144), (1, 1536, 6144), (40, 256, 2048), (64, 512, 2048)])
def test_dit_ffn_equals_the_four_launch_chain(m, d, f):
    """One-launch FFN == up GEMM (+GELU table) -> plain pack -> down GEMM
    (+residual), bit for bit; the workspace is left zeroed for reuse."""
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(m + d + f)
    x, _, b_up, qa, sa, qw_up, sw_up = quantized_problem(g, m, d, f, 8)
    _, _, b_dn, _, _, qw_dn, sw_dn = quantized_problem(g, m, f, d, 8)
    lut = device_lut("tanh")
    residual = randn_bf16(g, m, d).cuda()
    dev = lambda a: torch.from_numpy(a).cuda()   # noqa: E731
    up = SimpleNamespace(packed_weight=dev(qw_up), weight_scale=dev(sw_up), bias=b_up.cuda(),
                         out_features=f, in_features=d, _bias_mode=lambda: _lib.BIAS_ADD)
    down = SimpleNamespace(packed_weight=dev(qw_dn), weight_scale=dev(sw_dn), bias=b_dn.cuda(),
                           out_features=d, in_features=f, _bias_mode=lambda: _lib.BIAS_ADD)
    qa_d, sa_d = dev(qa), dev(sa)
    for _ in range(3):                      # repeated calls reuse the workspace
        got = ops.dit_ffn(qa_d, sa_d, up, down, lut, residual)
    h = ops.gemm(qa_d, sa_d, up.packed_weight, up.weight_scale, up.bias, 8, out_lut=lut, n_store=f)
    qh, sh = ops.quant_rows(h, 8)
    ref = ops.gemm(qh, sh, down.packed_weight, down.weight_scale, down.bias, 8, residual=residual, n_store=d)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    ws = ops.ffn_workspace(torch.device("cuda"), m, f)
    assert int(ws[:12].view(torch.int32).abs().sum()) == 0     # counters reset
    assert_status_clean()


@pytest.mark.parametrize("m,d,f", [(17, 1536, 6144), (40, 256, 2048)])
def test_dit_ffn_back_to_back_calls_on_one_workspace(m, d, f):
    """Two calls with different inputs, launched back to back on one stream
    and sharing the workspace: each output equals its own four-launch chain
    (the second call must not read the first call's codes or counters)."""
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(3 * m + d + f)
    _, _, b_up, qa1, sa1, qw_up, sw_up = quantized_problem(g, m, d, f, 8)
    _, _, b_dn, _, _, qw_dn, sw_dn = quantized_problem(g, m, f, d, 8)
    _, _, _, qa2, sa2, _, _ = quantized_problem(g, m, d, f, 8)
    lut = device_lut("tanh")
    dev = lambda a: torch.from_numpy(a).cuda()   # noqa: E731
    up = SimpleNamespace(packed_weight=dev(qw_up), weight_scale=dev(sw_up), bias=b_up.cuda(),
                         out_features=f, in_features=d, _bias_mode=lambda: _lib.BIAS_ADD)
    down = SimpleNamespace(packed_weight=dev(qw_dn), weight_scale=dev(sw_dn), bias=b_dn.cuda(),
                           out_features=d, in_features=f, _bias_mode=lambda: _lib.BIAS_ADD)
    inputs = [(dev(qa1), dev(sa1), randn_bf16(g, m, d).cuda()), (dev(qa2), dev(sa2), randn_bf16(g, m, d).cuda())]
    got = [ops.dit_ffn(qa, sa, up, down, lut, res) for qa, sa, res in inputs]
    for (qa, sa, res), out in zip(inputs, got):
        h = ops.gemm(qa, sa, up.packed_weight, up.weight_scale, up.bias, 8, out_lut=lut, n_store=f)
        qh, sh = ops.quant_rows(h, 8)
        ref = ops.gemm(qh, sh, down.packed_weight, down.weight_scale, down.bias, 8, residual=res, n_store=d)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert not torch.equal(got[0], got[1])
    assert_status_clean()


@pytest.mark.parametrize("bits", [8, 4])
def test_quant_codes_at_half_integer_boundaries(bits):
    """Rows whose values sit exactly on the rounding boundaries of the codes
    (v / s within an ulp of k + 1/2, ties to even): the packs multiply by the
    row's reciprocal and fall back to the IEEE division near a boundary, and
    must still equal rint(RN(v / s)) bit for bit."""
    limit = 127 if bits == 8 else 7
    halves = np.arange(-limit, limit, dtype=np.float32) + np.float32(0.5)
    rows = []
    for scale in (1.0, 0.5, 3.0, 2.0 ** -7, 1.5):
        row = np.concatenate([halves, [np.float32(limit)]]) * np.float32(scale)
        rows.append(np.resize(row, 1536))
    # Neighbours one bf16 step either side of each boundary.
    x = torch.from_numpy(np.stack(rows).astype(np.float32)).to(torch.bfloat16)
    up = torch.from_numpy(np.nextafter(np.stack(rows), np.float32(np.inf)).astype(np.float32)).to(torch.bfloat16)
    x = torch.cat([x, up, -x])
    q, s = ops.quant_rows(x.cuda(), bits)
    rq, rs = oracle.quant_rows(bits_of(x), bits)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(q.cpu().numpy(), rq)
    # The fused producers share the quantizer (modulation pack, zero shift).
    zero = torch.zeros(x.shape[0], 1536, dtype=torch.bfloat16)
    q2, s2, _ = ops.norm_quant_rows(x.cuda(), bits, scale=zero.cuda(), shift=zero.cuda(), tokens=1)
    rq2, rs2 = oracle.modulation_pack(bits_of(x), bits_of(zero), bits_of(zero), 1, bits)
    assert np.array_equal(q2.cpu().numpy(), rq2) and np.array_equal(s2.cpu().numpy(), rs2)
