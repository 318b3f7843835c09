"""numpy restatement of piR2's symmetric-row-v1 / NVFP4 / SmoothQuant maths.

Test infrastructure: used by tests/, smoke() and the benchmark's CPU baseline
as the checker, never by the product path.  Every function cites the
reference lines (paths relative to the piR2 repository) it restates.

All arithmetic is IEEE fp32 with one rounding per operation (numpy float32
elementwise ops never contract into FMAs); bf16 rounding is
round-to-nearest-even on the fp32 bit pattern.
"""

import numpy as np

__all__ = [
    "bf16_round",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "kpad_of",
    "npad_of",
    "pack_int4",
    "unpack_int4",
    "quant_rows",
    "quantize_weight",
    "int_matmul",
    "gemm_epilogue",
    "linear_w8a8",
    "rms_norm_pack",
    "torch_row_mean_config",
    "torch_row_mean",
    "rms_norm_tail_pack",
    "layer_norm_pack",
    "modulation_pack",
    "residual_norm_modulation_pack",
    "channel_scales",
    "e4m3_round",
    "e2m1_encode",
    "e2m1_decode",
    "nvfp4_sf_offset",
    "pack_nvfp4",
    "unpack_nvfp4",
    "nvfp4_gemm",
    "quant_fp8",
    "e4m3_decode",
    "fp8_gemm",
    "floating_values",
    "row_finite_max",
    "fp8_producer",
]

F32 = np.float32


# ----------------------------------------------------------------- bf16
def f32_to_bf16_bits(x):
    """fp32 -> bf16 bit pattern (uint16), round-to-nearest-even; NaN kept."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_bits_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(F32)


def bf16_round(x):
    """f32(bf16_rn(x))."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def kpad_of(k):
    return (k + 127) // 128 * 128


def npad_of(n):
    return (n + 7) // 8 * 8


# ----------------------------------------------------------------- int4
def pack_int4(q):
    """int8 codes in [-8, 7] -> bytes, low nibble = even column.

    integer.py:79-83 and :234-238 (`(q[0::2] & 15) | ((q[1::2] & 15) << 4)`).
    """
    q = np.asarray(q, dtype=np.int32)
    return ((q[..., 0::2] & 15) | ((q[..., 1::2] & 15) << 4)).astype(np.uint8)


def unpack_int4(b):
    b = np.asarray(b, dtype=np.uint8).astype(np.int32)
    lo = b & 15
    hi = b >> 4
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty(b.shape[:-1] + (b.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


# ----------------------------------------------------------------- activations
def _limit(bits):
    return (1 << (bits - 1)) - 1


def _row_scale(m, bits):
    # integer.py:69-71: where(max > 0, max * (1.0 / limit), 1.0), an fp32
    # multiply by the fp32 constant 1/limit.
    inv = F32(1.0) / F32(_limit(bits))
    return np.where(m > 0, (m * inv).astype(F32), F32(1.0)).astype(F32)


def _quantize(v, s, bits):
    # integer.py:74-75: nearbyint(div_rn(x, scale)) clamped to +-limit.
    lim = _limit(bits)
    with np.errstate(invalid="ignore", over="ignore"):
        q = np.rint((v / s[:, None]).astype(F32))
    return np.clip(q, -lim, lim).astype(np.int8)


def quant_rows(x_bits, bits, *, lut_bits=None, up_bits=None, smooth=None):
    """Per-row symmetric quantization (symmetric-row-v1).

    Restates `_activation_values` + `_prepare` (integer.py:27-94) and the
    native twin `prepare_integer` (integer_dispatch.cu:11-65):
      mode 0: v = f32(x); mode 2: v = f32(lut[x]); mode 1: v = f32(bf16(
      f32(lut[x]) * f32(up))); columns k..Kpad are 0; s = max|v| * (1/L)
      (1 if 0); q = clamp(rint(v / s), -L, L).
    `smooth` (fp32 [k]) applies the SmoothQuant input division
    bf16(bf16(v) / s) of thor/packing.py:69-73 before quantization.
    Inputs are bf16 bit patterns (uint16).  Returns (codes, scales): int8
    [rows, Kpad] for bits 8, packed uint8 [rows, Kpad/2] for bits 4.
    """
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    rows, k = x_bits.shape
    pad = kpad_of(k)
    if lut_bits is None:
        v = bf16_bits_to_f32(x_bits)
    else:
        lut_bits = np.asarray(lut_bits, dtype=np.uint16)
        v = bf16_bits_to_f32(lut_bits[x_bits])
        if up_bits is not None:
            v = bf16_round((v * bf16_bits_to_f32(up_bits)).astype(F32))
    if smooth is not None:
        v = bf16_round((bf16_round(v) / np.asarray(smooth, F32)[None, :]).astype(F32))
    full = np.zeros((rows, pad), dtype=F32)
    full[:, :k] = v
    s = _row_scale(np.abs(full).max(axis=1).astype(F32), bits)
    q = _quantize(full, s, bits)
    return (q if bits == 8 else pack_int4(q)), s


def quantize_weight(w, bits, *, scale_rule="cuda"):
    """Per-output-channel weight quantization and padding.

    Restates `IntegerLinear.from_linear` (integer.py:211-256):
    s_n = max_k |f32(w)| / L (1.0 for an all-zero row),
    q = clamp(round_half_even(w / s_n), -L, L), K zero-padded to Kpad and N to
    Npad (scales padded with 1.0), int4 nibble-packed low-first.

    `maximum / limit` divides a CUDA tensor by a Python scalar, which PyTorch
    evaluates on the GPU as a multiply by the fp32 reciprocal; that is the
    reference's effective arithmetic (scale_rule "cuda", the default).  CPU
    torch divides (scale_rule "divide").  `w / s` is a tensor-by-tensor IEEE
    division in both.  Returns (codes, scales[Npad]).
    """
    w = np.asarray(w, dtype=F32)
    n, k = w.shape
    lim = _limit(bits)
    m = np.abs(w).max(axis=1).astype(F32)
    if scale_rule == "cuda":
        raw = (m * (F32(1.0) / F32(lim))).astype(F32)
    elif scale_rule == "divide":
        raw = (m / F32(lim)).astype(F32)
    else:
        raise ValueError("scale_rule must be 'cuda' or 'divide'")
    s = np.where(m > 0, raw, F32(1.0)).astype(F32)
    q = np.clip(np.rint((w / s[:, None]).astype(F32)), -lim, lim).astype(np.int8)
    qp = np.zeros((npad_of(n), kpad_of(k)), dtype=np.int8)
    qp[:n, :k] = q
    sp = np.ones(npad_of(n), dtype=F32)
    sp[:n] = s
    return (qp if bits == 8 else pack_int4(qp)), sp


def int_matmul(qa, qw):
    """Exact int32 A @ W^T for int8 codes (float64 BLAS is exact here: every
    partial sum is an integer below 2^53)."""
    a = np.asarray(qa, dtype=np.float64)
    w = np.asarray(qw, dtype=np.float64)
    return np.rint(a @ w.T).astype(np.int64).astype(np.int32)


def gemm_epilogue(acc, sa, sw, bias_bits=None, bias_mode=1, out_lut_bits=None):
    """Dequant epilogue of pir2_integer::gemm (integer_gemm.cu:37-59, 73-76,
    164-168): y = bf16(f32(f32(i2f(acc) * sa[m]) * sw[n]) [+ f32(bias[n])]).

    bias_mode 0 skips the add (gemm_biasless without bias), 1 adds +0 (gemm
    with a null bias, turning -0 into +0), 2 adds the bias.  An optional
    activation table is applied to the bf16 result.  Returns bf16 bits.
    """
    accf = np.asarray(acc, dtype=np.int32).astype(F32)
    y = (accf * np.asarray(sa, F32)[:, None]).astype(F32)
    y = (y * np.asarray(sw, F32)[None, :]).astype(F32)
    if bias_mode == 1:
        y = (y + F32(0.0)).astype(F32)
    elif bias_mode == 2:
        y = (y + bf16_bits_to_f32(bias_bits)[None, :]).astype(F32)
    out = f32_to_bf16_bits(y)
    if out_lut_bits is not None:
        out = np.asarray(out_lut_bits, dtype=np.uint16)[out]
    return out


def linear_w8a8(x_bits, w_f32, bias_bits, bits, *, bias_mode=None, smooth=None, scale_rule="cuda"):
    """Whole quantized Linear: quantize rows, quantize weights, int GEMM,
    dequant epilogue.  Returns bf16 bits [rows, n]."""
    n = np.asarray(w_f32).shape[0]
    qa, sa = quant_rows(x_bits, bits, smooth=smooth)
    qw, sw = quantize_weight(w_f32, bits, scale_rule=scale_rule)
    if bits == 4:
        qa, qw = unpack_int4(qa), unpack_int4(qw)
    acc = int_matmul(qa, qw)
    if bias_mode is None:
        bias_mode = 2 if bias_bits is not None else 1
    bias_full = None
    if bias_bits is not None:
        bias_full = np.zeros(qw.shape[0], dtype=np.uint16)
        bias_full[:n] = bias_bits
    return gemm_epilogue(acc, sa, sw, bias_full, bias_mode)[:, :n]


# ----------------------------------------------------------------- producers
# Norm producers: the reference's reductions are tree sums in an unspecified
# order with approximate rsqrt, so these are tolerance oracles (the
# reference itself states the fused packs are not bitwise equal to native
# torch norms: modulation.py:163-165, tests/gpu/test_groot_norm_quant_gpu.py).
def _rsqrt(v):
    return (F32(1.0) / np.sqrt(v.astype(np.float64))).astype(F32)


def rms_norm_values(x_bits, gamma_bits, eps):
    """producers.py:19-53: n = bf16(x * rsqrt(mean(x^2) + eps)); v = bf16(n * g)."""
    x = bf16_bits_to_f32(x_bits)
    var = (np.sum(x.astype(np.float64) ** 2, axis=1) / x.shape[1]).astype(F32)
    inv = _rsqrt((var + F32(eps)).astype(F32))
    n = bf16_round((x * inv[:, None]).astype(F32))
    return bf16_round((n * bf16_bits_to_f32(gamma_bits)[None, :]).astype(F32))


def torch_row_mean_config(rows, k):
    """Threads per row (bw) and the fp32 mean factor of torch's CUDA row mean
    over a contiguous fp32 [rows, k] tensor (ATen/native/cuda/Reduce.cuh,
    setReduceConfig with 4-float input vectors), the reduction the reference's
    B200 RMS statistics use (rms_statistics.py:171-190: squares, then
    `squared.mean(-1)`).  None when torch would split a row across warps."""

    def last_pow2(n):
        return 1 << (int(n).bit_length() - 1)

    if k < 128 or k % 4 or rows < 1:
        return None
    dim0, dim1 = k // 4, rows
    d0 = last_pow2(dim0) if dim0 < 512 else 512
    d1 = last_pow2(dim1) if dim1 < 512 else 512
    bw = min(d0, 32)
    bh = min(d1, 512 // bw)
    bw = min(d0, 512 // bh)
    if -(-k // bw) >= min(bh * 16, 256):
        return None
    return bw, F32(F32(rows) / F32(rows * k))


def torch_row_mean(sq, bw, factor):
    """Row means of fp32 [rows, k] in the order of torch's CUDA reduction for
    that launch shape: virtual thread t of bw adds the 4-float vectors
    t, t + bw, ... into four accumulators (element i of each vector into
    accumulator i), combines them as ((a0 + a1) + a2) + a3, and the bw
    partials are added pairwise with halving offsets (bw/2, ..., 1); the
    mean is that sum times `factor`."""
    sq = np.asarray(sq, F32)
    rows, k = sq.shape
    vec = sq.reshape(rows, k // 4, 4)
    nvec = k // 4
    part = np.zeros((rows, bw), F32)
    for t in range(bw):
        acc = np.zeros((rows, 4), F32)
        for idx in range(t, nvec, bw):
            acc = (acc + vec[:, idx, :]).astype(F32)
        part[:, t] = (((acc[:, 0] + acc[:, 1]).astype(F32) + acc[:, 2]).astype(F32) + acc[:, 3]).astype(F32)
    width = bw
    while width > 1:
        half = width // 2
        part[:, :half] = (part[:, :half] + part[:, half:width]).astype(F32)
        width = half
    return (part[:, 0] * F32(factor)).astype(F32)


def rms_norm_tail_values(x_bits, gamma_bits, var, inv):
    """`_rms_tail_pack` (producers.py:19-53) given the row variance and its
    inverse root rsqrt(var + eps) as the device computes them:
    n = bf16(x * inv); v = bf16(n * gamma)."""
    x = bf16_bits_to_f32(x_bits)
    inv = np.asarray(inv, F32)
    n = bf16_round((x * inv[:, None]).astype(F32))
    return bf16_round((n * bf16_bits_to_f32(gamma_bits)[None, :]).astype(F32))


def rms_norm_tail_pack(x_bits, gamma_bits, var, inv, bits):
    return _pack_values(rms_norm_tail_values(x_bits, gamma_bits, var, inv), bits)


def layer_norm_values(x_f32, eps):
    """modulation.py:157-165: centred two-pass LayerNorm, bf16 output."""
    x = np.asarray(x_f32, F32)
    mean = (np.sum(x.astype(np.float64), axis=1) / x.shape[1]).astype(F32)
    c = (x - mean[:, None]).astype(F32)
    var = (np.sum(c.astype(np.float64) ** 2, axis=1) / x.shape[1]).astype(F32)
    return bf16_round((c * _rsqrt((var + F32(eps)).astype(F32))[:, None]).astype(F32))


def modulate_values(n_f32, scale_bits, shift_bits, tokens):
    """modulation.py:103-107: factor = bf16(1 + scale); p = bf16(n * factor);
    v = bf16(p + shift); scale/shift row = row // tokens."""
    rows = n_f32.shape[0]
    idx = np.arange(rows) // tokens
    s = bf16_bits_to_f32(scale_bits)[idx]
    h = bf16_bits_to_f32(shift_bits)[idx]
    factor = bf16_round((F32(1.0) + s).astype(F32))
    p = bf16_round((n_f32 * factor).astype(F32))
    return bf16_round((p + h).astype(F32))


def _pack_values(v, bits):
    rows, k = v.shape
    full = np.zeros((rows, kpad_of(k)), dtype=F32)
    full[:, :k] = v
    s = _row_scale(np.abs(full).max(axis=1).astype(F32), bits)
    q = _quantize(full, s, bits)
    return (q if bits == 8 else pack_int4(q)), s


def rms_norm_pack(x_bits, gamma_bits, eps, bits):
    return _pack_values(rms_norm_values(x_bits, gamma_bits, eps), bits)


def layer_norm_pack(x_bits, eps, bits):
    return _pack_values(layer_norm_values(bf16_bits_to_f32(x_bits), eps), bits)


def modulation_pack(x_bits, scale_bits, shift_bits, tokens, bits, *, eps=None):
    """`_prepare_modulation` / `_prepare_norm_modulation` (modulation.py:123-188)."""
    x = bf16_bits_to_f32(x_bits)
    n = x if eps is None else layer_norm_values(x, eps)
    return _pack_values(modulate_values(n, scale_bits, shift_bits, tokens), bits)


def residual_norm_modulation_pack(x_bits, y_bits, gate_bits, scale_bits, shift_bits, tokens, bits, eps):
    """`_prepare_residual_norm_modulation` (modulation.py:191-219):
    r = bf16(x + bf16(y * gate)); pack(modulate(LN(r))).  Returns (q, s, r bits)."""
    rows = np.asarray(x_bits).shape[0]
    idx = np.arange(rows) // tokens
    prod = bf16_round((bf16_bits_to_f32(y_bits) * bf16_bits_to_f32(gate_bits)[idx]).astype(F32))
    r = bf16_round((bf16_bits_to_f32(x_bits) + prod).astype(F32))
    q, s = _pack_values(modulate_values(layer_norm_values(r, eps), scale_bits, shift_bits, tokens), bits)
    return q, s, f32_to_bf16_bits(r)


# ----------------------------------------------------------------- SmoothQuant
def channel_scales(act_absmax, weights, alpha):
    """thor/smoothquant.py:27-45:
    s = clamp(amax^a / clamp(max_{w in group, n} |W_nc|, 1e-5)^(1-a), 1e-5)."""
    act = np.asarray(act_absmax, dtype=F32)
    wmax = np.max(np.stack([np.abs(np.asarray(w, F32)).max(axis=0) for w in weights]), axis=0)
    wmax = np.maximum(wmax, F32(1e-5)).astype(F32)
    num = np.power(act, F32(alpha)).astype(F32)
    den = np.power(wmax, F32(1.0 - alpha)).astype(F32)
    return np.maximum((num / den).astype(F32), F32(1e-5)).astype(F32)


# ----------------------------------------------------------------- NVFP4
def _e4m3_table():
    codes = np.arange(128, dtype=np.uint32)
    e = (codes >> 3) & 15
    m = codes & 7
    vals = np.where(e == 0, m / 512.0, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    vals[127] = np.nan  # 0x7F is NaN in e4m3fn
    return vals


_E4M3 = _e4m3_table()


def e4m3_round(v):
    """Non-negative fp32 -> e4m3fn code, round-to-nearest-even, satfinite.
    Returns (codes uint8, decoded fp32)."""
    v = np.asarray(v, dtype=np.float64)
    finite = _E4M3[:127]
    idx = np.searchsorted(finite, v)
    idx = np.clip(idx, 1, 126)
    lo, hi = finite[idx - 1], finite[idx]
    pick_hi = (v - lo > hi - v) | ((v - lo == hi - v) & ((idx % 2) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(v >= finite[126], 126, code)
    code = np.where(v <= 0, 0, code)
    return code.astype(np.uint8), _E4M3[code].astype(F32)


_E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_encode(v):
    """fp32 -> e2m1 code (4 bits), round-to-nearest-even, saturating to +-6;
    the sign bit is kept for negative inputs that round to zero."""
    v = np.asarray(v, dtype=np.float64)
    a = np.abs(v)
    idx = np.clip(np.searchsorted(_E2M1, a), 1, 7)
    lo, hi = _E2M1[idx - 1], _E2M1[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & ((idx % 2) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(a >= 6.0, 7, code)
    sign = (np.signbit(v)).astype(np.int64) << 3
    return (code | sign).astype(np.uint8)


def e2m1_decode(c):
    c = np.asarray(c, dtype=np.uint8)
    mag = _E2M1[c & 7]
    return np.where(c & 8, -mag, mag).astype(F32)


def nvfp4_sf_offset(row, sf, blocks_k):
    """Scale-factor byte offset, fp4_cutlass_linear.cu:686-690 and
    thor/packing.py:46-53 (128-row x 4-factor atoms of 512 bytes)."""
    row = np.asarray(row, dtype=np.int64)
    sf = np.asarray(sf, dtype=np.int64)
    return ((row >> 7) * blocks_k << 9) + ((row & 31) << 4) + (((row & 127) >> 5) << 2) + ((sf >> 2) << 9) + (sf & 3)


def pack_nvfp4(x_f32):
    """`_store_fp4_row` (thor/packing.py:24-54): per 16-block m = max|v|;
    s = m / 6 (IEEE; 1 if m == 0); e = e4m3(min(s, 448)); d = f32(e), or s if
    d <= 0; codes = e2m1(v * (1 / d)).  Returns (packed [rows, k/2], sf)."""
    v = np.asarray(x_f32, dtype=F32)
    rows, k = v.shape
    g = v.reshape(rows, k // 16, 16)
    m = np.abs(g).max(axis=2).astype(F32)
    s = np.where(m > 0, (m / F32(6.0)).astype(F32), F32(1.0)).astype(F32)
    code, d = e4m3_round(np.minimum(s, F32(448.0)))
    d = np.where(d > 0, d, s).astype(F32)
    r = (F32(1.0) / d).astype(F32)
    q = e2m1_encode((g * r[:, :, None]).astype(F32)).reshape(rows, k)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    blocks_k = (k // 16 + 3) // 4
    sf = np.zeros(((rows + 127) // 128 * 128) * blocks_k * 4, dtype=np.uint8)
    rr, jj = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    sf[nvfp4_sf_offset(rr, jj, blocks_k)] = code
    return packed, sf.reshape((rows + 127) // 128 * 128, blocks_k * 4)


def unpack_nvfp4(packed, sf, rows, k):
    """Dequantized fp32 values of an NVFP4 pack (codes * block factor)."""
    packed = np.asarray(packed, dtype=np.uint8)
    codes = np.empty((rows, k), dtype=np.uint8)
    codes[:, 0::2] = packed & 15
    codes[:, 1::2] = packed >> 4
    blocks_k = (k // 16 + 3) // 4
    rr, jj = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    fac = _E4M3[np.asarray(sf).reshape(-1)[nvfp4_sf_offset(rr, jj, blocks_k)]]
    return (e2m1_decode(codes).reshape(rows, k // 16, 16) * fac[:, :, None]).reshape(rows, k)


def nvfp4_gemm(pa, sfa, pw, sfw, m, n, k, bias_bits=None, alpha=1.0):
    """fp64 reference of the block-scaled FP4 GEMM: sum_k (a*sfa)(w*sfw),
    times alpha, plus bias, rounded to bf16 (fp4_cutlass_linear.cu:1358,
    alpha = 1).  Returns bf16 bits."""
    a = unpack_nvfp4(pa, sfa, m, k).astype(np.float64)
    w = unpack_nvfp4(pw, sfw, n, k).astype(np.float64)
    y = (a @ w.T) * alpha
    if bias_bits is not None:
        y = y + bf16_bits_to_f32(bias_bits).astype(np.float64)[None, :]
    return f32_to_bf16_bits(y.astype(F32))


# ----------------------------------------------------------------- FP8
def quant_fp8(x_bits, *, fast=False):
    """Per-tensor E4M3 quantization of bf16 values.

    Default: fp8_cutlass_linear.cu:61-120 (quantize_bf16, also the weight
    pack pack_linear_weight :1011-1024): amax of the finite |x| (fp32),
    scale = max(amax / 448, 1e-12), q = e4m3_rn_satfinite(clamp(x * (1 /
    scale), -448, 448)).  fast=True: thor/packing.py:451-519 (prepare_fp8):
    scale = max(amax * (1/448), 1e-12), q = e4m3(clamp(x / scale)); the
    division is IEEE round-to-nearest here.  A NaN input clamps to -448 as
    fminf(448, fmaxf(-448, NaN)) does.  Returns (codes uint8, scale fp32).
    """
    x = bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16)).astype(F32)
    a = np.abs(x)
    a = np.where(np.isfinite(a), a, F32(0))
    amax = F32(a.max()) if a.size else F32(0)
    if fast:
        scale = max(F32(amax * F32(1.0 / 448.0)), F32(1e-12))
        y = (x / F32(scale)).astype(F32)
    else:
        scale = max(F32(amax / F32(448.0)), F32(1e-12))
        inv = F32(F32(1.0) / F32(scale))
        y = (x * inv).astype(F32)
    y = np.where(np.isnan(y), F32(-448.0), y)
    y = np.clip(y, F32(-448.0), F32(448.0)).astype(F32)
    code, _ = e4m3_round(np.abs(y))
    code = np.where(np.signbit(y), code | np.uint8(0x80), code).astype(np.uint8)
    return code, F32(scale)


def e4m3_decode(codes):
    """E4M3fn codes -> float64 values."""
    c = np.asarray(codes, dtype=np.uint8)
    mag = _E4M3[c & 0x7F]
    return np.where(c & 0x80, -mag, mag)


def fp8_gemm(qa, sa, qw, sw, bias_bits=None):
    """fp64 reference of the E4M3 GEMM: (sum_k a[m,k] w[n,k]) * sa * sw
    [+ bias], for per-tensor scales sa, sw (the CUTLASS epilogue's
    scale_a * scale_b, fp8_cutlass_linear.cu:630-643)."""
    acc = e4m3_decode(qa) @ e4m3_decode(qw).T
    y = acc * float(sa) * float(sw)
    if bias_bits is not None:
        y = y + bf16_bits_to_f32(np.asarray(bias_bits, dtype=np.uint16)).astype(np.float64)
    return y


# ----------------------------------------------------------------- FP8 producers
def floating_values(x_bits, *, lut_bits=None, up_bits=None, smooth=None):
    """The bf16 values the Thor producers store before packing
    (thor/packing.py:57-82 `_store_producer`, :84-107 `_swiglu_pack`,
    :314-328 `_smooth_pack`, :352-369 `_gelu_pack`): v = f32(x), or
    f32(lut[x]), or bf16(f32(lut[x]) * f32(up)); then with `smooth`
    v = bf16(v / s) (IEEE division).  Returns fp32 (bf16-exact) [rows, k]."""
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    if lut_bits is None:
        v = bf16_bits_to_f32(x_bits)
    else:
        v = bf16_bits_to_f32(np.asarray(lut_bits, dtype=np.uint16)[x_bits])
        if up_bits is not None:
            v = bf16_round((v * bf16_bits_to_f32(up_bits)).astype(F32))
    if smooth is not None:
        v = bf16_round((bf16_round(v) / np.asarray(smooth, F32)[None, :]).astype(F32))
    return v.astype(F32)


def row_finite_max(v):
    """Each row's maximum finite |value| (packing.py:76-78; 0 for a row with
    none)."""
    a = np.abs(np.asarray(v, F32))
    return np.where(np.isfinite(a), a, F32(0)).max(axis=1).astype(F32)


def fp8_producer(values):
    """Second pass of the FP8 producers (`_finish_producer` with
    `_fp8_scale_and_cast`, packing.py:180-199, :461-482): the per-tensor
    scale from the row maxima and the E4M3 cast, i.e. prepare_fp8's
    arithmetic on the bf16 values.  Returns (codes, scale)."""
    return quant_fp8(f32_to_bf16_bits(np.asarray(values, F32)), fast=True)
