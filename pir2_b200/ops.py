"""Torch-facing wrappers of the C ABI: allocate outputs, validate, launch.

Every function runs on the current CUDA stream of the input's device, never
synchronizes and allocates only through torch's caching allocator, so all of
them can be captured in CUDA graphs (after the library has been loaded once).
Errors from the library are raised as ValueError (argument/alignment) or
RuntimeError (CUDA); there is no fallback implementation.
"""

import torch

from . import _lib

KPAD_MULTIPLE = 128
NPAD_MULTIPLE = 8


def kpad(k):
    return (k + KPAD_MULTIPLE - 1) // KPAD_MULTIPLE * KPAD_MULTIPLE


def npad(n):
    return (n + NPAD_MULTIPLE - 1) // NPAD_MULTIPLE * NPAD_MULTIPLE


# Optional launch recorder used by the benchmark to time individual GEMM
# launches with CUDA events (None in normal use).
launch_recorder = None


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _rows(x):
    """[rows, k] view and row stride of a tensor with unit last stride."""
    k = x.shape[-1]
    rows = x.numel() // k if k else 0
    try:
        matrix = x.view(rows, k)
    except RuntimeError as error:
        raise ValueError(
            "Activation leading dimensions must form regularly strided rows"
        ) from error
    return matrix, rows, k, (matrix.stride(0) if rows > 1 else max(k, matrix.stride(0)))


def quant_rows(x, bits, *, lut=None, up=None, smooth=None, out=None):
    """symmetric-row-v1 activation pack of bf16 rows -> (data, scales).

    mode: plain (no lut), LUT (lut only, e.g. GELU) or gated (lut and up,
    v = bf16(lut[x] * up), e.g. SiLU(gate) * up).
    """
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.stride(-1) != 1 or x.ndim < 2:
        raise ValueError("Expected CUDA BF16 rows with unit feature stride")
    matrix, rows, k, ldx = _rows(x)
    mode = _lib.MODE_PLAIN if lut is None else (_lib.MODE_LUT if up is None else _lib.MODE_GATED)
    ldu = 0
    if up is not None:
        if up.shape != x.shape or up.dtype != x.dtype or up.device != x.device or up.stride(-1) != 1:
            raise ValueError("Invalid gated activation input")
        _, _, _, ldu = _rows(up)
    if lut is not None and (lut.numel() != 65536 or lut.dtype != torch.bfloat16 or not lut.is_contiguous()):
        raise ValueError("Invalid activation lookup table")
    pad = kpad(k)
    if out is None:
        data = torch.empty(
            (rows, pad if bits == 8 else pad // 2),
            device=x.device,
            dtype=torch.int8 if bits == 8 else torch.uint8,
        )
        scales = torch.empty(rows, device=x.device, dtype=torch.float32)
    else:
        data, scales = out
    status = _lib.lib().pir2b_quant_rows(
        x.data_ptr(), ldx, _ptr(up), ldu, _ptr(lut), _ptr(smooth), mode, bits,
        rows, k, data.data_ptr(), scales.data_ptr(), _stream(x.device),
    )
    _lib.check(status, "pir2b_quant_rows")
    return data, scales


def quant_rows_max(x, x_max, bits):
    """symmetric-row-v1 pack of bf16 rows x [rows, k] whose maxima are known:
    x_max fp32 [rows, parts] partial maxima of |x| (the `max_out` of the GEMM
    that wrote x).  Same bytes and scales as `quant_rows(x, bits)`."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.stride(-1) != 1 or x.ndim < 2:
        raise ValueError("Expected CUDA BF16 rows with unit feature stride")
    matrix, rows, k, ldx = _rows(x)
    if x_max.dtype != torch.float32 or x_max.dim() != 2 or x_max.shape[0] != rows or not x_max.is_contiguous():
        raise ValueError("x_max must be contiguous fp32 [rows, parts]")
    pad = kpad(k)
    data = torch.empty((rows, pad if bits == 8 else pad // 2), device=x.device,
                       dtype=torch.int8 if bits == 8 else torch.uint8)
    scales = torch.empty(rows, device=x.device, dtype=torch.float32)
    status = _lib.lib().pir2b_quant_rows_max(
        x.data_ptr(), ldx, x_max.data_ptr(), x_max.shape[1], bits, rows, k, data.data_ptr(), scales.data_ptr(),
        _stream(x.device),
    )
    _lib.check(status, "pir2b_quant_rows_max")
    return data, scales


def _floating_buffers(rows, k, out_format, device, maxima_per_row=1):
    """Outputs of a floating producer: NVFP4 (packed E2M1 [rows, k/2],
    swizzled UE4M3 factors) or the FP8 first pass (bf16 values [rows, k],
    fp32 partial maxima, `maxima_per_row` per row)."""
    if out_format == _lib.OUT_NVFP4:
        data = torch.empty((rows, k // 2), device=device, dtype=torch.uint8)
        scales = torch.empty((-(-rows // 128) * 128, -(-(k // 16) // 4) * 4), device=device, dtype=torch.uint8)
    else:
        data = torch.empty((rows, k), device=device, dtype=torch.bfloat16)
        scales = torch.empty(rows * maxima_per_row, device=device, dtype=torch.float32)
    return data, scales


def fp8_value_slices(k):
    """Partial maxima per row of an FP8 first pass over rows of k values (one
    per 1024-value slice)."""
    return -(-k // 1024)


def floating_rows(x, out_format, *, lut=None, up=None, smooth=None):
    """The activation values of `quant_rows` (plain, LUT, SiLU * up, / smooth)
    to a floating output: `_lib.OUT_NVFP4` -> (packed, swizzled factors);
    `_lib.OUT_FP8_VALUES` -> (bf16 values, fp32 partial maxima: one per row
    and 1024-value slice), finished by `fp8_cast`."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.stride(-1) != 1 or x.ndim < 2:
        raise ValueError("Expected CUDA BF16 rows with unit feature stride")
    matrix, rows, k, ldx = _rows(x)
    mode = _lib.MODE_PLAIN if lut is None else (_lib.MODE_LUT if up is None else _lib.MODE_GATED)
    ldu = 0
    if up is not None:
        if up.shape != x.shape or up.dtype != x.dtype or up.device != x.device or up.stride(-1) != 1:
            raise ValueError("Invalid gated activation input")
        _, _, _, ldu = _rows(up)
    if lut is not None and (lut.numel() != 65536 or lut.dtype != torch.bfloat16 or not lut.is_contiguous()):
        raise ValueError("Invalid activation lookup table")
    data, scales = _floating_buffers(rows, k, out_format, x.device, fp8_value_slices(k))
    status = _lib.lib().pir2b_floating_rows(
        x.data_ptr(), ldx, _ptr(up), ldu, _ptr(lut), _ptr(smooth), mode, out_format,
        rows, k, data.data_ptr(), scales.data_ptr(), _stream(x.device),
    )
    _lib.check(status, "pir2b_floating_rows")
    return data, scales


def fp8_cast(values, maxima, *, replicate=None):
    """Second pass of the FP8 producers: bf16 values [rows, k] and the first
    pass's partial maxima -> (E4M3 codes uint8 [rows, k], scale fp32 [1], the
    scale replicated `replicate` times (default: once per row))."""
    if values.dtype != torch.bfloat16 or not values.is_cuda or values.dim() != 2 or not values.is_contiguous():
        raise ValueError("fp8_cast needs contiguous CUDA bf16 [rows, k] values")
    rows, k = values.shape
    if maxima.dtype != torch.float32 or maxima.numel() < 1 or not maxima.is_contiguous():
        raise ValueError("fp8_cast needs the fp32 partial maxima of the first pass")
    n_rep = rows if replicate is None else int(replicate)
    q = torch.empty((rows, k), device=values.device, dtype=torch.uint8)
    scale = torch.empty(1, device=values.device, dtype=torch.float32)
    rep = torch.empty(max(n_rep, 1), device=values.device, dtype=torch.float32)
    status = _lib.lib().pir2b_fp8_cast(
        values.data_ptr(), k, maxima.data_ptr(), maxima.numel(), rows, k, 1, q.data_ptr(), scale.data_ptr(),
        rep.data_ptr() if n_rep > 0 else None, n_rep, _stream(values.device),
    )
    _lib.check(status, "pir2b_fp8_cast")
    return q, scale, rep[:n_rep]


def norm_quant_rows(
    x,
    out_format,
    *,
    norm=_lib.NORM_NONE,
    eps=0.0,
    gamma=None,
    scale=None,
    shift=None,
    tokens=1,
    y=None,
    gate=None,
    smooth=None,
):
    """Fused [residual +] [RMS|LN norm] [+ AdaLN] [/ smooth] -> pack.

    x, y: contiguous bf16 [rows, k]; scale/shift/gate: bf16 rows indexed by
    row // tokens with a shared row stride.  Returns (data, scales, residual)
    where residual is the bf16 x + bf16(y * gate) when y is given.
    """
    if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("Fused producers need contiguous CUDA BF16 input")
    k = x.shape[-1]
    rows = x.numel() // k
    ld_mod = 0
    for t in (scale, shift, gate):
        if t is not None:
            if t.dtype != torch.bfloat16 or t.device != x.device or t.stride(-1) != 1:
                raise ValueError("Modulation operands must be CUDA BF16 with unit stride")
            ld_mod = t.stride(-2) if t.ndim >= 2 and t.shape[-2] > 1 else k
    if scale is not None and shift is not None and scale.stride(-2) != shift.stride(-2) and scale.shape[-2] > 1:
        raise ValueError("Scale and shift must share a row stride")
    residual = None
    if y is not None:
        if y.shape != x.shape or not y.is_contiguous() or y.dtype != x.dtype:
            raise ValueError("Residual operand must match the contiguous BF16 input")
        residual = torch.empty_like(x)
    if out_format in (_lib.OUT_NVFP4, _lib.OUT_FP8_VALUES):
        data, scales = _floating_buffers(rows, k, out_format, x.device)
    else:
        pad = kpad(k)
        data = torch.empty(
            (rows, pad if out_format == 8 else pad // 2),
            device=x.device,
            dtype=torch.int8 if out_format == 8 else torch.uint8,
        )
        scales = torch.empty(rows, device=x.device, dtype=torch.float32)
    status = _lib.lib().pir2b_norm_quant_rows(
        x.data_ptr(), _ptr(y), _ptr(gate), _ptr(residual), _ptr(gamma), _ptr(scale),
        _ptr(shift), ld_mod, tokens, _ptr(smooth), norm, float(eps), out_format,
        rows, k, data.data_ptr(), scales.data_ptr(), _stream(x.device),
    )
    _lib.check(status, "pir2b_norm_quant_rows")
    return data, scales, residual


def gemm(
    a, sa, w, sw, bias, bits, *, bias_mode=None, out_lut=None, residual=None, n_store=None, out=None, tactic=-1,
    max_out=None,
):
    """Quantized GEMM + dequant epilogue -> bf16 [m, n_store] (or into `out`).

    bias_mode defaults to piR2's `gemm` semantics: add the bias, or +0 when
    the bias is None.  Pass _lib.BIAS_NONE for `gemm_biasless` without bias.
    `residual` (bf16 [m, >= n_store], unit column stride) is added to the
    bf16 result in fp32 and rounded again (the residual epilogue).
    `max_out` (fp32 [m, npad/16]) also receives the output's per-16-channel
    maxima of |y| (see `gemm_rows`).
    """
    if max_out is not None:
        return _gemm_fused(
            w, sw, bias, bits, qa=a, sa=sa, bias_mode=bias_mode, out_lut=out_lut, residual=residual,
            n_store=n_store, out=out, max_out=max_out,
        )
    m = a.shape[0]
    n_pad = w.shape[0]
    k_pad = a.shape[1] * (2 if bits == 4 else 1)
    if n_store is None:
        n_store = n_pad
    if bias_mode is None:
        bias_mode = _lib.BIAS_ADD if bias is not None else _lib.BIAS_ZERO
    if out is None:
        out = torch.empty((m, n_store), device=a.device, dtype=torch.bfloat16)
    ldo = out.stride(0) if out.ndim == 2 else n_store
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("GEMM output must be BF16 with unit column stride")
    ldr = 0
    if residual is not None:
        residual = residual.reshape(m, -1) if residual.dim() != 2 else residual
        if residual.dtype != torch.bfloat16 or residual.stride(-1) != 1 or residual.shape[1] < n_store:
            raise ValueError("Residual must be BF16 [M, >= N] with unit column stride")
        ldr = residual.stride(0) if m > 1 else residual.shape[1]
    recorder = launch_recorder
    if recorder is not None:
        recorder.before(a.device)
    status = _lib.lib().pir2b_gemm(
        a.data_ptr(), sa.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias), bias_mode,
        _ptr(out_lut), _ptr(residual), ldr, bits, m, n_pad, k_pad, out.data_ptr(), ldo, n_store,
        int(tactic), _stream(a.device),
    )
    _lib.check(status, "pir2b_gemm")
    if recorder is not None:
        recorder.after(a.device, bits=bits, m=m, n=n_store, k=k_pad, npad=n_pad, residual=residual is not None,
                       bias=bias is not None)
    return out


def gemm_rows(x, w, sw, bias, *, x_max=None, bias_mode=None, out_lut=None, residual=None, n_store=None,
              out=None, max_out=None):
    """W8A8 GEMM of bf16 rows with the activation pack fused into the GEMM.

    x: bf16 [m <= 64, k] rows (unit column stride, k % 8 == 0); the result
    is bitwise `gemm(*quant_rows(x, 8), w, ...)` in one launch.  `x_max`
    (fp32 [m, parts], parts % 4 == 0) holds partial maxima of |x| covering
    each row, e.g. the `max_out` of the GEMM that wrote x; without it each
    CTA stages whole rows to find the maxima.  Raises ValueError when the
    rows do not fit the kernel (the caller packs separately then).
    """
    return _gemm_fused(
        w, sw, bias, 8, x=x, x_max=x_max, bias_mode=bias_mode, out_lut=out_lut, residual=residual,
        n_store=n_store, out=out, max_out=max_out,
    )


def _gemm_fused(w, sw, bias, bits, *, qa=None, sa=None, x=None, x_max=None, bias_mode=None, out_lut=None,
                residual=None, n_store=None, out=None, max_out=None):
    src = qa if qa is not None else x
    m = src.shape[0]
    n_pad = w.shape[0]
    if x is not None:
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
            raise ValueError("gemm_rows needs bf16 [m, k] rows with unit column stride")
        k = x.shape[1]
        k_pad = kpad(k)
        ldx = x.stride(0) if m > 1 else k
    else:
        k = 0
        k_pad = qa.shape[1] * (2 if bits == 4 else 1)
        ldx = 0
    if w.shape[1] * (2 if bits == 4 else 1) != k_pad:
        raise ValueError("weights do not match the activation width")
    if n_store is None:
        n_store = n_pad
    if bias_mode is None:
        bias_mode = _lib.BIAS_ADD if bias is not None else _lib.BIAS_ZERO
    if out is None:
        out = torch.empty((m, n_store), device=w.device, dtype=torch.bfloat16)
    ldo = out.stride(0) if out.ndim == 2 else n_store
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("GEMM output must be BF16 with unit column stride")
    ldr = 0
    if residual is not None:
        residual = residual.reshape(m, -1) if residual.dim() != 2 else residual
        if residual.dtype != torch.bfloat16 or residual.stride(-1) != 1 or residual.shape[1] < n_store:
            raise ValueError("Residual must be BF16 [M, >= N] with unit column stride")
        ldr = residual.stride(0) if m > 1 else residual.shape[1]
    parts = 0
    if x_max is not None:
        if x_max.dtype != torch.float32 or x_max.dim() != 2 or x_max.shape[0] != m or not x_max.is_contiguous():
            raise ValueError("x_max must be contiguous fp32 [m, parts]")
        parts = x_max.shape[1]
    if max_out is not None and (
        max_out.dtype != torch.float32 or max_out.shape != (m, n_pad // 16) or not max_out.is_contiguous()
    ):
        raise ValueError("max_out must be contiguous fp32 [m, npad / 16]")
    recorder = launch_recorder
    if recorder is not None:
        recorder.before(w.device)
    status = _lib.lib().pir2b_gemm_fused(
        _ptr(qa), _ptr(sa), _ptr(x), ldx, k, _ptr(x_max), parts, w.data_ptr(), sw.data_ptr(), _ptr(bias),
        bias_mode, _ptr(out_lut), _ptr(residual), ldr, bits, m, n_pad, k_pad, out.data_ptr(), ldo, n_store,
        _ptr(max_out), _stream(w.device),
    )
    _lib.check(status, "pir2b_gemm_fused")
    if recorder is not None:
        recorder.after(w.device, bits=bits, m=m, n=n_store, k=k_pad, npad=n_pad,
                       input="rows" if x is not None else "packed", k_logical=k, residual=residual is not None,
                       bias=bias is not None)
    return out


def interleave_gate_up(t, half):
    """Reorders the rows of a gate|up group tensor ([2*half, ...] or [2*half])
    into 128-row blocks gate_j, up_j (the SwiGLU GEMM's weight layout)."""
    if t.shape[0] != 2 * half or half % 128:
        raise ValueError("gate|up interleave needs 2*half rows with half % 128 == 0")
    g, u = t[:half], t[half:]
    parts = torch.stack((g.reshape(half // 128, 128, *t.shape[1:]), u.reshape(half // 128, 128, *t.shape[1:])), 1)
    return parts.reshape(t.shape).contiguous()


def gemm_swiglu(a, sa, w, sw, bias, silu_lut, *, half_n, bias_mode=None, out=None, max_out=None):
    """W8A8 gate|up GEMM writing bf16(silu(gate) * up) [m, half_n]; w, sw
    and bias in the interleaved layout of `interleave_gate_up`.  `max_out`
    (fp32 [m, half_n / 16]) also receives the output's per-16-column
    maxima of |h| (for `quant_rows_max`)."""
    m = a.shape[0]
    k_pad = a.shape[1]
    if w.dtype != torch.int8 or w.shape[1] != k_pad or w.shape[0] != 2 * half_n:
        raise ValueError("SwiGLU GEMM needs int8 weights [2*half_n, Kpad] matching the activations")
    if bias_mode is None:
        bias_mode = _lib.BIAS_NONE if bias is None else _lib.BIAS_ADD
    if out is None:
        out = torch.empty((m, half_n), device=a.device, dtype=torch.bfloat16)
    if max_out is not None and (
        max_out.dtype != torch.float32 or max_out.shape != (m, half_n // 16) or not max_out.is_contiguous()
    ):
        raise ValueError("max_out must be contiguous fp32 [m, half_n / 16]")
    recorder = launch_recorder
    if recorder is not None:
        recorder.before(a.device)
    status = _lib.lib().pir2b_gemm_swiglu(
        a.data_ptr(), sa.data_ptr(), w.data_ptr(), sw.data_ptr(), _ptr(bias), bias_mode,
        silu_lut.data_ptr(), m, half_n, k_pad, out.data_ptr(), out.stride(0), _ptr(max_out), _stream(a.device),
    )
    _lib.check(status, "pir2b_gemm_swiglu")
    if recorder is not None:
        recorder.after(a.device, bits=8, m=m, n=2 * half_n, k=k_pad, npad=2 * half_n, out_n=half_n,
                       bias=bias is not None)
    return out


_FFN_WORKSPACES = {}


def ffn_workspace(device, m, f):
    """Zero-initialised workspace for dit_ffn, one per (device, size) and
    reused by every stream-ordered call (each call leaves it zeroed)."""
    size = int(_lib.lib().pir2b_dit_ffn_workspace(m, f))
    key = (torch.device(device), size)
    if key not in _FFN_WORKSPACES:
        _FFN_WORKSPACES[key] = torch.zeros(size, device=device, dtype=torch.uint8)
    return _FFN_WORKSPACES[key]


def dit_ffn(qa, sa, up, down, gelu_lut, residual, *, out=None):
    """residual + down(pack(gelu(up(x)))) for a packed x [m, d] (int8 codes,
    fp32 scales).  `up` and `down` are W8A8 IntegerLinear-like objects
    (packed_weight, weight_scale, bias, bias mode, in/out features)."""
    m, d = qa.shape
    f = up.out_features
    res = residual.reshape(m, d)
    if res.dtype != torch.bfloat16 or res.stride(-1) != 1:
        raise ValueError("dit_ffn residual must be bf16 rows")
    if out is None:
        out = torch.empty((m, d), device=qa.device, dtype=torch.bfloat16)
    ws = ffn_workspace(qa.device, m, f)
    status = _lib.lib().pir2b_dit_ffn(
        qa.data_ptr(), sa.data_ptr(), up.packed_weight.data_ptr(), up.weight_scale.data_ptr(),
        _ptr(up.bias), up._bias_mode(), gelu_lut.data_ptr(), down.packed_weight.data_ptr(),
        down.weight_scale.data_ptr(), _ptr(down.bias), down._bias_mode(), res.data_ptr(),
        res.stride(0), m, d, f, out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(),
        _stream(qa.device),
    )
    _lib.check(status, "pir2b_dit_ffn")
    return out


def pack_nvfp4(x):
    """NVFP4 pack of contiguous bf16 rows -> (packed [rows, k/2], swizzled sf)."""
    data, scales, _ = norm_quant_rows(x.reshape(-1, x.shape[-1]).contiguous(), _lib.OUT_NVFP4)
    return data, scales


def qk_norm_rope(qkv, q_weight, k_weight, cos, sin, *, tokens, hq, hk, eps, head_dim=128):
    """Fused q/k RMSNorm + RoPE of a grouped q|k|v projection output.

    qkv: bf16 [B*T, >= (hq + 2hk) * head_dim] rows with unit column stride.
    Returns q [B, hq, T, D], k [B, hk, T, D], v [B, hk, T, D] (contiguous).
    """
    matrix, rows, _, ld = _rows(qkv)
    b = rows // tokens
    q = torch.empty((b, hq, tokens, head_dim), device=qkv.device, dtype=torch.bfloat16)
    k = torch.empty((b, hk, tokens, head_dim), device=qkv.device, dtype=torch.bfloat16)
    v = torch.empty((b, hk, tokens, head_dim), device=qkv.device, dtype=torch.bfloat16)
    status = _lib.lib().pir2b_qk_norm_rope(
        matrix.data_ptr(), ld, q_weight.data_ptr(), k_weight.data_ptr(), cos.data_ptr(), sin.data_ptr(),
        rows, tokens, hq, hk, head_dim, float(eps), q.data_ptr(), k.data_ptr(), v.data_ptr(),
        _stream(qkv.device),
    )
    _lib.check(status, "pir2b_qk_norm_rope")
    return q, k, v


def unpack_int4(packed, out=None):
    """Low-nibble-first int4 codes uint8 [rows, k/2] -> int8 [rows, k]
    (sign-extended, one code per byte): the int8 container of the same
    values, for the int8 GEMM."""
    if packed.dtype != torch.uint8 or packed.dim() != 2 or packed.stride(1) != 1 or not packed.is_contiguous():
        raise ValueError("unpack_int4 needs contiguous uint8 [rows, k/2] codes")
    rows, half = packed.shape
    if out is None:
        out = torch.empty((rows, 2 * half), device=packed.device, dtype=torch.int8)
    if out.shape != (rows, 2 * half) or out.dtype != torch.int8 or not out.is_contiguous():
        raise ValueError("unpack_int4 output must be contiguous int8 [rows, k]")
    status = _lib.lib().pir2b_unpack_int4(packed.data_ptr(), rows, 2 * half, out.data_ptr(), _stream(packed.device))
    _lib.check(status, "pir2b_unpack_int4")
    return out


def attention_causal(q, k, v, *, scale=None, out=None):
    """Causal grouped-query attention, head_dim 128.

    q: bf16 [B, hq, T, 128], k and v: bf16 [B, hk, T, 128] contiguous (the
    layout `qk_norm_rope` returns).  Returns bf16 [B*T, hq*128] rows, the
    o_proj input, equal to SDPA(q, k, v, is_causal=True, enable_gqa=True)
    transposed to [B, T, hq*128] within bf16 tolerance.
    """
    b, hq, t, d = q.shape
    hk = k.shape[1]
    if k.shape != (b, hk, t, d) or v.shape != k.shape:
        raise ValueError("attention_causal: k and v must be [B, hk, T, D] like q")
    for x in (q, k, v):
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("attention_causal: q, k, v must be contiguous bf16")
    if out is None:
        out = torch.empty((b * t, hq * d), device=q.device, dtype=torch.bfloat16)
    if scale is None:
        scale = d ** -0.5
    status = _lib.lib().pir2b_attention_causal(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), b, t, hq, hk, d, float(scale), out.data_ptr(),
        out.stride(0), _stream(q.device),
    )
    _lib.check(status, "pir2b_attention_causal")
    return out


def quant_fp8(x, *, fast=False, replicate=None, weights=False):
    """Per-tensor E4M3 quantization of bf16 rows x [rows, k] (k % 8 == 0):
    activations with k % 16 == 0 and k <= 8192 in two launches (partial
    maxima, then scale and cast), weights and other widths in the one-launch
    cluster quantizer; both give the same bits.

    Returns (codes uint8 [rows, k], scale fp32 [1], replicated fp32
    [replicate]) -- the replicated vector (default: one per row) is the
    per-row or per-channel scale the FP8 GEMM reads.  fast=True selects
    piR2's prepare_fp8 arithmetic instead of quantize_bf16's.  weights=True
    when the codes are GEMM weights (the GEMMs read weights before their
    programmatic-dependent wait; this launch then does not let the next
    kernel start early).
    """
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("quant_fp8 needs CUDA bf16 [rows, k] rows with unit column stride")
    rows, k = x.shape
    n_rep = rows if replicate is None else int(replicate)
    q = torch.empty((rows, k), device=x.device, dtype=torch.uint8)
    scale = torch.empty(1, device=x.device, dtype=torch.float32)
    rep = torch.empty(max(n_rep, 1), device=x.device, dtype=torch.float32)
    ldx = x.stride(0) if rows > 1 else k
    if not weights and k % 16 == 0 and k <= 8192 and ldx % 8 == 0 and x.data_ptr() % 16 == 0:
        # Activations: two parallel launches, one CTA per row for the row
        # maxima, then the grid-wide scale and cast reading x in place.
        row_max = torch.empty(rows * fp8_value_slices(k), device=x.device, dtype=torch.float32)
        status = _lib.lib().pir2b_floating_rows(
            x.data_ptr(), ldx, None, 0, None, None, _lib.MODE_PLAIN, _lib.OUT_FP8_VALUES, rows, k, None,
            row_max.data_ptr(), _stream(x.device),
        )
        _lib.check(status, "pir2b_floating_rows")
        status = _lib.lib().pir2b_fp8_cast(
            x.data_ptr(), ldx, row_max.data_ptr(), row_max.numel(), rows, k, 1 if fast else 0, q.data_ptr(),
            scale.data_ptr(),
            rep.data_ptr() if n_rep > 0 else None, n_rep, _stream(x.device),
        )
        _lib.check(status, "pir2b_fp8_cast")
        return q, scale, rep[:n_rep]
    status = _lib.lib().pir2b_quant_fp8(
        x.data_ptr(), ldx, rows, k, 1 if fast else 0, 1 if weights else 0, q.data_ptr(), scale.data_ptr(),
        rep.data_ptr() if n_rep > 0 else None, n_rep, _stream(x.device),
    )
    _lib.check(status, "pir2b_quant_fp8")
    return q, scale, rep[:n_rep]


def gemm_fp8(qa, sa_rows, qw, sw_cols, bias=None, *, n, residual=None, out=None, out_lut=None, max_out=None):
    """E4M3 GEMM (fp32 accumulate) -> bf16 [m, n]: bf16(f32(acc * sa[m]) *
    sw[c] + bias[c]) with the replicated per-tensor scale vectors of
    `quant_fp8`; `out_lut` maps the result through an activation table;
    `max_out` (fp32 [m, npad / 16], m <= 32) receives per-16-column maxima
    of the finite |out| for `fp8_cast`."""
    m, kpad = qa.shape
    npad = qw.shape[0]
    if qw.shape[1] != kpad or qa.dtype != torch.uint8 or qw.dtype != torch.uint8:
        raise ValueError("FP8 operands must be uint8 E4M3 codes with matching K")
    if out is None:
        out = torch.empty((m, n), device=qa.device, dtype=torch.bfloat16)
    ldr = 0
    if residual is not None:
        residual = residual.reshape(m, -1)
        ldr = residual.stride(0) if m > 1 else residual.shape[1]
    bias_mode = _lib.BIAS_ADD if bias is not None else _lib.BIAS_NONE
    recorder = launch_recorder
    if recorder is not None:
        recorder.before(qa.device)
    if max_out is not None and (
        max_out.dtype != torch.float32 or max_out.shape != (m, npad // 16) or not max_out.is_contiguous()
    ):
        raise ValueError("max_out must be contiguous fp32 [m, npad / 16]")
    status = _lib.lib().pir2b_gemm_fp8(
        qa.data_ptr(), sa_rows.data_ptr(), qw.data_ptr(), sw_cols.data_ptr(), _ptr(bias), bias_mode,
        _ptr(residual), ldr, m, npad, kpad, out.data_ptr(), out.stride(0), n, _ptr(out_lut), _ptr(max_out),
        _stream(qa.device),
    )
    _lib.check(status, "pir2b_gemm_fp8")
    if recorder is not None:
        recorder.after(qa.device, bits="fp8", m=m, n=n, k=kpad, npad=npad, residual=residual is not None,
                       bias=bias is not None)
    return out


def gemm_nvfp4(a_packed, a_sf, w_packed, w_sf, bias=None, *, n, alpha=1.0, out=None):
    """NVFP4 GEMM: bf16(alpha * sum (a * sfa)(w * sfw) [+ bias]) -> [m, n].

    a_packed: uint8 [m, k/2], a_sf: swizzled UE4M3 factors (rows padded to
    128); w_packed: uint8 [n, k/2], w_sf likewise (the layouts of pack_nvfp4).
    """
    m = a_packed.shape[0]
    k = a_packed.shape[1] * 2
    if w_packed.shape[1] * 2 != k or w_packed.shape[0] < n:
        raise ValueError("NVFP4 operand shapes do not match")
    if out is None:
        out = torch.empty((m, n), device=a_packed.device, dtype=torch.bfloat16)
    recorder = launch_recorder
    if recorder is not None:
        recorder.before(a_packed.device)
    status = _lib.lib().pir2b_gemm_nvfp4(
        a_packed.data_ptr(), a_sf.data_ptr(), w_packed.data_ptr(), w_sf.data_ptr(), _ptr(bias),
        float(alpha), m, n, k, out.data_ptr(), out.stride(0), _stream(a_packed.device),
    )
    _lib.check(status, "pir2b_gemm_nvfp4")
    if recorder is not None:
        recorder.after(a_packed.device, bits="fp4", m=m, n=n, k=k, npad=n)
    return out


def attention_rows(q, k, v, *, batch, heads, head_dim, scale=None, out=None):
    """Unmasked attention over projection rows.

    q: bf16 [batch*T, >= heads*head_dim] rows; k, v: bf16 [batch*S, ...]
    rows (any row stride with unit column stride).  Returns bf16
    [batch*T, heads*head_dim] rows ready for the output projection.
    """
    qm, qrows, _, ldq = _rows(q)
    km, krows, _, ldk = _rows(k)
    vm, vrows, _, ldv = _rows(v)
    if qrows % batch or krows % batch or krows != vrows:
        raise ValueError("attention_rows: row counts must be multiples of the batch")
    tq, skv = qrows // batch, krows // batch
    width = heads * head_dim
    if out is None:
        out = torch.empty((qrows, width), device=q.device, dtype=torch.bfloat16)
    if scale is None:
        scale = head_dim ** -0.5
    status = _lib.lib().pir2b_attention_rows(
        qm.data_ptr(), ldq, km.data_ptr(), ldk, vm.data_ptr(), ldv, out.data_ptr(), out.stride(0),
        batch, tq, skv, heads, head_dim, float(scale), _stream(q.device),
    )
    _lib.check(status, "pir2b_attention_rows")
    return out
