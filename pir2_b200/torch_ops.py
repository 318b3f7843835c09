"""torch.ops registrations with piR2's native op schemas.

Importing this module (or calling `register()`) defines, for the CUDA
dispatch key, the ops piR2's Python code calls, backed by libpir2b.so:

* `pir2_integer::gemm` / `gemm_biasless`
  (coexecution/kernels/ampere_ada/csrc/integer_gemm.cu:185-195): same
  schema, same checks (K % 128, N % 8, contiguity, dtypes, devices), output
  `[M, Npad]` bf16; `gemm` adds +0 for a null bias, `gemm_biasless` does not.
* `pir2_integer_dispatch::linear` / `prepare`
  (coexecution/kernels/ampere_ada/csrc/integer_dispatch.cu:127-136).
* `pir2_integer_epilogue::gemm` (residual epilogue: bf16(bf16(y) + r)) and
  `group_gemm` (segmented [Q rows][K rows][V rows] output), with
  `source_identity` (coexecution/kernels/ampere_ada/csrc/integer_epilogue.cu:
  189-341): the same schemas, limits and error messages.
* `pir2_cutlass_fp4`: the ops the reference's FP4 loader requires
  (coexecution/kernels/blackwell/fp4_linear.py:8-15; schemas at
  coexecution/kernels/blackwell/csrc/fp4_cutlass_linear.cu:2968-3065) plus
  `linear_forward_packed_gemm_bf16` and `get_decode_policy`, on this
  library's NVFP4 pack and tcgen05 block-scaled GEMM.

Tactic arguments are accepted and validated with the reference's ranges;
the B200 kernels plan their tiles per call, and results do not depend on
the tactic.  Do not load piR2's own extensions for these namespaces in the
same process.
"""

import torch

from . import _lib, ops

_LIBS = []


def _check_gemm(a, sa, b, sb, bias, bits):
    if bits not in (4, 8):
        raise RuntimeError("bits must be 4 or 8")
    tensors = (a, sa, b, sb)
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("CUDA tensors required")
    if any(t.device != a.device for t in tensors):
        raise RuntimeError("Devices must match")
    if a.dim() != 2 or b.dim() != 2 or a.size(1) != b.size(1):
        raise RuntimeError("Invalid packed matrix shapes")
    if not all(t.is_contiguous() for t in tensors):
        raise RuntimeError("Contiguous tensors required")
    storage = torch.uint8 if bits == 4 else torch.int8
    if a.dtype != storage or b.dtype != storage:
        raise RuntimeError("Invalid integer storage dtype")
    if (
        sa.dtype != torch.float32
        or sb.dtype != torch.float32
        or sa.dim() != 1
        or sb.dim() != 1
        or sa.size(0) != a.size(0)
        or sb.size(0) != b.size(0)
    ):
        raise RuntimeError("Invalid scale buffers")
    if a.size(0) <= 0 or b.size(0) <= 0 or b.size(0) % 8 or (a.size(1) * (2 if bits == 4 else 1)) % 128:
        raise RuntimeError("GEMM requires padded K%128=0, N%8=0 and nonempty matrices")
    if bias is not None and (
        bias.device != a.device or bias.dtype != torch.bfloat16 or not bias.is_contiguous() or bias.dim() != 1 or bias.size(0) != b.size(0)
    ):
        raise RuntimeError("Invalid BF16 bias")


def _gemm(a, sa, b, sb, bias, bits, tactic, biasless):
    _check_gemm(a, sa, b, sb, bias, bits)
    if tactic not in range(8):
        raise RuntimeError("Unknown integer GEMM tactic")
    if bias is not None:
        mode = _lib.BIAS_ADD
    else:
        mode = _lib.BIAS_NONE if biasless else _lib.BIAS_ZERO
    with torch.cuda.device(a.device):
        return ops.gemm(a, sa, b, sb, bias, bits, bias_mode=mode, n_store=b.size(0), tactic=tactic)


def _prepare(x, lut, up, bits):
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.dim() < 2:
        raise RuntimeError("Preparation requires CUDA BF16 rows")
    if bits not in (4, 8) or x.size(-1) <= 0 or x.size(-1) > 8192 or x.stride(-1) != 1:
        raise RuntimeError("Invalid precision or input row width/stride")
    if lut is not None and (lut.device != x.device or lut.dtype != torch.bfloat16 or not lut.is_contiguous() or lut.numel() != 65536):
        raise RuntimeError("Invalid activation lookup table")
    if up is not None and (up.device != x.device or up.dtype != torch.bfloat16 or up.shape != x.shape or up.stride(-1) != 1):
        raise RuntimeError("Invalid activation multiplier")
    if up is not None and lut is None:
        raise RuntimeError("An activation multiplier needs a lookup table")
    with torch.cuda.device(x.device):
        return ops.quant_rows(x, bits, lut=lut, up=up)


# ------------------------------------------------------------------ epilogue ops
def _check_epilogue(a, sa, b, sb, bias, bits, tactic, what, max_m):
    if bits not in (4, 8):
        raise RuntimeError("bits must be 4 or 8")
    if tactic not in (0, 2, 7):
        raise RuntimeError(f"{what} epilogue tactic must be 0, 2 or 7")
    tensors = (a, sa, b, sb)
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("CUDA tensors required")
    if any(t.device != a.device for t in tensors):
        raise RuntimeError("Devices must match")
    if a.dim() != 2 or b.dim() != 2 or a.size(1) != b.size(1):
        raise RuntimeError("Invalid packed matrix shapes")
    if not all(t.is_contiguous() for t in tensors):
        raise RuntimeError("Contiguous packed buffers required")
    storage = torch.uint8 if bits == 4 else torch.int8
    if a.dtype != storage or b.dtype != storage:
        raise RuntimeError("Invalid integer storage dtype")
    if (
        sa.dtype != torch.float32 or sb.dtype != torch.float32 or sa.dim() != 1 or sb.dim() != 1
        or sa.size(0) != a.size(0) or sb.size(0) != b.size(0)
    ):
        raise RuntimeError("Invalid scale buffers")
    m, n, k = a.size(0), b.size(0), a.size(1) * (2 if bits == 4 else 1)
    if not (m <= max_m and 0 < n <= 8192 and n % 8 == 0 and 128 <= k <= 8192 and k % 128 == 0):
        if max_m == 64:
            raise RuntimeError(
                "Residual epilogue requires M<=64, padded N<=8192 with N%8=0, and 128<=K<=8192 with K%128=0"
            )
        raise RuntimeError("Group epilogue requires M<=4096, N<=8192 with N%8=0, and 128<=K<=8192 with K%128=0")
    if a.data_ptr() % 16 or b.data_ptr() % 16 or sb.data_ptr() % 16:
        raise RuntimeError("Packed matrices and weight scales require 16-byte alignment")
    if bias is not None and (
        bias.device != a.device or bias.dtype != torch.bfloat16 or not bias.is_contiguous() or bias.dim() != 1
        or bias.size(0) != n or bias.data_ptr() % 16
    ):
        raise RuntimeError("Invalid aligned BF16 bias")
    return m, n


def _bias_mode(bias, biasless):
    if bias is not None:
        return _lib.BIAS_ADD
    return _lib.BIAS_NONE if biasless else _lib.BIAS_ZERO


def _residual_gemm(a, sa, b, sb, bias, bits, tactic, biasless, residual):
    m, n = _check_epilogue(a, sa, b, sb, bias, bits, tactic, "Residual", 64)
    if not (
        residual.is_cuda and residual.device == a.device and residual.dtype == torch.bfloat16
        and residual.is_contiguous() and residual.dim() == 2 and residual.size(0) == m
        and residual.size(1) == n and residual.data_ptr() % 16 == 0
    ):
        raise RuntimeError("Invalid aligned CUDA BF16 [M,Npad] residual")
    with torch.cuda.device(a.device):
        if m == 0:
            return torch.empty((0, n), device=a.device, dtype=torch.bfloat16)
        return ops.gemm(a, sa, b, sb, bias, bits, bias_mode=_bias_mode(bias, biasless), residual=residual, n_store=n)


def _group_gemm(a, sa, b, sb, bias, bits, tactic, biasless, sizes):
    """Segmented output: segment s is a contiguous [M, sizes[s]] matrix
    placed after the previous segments (integer_epilogue.cu:90-115)."""
    m, n = _check_epilogue(a, sa, b, sb, bias, bits, tactic, "Group", 4096)
    sizes = list(sizes)
    if len(sizes) not in (2, 3):
        raise RuntimeError("Group epilogue requires two or three segments")
    if any(w <= 0 or w > n or w % 8 for w in sizes):
        raise RuntimeError("Group epilogue requires positive aligned segment widths")
    if sum(sizes) != n:
        raise RuntimeError("Group epilogue widths must cover physical N")
    with torch.cuda.device(a.device):
        if m == 0:
            return torch.empty((0,), device=a.device, dtype=torch.bfloat16)
        out = torch.empty((m * n,), device=a.device, dtype=torch.bfloat16)
        mode = _bias_mode(bias, biasless)
        offset = 0
        # One launch per segment: each writes its [M, width] block directly.
        for width in sizes:
            seg = out[m * offset : m * (offset + width)].view(m, width)
            ops.gemm(
                a, sa, b[offset : offset + width], sb[offset : offset + width],
                None if bias is None else bias[offset : offset + width], bits, bias_mode=mode,
                n_store=width, out=seg,
            )
            offset += width
        return out


# ------------------------------------------------------------------ FP4 ops
_FP4_ELEMENTS_PER_ACCESS = 32
_FP4_SF_VEC = 16
_decode_policy = [0]


def _fp4_scale_shape(rows, cols):
    return (-(-rows // 128) * 128, -(-(-(-cols // _FP4_SF_VEC)) // 4) * 4)


def _fp4_pack(x, rows, cols, zero_padding):
    """NVFP4 pack of bf16 rows (E2M1 pairs, UE4M3 block-16 factors in the
    128x4 swizzled layout of fp4_cutlass_linear.cu:686-690)."""
    packed = torch.empty((rows, cols // 2), device=x.device, dtype=torch.uint8)
    make = torch.zeros if zero_padding else torch.empty
    scales = make(_fp4_scale_shape(rows, cols), device=x.device, dtype=torch.uint8)
    status = _lib.lib().pir2b_pack_nvfp4(
        x.data_ptr(), rows, cols, packed.data_ptr(), scales.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream
    )
    _lib.check(status, "pir2_cutlass_fp4 pack")
    return packed, scales


def _fp4_supports_device(cc):
    # This library is built for sm_100a only.
    return cc == 100


def _fp4_set_decode_policy(policy):
    if not 0 <= policy <= 3:
        raise RuntimeError(
            f"FP4 decode policy must be 0 (balanced), 1 (low_clock), 2 (mid_clock), or 3 (legacy), got {policy}"
        )
    _decode_policy[0] = policy


def _fp4_get_decode_policy():
    return _decode_policy[0]


def _fp4_pack_weight(weight, role, target_name):
    if not weight.is_cuda:
        raise RuntimeError("weight must be CUDA")
    if weight.dim() != 2:
        raise RuntimeError("weight must be rank-2 [out_features, in_features]")
    if not weight.is_contiguous():
        raise RuntimeError("weight must be contiguous")
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("weight must be bf16 (this build packs bf16 weights only)")
    rows, cols = weight.shape
    if rows % 32:
        raise RuntimeError(f"CUTLASS FP4 GEMM requires out_features divisible by 32, got {rows}")
    if cols % _FP4_ELEMENTS_PER_ACCESS:
        raise RuntimeError(f"CUTLASS FP4 GEMM requires in_features divisible by 32, got {cols}")
    with torch.cuda.device(weight.device):
        packed, scales = _fp4_pack(weight, rows, cols, True)
    metadata = torch.tensor([rows, cols], dtype=torch.int64)
    return [packed, scales, metadata]


def _fp4_pack_activation(x):
    if not x.is_cuda:
        raise RuntimeError("input must be CUDA")
    if x.dtype != torch.bfloat16:
        raise RuntimeError("CUTLASS FP4 activation packing supports bf16 input only")
    if not x.is_contiguous():
        raise RuntimeError("input must be contiguous")
    if x.dim() < 1:
        raise RuntimeError("input must have at least one dimension")
    cols = x.size(-1)
    if cols % _FP4_ELEMENTS_PER_ACCESS:
        raise RuntimeError(f"CUTLASS FP4 GEMM requires in_features divisible by 32, got {cols}")
    leading = x.numel() // cols if cols else 0
    if leading <= 0:
        raise RuntimeError("input must contain at least one row")
    with torch.cuda.device(x.device):
        return list(_fp4_pack(x.reshape(leading, cols), leading, cols, False))


def _fp4_forward(packed_input, input_scale, packed_weight, weight_scale, metadata, bias, role, target_name, tactic=0):
    if tactic not in (0, 1, 2, 3):
        raise RuntimeError(f"unknown CUTLASS FP4 GEMM tactic {tactic}")
    tensors = (packed_input, input_scale, packed_weight, weight_scale)
    if not (packed_input.is_cuda and input_scale.is_cuda):
        raise RuntimeError("packed input and scale must be CUDA")
    if not (packed_weight.is_cuda and weight_scale.is_cuda):
        raise RuntimeError("packed weight and scale must be CUDA")
    if any(t.dtype != torch.uint8 for t in tensors):
        raise RuntimeError("packed inputs, weights, and scales must be uint8")
    if not (packed_input.is_contiguous() and input_scale.is_contiguous()):
        raise RuntimeError("packed input and scale must be contiguous")
    if any(t.device != packed_input.device for t in tensors):
        raise RuntimeError("packed input, weights, and scales must share a CUDA device")
    if packed_input.dim() != 2:
        raise RuntimeError("packed input must be rank-2 [rows, packed_k]")
    meta = metadata.cpu()
    if meta.dtype != torch.int64:
        raise RuntimeError("metadata must be int64")
    if meta.numel() < 2:
        raise RuntimeError("metadata must contain rows and cols")
    rows, cols = int(meta[0]), int(meta[1])
    leading = packed_input.size(0)
    if leading <= 0:
        raise RuntimeError("packed input must contain at least one row")
    if packed_input.size(1) != cols // 2:
        raise RuntimeError("packed input width does not match weight in_features")
    if rows % 32 or cols % _FP4_ELEMENTS_PER_ACCESS:
        raise RuntimeError("CUTLASS FP4 GEMM dimensions must be divisible by 32")
    need = _fp4_scale_shape(leading, cols)
    if input_scale.numel() < need[0] * need[1]:
        raise RuntimeError("packed input scale buffer is too small")
    if bias is not None:
        if not bias.is_cuda:
            raise RuntimeError("bias must be CUDA")
        if bias.device != packed_input.device:
            raise RuntimeError("bias and packed input must be on the same CUDA device")
        if bias.dtype != torch.bfloat16:
            raise RuntimeError("bias must be bf16")
        if bias.numel() != rows:
            raise RuntimeError("bias size must match out_features")
        bias = bias.contiguous()
    with torch.cuda.device(packed_input.device):
        if leading == 1 and bias is not None:
            # One token: the bias is added to the rounded bf16 product by a
            # separate step (fp4_cutlass_linear.cu:1808-1828).
            y = ops.gemm_nvfp4(packed_input, input_scale, packed_weight, weight_scale, None, n=rows)
            return y + bias
        return ops.gemm_nvfp4(packed_input, input_scale, packed_weight, weight_scale, bias, n=rows)


def _fp4_swap_ab(a, z, w, ws, bias):
    if a.dim() != 2 or w.dim() != 2 or a.size(1) != w.size(1):
        raise RuntimeError("Swap-AB packed input/weight shapes mismatch")
    for t in (a, z, w, ws):
        if not (t.is_cuda and t.device == a.device and t.dtype == torch.uint8 and t.is_contiguous()):
            raise RuntimeError("Swap-AB requires contiguous CUDA uint8 buffers on one device")
    m, n, packed_k = a.size(0), w.size(0), a.size(1)
    if not (m == 41 and n == 1536 and packed_k in (128, 768)):
        raise RuntimeError("Swap-AB supports only (M,K,N)=(41,256,1536)/(41,1536,1536)")
    k = packed_k * 2
    if z.numel() < -(-m // 128) * 128 * (-(-k // 64)) * 4 or ws.numel() < -(-n // 128) * 128 * (-(-k // 64)) * 4:
        raise RuntimeError("Swap-AB scale buffer too small")
    if not (
        bias.is_cuda and bias.device == a.device and bias.dtype == torch.bfloat16 and bias.is_contiguous()
        and bias.dim() == 1 and bias.numel() == n and not bias.requires_grad
    ):
        raise RuntimeError("Swap-AB requires a contiguous BF16 output-channel bias without autograd")
    if any(t.data_ptr() % 16 for t in (a, z, w, ws, bias)):
        raise RuntimeError("Swap-AB requires 16-byte aligned packed, scale and bias buffers")
    with torch.cuda.device(a.device):
        return ops.gemm_nvfp4(a, z, w, ws, bias, n=n)


def register():
    if _LIBS:
        return
    schema = "(Tensor a, Tensor sa, Tensor b, Tensor sb, Tensor? bias, int bits, int tactic) -> Tensor"
    integer = torch.library.Library("pir2_integer", "DEF")
    integer.define("gemm" + schema)
    integer.define("gemm_biasless" + schema)
    integer.impl("gemm", lambda a, sa, b, sb, bias, bits, tactic: _gemm(a, sa, b, sb, bias, bits, tactic, False), "CUDA")
    integer.impl(
        "gemm_biasless", lambda a, sa, b, sb, bias, bits, tactic: _gemm(a, sa, b, sb, bias, bits, tactic, True), "CUDA"
    )
    dispatch = torch.library.Library("pir2_integer_dispatch", "DEF")
    dispatch.define(
        "linear(Tensor x, Tensor w, Tensor ws, Tensor? bias, Tensor? lut, Tensor? up, int bits, int tactic) -> Tensor"
    )
    dispatch.define("prepare(Tensor x, Tensor? lut, Tensor? up, int bits) -> (Tensor, Tensor)")

    def linear(x, w, ws, bias, lut, up, bits, tactic):
        q, s = _prepare(x, lut, up, bits)
        return _gemm(q, s, w, ws, bias, bits, tactic, True)

    dispatch.impl("linear", linear, "CUDA")
    dispatch.impl("prepare", _prepare, "CUDA")

    epilogue = torch.library.Library("pir2_integer_epilogue", "DEF")
    epilogue.define("source_identity() -> str")
    epilogue.define(
        "gemm(Tensor a, Tensor sa, Tensor b, Tensor sb, Tensor? bias, int bits, int tactic, bool biasless, "
        "Tensor residual) -> Tensor"
    )
    epilogue.define(
        "group_gemm(Tensor a, Tensor sa, Tensor b, Tensor sb, Tensor? bias, int bits, int tactic, bool biasless, "
        "int[] sizes) -> Tensor"
    )
    epilogue.impl("source_identity", lambda: f"pir2b-sm100a-{_lib.lib().pir2b_version()}", "CompositeExplicitAutograd")
    epilogue.impl("gemm", _residual_gemm, "CUDA")
    epilogue.impl("group_gemm", _group_gemm, "CUDA")

    fp4 = torch.library.Library("pir2_cutlass_fp4", "DEF")
    fp4.define("supports_device(int cc) -> bool")
    fp4.define("set_decode_policy(int policy) -> ()")
    fp4.define("get_decode_policy() -> int")
    fp4.define("pack_linear_weight_gemm_bf16(Tensor weight, str role, str target_name) -> Tensor[]")
    fp4.define("pack_activation_gemm_bf16(Tensor input) -> Tensor[]")
    fp4.define(
        "linear_forward_packed_gemm_bf16(Tensor packed_input, Tensor input_scale, Tensor packed_weight, "
        "Tensor weight_scale, Tensor metadata, Tensor? bias, str role, str target_name) -> Tensor"
    )
    fp4.define(
        "linear_forward_packed_gemm_bf16_tactic(Tensor packed_input, Tensor input_scale, Tensor packed_weight, "
        "Tensor weight_scale, Tensor metadata, Tensor? bias, str role, str target_name, int tactic) -> Tensor"
    )
    fp4.define("linear_forward_packed_gemm_bf16_swap_ab(Tensor a, Tensor z, Tensor w, Tensor ws, Tensor bias) -> Tensor")
    for name, fn in (
        ("supports_device", _fp4_supports_device),
        ("set_decode_policy", _fp4_set_decode_policy),
        ("get_decode_policy", _fp4_get_decode_policy),
    ):
        fp4.impl(name, fn, "CompositeExplicitAutograd")
    fp4.impl("pack_linear_weight_gemm_bf16", _fp4_pack_weight, "CUDA")
    fp4.impl("pack_activation_gemm_bf16", _fp4_pack_activation, "CUDA")
    fp4.impl("linear_forward_packed_gemm_bf16", _fp4_forward, "CUDA")
    fp4.impl("linear_forward_packed_gemm_bf16_tactic", _fp4_forward, "CUDA")
    fp4.impl("linear_forward_packed_gemm_bf16_swap_ab", _fp4_swap_ab, "CUDA")
    _LIBS.extend([integer, dispatch, epilogue, fp4])


register()
