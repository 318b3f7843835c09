"""torch.ops registrations with piR2's native op schemas.

Importing this module (or calling `register()`) defines, for the CUDA
dispatch key, the ops piR2's Python code calls, backed by libpir2b.so:

* `pir2_integer::gemm` / `gemm_biasless`
  (coexecution/kernels/ampere_ada/csrc/integer_gemm.cu:185-195): same
  schema, same checks (K % 128, N % 8, contiguity, dtypes, devices), output
  `[M, Npad]` bf16; `gemm` adds +0 for a null bias, `gemm_biasless` does not.
* `pir2_integer_dispatch::linear` / `prepare`
  (coexecution/kernels/ampere_ada/csrc/integer_dispatch.cu:127-136).

The tactic argument is accepted and validated (0..7); the B200 kernel picks
its tile shape per call.  Do not load piR2's own extensions for these
namespaces in the same process.
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
    _LIBS.extend([integer, dispatch])


register()
