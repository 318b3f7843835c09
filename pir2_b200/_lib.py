"""ctypes binding of libpir2b.so, the sm_100a C-ABI library (include/pir2b.h).

Loading fails loudly: there is no CPU or eager fallback anywhere in the
package, so a missing or stale library is an ImportError-class failure the
caller sees, never a silently slower path (piR2 keeps the same rule:
coexecution/optimization/capabilities.py:1-7).
"""

import ctypes
import os
from functools import lru_cache

LIB_NAME = "libpir2b.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

OK, EINVAL, EALIGN, ECUDA = 0, 1, 2, -1

MODE_PLAIN, MODE_GATED, MODE_LUT = 0, 1, 2
BIAS_NONE, BIAS_ZERO, BIAS_ADD = 0, 1, 2
NORM_NONE, NORM_RMS, NORM_LN = 0, 1, 2
OUT_INT8, OUT_INT4, OUT_NVFP4 = 8, 4, 16
OUT_FP8_VALUES = 32   # FP8 producers' first pass: bf16 values + fp32 row maxima
STATUS_TIMEOUT_PROBE = 0x105   # device status word left by pir2b_wait_probe

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# Exported entry points and their argument types, in header order.
SIGNATURES = {
    "pir2b_version": [],
    "pir2b_last_error": [],
    "pir2b_device_status": [ctypes.POINTER(_I), _P],
    "pir2b_wait_probe": [_P, _P],
    "pir2b_quant_rows": [_P, _I64, _P, _I64, _P, _P, _I, _I, _I64, _I64, _P, _P, _P],
    "pir2b_quant_rows_max": [_P, _I64, _P, _I64, _I, _I64, _I64, _P, _P, _P],
    "pir2b_floating_rows": [_P, _I64, _P, _I64, _P, _P, _I, _I, _I64, _I64, _P, _P, _P],
    "pir2b_fp8_cast": [_P, _I64, _P, _I64, _I64, _I64, _I, _P, _P, _P, _I64, _P],
    "pir2b_norm_quant_rows": [
        _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _P, _I, _F, _I, _I64, _I64, _P, _P, _P,
    ],
    "pir2b_gemm": [
        _P, _P, _P, _P, _P, _I, _P, _P, _I64, _I, _I64, _I64, _I64, _P, _I64, _I64, _I, _P,
    ],
    "pir2b_gemm_fused": [
        _P, _P, _P, _I64, _I64, _P, _I64, _P, _P, _P, _I, _P, _P, _I64, _I, _I64, _I64, _I64, _P, _I64,
        _I64, _P, _P,
    ],
    "pir2b_quant_fp8": [_P, _I64, _I64, _I64, _I, _I, _P, _P, _P, _I64, _P],
    "pir2b_gemm_fp8": [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P],
    "pir2b_pack_nvfp4": [_P, _I64, _I64, _P, _P, _P],
    "pir2b_gemm_nvfp4": [_P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _P, _I64, _P],
    "pir2b_dit_ffn_workspace": [_I64, _I64],
    "pir2b_dit_ffn": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _P],
    "pir2b_dit_ffn_static": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I64, _P],
    "pir2b_gemm_swiglu": [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _I64, _P, _I64, _P, _P],
    "pir2b_attention_rows": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _I, _F, _P],
    "pir2b_unpack_int4": [_P, _I64, _I64, _P, _P],
    "pir2b_attention_causal": [_P, _P, _P, _I64, _I64, _I, _I, _I, _F, _P, _I64, _P],
    "pir2b_qk_norm_rope": [_P, _I64, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _F, _P, _P, _P, _P],
}


class Pir2bError(RuntimeError):
    """A non-zero status from the C ABI; `.status` holds the code."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


@lru_cache(maxsize=1)
def lib():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m pir2_b200.build` "
            "(there is no fallback implementation)"
        )
    handle = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = argtypes
        fn.restype = {"pir2b_last_error": ctypes.c_char_p, "pir2b_dit_ffn_workspace": _I64}.get(name, _I)
    return handle


def check(status, what):
    if status != OK:
        message = lib().pir2b_last_error().decode(errors="replace")
        error = ValueError if status in (EINVAL, EALIGN) else RuntimeError
        if error is ValueError:
            raise ValueError(f"{what}: {message}")
        raise Pir2bError(status, f"{what}: {message}")


def wait_probe(result, stream=None):
    """Launches the bounded-wait self-test kernel: one thread waits on an
    mbarrier nothing arrives at, gives up after its ~1 s budget, sets the
    device status word to STATUS_TIMEOUT_PROBE and writes 0 to `result`
    (a CUDA int32 tensor of one element)."""
    import torch

    if not result.is_cuda or result.dtype != torch.int32 or result.numel() != 1:
        raise ValueError("wait_probe needs a one-element CUDA int32 tensor")
    handle = (stream or torch.cuda.current_stream()).cuda_stream
    check(lib().pir2b_wait_probe(result.data_ptr(), handle), "wait_probe")


def device_status(stream=None):
    """Reads and clears the device-side wait-timeout word (0 means clean)."""
    import torch

    value = ctypes.c_int(0)
    handle = (stream or torch.cuda.current_stream()).cuda_stream
    check(lib().pir2b_device_status(ctypes.byref(value), handle), "device_status")
    return value.value


def set_pair_mode(mode):
    """Plan override for tests and measurement: 0 lets the GEMM planner
    choose, 1 takes 2-SM tiles wherever they fit, 2 never takes them.
    Returns the previous mode."""
    previous = lib().pir2b_set_pair_mode(int(mode))
    if previous < 0:
        check(previous, "set_pair_mode")
    return previous


def set_few_mode(mode):
    """Plan override for tests and measurement: 0 lets the planner choose
    the few-token kernel, 1 takes it for every GEMM of at most 32 token
    rows, 2 never.  Returns the previous mode."""
    previous = lib().pir2b_set_few_mode(int(mode))
    if previous < 0:
        check(previous, "set_few_mode")
    return previous
