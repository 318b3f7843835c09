"""B200-native (sm_100a) implementation of piR2's quantized-Linear hot path.

The symmetric-row-v1 W8A8 / W4A4 Linear replacements and the NVFP4 path
that piR2 patches into the GR00T VLM decoder and DiT action head, behind the
same plugin API (TransformerINT / IntegerLinear / PackedActivation, the
OptimizationConfig flags and the configs/quantization tactic files).  All
device work runs in hand-written CUDA kernels of libpir2b.so (C ABI,
include/pir2b.h); there is no CPU or eager fallback.
"""

__version__ = "0.1.0"
