"""OptimizationConfig and its CLI flags (GPU-free).

Same fields, defaults and cross-field validation as piR2's
coexecution/optimization/config.py:7-231, so existing command lines and
config objects keep working.  Flags for subsystems outside the quantized
Linear path (vision channels-last, tokenizer cache, input/image
preparation, static VLM, compiled host guards, FP8) are parsed and rejected
by GrootOptimizations with a clear error rather than silently ignored.
"""

import argparse
from dataclasses import dataclass
from pathlib import Path

OUT_OF_SCOPE_FLAGS = (
    "vision_channels_last",
    "input_preparation",
    "tokenizer_cache",
    "static_vlm",
    "vlm_graph",
    "image_array_preparation",
    "compiled_host_guards",
)


@dataclass(frozen=True)
class OptimizationConfig:
    precision: str = "bf16"
    fusion: bool = False
    dit_graph: bool = False
    action_graph: bool = False
    action_kv_reuse: bool = False
    scope: str = "transformer"
    category_id: int | None = None
    coverage: Path | None = None
    tactics: Path | None = None
    group_tactics: Path | None = None
    shape_tactics: Path | None = None
    group_conditioning: bool = False
    vision_channels_last: bool = False
    norm_modulation_quant: bool = False
    residual_norm_quant: bool = False
    fp8_fast_quant: bool = False
    fp4_swap_ab: bool = False
    fp_shared_inputs: bool = False
    fp_grouped: bool = False
    fp_swiglu: bool = False
    fp_gelu: bool = False
    fp_rmsnorm: bool = False
    fp_smoothquant: Path | None = None
    component: str = "all"
    input_preparation: bool = False
    tokenizer_cache: bool = False
    static_vlm: bool = False
    vlm_graph: bool = False
    image_array_preparation: bool = False
    compiled_host_guards: bool = False
    fusion_mode: str = "all"
    operator_profile: Path | None = None
    # Packed-weight cache file (weight_cache): loaded when present and valid
    # for these weights, written after quantizing when absent.
    packed_weights: Path | None = None

    def __post_init__(self):
        floating = ("fp8", "fp4")
        checks = [
            (type(self.action_kv_reuse) is not bool, "Action K/V reuse must be a bool"),
            (self.action_kv_reuse and not self.action_graph, "Action K/V reuse requires --action-cuda-graph"),
            (
                self.action_graph and self.precision not in ("bf16", "w8a8", "w4a4"),
                "Action graph requires BF16, W8A8 or W4A4",
            ),
            (self.vlm_graph and not self.static_vlm, "VLM graph requires static_vlm"),
            (
                self.fusion_mode not in ("vision_rope", "text_rope", "rope", "rmsnorm", "rope_rms", "all"),
                "Unknown operator fusion mode",
            ),
            (self.fusion_mode != "all" and not self.fusion, "Selective mode requires operator fusion"),
            (
                self.fusion_mode != "all" and (self.group_conditioning or self.norm_modulation_quant),
                "DiT producer options require all operator fusion",
            ),
            (
                self.operator_profile is not None and not (self.fusion or self.precision != "bf16"),
                "Operator profile requires fusion or low-bit precision",
            ),
            (
                self.precision not in ("bf16", "w8a8", "w4a4", "fp8", "fp4"),
                "Precision must be bf16, w8a8, w4a4, fp8 or fp4",
            ),
            (self.fp8_fast_quant and self.precision != "fp8", "Fast FP8 quantization requires precision=fp8"),
            (
                self.fp_smoothquant is not None and self.precision not in floating,
                "SmoothQuant profile requires precision=fp8 or fp4",
            ),
            (
                (self.fp_gelu or self.fp_rmsnorm) and self.precision not in floating,
                "Floating producers require precision=fp8 or fp4",
            ),
            (self.fp4_swap_ab and self.precision != "fp4", "FP4 Swap-AB requires precision=fp4"),
            (
                self.fp_shared_inputs and self.precision not in floating,
                "Shared floating inputs require precision=fp8 or fp4",
            ),
            (
                (self.fp_grouped or self.fp_swiglu) and self.precision not in floating,
                "Floating fusion requires precision=fp8 or fp4",
            ),
            (self.scope not in ("transformer", "all"), "Quantization scope must be transformer or all"),
            (self.component not in ("all", "vlm", "dit"), "Quantization component must be all, vlm or dit"),
            (
                self.component == "vlm"
                and (self.category_id is not None or self.group_conditioning or self.norm_modulation_quant),
                "Category, condition and norm producers require the DiT component",
            ),
            (self.category_id is not None and self.category_id < 0, "Category ID must be nonnegative"),
            (self.category_id is not None and self.scope != "all", "Category projections require scope=all"),
            (
                self.precision in floating
                and (
                    self.category_id is not None
                    or self.tactics is not None
                    or self.group_tactics is not None
                    or self.shape_tactics is not None
                    or self.group_conditioning
                ),
                "Floating precision does not support integer tactic, category or condition grouping flags",
            ),
            (
                self.group_conditioning and (not self.fusion or self.scope != "all" or self.precision == "bf16"),
                "Condition grouping requires fusion, scope=all and integer precision",
            ),
            (
                self.norm_modulation_quant and (not self.fusion or self.precision == "bf16"),
                "Norm quantization fusion requires fusion and low-bit precision",
            ),
            (self.residual_norm_quant and not self.norm_modulation_quant, "Residual fusion requires norm_modulation_quant"),
            (
                self.packed_weights is not None and self.precision not in ("w8a8", "w4a4"),
                "A packed-weight cache requires precision=w8a8 or w4a4",
            ),
        ]
        for failed, message in checks:
            if failed:
                raise ValueError(message)

    @property
    def enabled(self):
        return (
            self.precision != "bf16"
            or self.fusion
            or self.dit_graph
            or self.action_graph
            or any(getattr(self, flag) for flag in OUT_OF_SCOPE_FLAGS)
        )

    def validate_variant(self, variant):
        if self.action_graph and variant != "flow":
            raise ValueError("Action graph requires non-streaming Flow4")
        if variant == "pir2" and self.group_conditioning:
            raise ValueError("Streaming piR2 condition grouping is not validated")


def add_optimization_arguments(parser):
    parser.add_argument("--inference-precision", choices=["bf16", "w8a8", "w4a4", "fp8", "fp4"], default="bf16")
    parser.add_argument("--operator-fusion", action="store_true")
    parser.add_argument(
        "--operator-fusion-mode",
        choices=["vision_rope", "text_rope", "rope", "rmsnorm", "rope_rms", "all"],
        default="all",
    )
    parser.add_argument("--operator-profile", type=Path)
    parser.add_argument("--dit-cuda-graph", action="store_true")
    parser.add_argument("--action-cuda-graph", action="store_true")
    parser.add_argument("--action-kv-reuse", action="store_true")
    parser.add_argument("--quantization-scope", choices=["transformer", "all"], default="transformer")
    parser.add_argument("--quantization-component", choices=["all", "vlm", "dit"], default="all")
    parser.add_argument("--quantization-category-id", type=int)
    parser.add_argument("--quantization-coverage", type=Path)
    parser.add_argument("--quantization-tactics", type=Path)
    parser.add_argument("--quantization-group-tactics", type=Path)
    parser.add_argument("--quantization-shape-tactics", type=Path)
    parser.add_argument("--group-conditioning", action="store_true")
    for flag in (
        "--vision-channels-last",
        "--input-preparation",
        "--tokenizer-cache",
        "--static-vlm",
        "--vlm-cuda-graph",
        "--image-array-preparation",
        "--compiled-host-guards",
        "--norm-modulation-quant",
        "--residual-norm-quant",
        "--fp8-fast-quant",
        "--fp4-swap-ab",
        "--fp-shared-inputs",
        "--fp-grouped",
        "--fp-swiglu",
        "--fp-gelu",
        "--fp-rmsnorm",
    ):
        parser.add_argument(flag, action="store_true")
    parser.add_argument("--fp-smoothquant", type=Path, help="Calibrated, weight-bound FP4 smoothing profile")


def optimization_config(args):
    return OptimizationConfig(
        precision=args.inference_precision,
        fusion=args.operator_fusion,
        fusion_mode=args.operator_fusion_mode,
        operator_profile=args.operator_profile,
        dit_graph=args.dit_cuda_graph,
        action_graph=args.action_cuda_graph,
        action_kv_reuse=args.action_kv_reuse,
        scope=args.quantization_scope,
        component=args.quantization_component,
        category_id=args.quantization_category_id,
        coverage=args.quantization_coverage,
        tactics=args.quantization_tactics,
        group_tactics=args.quantization_group_tactics,
        shape_tactics=args.quantization_shape_tactics,
        group_conditioning=args.group_conditioning,
        vision_channels_last=args.vision_channels_last,
        input_preparation=args.input_preparation,
        tokenizer_cache=args.tokenizer_cache,
        static_vlm=args.static_vlm,
        vlm_graph=args.vlm_cuda_graph,
        image_array_preparation=args.image_array_preparation,
        compiled_host_guards=args.compiled_host_guards,
        norm_modulation_quant=args.norm_modulation_quant,
        residual_norm_quant=args.residual_norm_quant,
        fp8_fast_quant=args.fp8_fast_quant,
        fp4_swap_ab=args.fp4_swap_ab,
        fp_shared_inputs=args.fp_shared_inputs,
        fp_grouped=args.fp_grouped,
        fp_swiglu=args.fp_swiglu,
        fp_gelu=args.fp_gelu,
        fp_rmsnorm=args.fp_rmsnorm,
        fp_smoothquant=args.fp_smoothquant,
    )


def parser():
    p = argparse.ArgumentParser()
    add_optimization_arguments(p)
    return p
