"""Transactional installation of the quantized path into a GR00T policy.

Mirrors the quantized-Linear part of `GrootOptimizations`
(coexecution/optimization/session.py:20-562): `with GrootOptimizations(
policy, OptimizationConfig(precision="w8a8", ...)):` validates an eval BF16
CUDA model, selects the executed projections (scope, component, coverage),
builds the integer controller, the AdaLN/RMSNorm producers and the tactic
assignment, swaps the forwards, and restores everything on exit or on any
exception during installation.  `evidence()` reports configuration hashes,
coverage and the loaded library's identity.
"""

import hashlib
from contextlib import ExitStack
from dataclasses import asdict
from pathlib import Path
from types import SimpleNamespace

from . import _lib
from .config import OUT_OF_SCOPE_FLAGS, OptimizationConfig
from .tactics import apply_tactics, read_json

CONFIG_FILES = ("coverage", "tactics", "group_tactics", "shape_tactics", "operator_profile", "fp_smoothquant")


def selected_component(name, component):
    """S2 is the backbone; S1 includes every action-head projection."""
    if component not in ("all", "vlm", "dit"):
        raise ValueError("Quantization component must be all, vlm or dit")
    return component == "all" or name.startswith("backbone." if component == "vlm" else "action_head.")


def backend_evidence():
    path = _lib.LIB_PATH
    digest = hashlib.sha256(Path(path).read_bytes()).hexdigest()
    return {
        "backend_id": "pir2_integer",
        "backend_revision": digest[:16],
        "device_arch": "sm_100a",
        "library": path,
        "library_sha256": digest,
        "library_version": _lib.lib().pir2b_version(),
    }


class GrootOptimizations:
    def __init__(self, policy, config=None):
        self.policy = policy
        self.config = OptimizationConfig() if config is None else config
        self.stack = ExitStack()
        self.coverage = {}
        self.backend = {}
        self.controller = None
        self.extra = None
        self.producers = None
        self.residual = None
        self.pointwise = None
        self.attention = None
        self.swiglu = None
        self.floating = None
        self._active = False
        self._configuration_file_hashes = {}

    def __enter__(self):
        if self._active:
            raise RuntimeError("Optimization session is already active")
        self._active = True
        if not self.config.enabled:
            return self
        try:
            self._install()
        except BaseException:
            self.close()
            raise
        return self

    def _install(self):
        import torch

        model = self.policy.model
        params = next(model.parameters())
        if model.training or params.dtype != torch.bfloat16:
            raise ValueError("Optimizations require an eval-mode BF16 model")
        if params.device.type != "cuda":
            raise ValueError("Optimizations require CUDA")
        enabled = [flag for flag in OUT_OF_SCOPE_FLAGS if getattr(self.config, flag)]
        if enabled:
            raise ValueError(f"Not part of the B200 quantized-Linear build: {', '.join(enabled)}")
        self._configuration_file_hashes = {
            key: hashlib.sha256(Path(path).read_bytes()).hexdigest()
            for key in CONFIG_FILES
            if (path := getattr(self.config, key)) is not None
        }
        self.backend = backend_evidence()
        if self.config.precision == "bf16":
            return
        from .projections import inventory

        expanded = self.config.scope == "all"
        sites = inventory(model, expanded=expanded)[0]
        recorded = read_json(self.config.coverage, {}).get("linears", {})
        candidates = recorded if self.config.coverage is not None else sites
        executed = {n: v for n, v in candidates.items() if selected_component(n, self.config.component) and n in sites}
        categories = {
            name: (module, self.config.category_id)
            for name, module in model.named_modules()
            if type(module).__name__ == "CategorySpecificLinear"
            and self.config.category_id is not None
            and selected_component(name, self.config.component)
        }
        if not executed and not categories:
            raise ValueError("Quantization selected no matching projections")
        self.coverage = {
            "executed": len(executed),
            "available": len(sites),
            "categories": sorted(categories),
        }
        if self.config.precision in ("fp4", "fp8"):
            from .floating import FloatingProjections, aligned_for

            precision = self.config.precision
            smoothing = None
            if self.config.fp_smoothquant is not None:
                from .smoothquant import load_profile

                modules = dict(model.named_modules())
                selected = {
                    n: (modules[n], *sites[n][1:])
                    for n in executed
                    if aligned_for(precision, modules[n].in_features, modules[n].out_features)
                }
                groups = inventory(model, expanded=expanded)[1]
                smoothing, self.coverage["smoothquant"] = load_profile(
                    self.config.fp_smoothquant, selected, groups, self.config.precision
                )
            # coexecution/optimization/session.py:159-193: the floating
            # projections with their producers, then the DiT norm / residual
            # producers when norm_modulation_quant is set.
            self.floating = FloatingProjections(
                model,
                executed,
                smoothing=smoothing,
                precision=precision,
                fast_fp8=self.config.fp8_fast_quant,
                shared_inputs=self.config.fp_shared_inputs,
                grouped=self.config.fp_grouped,
                swiglu=self.config.fp_swiglu,
                gelu=self.config.fp_gelu,
                rmsnorm=self.config.fp_rmsnorm,
                groups=inventory(model, expanded=expanded)[1],
            )
            self.stack.callback(self.floating.close)
            self.floating.set()
            self.coverage["shared_input_groups"] = len(self.floating.groups)
            self.coverage["floating"] = self.floating.coverage
            if self.config.norm_modulation_quant:
                from .floating import FloatingConnections

                connections = FloatingConnections(model, self.floating, residual=self.config.residual_norm_quant)
                self.stack.callback(connections.close)
                connections.set()
                self.coverage["norm_quantization_fusion"] = {
                    "attention_producers": len(connections.norms),
                    "residual_ffn_producers": len(connections.blocks),
                }
            if self.config.fusion and self.config.fusion_mode in ("all", "rope_rms"):
                from .floating import FloatingTextFusion

                self.pointwise = FloatingTextFusion(model, self.floating)
                self.stack.callback(self.pointwise.close)
                self.pointwise.set()
                self.coverage["text_attention_fusion"] = len(self.pointwise.targets)
            if self.config.fusion and self.config.fusion_mode == "all":
                from .pointwise import DiTAttentionFusion

                self.attention = DiTAttentionFusion(model.action_head.model)
                self.stack.callback(self.attention.close)
                self.attention.set()
            return
        from .connections import AdditionalConnections
        from .producers import QuantizationProducers
        from .transformer import TransformerINT

        packed = None
        cache = self.config.packed_weights
        if cache is not None and Path(cache).exists():
            from . import weight_cache

            modules = dict(model.named_modules())
            packed = weight_cache.load(cache, {n: modules[n] for n in executed}, next(model.parameters()).device)
            self.coverage["packed_weights"] = {"path": str(cache), "loaded": True}
        self.controller = TransformerINT(
            model,
            set(executed),
            native=True,
            expanded=expanded,
            condition_group=self.config.group_conditioning,
            packed=packed,
        )
        if cache is not None and packed is None:
            from . import weight_cache

            weight_cache.save(self.controller, cache)
            self.coverage["packed_weights"] = {"path": str(cache), "loaded": False, "written": True}
        self.stack.callback(self.controller.close)
        self.extra = AdditionalConnections(SimpleNamespace(model=model), self.controller, categories)
        self.stack.callback(self.extra.close)
        apply_tactics(self.controller, self.extra, self.config, recorded, backend_evidence=self.backend)
        self.controller.set(self.config.precision)
        if self.config.fusion:
            # The residual fusion of this build (ResidualFusion: residual adds
            # in the GEMM epilogues, norm3 + pack fused) replaces the
            # block-level residual + norm3 + pack of AdditionalConnections.
            self.extra.set(
                self.config.precision,
                expanded=expanded,
                fuse=True,
                norm_quant=self.config.norm_modulation_quant,
                residual_quant=False,
            )
            if self.config.residual_norm_quant:
                from .fusion import ResidualFusion

                self.residual = ResidualFusion(model, self.controller)
                self.stack.callback(self.residual.close)
                self.residual.set({"w8a8": 8, "w4a4": 4}[self.config.precision])
            if self.config.precision == "w8a8":
                from .fusion import SwiGLUFusion

                self.swiglu = SwiGLUFusion(model, self.controller)
                self.stack.callback(self.swiglu.close)
                self.swiglu.set()
            if self.config.fusion_mode in ("all", "rope_rms"):
                from .pointwise import TextAttentionFusion

                self.pointwise = TextAttentionFusion(model, self.controller)
                self.stack.callback(self.pointwise.close)
                self.pointwise.set({"w8a8": 8, "w4a4": 4}[self.config.precision])
            if self.config.fusion_mode == "all":
                from .pointwise import DiTAttentionFusion

                self.attention = DiTAttentionFusion(model.action_head.model)
                self.stack.callback(self.attention.close)
                self.attention.set()
            self.producers = QuantizationProducers(model, self.controller)
            if self.producers.norms:
                self.stack.callback(self.producers.close)
                self.producers.set({"w8a8": 8, "w4a4": 4}[self.config.precision])
        elif categories:
            self.extra.set(self.config.precision, expanded=expanded, fuse=False)

    def evidence(self):
        config = asdict(self.config)
        for key in CONFIG_FILES:
            path = config[key]
            actual = None if path is None else hashlib.sha256(Path(path).read_bytes()).hexdigest()
            if key in self._configuration_file_hashes and actual != self._configuration_file_hashes[key]:
                raise RuntimeError(f"Installed optimization configuration file changed: {key}")
            config[key] = None if path is None else {"sha256": actual}
        if config.get("packed_weights") is not None:
            config["packed_weights"] = str(config["packed_weights"])
        return {
            "config": config,
            "coverage": self.coverage,
            "backend": self.backend,
            "producers": None if self.producers is None else self.producers.evidence(),
            "scope": "Serial inference; parity tests do not establish task quality",
        }

    def close(self):
        try:
            self.stack.close()
        finally:
            self._active = False

    def __exit__(self, *exception):
        self.close()
