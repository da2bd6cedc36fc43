"""Quantization configs — same dataclasses, fields and defaults as the
reference (``src/qi/quantization/config.py:21-115``), extended for the B200
backend:

* backend ``"b200"`` (the native sm_100a kernels of this package); the
  reference's native backend names (``"int8_w8a8"``, ``"flashrt_fp8"``,
  ``"cuda_ext"``) are accepted and served by the same kernels;
* ``WeightActivationQuantConfig.quant_dtype`` gains ``"nvfp4"`` (W4A4: E2M1
  values, E4M3 scale per 16 elements along K, fp32 per-tensor scale);
* FP8 on the B200 backend also allows per-token activations and
  per-channel weights (the reference only has per-tensor, ``config.py:95-96``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

# Linear layers of the Wan2.2 MoT DiT block that are quantized
# (config.py:7-18 of the reference).
_TARGET_MODULES = (
    "self_attn.q",
    "self_attn.k",
    "self_attn.v",
    "self_attn.o",
    "cross_attn.q",
    "cross_attn.k",
    "cross_attn.v",
    "cross_attn.o",
    "ffn.0",
    "ffn.2",
)

NATIVE_BACKENDS = ("b200", "int8_w8a8", "flashrt_fp8", "cuda_ext")


@dataclass
class WeightOnlyQuantConfig:
    enabled: bool = False
    algo: Literal["awq", "rtn"] = "awq"
    quant_dtype: Literal["int"] = "int"
    bits: int = 8
    group_size: int = 128
    symmetric: bool = True
    backend: Literal["reference", "cuda_ext", "b200"] = "reference"

    target_expert: Literal["all", "both", "action", "video"] = "all"
    action_expert_markers: tuple[str, ...] = ("action_expert", "action")
    video_expert_markers: tuple[str, ...] = ("video_expert", "video", "dit")
    target_modules: tuple[str, ...] = _TARGET_MODULES
    skip_modules: tuple[str, ...] = ()
    quantize_ffn: bool = True
    quantize_attn_proj: bool = True

    keep_output_dtype: Literal["input", "fp16", "bf16", "fp32"] = "input"

    awq_alpha: float = 0.5
    awq_scale_eps: float = 1e-4

    def validate(self) -> None:
        if self.quant_dtype != "int":
            raise ValueError(
                'WeightOnlyQuantConfig only supports quant_dtype="int". '
                "Use WeightActivationQuantConfig for W8A8 / W4A4 quantization."
            )
        if self.bits not in (4, 8):
            raise ValueError(f"`bits` must be 4 or 8, got {self.bits}.")
        if self.group_size == 0 or self.group_size < -1:
            raise ValueError(f"`group_size` must be positive or -1, got {self.group_size}.")
        if not 0.0 <= float(self.awq_alpha) <= 1.0:
            raise ValueError(f"`awq_alpha` must be in [0, 1], got {self.awq_alpha}.")
        if self.backend in NATIVE_BACKENDS and self.bits == 4:
            if self.group_size != -1 and self.group_size % 8 != 0:
                raise ValueError("The B200 W4A16 kernels need group_size % 8 == 0 (or -1).")


@dataclass
class WeightActivationQuantConfig:
    enabled: bool = False
    algo: Literal["rtn", "smoothquant"] = "rtn"
    quant_dtype: Literal["fp8", "int", "nvfp4"] = "fp8"
    bits: int = 8
    activation_bits: int = 8
    backend: Literal["flashrt_fp8", "reference", "int8_w8a8", "b200"] = "flashrt_fp8"
    activation_granularity: Literal["per_tensor", "per_token"] = "per_tensor"
    weight_granularity: Literal["per_tensor", "per_channel"] = "per_tensor"
    group_size: int = -1
    symmetric: bool = True

    target_expert: Literal["all", "both", "action", "video"] = "all"
    action_expert_markers: tuple[str, ...] = ("action_expert", "action")
    video_expert_markers: tuple[str, ...] = ("video_expert", "video", "dit")
    target_modules: tuple[str, ...] = _TARGET_MODULES
    skip_modules: tuple[str, ...] = ()
    quantize_ffn: bool = True
    quantize_attn_proj: bool = True

    keep_output_dtype: Literal["input", "fp16", "bf16", "fp32"] = "input"

    smoothquant_alpha: float = 0.5
    smoothquant_scale_eps: float = 1e-4
    activation_scale: float = 1.0

    def validate(self) -> None:
        if self.quant_dtype == "nvfp4":
            if self.bits != 4 or self.activation_bits != 4:
                raise ValueError("NVFP4 W4A4 requires bits=4 and activation_bits=4.")
            if self.backend != "b200":
                raise ValueError(f'NVFP4 W4A4 requires backend="b200", got {self.backend}.')
            if self.algo != "rtn":
                raise ValueError("NVFP4 W4A4 supports algo=\"rtn\" only.")
            if self.group_size not in (-1, 16):
                raise ValueError("NVFP4 block size is fixed at 16 elements.")
            return
        if self.bits != 8:
            raise ValueError(f"W8A8 requires `bits=8`, got {self.bits}.")
        if self.activation_bits != 8:
            raise ValueError(f"W8A8 requires `activation_bits=8`, got {self.activation_bits}.")
        if self.algo not in ("rtn", "smoothquant"):
            raise ValueError(f"Unsupported W8A8 algo: {self.algo}.")
        if self.quant_dtype == "fp8":
            if self.backend not in ("flashrt_fp8", "b200"):
                raise ValueError(f'FP8 W8A8 requires backend="flashrt_fp8" or "b200", got {self.backend}.')
            if self.backend == "flashrt_fp8" and (
                self.activation_granularity != "per_tensor" or self.weight_granularity != "per_tensor"
            ):
                raise ValueError("FP8 W8A8 currently supports per_tensor activation and weight scales only.")
        elif self.quant_dtype == "int":
            if self.backend not in ("reference", "int8_w8a8", "b200"):
                raise ValueError(
                    f'INT8 W8A8 requires backend="reference", "int8_w8a8" or "b200", got {self.backend}.'
                )
            if self.activation_granularity != "per_token":
                raise ValueError('INT8 W8A8 currently requires activation_granularity="per_token".')
            if self.weight_granularity != "per_channel":
                raise ValueError('INT8 W8A8 currently requires weight_granularity="per_channel".')
            if self.group_size != -1:
                raise ValueError("INT8 W8A8 per-channel weights require group_size=-1.")
            if not self.symmetric:
                raise ValueError("INT8 W8A8 currently requires symmetric quantization.")
        else:
            raise ValueError(f"Unsupported W8A8 quant_dtype: {self.quant_dtype}.")
        if not 0.0 <= float(self.smoothquant_alpha) <= 1.0:
            raise ValueError(f"`smoothquant_alpha` must be in [0, 1], got {self.smoothquant_alpha}.")
        if float(self.smoothquant_scale_eps) <= 0:
            raise ValueError("`smoothquant_scale_eps` must be positive.")
        if float(self.activation_scale) <= 0:
            raise ValueError("`activation_scale` must be positive.")
