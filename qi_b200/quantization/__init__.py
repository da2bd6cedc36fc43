"""Quantized-linear API with the names of ``qi.quantization`` (reference
``src/qi/quantization/__init__.py``), served by the B200 kernels."""

from .checkpoint import (
    checkpoint_format,
    checkpoint_is_quantized,
    load_checkpoint_payload,
    load_quantized_checkpoint,
    prepare_model_for_quantized_checkpoint,
    quant_config_from_metadata,
    quantize_loaded_model,
    save_quantized_checkpoint,
)
from .config import WeightActivationQuantConfig, WeightOnlyQuantConfig
from .modules import WeightOnlyLinear
from .quantize import (
    QuantizedLinearWeight,
    dequantize_weight,
    quantize_linear_weight,
    quantize_weight_awq,
    quantize_weight_fp8_rtn,
    quantize_weight_fp8_smoothquant,
    quantize_weight_int8_smoothquant,
    quantize_weight_nvfp4,
    quantize_weight_rtn,
)
from .swap import (
    fuse_ffn_gelu,
    prepare_model_for_weight_only_load,
    replace_linear_with_weight_only,
    should_quantize,
    verify_loaded_buffers,
)

__all__ = [
    "QuantizedLinearWeight", "WeightOnlyLinear", "WeightActivationQuantConfig", "WeightOnlyQuantConfig",
    "checkpoint_format", "checkpoint_is_quantized", "load_quantized_checkpoint", "dequantize_weight", "fuse_ffn_gelu", "load_checkpoint_payload",
    "prepare_model_for_quantized_checkpoint", "prepare_model_for_weight_only_load", "quant_config_from_metadata",
    "quantize_linear_weight", "quantize_loaded_model", "quantize_weight_awq", "quantize_weight_fp8_rtn",
    "quantize_weight_fp8_smoothquant", "quantize_weight_int8_smoothquant", "quantize_weight_nvfp4",
    "quantize_weight_rtn", "replace_linear_with_weight_only", "save_quantized_checkpoint", "should_quantize",
    "verify_loaded_buffers",
]
