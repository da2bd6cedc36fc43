"""Quantized checkpoint format — the reference's (``src/qi/quantization/
checkpoint.py:13-98``): a ``torch.save`` dict with the model's state dict under
``"mot"`` / ``"dit"`` / ``"model"`` and metadata under ``"qi_quantization"``
= ``{"format": "qi.weight_activation.v1" | "qi.weight_only.v1", "config":
asdict(cfg), "source_checkpoint": ...}``.  The B200 formats use the same
keys; their packed buffers are ordinary state-dict entries.
"""

from __future__ import annotations

from dataclasses import asdict
from pathlib import Path
from typing import Any, Mapping

import torch
import torch.nn as nn

from .config import WeightActivationQuantConfig, WeightOnlyQuantConfig
from .swap import prepare_model_for_weight_only_load, replace_linear_with_weight_only

METADATA_KEY = "qi_quantization"
FORMAT_WEIGHT_ACTIVATION = "qi.weight_activation.v1"
FORMAT_WEIGHT_ONLY = "qi.weight_only.v1"
_CONTAINERS = ("mot", "dit", "model")


def quant_config_from_metadata(metadata: Mapping[str, Any]):
    payload = dict(metadata.get("config", metadata))
    is_wa = metadata.get("format") == FORMAT_WEIGHT_ACTIVATION or payload.get("quant_dtype") in ("fp8", "nvfp4")
    cls = WeightActivationQuantConfig if is_wa else WeightOnlyQuantConfig
    payload = {k: v for k, v in payload.items() if k in cls.__dataclass_fields__}
    for key in ("action_expert_markers", "video_expert_markers", "target_modules", "skip_modules"):
        if isinstance(payload.get(key), list):
            payload[key] = tuple(payload[key])
    return cls(**payload)


def checkpoint_is_quantized(payload: Mapping[str, Any]) -> bool:
    return METADATA_KEY in payload


def prepare_model_for_quantized_checkpoint(model: nn.Module, payload: Mapping[str, Any],
                                           backend: str | None = None):
    """Swap quantized layers in before loading.  ``backend`` overrides the one
    recorded in the checkpoint (e.g. load an ``int8_w8a8`` checkpoint onto
    ``b200``)."""
    if not checkpoint_is_quantized(payload):
        raise ValueError("Checkpoint is missing quantization metadata.")
    cfg = quant_config_from_metadata(payload[METADATA_KEY])
    if backend is not None:
        cfg.backend = backend
    for key in _CONTAINERS:
        if key in payload:
            target = model if key == "model" else getattr(model, key)
            prepare_model_for_weight_only_load(target, cfg, state_dict=payload[key])
            break
    else:
        prepare_model_for_weight_only_load(model, cfg)
    return cfg


def load_checkpoint_payload(path: str | Path) -> dict[str, Any]:
    payload = torch.load(path, map_location="cpu")
    if not isinstance(payload, dict):
        raise ValueError(f"Checkpoint payload must be a dict, got {type(payload)} from {path}.")
    return payload


def quantize_loaded_model(model: nn.Module, cfg, act_stats=None) -> nn.Module:
    replace_linear_with_weight_only(model, cfg, act_stats=act_stats)
    return model


def save_quantized_checkpoint(model, output_path: str | Path, cfg, source_payload: Mapping[str, Any] | None = None,
                              source_checkpoint: str | Path | None = None) -> None:
    payload: dict[str, Any] = dict(source_payload or {})
    if hasattr(model, "mot"):
        payload["mot"] = model.mot.state_dict()
    elif hasattr(model, "dit"):
        payload["dit"] = model.dit.state_dict()
    else:
        payload["model"] = model.state_dict()
    if getattr(model, "proprio_encoder", None) is not None:
        payload["proprio_encoder"] = model.proprio_encoder.state_dict()
    payload.pop("optimizer", None)
    payload[METADATA_KEY] = {
        "format": FORMAT_WEIGHT_ACTIVATION if isinstance(cfg, WeightActivationQuantConfig) else FORMAT_WEIGHT_ONLY,
        "config": asdict(cfg),
        "source_checkpoint": None if source_checkpoint is None else str(source_checkpoint),
    }
    output_path = Path(output_path)
    output_path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, output_path)
