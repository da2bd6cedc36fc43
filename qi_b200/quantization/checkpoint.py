"""Quantized checkpoints: the reference's format (read and written) and a
versioned format whose buffers are already in this library's kernel layouts.

A checkpoint is one ``torch.save`` dict.  Its keys, as the reference defines
them (``src/qi/quantization/checkpoint.py:13-98``), are kept so a checkpoint
moves between the two code bases:

==================  =========================================================
key                 value
==================  =========================================================
``"mot"``           state dict of ``model.mot``  (first that the model has,
``"dit"``           ... or of ``model.dit``       in this order)
``"model"``         ... or of the model itself
``"proprio_encoder"`` state dict of ``model.proprio_encoder``, when present
``"optimizer"``     never written (dropped from a source payload)
``"qi_quantization"`` metadata: ``format``, ``config`` (the quantization
                    config's fields), ``source_checkpoint`` (path or None)
                    and, in the packed formats, ``layouts``
==================  =========================================================

Formats (``metadata["format"]``):

* ``qi.weight_only.v1`` / ``qi.weight_activation.v1`` -- the reference's.
  Weight-only INT4 keeps one code per int8 with fp32 scales and int16 zero
  points.  Loading one for the B200 backend repacks INT4 layers into the
  packed layout (8 codes per int32, fp16 scales, packed uint4 zero points).
* ``qi_b200.weight_only.packed.v2`` / ``qi_b200.weight_activation.packed.v2``
  -- written whenever a model holds a packed buffer (W4A16 or NVFP4).  The
  buffers are stored exactly as the kernels read them (``LAYOUTS``), so
  loading copies bytes and repacks nothing.  The loader refuses a packed
  checkpoint whose layout names differ from this library's, and any format
  string it does not know.
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
FORMAT_WEIGHT_ONLY = "qi.weight_only.v1"
FORMAT_WEIGHT_ACTIVATION = "qi.weight_activation.v1"
FORMAT_PACKED_WEIGHT_ONLY = "qi_b200.weight_only.packed.v2"
FORMAT_PACKED_WEIGHT_ACTIVATION = "qi_b200.weight_activation.packed.v2"
_WA_FORMATS = (FORMAT_WEIGHT_ACTIVATION, FORMAT_PACKED_WEIGHT_ACTIVATION)
_PACKED_FORMATS = (FORMAT_PACKED_WEIGHT_ONLY, FORMAT_PACKED_WEIGHT_ACTIVATION)
KNOWN_FORMATS = (FORMAT_WEIGHT_ONLY, FORMAT_WEIGHT_ACTIVATION) + _PACKED_FORMATS

# Names of the on-disk layouts of the packed formats (kernel-ready bytes).
LAYOUTS = {
    "w4a16": "qweight_packed int32 [N, K/8] (code k in bits 4(k%8) of word k/8); "
             "scale_factors fp16 [N, G]; zeros int32 [N, ceil(G/8)] (uint4 zero g in bits 4(g%8))",
    "nvfp4": "qweight_packed uint8 [N, K/2] (E2M1, even k in the low nibble); scale_factors E4M3 in "
             "512-byte atoms of 128 rows x 4 (row r0 + 32 r1 at byte 16 r0 + 4 r1 + j); weight_global_scale fp32 [1]",
}

# Container keys in the order a model is probed for them; None = the model itself.
_CONTAINERS = (("mot", "mot"), ("dit", "dit"), ("model", None))


def _container(model: nn.Module):
    """(payload key, module) whose state dict a checkpoint of ``model`` holds."""
    for key, attr in _CONTAINERS:
        if attr is None or hasattr(model, attr):
            return key, model if attr is None else getattr(model, attr)
    return "model", model


def _payload_container(model: nn.Module, payload: Mapping[str, Any]):
    """(payload key, module of ``model``) for the first container key the
    payload holds; (None, model) when it holds none."""
    for key, attr in _CONTAINERS:
        if key in payload:
            return key, model if attr is None else getattr(model, attr)
    return None, model


def checkpoint_is_quantized(payload: Mapping[str, Any]) -> bool:
    return METADATA_KEY in payload


def checkpoint_format(payload: Mapping[str, Any]) -> str:
    """The payload's format string; ValueError for a format this library cannot read."""
    meta = payload.get(METADATA_KEY)
    if not isinstance(meta, Mapping):
        raise ValueError("Checkpoint is missing quantization metadata.")
    fmt = meta.get("format", FORMAT_WEIGHT_ONLY)
    if fmt not in KNOWN_FORMATS:
        raise ValueError(f"Unsupported quantized checkpoint format {fmt!r}; this library reads {KNOWN_FORMATS}.")
    if fmt in _PACKED_FORMATS:
        theirs = meta.get("layouts", {})
        for name, layout in theirs.items():
            if LAYOUTS.get(name) != layout:
                raise ValueError(f"Packed checkpoint layout {name!r} differs from this library's: {layout!r}.")
    return fmt


def quant_config_from_metadata(metadata: Mapping[str, Any]):
    """Rebuild the quantization config recorded in a checkpoint's metadata
    (a config dict, or metadata holding one under ``"config"``)."""
    fields = dict(metadata.get("config", metadata))
    weight_activation = metadata.get("format") in _WA_FORMATS or fields.get("quant_dtype") in ("fp8", "nvfp4")
    cls = WeightActivationQuantConfig if weight_activation else WeightOnlyQuantConfig
    known = cls.__dataclass_fields__
    kwargs = {}
    for name, value in fields.items():
        if name in known:
            kwargs[name] = tuple(value) if isinstance(value, list) else value
    return cls(**kwargs)


def _repack_reference_int4(state: dict, cfg) -> dict:
    """Reference weight-only INT4 entries (``<layer>.qweight`` int8 codes,
    ``.scales`` fp32, ``.zeros`` int16 or absent) -> the packed entries the
    B200 modules hold.  Other entries pass through."""
    from .quantize import pack_w4a16

    out = dict(state)
    for key, q in state.items():
        if not key.endswith(".qweight") or not isinstance(q, torch.Tensor) or q.dtype != torch.int8:
            continue
        layer = key[: -len("qweight")]
        s = state.get(layer + "scales")
        if s is None:
            continue
        z = state.get(layer + "zeros")
        qp, s16, zp = pack_w4a16(q, s.reshape(q.shape[0], -1).float(), None if z is None else z.reshape(q.shape[0], -1))
        for k in ("qweight", "scales", "zeros"):
            out.pop(layer + k, None)
        out[layer + "qweight_packed"], out[layer + "scale_factors"], out[layer + "zeros"] = qp, s16, zp
    return out


def prepare_model_for_quantized_checkpoint(model: nn.Module, payload: dict, backend: str | None = None):
    """Swap quantized layers into ``model`` shaped for ``payload``'s buffers.
    ``backend`` overrides the recorded one (e.g. load a reference
    ``int8_w8a8`` checkpoint onto ``b200``).  A reference INT4 weight-only
    checkpoint loaded for the B200 backend has its container state dict
    repacked in place into the kernels' layout.  Returns the config."""
    fmt = checkpoint_format(payload)
    cfg = quant_config_from_metadata(payload[METADATA_KEY])
    if backend is not None:
        cfg.backend = backend
    key, target = _payload_container(model, payload)
    state = payload.get(key) if key is not None else None
    native_int4 = (not isinstance(cfg, WeightActivationQuantConfig) and cfg.bits == 4
                   and cfg.backend in ("b200", "cuda_ext"))
    if state is not None and native_int4 and fmt not in _PACKED_FORMATS:
        state = payload[key] = _repack_reference_int4(state, cfg)
    prepare_model_for_weight_only_load(target, cfg, state_dict=state)
    return cfg


def load_quantized_checkpoint(model: nn.Module, payload: dict, backend: str | None = None, strict: bool = True):
    """``prepare_model_for_quantized_checkpoint`` then load the container's
    state dict (and ``proprio_encoder``'s, when both sides have one)."""
    from .swap import verify_loaded_buffers

    cfg = prepare_model_for_quantized_checkpoint(model, payload, backend)
    key, target = _payload_container(model, payload)
    if key is not None:
        target.load_state_dict(payload[key], strict=strict)
        verify_loaded_buffers(target, payload[key])
    if "proprio_encoder" in payload and getattr(model, "proprio_encoder", None) is not None:
        model.proprio_encoder.load_state_dict(payload["proprio_encoder"], strict=strict)
    return cfg


def load_checkpoint_payload(path: str | Path) -> dict[str, Any]:
    obj = torch.load(path, map_location="cpu")
    if isinstance(obj, dict):
        return obj
    raise ValueError(f"{path}: expected a checkpoint dict, found {type(obj).__name__}.")


def quantize_loaded_model(model: nn.Module, cfg, act_stats=None) -> nn.Module:
    """Quantize a model whose float weights are loaded (swap in WeightOnlyLinear)."""
    return replace_linear_with_weight_only(model, cfg, act_stats=act_stats)


def _holds_packed_buffers(module: nn.Module) -> bool:
    return any(name.endswith("qweight_packed") for name, _ in module.named_buffers())


def save_quantized_checkpoint(model, output_path: str | Path, cfg, source_payload: Mapping[str, Any] | None = None,
                              source_checkpoint: str | Path | None = None) -> str:
    """Write ``model``'s quantized state (see the key table above) and return
    the format written: the packed v2 format when the model holds packed
    buffers, else the reference's v1."""
    key, target = _container(model)
    packed = _holds_packed_buffers(target)
    weight_activation = isinstance(cfg, WeightActivationQuantConfig)
    fmt = ((FORMAT_PACKED_WEIGHT_ACTIVATION if weight_activation else FORMAT_PACKED_WEIGHT_ONLY) if packed
           else (FORMAT_WEIGHT_ACTIVATION if weight_activation else FORMAT_WEIGHT_ONLY))
    meta = {"format": fmt, "config": asdict(cfg),
            "source_checkpoint": str(source_checkpoint) if source_checkpoint is not None else None}
    if packed:
        meta["layouts"] = dict(LAYOUTS)
    payload = {k: v for k, v in (source_payload or {}).items() if k != "optimizer"}
    payload[key] = target.state_dict()
    encoder = getattr(model, "proprio_encoder", None)
    if encoder is not None:
        payload["proprio_encoder"] = encoder.state_dict()
    payload[METADATA_KEY] = meta
    path = Path(output_path)
    path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, path)
    return fmt
