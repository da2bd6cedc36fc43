"""Module swap: replace selected ``nn.Linear`` layers with ``WeightOnlyLinear``.

Same selection rules and entry points as the reference
(``src/qi/quantization/swap.py:49-233``): ``should_quantize`` (enabled flag,
expert markers, skip list, target-module substrings, ffn/attention toggles),
``replace_linear_with_weight_only`` (quantize now) and
``prepare_model_for_weight_only_load`` (empty buffers shaped like the
checkpoint's, filled later by ``load_state_dict``).

Additions for the B200 backend:
* load-time preparation knows the packed W4A16 / NVFP4 / per-channel FP8
  buffer shapes (taken from the checkpoint's state dict when present);
* ``verify_loaded_buffers`` catches the reference's silent failure mode
  (``load_state_dict(strict=False)`` leaves a missing buffer uninitialised);
* ``fuse_ffn_gelu`` moves the FFN's GELU(tanh) into the ``ffn.0`` epilogue.
"""

from __future__ import annotations

import math
from collections.abc import Mapping

import torch
import torch.nn as nn

from .backends import get_backend
from .modules import WeightOnlyLinear
from .quantize import effective_group_size, quantize_linear_weight


def _markers(markers) -> tuple[str, ...]:
    return tuple(str(m).lower() for m in markers if str(m).strip())


def _matches_target_expert(name: str, cfg) -> bool:
    scope = str(getattr(cfg, "target_expert", "all")).lower()
    if scope in ("all", "both"):
        return True
    lname = name.lower()
    if scope == "action":
        return any(m in lname for m in _markers(getattr(cfg, "action_expert_markers", ("action_expert", "action"))))
    if scope == "video":
        return any(m in lname for m in _markers(getattr(cfg, "video_expert_markers", ("video_expert", "video", "dit"))))
    raise ValueError(f"Unsupported target_expert: {scope}")


_FFN_MARKERS = ("fc1", "fc2", "ffn", "mlp", "feed_forward")
_ATTN_MARKERS = ("q_proj", "k_proj", "v_proj", "o_proj", "attn", "attention")


def _matches_module_kind(name: str, cfg) -> bool:
    lname = name.lower()
    if not getattr(cfg, "quantize_ffn", True) and any(m in lname for m in _FFN_MARKERS):
        return False
    if not getattr(cfg, "quantize_attn_proj", True) and any(m in lname for m in _ATTN_MARKERS):
        return False
    return True


def should_quantize(name: str, module: nn.Module, cfg) -> bool:
    if not getattr(cfg, "enabled", True) or not isinstance(module, nn.Linear):
        return False
    if not _matches_target_expert(name, cfg):
        return False
    if any(s and s in name for s in getattr(cfg, "skip_modules", ())):
        return False
    targets = getattr(cfg, "target_modules", ())
    if targets and not any(t and t in name for t in targets):
        return False
    return _matches_module_kind(name, cfg)


def _stats_for_module(act_stats, name: str):
    if act_stats is None or not isinstance(act_stats, Mapping):
        return act_stats
    if name in act_stats:
        return act_stats[name]
    hits = [v for k, v in act_stats.items() if name.endswith(str(k))]
    if len(hits) == 1:
        return hits[0]
    raise ValueError(f"Missing activation stats for module {name!r}; collect them with the same target modules.")


def _named_linear_children(model: nn.Module):
    for parent_name, parent in model.named_modules():
        for child_name, child in list(parent.named_children()):
            full = f"{parent_name}.{child_name}" if parent_name else child_name
            yield parent, child_name, full, child


def replace_linear_with_weight_only(model: nn.Module, cfg, act_stats=None) -> nn.Module:
    if hasattr(cfg, "validate"):
        cfg.validate()
    backend = get_backend(cfg.backend)
    for parent, child_name, full, child in list(_named_linear_children(model)):
        if not should_quantize(full, child, cfg):
            continue
        q = quantize_linear_weight(child.weight.detach(), cfg=cfg, act_stats=_stats_for_module(act_stats, full))
        ql = WeightOnlyLinear.from_linear(child, q, cfg=cfg, backend=backend)
        ql.train(child.training)
        setattr(parent, child_name, ql)
    return model


def _state_tensor(sd, container_key, module_name, key):
    if sd is None:
        return None
    prefix = f"{module_name}." if module_name else ""
    if container_key:
        prefix = f"{container_key}.{prefix}"
    v = sd.get(prefix + key)
    return v if isinstance(v, torch.Tensor) else None


def _empty_like_state(sd, ck, name, key, default_shape=None, default_dtype=None):
    t = _state_tensor(sd, ck, name, key)
    if t is not None:
        return torch.empty_like(t)
    if default_shape is None:
        return None
    return torch.empty(default_shape, dtype=default_dtype)


def _first(*vals):
    for v in vals:
        if v is not None:
            return v
    return None


def prepare_model_for_weight_only_load(model: nn.Module, cfg, state_dict: Mapping | None = None,
                                       container_key: str | None = None) -> nn.Module:
    """Swap in ``WeightOnlyLinear`` layers with empty (CPU) buffers shaped like
    the checkpoint's, so ``load_state_dict`` can fill them."""
    if hasattr(cfg, "validate"):
        cfg.validate()
    backend = get_backend(cfg.backend)
    qdt = getattr(cfg, "quant_dtype", "int")
    for parent, child_name, full, child in list(_named_linear_children(model)):
        if not should_quantize(full, child, cfg):
            continue
        N, K = child.weight.shape
        g = effective_group_size(int(getattr(cfg, "group_size", -1)), K)
        G = math.ceil(K / g)
        bufs = dict(qweight=None, scales=None, zeros=None, qweight_packed=None, scale_factors=None,
                    weight_global_scale=None, weight_fp8=None, weight_scale=None, activation_scale=None)
        E = lambda key, shape=None, dtype=None: _empty_like_state(state_dict, container_key, full, key, shape, dtype)
        if qdt == "fp8":
            # aliases of the reference loader (swap.py:182-199)
            bufs["weight_fp8"] = _first(E("weight_fp8"), E("qweight_packed"), torch.empty((N, K), dtype=torch.uint8))
            bufs["weight_scale"] = _first(E("weight_scale"), E("weight_global_scale"), torch.empty((1,)))
            bufs["activation_scale"] = _first(E("activation_scale"), E("scale_factors"), torch.empty((1,)))
        elif qdt == "nvfp4":
            bufs["qweight_packed"] = E("qweight_packed", (N, K // 2), torch.uint8)
            sf_bytes = -(-N // 128) * 128 * (-(-(K // 16) // 4) * 4)
            bufs["scale_factors"] = E("scale_factors", (sf_bytes,), torch.uint8)
            bufs["weight_global_scale"] = E("weight_global_scale", (1,), torch.float32)
            bufs["activation_scale"] = E("activation_scale")
        elif getattr(cfg, "backend", "") in ("b200", "cuda_ext") and cfg.bits == 4:
            bufs["qweight_packed"] = E("qweight_packed", (N, K // 8), torch.int32)
            bufs["scale_factors"] = E("scale_factors", (N, G), torch.float16)
            bufs["zeros"] = E("zeros", (N, -(-G // 8)), torch.int32)
        else:
            bufs["qweight"] = torch.empty((N, K), dtype=torch.int8)
            bufs["scales"] = torch.empty((N, G), dtype=torch.float32)
            if not getattr(cfg, "symmetric", True) or _state_tensor(state_dict, container_key, full, "zeros") is not None:
                bufs["zeros"] = torch.empty((N, G), dtype=torch.int16)
        input_scale = None
        if cfg.algo in ("awq", "smoothquant") or _state_tensor(state_dict, container_key, full, "input_scale") is not None:
            input_scale = torch.empty((K,), dtype=torch.float32)
        ql = WeightOnlyLinear(
            **bufs, input_scale=input_scale, bias=child.bias.detach() if child.bias is not None else None,
            in_features=child.in_features, out_features=child.out_features, bits=cfg.bits,
            group_size=int(getattr(cfg, "group_size", -1)), symmetric=bool(getattr(cfg, "symmetric", True)),
            backend=backend, activation_granularity=getattr(cfg, "activation_granularity", None),
            weight_granularity=getattr(cfg, "weight_granularity", None),
            keep_output_dtype=getattr(cfg, "keep_output_dtype", "input"),
        )
        ql.train(child.training)
        setattr(parent, child_name, ql)
    return model


def verify_loaded_buffers(model: nn.Module, state_dict: Mapping, container_key: str | None = None) -> None:
    """Raise if any ``WeightOnlyLinear`` buffer has no entry in ``state_dict``."""
    missing = []
    for name, mod in model.named_modules():
        if not isinstance(mod, WeightOnlyLinear):
            continue
        for bname, _ in mod.named_buffers(recurse=False):
            if _state_tensor(state_dict, container_key, name, bname) is None:
                missing.append(f"{name}.{bname}")
    if missing:
        raise ValueError(f"quantized checkpoint is missing {len(missing)} buffers, e.g. {missing[:4]}")


def fuse_ffn_gelu(model: nn.Module) -> int:
    """For every ``nn.Sequential(Linear, GELU(tanh), Linear)`` whose first layer
    is a ``WeightOnlyLinear``, run the GELU in that layer's epilogue and make
    the GELU an identity.  Returns the number of fused blocks."""
    n = 0
    for mod in model.modules():
        if isinstance(mod, nn.Sequential) and len(mod) == 3 and isinstance(mod[0], WeightOnlyLinear) \
                and isinstance(mod[1], nn.GELU) and mod[1].approximate == "tanh":
            mod[0].fuse_gelu = True
            mod[1] = nn.Identity()
            n += 1
    return n
