"""``WeightOnlyLinear``: the quantized ``nn.Linear`` replacement.

Same constructor, buffer names and forward contract as the reference
(``src/qi/quantization/modules.py:7-133``): every quantization tensor is a
registered buffer (so ``state_dict`` / checkpoints carry it) and ``forward``
hands all of them to ``backend.linear`` by keyword.  Which buffers a format
uses is listed in ``qi_b200/quantization/quantize.py``.
"""

from __future__ import annotations

import torch
import torch.nn as nn

_BUFFERS = ("qweight", "scales", "qweight_packed", "scale_factors", "weight_global_scale", "activation_scale",
            "weight_scale", "weight_fp8", "zeros", "input_scale")
_FLOAT_BUFFERS = ("weight_global_scale", "activation_scale", "weight_scale", "input_scale")


class WeightOnlyLinear(nn.Module):
    def __init__(self, qweight, scales, zeros, bias, in_features: int, out_features: int, bits: int,
                 group_size: int, symmetric: bool, backend, input_scale=None, qweight_packed=None,
                 scale_factors=None, weight_global_scale=None, activation_scale=None, weight_scale=None,
                 weight_fp8=None, activation_granularity: str | None = None,
                 weight_granularity: str | None = None, keep_output_dtype: str = "input"):
        super().__init__()
        given = dict(qweight=qweight, scales=scales, qweight_packed=qweight_packed, scale_factors=scale_factors,
                     weight_global_scale=weight_global_scale, activation_scale=activation_scale,
                     weight_scale=weight_scale, weight_fp8=weight_fp8, zeros=zeros, input_scale=input_scale)
        for name in _BUFFERS:
            t = given[name]
            if t is None:
                setattr(self, name, None)
            else:
                t = t.contiguous()
                self.register_buffer(name, t.float() if name in _FLOAT_BUFFERS else t)
        if bias is None:
            self.bias = None
        else:
            self.register_buffer("bias", bias.detach().clone())
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.bits = int(bits)
        self.group_size = int(group_size)
        self.symmetric = bool(symmetric)
        self.backend = backend
        self.activation_granularity = activation_granularity
        self.weight_granularity = weight_granularity
        self.keep_output_dtype = keep_output_dtype
        # Set by fuse_ffn_gelu(): the following GELU(tanh) runs in this
        # layer's epilogue and the model's nn.GELU becomes an identity.
        self.fuse_gelu = False

    @classmethod
    def from_linear(cls, linear: nn.Linear, quantized, cfg, backend) -> "WeightOnlyLinear":
        return cls(
            qweight=quantized.qweight, scales=quantized.scales, zeros=quantized.zeros,
            input_scale=quantized.input_scale,
            qweight_packed=getattr(quantized, "qweight_packed", None),
            scale_factors=getattr(quantized, "scale_factors", None),
            weight_global_scale=getattr(quantized, "weight_global_scale", None),
            activation_scale=getattr(quantized, "activation_scale", None),
            weight_scale=getattr(quantized, "weight_scale", None),
            weight_fp8=getattr(quantized, "weight_fp8", None),
            bias=linear.bias.detach() if linear.bias is not None else None,
            in_features=linear.in_features, out_features=linear.out_features, bits=cfg.bits,
            group_size=int(getattr(cfg, "group_size", -1)), symmetric=bool(getattr(cfg, "symmetric", True)),
            backend=backend, activation_granularity=getattr(cfg, "activation_granularity", None),
            weight_granularity=getattr(cfg, "weight_granularity", None),
            keep_output_dtype=getattr(cfg, "keep_output_dtype", "input"),
        )

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, bits={self.bits}, "
                f"group_size={self.group_size}, backend={type(self.backend).__name__}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        extra = {"gelu": True} if self.fuse_gelu else {}
        return self.backend.linear(
            x=x, qweight=self.qweight, scales=self.scales, zeros=self.zeros, bias=self.bias, bits=self.bits,
            group_size=self.group_size, symmetric=self.symmetric, input_scale=self.input_scale,
            qweight_packed=self.qweight_packed, scale_factors=self.scale_factors,
            weight_global_scale=self.weight_global_scale, activation_scale=self.activation_scale,
            weight_scale=self.weight_scale, weight_fp8=self.weight_fp8,
            activation_granularity=self.activation_granularity, weight_granularity=self.weight_granularity,
            keep_output_dtype=self.keep_output_dtype,
            **extra,
        )
