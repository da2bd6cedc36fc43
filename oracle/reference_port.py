"""CPU port of the reference's own PyTorch path for a quantized linear
(TEST / BASELINE INFRASTRUCTURE ONLY: used by tests and by ``bench.py``'s
``cpu_baseline`` leg and ``--impl reference`` arm, never by the product).

The reference's dequantise-then-matmul backend cannot travel to the GPU box,
so its algorithm is restated here step for step with the same torch CPU
operations:

* ``ReferenceBackend.linear``  — ``src/qi/quantization/backends/reference.py:48-91``
  (compute dtype, ``x / input_scale``, per-token fake quantization in the
  compute dtype, ``dequantize_weight``, ``F.linear``);
* ``dequantize_weight``        — ``src/qi/quantization/quantize.py:81-119``
  (a Python loop over K-groups building the fp32 ``(q - z) * s`` block and
  casting it to the compute dtype on every call).

For formats the reference has no CPU kernel for (per-token FP8, NVFP4) the
same shape of computation is used: dequantise the stored weight to the
compute dtype, fake-quantise the activation the way the kernel quantizes it,
``F.linear``, then the fused epilogue (GELU) in torch.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _dequantize_loop(qweight, scales, zeros, group_size, symmetric, dtype):
    """Group loop of quantize.py:107-117."""
    N, K = qweight.shape
    g = K if (group_size <= 0 or group_size > K) else group_size
    G = math.ceil(K / g)
    w = torch.empty((N, K), dtype=dtype)
    qf = qweight.float()
    for gi in range(G):
        s, e = gi * g, min((gi + 1) * g, K)
        sc = scales[:, gi].float()[:, None]
        blk = qf[:, s:e] * sc if symmetric else (qf[:, s:e] - zeros[:, gi].float()[:, None]) * sc
        w[:, s:e] = blk.to(dtype)
    return w


def reference_linear(x, qweight, scales, zeros, bias, bits, group_size, symmetric,
                     input_scale=None, activation_granularity=None):
    """``ReferenceBackend.linear`` (reference.py:48-91), output dtype = input dtype."""
    out_dtype = x.dtype
    cdt = torch.float32 if x.dtype == torch.float32 else out_dtype
    xc = x.to(cdt)
    if input_scale is not None:
        xc = xc / input_scale.to(cdt)
    if activation_granularity == "per_token":
        qmax = 2 ** (bits - 1) - 1
        ts = xc.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8) / qmax
        xc = torch.round(xc / ts).clamp(-qmax, qmax) * ts
    w = _dequantize_loop(qweight, scales, zeros, group_size, symmetric, cdt)
    b = None if bias is None else bias.to(cdt)
    return F.linear(xc, w, b).to(out_dtype)


def fp8_linear_port(x_bf16, weight_fp8_u8, weight_scale, bias=None, gelu=False):
    """Per-token FP8 W8A8 linear in the reference's style (dequantise, fake
    quantise, ``F.linear``), fp32 compute, bf16 out."""
    xf = x_bf16.float()
    s = (xf.abs().amax(dim=1, keepdim=True) / 448.0).clamp(min=1e-12)
    xq = (xf / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s
    w = weight_fp8_u8.view(torch.float8_e4m3fn).float() * weight_scale.float().reshape(-1, 1)
    y = F.linear(xq, w, None if bias is None else bias.float()).to(torch.bfloat16)
    if gelu:
        y = F.gelu(y.float(), approximate="tanh").to(torch.bfloat16)
    return y


_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _nvfp4_dequant(packed_u8, sf_u8_rowmajor, g):
    """[R, K/2] packed E2M1 + [R, K/16] E4M3 scales + fp32 g -> fp32 [R, K]."""
    lo = _E2M1[(packed_u8 & 0xF).long()]
    hi = _E2M1[(packed_u8 >> 4).long()]
    v = torch.stack([lo, hi], dim=-1).reshape(packed_u8.shape[0], -1)
    s = sf_u8_rowmajor.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return v * s * g.float()


def nvfp4_linear_port(x_bf16, w_packed, w_sf_rowmajor, w_g, bias=None):
    """NVFP4 W4A4 linear in the reference's style: fake-quantise the
    activation (per-tensor global scale), dequantise the weight, ``F.linear``
    in fp32, bf16 out."""
    from qi_b200.quantization.quantize import quantize_nvfp4

    xp, xsf, xg = quantize_nvfp4(x_bf16.float())
    xq = _nvfp4_dequant(xp, xsf, xg)
    w = _nvfp4_dequant(w_packed, w_sf_rowmajor, w_g)
    return F.linear(xq, w, None if bias is None else bias.float()).to(torch.bfloat16)
