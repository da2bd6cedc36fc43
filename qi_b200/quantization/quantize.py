"""Weight quantizers and the packed weight layouts of the B200 backend.

Offline (quantize-checkpoint time) code, torch on any device.  The integer
and FP8 per-tensor quantizers give the same bytes as the reference's
(``src/qi/quantization/quantize.py:32-284``,
``backends/flashrt_fp8_ops.py:38-48``), vectorised over groups instead of a
Python loop.  New here: per-channel FP8, NVFP4, and the packed INT4 layout
the W4A16 kernels read:

* ``qweight_packed`` int32 [N, K/8]: element k = 8w + j in bits 4j..4j+3 of word w
* ``scale_factors`` fp16 [N, G]: group scales (G = ceil(K / group_size))
* ``zeros`` int32 [N, ceil(G/8)]: uint4 zero points packed the same way

NVFP4 (W4A4) layout:

* ``qweight_packed`` uint8 [N, K/2]: two E2M1 codes per byte, element 2j in
  the low nibble
* ``scale_factors`` uint8: E4M3 block-16 scales in the tensor-core
  scale-factor atom layout (512-byte atoms of 128 rows x 4 scales, atoms
  K-fastest; row r0 + 32*r1 at byte r0*16 + r1*4 + j)
* ``weight_global_scale`` fp32 [1]: g_w = max(amax(W), tiny) / (6 * 448)
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Mapping

import torch

FP8_E4M3_MAX = 448.0
FP8_SCALE_FLOOR = 1e-12
NVFP4_BLOCK = 16


@dataclass
class QuantizedLinearWeight:
    qweight: torch.Tensor | None
    scales: torch.Tensor | None
    zeros: torch.Tensor | None
    input_scale: torch.Tensor | None = None
    qweight_packed: torch.Tensor | None = None
    scale_factors: torch.Tensor | None = None
    weight_global_scale: torch.Tensor | None = None
    weight_fp8: torch.Tensor | None = None
    weight_scale: torch.Tensor | None = None
    activation_scale: torch.Tensor | None = None


def effective_group_size(group_size: int, in_features: int) -> int:
    """Non-positive or oversized groups mean one group per row (quantize.py:26-29)."""
    if group_size <= 0 or group_size > in_features:
        return in_features
    return int(group_size)


def _groups(w: torch.Tensor, g: int):
    """Yield (start, end, block) with full groups batched into one [N, n, g] view."""
    N, K = w.shape
    full = K // g
    if full:
        yield 0, full * g, w[:, : full * g].reshape(N, full, g)
    if full * g < K:
        yield full * g, K, w[:, full * g :].reshape(N, 1, K - full * g)


def quantize_weight_rtn(weight: torch.Tensor, bits: int = 8, group_size: int = 128, symmetric: bool = True):
    """Round-to-nearest quantization (reference ``quantize.py:32-78``).

    Returns (qweight int8 [N,K], scales fp32 [N,G], zeros int16 [N,G] | None);
    bit-identical to the reference (same fp32 operations, torch.round = half
    to even)."""
    if weight.dim() != 2:
        raise ValueError(f"Expected a 2D linear weight, got shape {tuple(weight.shape)}.")
    if bits not in (4, 8):
        raise ValueError(f"`bits` must be 4 or 8, got {bits}.")
    N, K = weight.shape
    g = effective_group_size(group_size, K)
    G = math.ceil(K / g)
    w = weight.detach().float()
    qweight = torch.empty((N, K), dtype=torch.int8, device=w.device)
    scales = torch.empty((N, G), dtype=torch.float32, device=w.device)
    zeros = None if symmetric else torch.empty((N, G), dtype=torch.int16, device=w.device)
    for start, end, blk in _groups(w, g):
        g0 = start // g
        ng = blk.shape[1]
        if symmetric:
            qmax = 2 ** (bits - 1) - 1
            s = blk.abs().amax(dim=2).clamp(min=1e-8) / qmax
            q = torch.round(blk / s[..., None]).clamp(-qmax, qmax)
        else:
            qmax = 2**bits - 1
            bmin, bmax = blk.amin(dim=2), blk.amax(dim=2)
            s = ((bmax - bmin) / max(qmax, 1)).clamp(min=1e-8)
            z = torch.round(0 - bmin / s).clamp(0, qmax)
            q = torch.round(blk / s[..., None] + z[..., None]).clamp(0, qmax)
            zeros[:, g0 : g0 + ng] = z.to(torch.int16)
        qweight[:, start:end] = q.reshape(N, end - start).to(torch.int8)
        scales[:, g0 : g0 + ng] = s
    return qweight, scales, zeros


def dequantize_weight(qweight, scales, zeros, bits: int, group_size: int, symmetric: bool = True, dtype=None):
    """w = (q - z) * s in fp32, cast to ``dtype`` (reference ``quantize.py:81-119``)."""
    if qweight.dim() != 2:
        raise ValueError(f"Expected a 2D qweight, got shape {tuple(qweight.shape)}.")
    N, K = qweight.shape
    g = effective_group_size(group_size, K)
    G = math.ceil(K / g)
    if scales.shape != (N, G):
        raise ValueError(f"Expected scales shape {(N, G)}, got {tuple(scales.shape)}.")
    if not symmetric and zeros is None:
        raise ValueError("Asymmetric dequantization requires zeros.")
    s = scales.float().repeat_interleave(g, dim=1)[:, :K]
    q = qweight.float()
    if zeros is not None and not symmetric:
        q = q - zeros.float().repeat_interleave(g, dim=1)[:, :K]
    return (q * s).to(dtype or torch.float16)


# ---------------------------------------------------------------------------
# activation-aware input scales (AWQ / SmoothQuant), reference quantize.py:122-198
# ---------------------------------------------------------------------------


def _resolve_act_stats(act_stats, in_features: int, device) -> torch.Tensor:
    if act_stats is None:
        raise ValueError("Activation-aware quantization requires calibration activation statistics.")
    if isinstance(act_stats, Mapping):
        for key in ("abs_mean", "mean_abs", "abs_max", "amax", "max_abs"):
            if key in act_stats:
                act_stats = act_stats[key]
                break
        else:
            raise ValueError("act_stats mapping must contain one of abs_mean, mean_abs, abs_max, amax, or max_abs.")
    act = torch.as_tensor(act_stats, dtype=torch.float32, device=device).flatten()
    if act.numel() != in_features:
        raise ValueError(f"Expected activation stats with {in_features} values, got {act.numel()}.")
    return act


def _activation_scale_from_stats(act_stats, device, fallback: float = 1.0) -> torch.Tensor:
    """Static FP8 activation scale = global |x| max / 448 (reference quantize.py:140-155)."""
    src = None
    if isinstance(act_stats, Mapping):
        for key in ("global_abs_max", "abs_max", "amax", "max_abs", "abs_mean", "mean_abs"):
            if key in act_stats:
                src = act_stats[key]
                break
    elif act_stats is not None:
        src = act_stats
    scale = float(fallback) if src is None else float(torch.as_tensor(src, dtype=torch.float32).abs().max()) / 448.0
    return torch.tensor([max(scale, FP8_SCALE_FLOOR)], dtype=torch.float32, device=device)


def awq_input_scale(weight: torch.Tensor, act_stats, alpha: float, eps: float) -> torch.Tensor:
    """Per-input-channel smoothing scale s_k = a_k^alpha / w_k^(1-alpha),
    normalised by sqrt(max*min) (reference quantize.py:158-164)."""
    act = _resolve_act_stats(act_stats, weight.shape[1], weight.device).clamp(min=eps)
    wcol = weight.detach().float().abs().amax(dim=0).clamp(min=eps)
    s = act.pow(float(alpha)) / wcol.pow(1.0 - float(alpha))
    s = s / torch.sqrt(s.amax() * s.amin()).clamp(min=eps)
    return s.clamp(min=eps).to(torch.float32)


def quantize_weight_awq(weight, act_stats, bits=4, group_size=128, symmetric=True, alpha=0.5, eps=1e-4):
    input_scale = awq_input_scale(weight, act_stats, alpha, eps)
    q, s, z = quantize_weight_rtn(weight.detach().float() * input_scale[None, :], bits, group_size, symmetric)
    return QuantizedLinearWeight(qweight=q, scales=s, zeros=z, input_scale=input_scale)


def quantize_weight_int8_smoothquant(weight, act_stats, alpha=0.5, eps=1e-4):
    input_scale = awq_input_scale(weight, act_stats, alpha, eps)
    q, s, z = quantize_weight_rtn(weight.detach().float() * input_scale[None, :], 8, -1, True)
    return QuantizedLinearWeight(qweight=q, scales=s, zeros=z, input_scale=input_scale)


# ---------------------------------------------------------------------------
# FP8 E4M3
# ---------------------------------------------------------------------------


def quantize_to_fp8_e4m3(t: torch.Tensor):
    """Per-tensor: s = max(amax/448, 1e-12), q = e4m3(clamp(x/s, +-448))
    (reference flashrt_fp8_ops.py:38-48).  Returns (uint8 codes, fp32 [1])."""
    amax = float(t.detach().float().abs().max()) if t.numel() else 0.0
    scale = max(amax / FP8_E4M3_MAX, FP8_SCALE_FLOOR)
    q = t.detach().float().div(scale).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX)
    return q.to(torch.float8_e4m3fn).view(torch.uint8).contiguous(), torch.tensor(
        [scale], dtype=torch.float32, device=t.device
    )


def quantize_to_fp8_e4m3_rowwise(t: torch.Tensor):
    """Per-row (per output channel): s_n = max(amax_n/448, 1e-12) in fp32,
    q = e4m3(clamp(w/s_n, +-448)).  Returns (uint8 [N,K], fp32 [N])."""
    w = t.detach().float()
    s = (w.abs().amax(dim=1) / FP8_E4M3_MAX).clamp(min=FP8_SCALE_FLOOR)
    q = (w / s[:, None]).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX)
    return q.to(torch.float8_e4m3fn).view(torch.uint8).contiguous(), s.contiguous()


def quantize_weight_fp8_rtn(weight: torch.Tensor, activation_scale: float = 1.0, per_channel: bool = False):
    wq, ws = quantize_to_fp8_e4m3_rowwise(weight) if per_channel else quantize_to_fp8_e4m3(weight.contiguous())
    act = torch.tensor([float(activation_scale)], dtype=torch.float32, device=weight.device).clamp(min=1e-12)
    return QuantizedLinearWeight(qweight=None, scales=None, zeros=None, weight_fp8=wq, weight_scale=ws,
                                 activation_scale=act)


def quantize_weight_fp8_smoothquant(weight, act_stats, alpha=0.5, eps=1e-4, per_channel: bool = False):
    input_scale = awq_input_scale(weight, act_stats, alpha, eps)
    out = quantize_weight_fp8_rtn(weight.detach().float() * input_scale[None, :], 1.0, per_channel)
    out.input_scale = input_scale
    out.activation_scale = _activation_scale_from_stats(act_stats, weight.device)
    return out


# ---------------------------------------------------------------------------
# NVFP4
# ---------------------------------------------------------------------------

_E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _round_e2m1(v: torch.Tensor) -> torch.Tensor:
    """|v| <= 6 -> E2M1 code (sign bit 3), round to nearest, ties to even code."""
    grid = torch.tensor(_E2M1_GRID, dtype=torch.float32, device=v.device)
    a = v.abs()
    hi = torch.searchsorted(grid, a.contiguous(), right=False).clamp(0, 7)
    lo = (hi - 1).clamp(0, 7)
    d_lo = a - grid[lo]
    d_hi = grid[hi] - a
    pick_hi = torch.where(d_hi == d_lo, (hi % 2) == 0, d_hi < d_lo)
    code = torch.where(pick_hi, hi, lo).to(torch.uint8)
    return code | (torch.signbit(v).to(torch.uint8) << 3)


def sf_atom_layout(sf: torch.Tensor) -> torch.Tensor:
    """[R, S] E4M3 block scales -> flat uint8 in the scale-factor atom layout
    (rows padded to 128, scale columns to 4)."""
    R, S = sf.shape
    Rp, Sp = -(-R // 128) * 128, -(-S // 4) * 4
    pad = torch.zeros((Rp, Sp), dtype=torch.uint8, device=sf.device)
    pad[:R, :S] = sf
    t = pad.reshape(Rp // 128, 4, 32, Sp // 4, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().reshape(-1)


def nvfp4_global_scale(amax: torch.Tensor) -> torch.Tensor:
    return (amax.float() / (6.0 * FP8_E4M3_MAX)).clamp(min=1e-12).reshape(1)


def quantize_nvfp4(t: torch.Tensor, global_scale: torch.Tensor | None = None):
    """NVFP4 along K: sf_b = e4m3(amax_b / (6 g)), q = e2m1(clamp(x / (sf_b g), +-6)).

    Returns (packed uint8 [R, K/2], sf uint8 [R, K/16] row-major, g fp32 [1])."""
    x = t.detach().float()
    R, K = x.shape
    if K % NVFP4_BLOCK:
        raise ValueError("NVFP4 needs K % 16 == 0.")
    g = nvfp4_global_scale(x.abs().amax()) if global_scale is None else global_scale.float().reshape(1)
    xb = x.reshape(R, K // NVFP4_BLOCK, NVFP4_BLOCK)
    sf_val = (xb.abs().amax(dim=2) / (6.0 * g)).clamp(max=FP8_E4M3_MAX)
    sf = sf_val.to(torch.float8_e4m3fn)
    denom = sf.float() * g
    v = torch.where(denom[..., None] > 0, xb / denom[..., None], torch.zeros_like(xb)).clamp(-6.0, 6.0)
    nib = _round_e2m1(v).reshape(R, K)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    return packed, sf.view(torch.uint8).contiguous(), g


def quantize_weight_nvfp4(weight: torch.Tensor) -> QuantizedLinearWeight:
    packed, sf, g = quantize_nvfp4(weight)
    return QuantizedLinearWeight(qweight=None, scales=None, zeros=None, qweight_packed=packed,
                                 scale_factors=sf_atom_layout(sf), weight_global_scale=g)


# ---------------------------------------------------------------------------
# packed INT4 (W4A16)
# ---------------------------------------------------------------------------


def pack_int4_rows(q: torch.Tensor) -> torch.Tensor:
    """uint4 values [R, C] (C % 8 == 0) -> int32 [R, C/8]; element 8w+j in bits 4j..4j+3."""
    R, C = q.shape
    if C % 8:
        raise ValueError("pack_int4_rows needs a multiple of 8 columns.")
    v = (q.to(torch.int64) & 0xF).reshape(R, C // 8, 8)
    shifts = torch.arange(0, 32, 4, device=q.device, dtype=torch.int64)
    words = (v << shifts).sum(dim=2)
    return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32).contiguous()


def pack_w4a16(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None):
    """Reference weight-only INT4 tensors (quantize.py:32-78: one int8 per
    value, fp32 scales [N, G], int16 zeros [N, G] or None when symmetric) ->
    (qweight_packed, scale_factors fp16, zeros packed).  Symmetric codes
    q in [-7, 7] are stored as q + 8 with zero point 8, which dequantizes to
    the same (q + 8 - 8) * s."""
    N, K = qweight.shape
    G = scales.shape[1]
    q = qweight.to(torch.int16)
    Gp = -(-G // 8) * 8
    z = torch.zeros((N, Gp), dtype=torch.int32, device=qweight.device)
    if zeros is not None:
        z[:, :G] = zeros.to(torch.int32)
    else:
        q = q + 8
        z[:, :G] = 8
    if int(q.min()) < 0 or int(q.max()) > 15:
        raise ValueError("INT4 codes out of range for the packed layout.")
    qp = pack_int4_rows(q)
    s16 = scales.to(torch.float16).contiguous()
    return qp, s16, pack_int4_rows(z)


def quantize_weight_w4a16(weight: torch.Tensor, group_size: int, symmetric: bool, input_scale=None):
    w = weight.detach().float()
    if input_scale is not None:
        w = w * input_scale[None, :]
    q, s, z = quantize_weight_rtn(w, 4, group_size, symmetric)
    qp, s16, zp = pack_w4a16(q, s, z)
    return QuantizedLinearWeight(qweight=None, scales=None, zeros=zp, qweight_packed=qp, scale_factors=s16,
                                 input_scale=input_scale)


# ---------------------------------------------------------------------------
# dispatcher (reference quantize.py:232-284, plus the B200 formats)
# ---------------------------------------------------------------------------


def quantize_linear_weight(weight: torch.Tensor, cfg, act_stats=None) -> QuantizedLinearWeight:
    if hasattr(cfg, "validate"):
        cfg.validate()
    native = getattr(cfg, "backend", "reference") in ("b200", "cuda_ext")
    qdt = getattr(cfg, "quant_dtype", "int")

    if qdt == "nvfp4":
        return quantize_weight_nvfp4(weight)

    if qdt == "int" and hasattr(cfg, "activation_granularity"):
        if cfg.algo == "rtn":
            q, s, z = quantize_weight_rtn(weight, bits=8, group_size=-1, symmetric=True)
            return QuantizedLinearWeight(qweight=q, scales=s, zeros=z)
        if cfg.algo == "smoothquant":
            return quantize_weight_int8_smoothquant(weight, act_stats, getattr(cfg, "smoothquant_alpha", 0.5),
                                                    getattr(cfg, "smoothquant_scale_eps", 1e-4))
        raise ValueError(f"Unknown INT8 W8A8 quantization algo: {cfg.algo}")

    if qdt == "fp8":
        per_channel = getattr(cfg, "weight_granularity", "per_tensor") == "per_channel"
        if cfg.algo == "rtn":
            return quantize_weight_fp8_rtn(weight, getattr(cfg, "activation_scale", 1.0), per_channel)
        if cfg.algo == "smoothquant":
            return quantize_weight_fp8_smoothquant(weight, act_stats, getattr(cfg, "smoothquant_alpha", 0.5),
                                                   getattr(cfg, "smoothquant_scale_eps", 1e-4), per_channel)
        raise ValueError(f"Unknown W8A8 quantization algo: {cfg.algo}")

    # weight-only
    if native and cfg.bits == 4:
        input_scale = None
        if cfg.algo == "awq":
            input_scale = awq_input_scale(weight, act_stats, getattr(cfg, "awq_alpha", 0.5),
                                          getattr(cfg, "awq_scale_eps", 1e-4))
        elif cfg.algo != "rtn":
            raise ValueError(f"Unknown quantization algo: {cfg.algo}")
        return quantize_weight_w4a16(weight, cfg.group_size, cfg.symmetric, input_scale)
    if cfg.algo == "rtn":
        q, s, z = quantize_weight_rtn(weight, bits=cfg.bits, group_size=cfg.group_size, symmetric=cfg.symmetric)
        return QuantizedLinearWeight(qweight=q, scales=s, zeros=z)
    if cfg.algo == "awq":
        return quantize_weight_awq(weight, act_stats, cfg.bits, cfg.group_size, cfg.symmetric,
                                   getattr(cfg, "awq_alpha", 0.5), getattr(cfg, "awq_scale_eps", 1e-4))
    raise ValueError(f"Unknown quantization algo: {cfg.algo}")
