"""Torch-tensor front end of the C ABI (``include/qi_b200.h``).

The host-side counterpart of the reference's torch extension glue
(``src/qi/quantization/csrc/int8_w8a8/bindings.cpp:87-165``): it validates
tensors (CUDA, contiguous, dtype, same device — ``TORCH_CHECK``-style
``ValueError`` here), allocates outputs and workspaces with torch's caching
allocator, and launches on torch's current stream.  No host synchronization,
so every function here is safe inside ``torch.cuda.graph`` capture.
"""

from __future__ import annotations

import torch

from . import _lib

_U8 = torch.uint8


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check(t: torch.Tensor, name: str, dtype=None, dim=None, device=None) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor.")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous.")
    if dtype is not None and t.dtype not in (dtype if isinstance(dtype, tuple) else (dtype,)):
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}.")
    if dim is not None and t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D, got shape {tuple(t.shape)}.")
    if device is not None and t.device != device:
        raise ValueError(f"{name} must be on {device}, got {t.device}.")


# ---------------------------------------------------------------------------
# activation quantizers
# ---------------------------------------------------------------------------


def quantize_int8_rowwise(x: torch.Tensor, out: torch.Tensor | None = None,
                          scales: torch.Tensor | None = None):
    """bf16 [M,K] -> (int8 [M,K], fp32 [M]) with the reference K1 semantics."""
    _check(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    q = out if out is not None else torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = scales if scales is not None else torch.empty((M,), dtype=torch.float32, device=x.device)
    _lib.call("qi_b200_quantize_int8_rowwise", _ptr(x), _ptr(q), _ptr(s), M, K, _stream(x.device))
    return q, s


def quantize_fp8_rowwise(x: torch.Tensor):
    """bf16 [M,K] -> (e4m3 codes uint8 [M,K], fp32 [M]) per-token scales."""
    _check(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    q = torch.empty((M, K), dtype=_U8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    _lib.call("qi_b200_quantize_fp8_rowwise", _ptr(x), _ptr(q), _ptr(s), M, K, _stream(x.device))
    return q, s


def quantize_fp8_static(x: torch.Tensor, scale: torch.Tensor):
    """bf16 [M,K] -> e4m3 codes with a calibrated per-tensor scale (device fp32 [1])."""
    _check(x, "x", torch.bfloat16, 2)
    _check(scale, "scale", torch.float32, device=x.device)
    M, K = x.shape
    q = torch.empty((M, K), dtype=_U8, device=x.device)
    _lib.call("qi_b200_quantize_fp8_static", _ptr(x), _ptr(scale), _ptr(q), M, K, _stream(x.device))
    return q


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------


def gemm(kind: int, a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor | None,
         b_scale: torch.Tensor | None, bias: torch.Tensor | None = None, *, gelu: bool = False,
         raw_acc: bool = False, out: torch.Tensor | None = None, tile_n: int = 0) -> torch.Tensor:
    """D = epi(A[M,K] . B[N,K]^T); see ``qi_b200_gemm`` in include/qi_b200.h.

    Scales of one element broadcast (per tensor); otherwise a_scale is [M]
    and b_scale is [N].  ``raw_acc`` returns the 32-bit accumulators (int32
    for INT8, fp32 otherwise) instead of bf16.
    """
    dt = {_lib.KIND_INT8: (torch.int8,), _lib.KIND_FP8_E4M3: (torch.uint8, torch.float8_e4m3fn),
          _lib.KIND_BF16: (torch.bfloat16,)}[kind]
    _check(a, "A", dt, 2)
    _check(b, "B", dt, 2, a.device)
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError(f"K mismatch: A has K={K}, B has K={b.shape[1]}.")

    def scale_arg(s, n, name):
        if s is None:
            return None, 0
        _check(s, name, torch.float32, device=a.device)
        if s.numel() == 1:
            return s, 0
        if s.numel() != n:
            raise ValueError(f"{name} must have 1 or {n} elements, got {s.numel()}.")
        return s, 1

    sa, sa_stride = scale_arg(a_scale, M, "a_scale")
    sb, sb_stride = scale_arg(b_scale, N, "b_scale")
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=a.device)
        if bias.numel() != N:
            raise ValueError(f"bias must have {N} values, got {bias.numel()}.")
    if out is None:
        odt = (torch.int32 if kind == _lib.KIND_INT8 else torch.float32) if raw_acc else torch.bfloat16
        out = torch.empty((M, N), dtype=odt, device=a.device)
    flags = (_lib.EPI_GELU if gelu else 0) | (_lib.EPI_RAW_ACC if raw_acc else 0)
    _lib.call("qi_b200_gemm", kind, _ptr(a), _ptr(b), _ptr(sa), sa_stride, _ptr(sb), sb_stride,
              _ptr(bias), _ptr(out), out.stride(0), M, N, K, flags, tile_n, _stream(a.device))
    return out


# ---------------------------------------------------------------------------
# whole linears
# ---------------------------------------------------------------------------


def int8_linear(x_bf16_2d: torch.Tensor, qweight: torch.Tensor, weight_scales: torch.Tensor,
                bias: torch.Tensor | None = None, gelu: bool = False) -> torch.Tensor:
    """Same contract as the reference torch op
    ``qi_int8_w8a8::linear(Tensor x_bf16_2d, Tensor qweight, Tensor weight_scales, Tensor? bias)``
    (``bindings.cpp:87-165``); ``gelu`` additionally fuses GELU(tanh) into the epilogue."""
    _check(x_bf16_2d, "x_bf16_2d", torch.bfloat16, 2)
    dev = x_bf16_2d.device
    _check(qweight, "qweight", torch.int8, 2, dev)
    _check(weight_scales, "weight_scales", torch.float32, 1, dev)
    M, K = x_bf16_2d.shape
    N = qweight.shape[0]
    if qweight.shape[1] != K:
        raise ValueError("qweight K dimension must match x_bf16_2d.")
    if weight_scales.shape[0] != N:
        raise ValueError("weight_scales length must match qweight N dimension.")
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=dev)
        if bias.numel() != N:
            raise ValueError("bias length must match qweight N dimension.")
    ws_q = torch.empty((M, K), dtype=torch.int8, device=dev)
    ws_s = torch.empty((M,), dtype=torch.float32, device=dev)
    if gelu:
        quantize_int8_rowwise(x_bf16_2d, ws_q, ws_s)
        return gemm(_lib.KIND_INT8, ws_q, qweight, ws_s, weight_scales, bias, gelu=True)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _lib.call("qi_b200_int8_linear", _ptr(x_bf16_2d), _ptr(qweight), _ptr(weight_scales), _ptr(bias),
              _ptr(out), _ptr(ws_q), _ptr(ws_s), M, N, K, _stream(dev))
    return out


def fp8_linear(x_bf16_2d: torch.Tensor, weight_fp8: torch.Tensor, weight_scale: torch.Tensor,
               activation_scale: torch.Tensor | None = None, bias: torch.Tensor | None = None,
               gelu: bool = False) -> torch.Tensor:
    """FP8-E4M3 W8A8 linear.  ``activation_scale`` (fp32 [1]) selects static
    per-tensor activation quantization; ``None`` selects dynamic per-token.
    ``weight_scale`` is fp32 [1] (per tensor) or [N] (per channel)."""
    _check(x_bf16_2d, "x_bf16_2d", torch.bfloat16, 2)
    dev = x_bf16_2d.device
    _check(weight_fp8, "weight_fp8", (torch.uint8, torch.float8_e4m3fn), 2, dev)
    _check(weight_scale, "weight_scale", torch.float32, device=dev)
    M, K = x_bf16_2d.shape
    N = weight_fp8.shape[0]
    if weight_fp8.shape[1] != K:
        raise ValueError(f"FP8 K mismatch: activation K={K}, weight K={weight_fp8.shape[1]}.")
    if weight_scale.numel() not in (1, N):
        raise ValueError(f"weight_scale must have 1 or {N} values.")
    if activation_scale is not None:
        _check(activation_scale, "activation_scale", torch.float32, device=dev)
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=dev)
    ws_q = torch.empty((M, K), dtype=_U8, device=dev)
    ws_s = None if activation_scale is not None else torch.empty((M,), dtype=torch.float32, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _lib.call("qi_b200_fp8_linear", _ptr(x_bf16_2d), _ptr(weight_fp8), _ptr(weight_scale),
              int(weight_scale.numel() == N and N > 1), _ptr(activation_scale), _ptr(bias), _ptr(out),
              _ptr(ws_q), _ptr(ws_s), M, N, K, _lib.EPI_GELU if gelu else 0, _stream(dev))
    return out
