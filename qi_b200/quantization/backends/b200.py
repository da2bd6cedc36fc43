"""``B200Backend``: the ``QuantBackend.linear`` implementation
(protocol: reference ``src/qi/quantization/backends/reference.py:11-33``)
backed by the sm_100a kernels of ``libqi_b200``.

The format is chosen from the buffers a ``WeightOnlyLinear`` carries:

====================  ==========================================================
format                buffers
====================  ==========================================================
INT8 W8A8             qweight int8 [N,K], scales fp32 [N,1] or [N]; per-token acts
weight-only (W8A16,   qweight int8 [N,K] codes, scales fp32 [N,G], zeros int16
INT4 unpacked)        [N,G] or None: the reference's own layout (``cuda_ext``)
FP8-E4M3 W8A8         weight_fp8 (or qweight_packed uint8) [N,K], weight_scale
                      fp32 [1] or [N]; activation_scale fp32 [1] (static) or
                      activation_granularity="per_token" (dynamic)
W4A16 INT4            qweight_packed int32 [N,K/8], scale_factors fp16 [N,G],
                      zeros int32 [N,ceil(G/8)]
NVFP4 W4A4            qweight_packed uint8 [N,K/2], scale_factors uint8 (atoms),
                      weight_global_scale fp32 [1]
====================  ==========================================================

Error behaviour follows the reference backends: a missing / unusable native
library raises ``B200Unavailable`` (a ``RuntimeError``, like
``Int8W8A8Unavailable`` at ``backends/int8_w8a8_ops.py:15-59``); bad shapes or
buffers raise ``ValueError``.  There is no CPU or PyTorch fallback.
The backend object is stateless, so one instance can be shared by every
layer of a model (``swap.py:133,161`` of the reference shares it).
"""

from __future__ import annotations

import torch

from ... import _lib
from ... import kernels as K


class B200Unavailable(RuntimeError):
    pass


def _hardware_note() -> str:
    if not torch.cuda.is_available():
        return " CUDA is not available."
    major, minor = torch.cuda.get_device_capability()
    return f" Current GPU is {torch.cuda.get_device_name()} sm_{major}{minor}; the kernels need sm_100 (B200)."


def load_b200_ops(required: bool = True):
    try:
        lib = _lib.load()
        if torch.cuda.is_available() and torch.cuda.get_device_capability() != (10, 0):
            raise _lib.QiB200Unavailable("device is not sm_100")
        return lib
    except _lib.QiB200Unavailable as e:
        if required:
            raise B200Unavailable(f"qi_b200 kernels are not available: {e}." + _hardware_note()) from e
        return None


def _output_dtype(x: torch.Tensor, keep_output_dtype: str) -> torch.dtype:
    if keep_output_dtype == "input":
        return x.dtype
    if keep_output_dtype == "fp16":
        return torch.float16
    if keep_output_dtype == "bf16":
        return torch.bfloat16
    if keep_output_dtype == "fp32":
        return torch.float32
    raise ValueError(f"Unsupported keep_output_dtype: {keep_output_dtype}")


def _bias_bf16(bias, n, device):
    if bias is None:
        return None
    if bias.numel() != n:
        raise ValueError(f"Expected bias with {n} values, got {bias.numel()}.")
    b = bias.reshape(-1)
    if b.device != device or b.dtype != torch.bfloat16 or not b.is_contiguous():
        b = b.to(device=device, dtype=torch.bfloat16).contiguous()
    return b


class B200Backend:
    """Quantized linear on B200 tensor cores (tcgen05).

    ``check_errors=True`` reads the device status word after every call and
    raises ``QiB200DeviceError`` if a kernel gave up a bounded wait (its
    output is then incomplete).  That read synchronizes the host with the
    device, so it is off by default; callers that run many layers check once
    per step instead (``qi_b200._lib.raise_on_device_error``, which
    ``DiTStepRunner.check`` and ``bench.py`` call)."""

    def __init__(self, gelu: bool = False, check_errors: bool = False) -> None:
        self._lib = load_b200_ops(required=False)
        self.fuse_gelu = gelu
        self.check_errors = check_errors

    def linear(self, x, qweight, scales, zeros, bias, bits, group_size, symmetric, input_scale,
               keep_output_dtype, qweight_packed=None, scale_factors=None, weight_global_scale=None,
               activation_scale=None, weight_scale=None, weight_fp8=None, activation_granularity=None,
               weight_granularity=None, gelu: bool | None = None) -> torch.Tensor:
        if self._lib is None:
            self._lib = load_b200_ops(required=True)
        if not x.is_cuda:
            raise ValueError("B200 backend requires CUDA tensors.")
        gelu = self.fuse_gelu if gelu is None else gelu
        out_dtype = _output_dtype(x, keep_output_dtype)
        xk = x
        int8_path = (weight_fp8 is None and qweight_packed is None and bits == 8
                     and activation_granularity == "per_token")
        # SmoothQuant / AWQ smoothing (int8_w8a8_ops.py:138-139): on the INT8 path
        # with bf16 input it runs inside the activation quantizer (same bf16 division)
        fuse_smooth = input_scale is not None and int8_path and x.dtype == torch.bfloat16
        if input_scale is not None and not fuse_smooth:
            xk = xk / input_scale.to(device=x.device, dtype=x.dtype)
        k_in = int(xk.shape[-1])
        x2 = xk.reshape(-1, k_in).to(torch.bfloat16).contiguous()

        if weight_fp8 is not None or (qweight_packed is not None and qweight_packed.dtype == torch.uint8
                                      and weight_global_scale is None and scale_factors is None):
            y = self._fp8(x2, weight_fp8 if weight_fp8 is not None else qweight_packed,
                          weight_scale if weight_scale is not None else weight_global_scale,
                          activation_scale, activation_granularity, bias, gelu)
        elif qweight_packed is not None and qweight_packed.dtype == torch.uint8:
            if scale_factors is None or weight_global_scale is None:
                raise ValueError("NVFP4 backend requires scale_factors and weight_global_scale buffers.")
            n = qweight_packed.shape[0]
            y = K.nvfp4_linear(x2, qweight_packed.contiguous(), scale_factors.contiguous(),
                               weight_global_scale.contiguous().float(),
                               None if activation_scale is None else activation_scale.contiguous().float(),
                               _bias_bf16(bias, n, x2.device), per_row=activation_granularity == "per_token",
                               gelu=gelu)
        elif qweight_packed is not None and qweight_packed.dtype == torch.int32:
            y = self._w4a16(x2, qweight_packed, scale_factors, zeros, group_size, bias)
            if gelu:
                raise ValueError("GELU fusion is not available on the W4A16 path.")
        elif bits == 8 and activation_granularity == "per_token":
            y = self._int8(x2, qweight, scales, group_size, symmetric, weight_granularity, bias, gelu,
                           input_scale if fuse_smooth else None)
        elif qweight is not None and qweight.dtype == torch.int8 and bits in (2, 3, 4, 5, 6, 7, 8):
            # weight-only on the reference's own buffers (W8A16, or INT4 one value per byte):
            # ReferenceBackend.linear's dequantise-then-matmul (reference.py:48-91) on the GPU
            if scales is None:
                raise ValueError("weight-only backend requires scales.")
            n = qweight.shape[0]
            y = K.weight_only_linear(x2, qweight.contiguous(), scales, None if symmetric else zeros, int(group_size),
                                     _bias_bf16(bias, n, x2.device))
            if gelu:
                y = torch.nn.functional.gelu(y.float(), approximate="tanh").to(torch.bfloat16)
        else:
            raise ValueError(
                "B200 backend: unsupported buffer combination (bits=%s, activation_granularity=%s, packed=%s)"
                % (bits, activation_granularity, None if qweight_packed is None else qweight_packed.dtype))
        if self.check_errors:
            _lib.raise_on_device_error()
        return y.reshape(*x.shape[:-1], y.shape[-1]).to(out_dtype)

    # -- formats ------------------------------------------------------------

    def _int8(self, x2, qweight, scales, group_size, symmetric, weight_granularity, bias, gelu, input_scale=None):
        if group_size != -1:
            raise ValueError("INT8 W8A8 backend requires per-channel weights with group_size=-1.")
        if not symmetric:
            raise ValueError("INT8 W8A8 backend requires symmetric quantization.")
        if weight_granularity != "per_channel":
            raise ValueError("INT8 W8A8 backend requires per-token activations and per-channel weights.")
        if qweight is None or scales is None:
            raise ValueError("INT8 W8A8 backend requires qweight and per-channel scales.")
        if qweight.dim() != 2 or qweight.shape[1] != x2.shape[1]:
            raise ValueError(f"INT8 W8A8 K mismatch: activation K={x2.shape[1]}, weight {tuple(qweight.shape)}.")
        n = qweight.shape[0]
        ws = scales
        if ws.dim() == 2:
            if ws.shape != (n, 1):
                raise ValueError(f"Expected per-channel scales shape {(n, 1)}, got {tuple(ws.shape)}.")
            ws = ws[:, 0]
        ws = ws.contiguous().float()
        return K.int8_linear(x2, qweight.contiguous(), ws, _bias_bf16(bias, n, x2.device), gelu=gelu,
                             input_scale=input_scale)

    def _w4a16(self, x2, qp, s16, zp, group_size, bias):
        if s16 is None or zp is None:
            raise ValueError("W4A16 backend requires scale_factors (fp16) and packed zeros.")
        if zp.dtype != torch.int32:
            raise ValueError("W4A16 backend requires zeros packed as int32 (8 uint4 per word); "
                             "repack reference tensors with qi_b200.quantization.quantize.pack_w4a16.")
        n = qp.shape[0]
        return K.w4a16_linear(x2, qp.contiguous(), s16.contiguous(), zp.contiguous(), int(group_size),
                              _bias_bf16(bias, n, x2.device))

    def _fp8(self, x2, wq, ws, act_scale, activation_granularity, bias, gelu):
        if wq is None or ws is None:
            raise ValueError("FP8 backend requires weight_fp8 and weight_scale buffers.")
        if wq.dim() != 2 or wq.shape[1] != x2.shape[1]:
            raise ValueError(f"FP8 K mismatch: activation K={x2.shape[1]}, weight {tuple(wq.shape)}.")
        n = wq.shape[0]
        static = None if activation_granularity == "per_token" else act_scale
        if static is None and activation_granularity != "per_token":
            raise ValueError("FP8 backend requires activation_scale (static) or per_token activations.")
        return K.fp8_linear(x2, wq.contiguous(), ws.contiguous().float(),
                            None if static is None else static.contiguous().float(),
                            _bias_bf16(bias, n, x2.device), gelu=gelu)
