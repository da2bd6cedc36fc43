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
                          scales: torch.Tensor | None = None, input_scale: torch.Tensor | None = None):
    """bf16 [M,K] -> (int8 [M,K], fp32 [M]) with the reference K1 semantics.
    ``input_scale`` (fp32 [K]) first divides x as the reference's SmoothQuant
    path does, in bf16 (``int8_w8a8_ops.py:138-139``), inside the same kernel."""
    _check(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    q = out if out is not None else torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = scales if scales is not None else torch.empty((M,), dtype=torch.float32, device=x.device)
    if input_scale is not None:
        isc = input_scale.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
        if isc.numel() != K:
            raise ValueError(f"input_scale must have {K} values, got {isc.numel()}.")
        _lib.call("qi_b200_quantize_int8_rowwise_smooth", _ptr(x), _ptr(isc), _ptr(q), _ptr(s), M, K,
                  _stream(x.device))
        return q, s
    _lib.call("qi_b200_quantize_int8_rowwise", _ptr(x), _ptr(q), _ptr(s), M, K, _stream(x.device))
    return q, s


def int8_row_scales(x: torch.Tensor) -> torch.Tensor:
    """bf16 [M,K] -> fp32 [M] per-row INT8 scales max(amax/127, 1e-10), no codes."""
    _check(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    _lib.call("qi_b200_int8_row_scales", _ptr(x), _ptr(s), M, K, _stream(x.device))
    return s


def quantize_int8_rowwise_given(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """bf16 [M,K] -> int8 [M,K] with caller-provided per-row scales (fp32 [M])."""
    _check(x, "x", torch.bfloat16, 2)
    _check(scales, "scales", torch.float32, 1, x.device)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    _lib.call("qi_b200_quantize_int8_rowwise_given", _ptr(x), _ptr(scales), _ptr(q), M, K, _stream(x.device))
    return q


def int8_epilogue(acc: torch.Tensor, act_scale: torch.Tensor, weight_scale: torch.Tensor,
                  bias: torch.Tensor | None = None, gelu: bool = False) -> torch.Tensor:
    """int32 [M,N] accumulators -> bf16 with the INT8 GEMM epilogue."""
    _check(acc, "acc", torch.int32, 2)
    M, N = acc.shape
    out = torch.empty((M, N), dtype=torch.bfloat16, device=acc.device)
    _lib.call("qi_b200_int8_epilogue", _ptr(acc), _ptr(act_scale), _ptr(weight_scale), _ptr(bias), _ptr(out),
              M, N, _lib.EPI_GELU if gelu else 0, _stream(acc.device))
    return out


def resid_ln_quant(x: torch.Tensor, y: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                   ln_w: torch.Tensor | None = None, ln_b: torch.Tensor | None = None,
                   mod_scale1: torch.Tensor | None = None, mod_shift: torch.Tensor | None = None,
                   eps: float = 1e-6, quant: bool = True, q: torch.Tensor | None = None,
                   s: torch.Tensor | None = None, xn: torch.Tensor | None = None):
    """Fused residual update / LayerNorm / modulate / INT8 quantization of
    the rows of ``x`` [M, D] bf16 (``x`` is updated in place when ``y`` is
    given).  Returns (q int8 [M, D], s fp32 [M]) or (None, None)."""
    _check(x, "x", torch.bfloat16, 2)
    M, D = x.shape
    dev = x.device
    if y is not None:
        _check(y, "y", torch.bfloat16, 2, dev) if y.is_contiguous() else None
        if y.shape[0] != M or y.stride(1) != 1 or y.shape[1] != D:
            raise ValueError("y must be [M, D] with unit column stride.")
    for t, nm in ((gate, "gate"), (ln_w, "ln_w"), (ln_b, "ln_b"), (mod_scale1, "mod_scale1"),
                  (mod_shift, "mod_shift")):
        if t is not None:
            _check(t, nm, torch.bfloat16, device=dev)
            if t.numel() != D:
                raise ValueError(f"{nm} must have {D} values.")
    if quant:
        q = q if q is not None else torch.empty((M, D), dtype=torch.int8, device=dev)
        s = s if s is not None else torch.empty((M,), dtype=torch.float32, device=dev)
    _lib.call("qi_b200_resid_ln_quant", _ptr(x), _ptr(y), 0 if y is None else y.stride(0), _ptr(gate), _ptr(ln_w),
              _ptr(ln_b), _ptr(mod_scale1), _ptr(mod_shift), _ptr(q) if quant else None,
              _ptr(s) if quant else None, _ptr(xn), M, D, float(eps), _stream(dev))
    return (q, s) if quant else (None, None)


def rms_rope(inputs, weights, rope: torch.Tensor | None, head_dim: int, eps: float = 1e-6, outs=None):
    """RMSNorm (+ RoPE) of one or two [M, A] bf16 row blocks (row stride may
    exceed A, e.g. column slices of a fused QKV output).  Returns the
    normalized contiguous [M, A] tensors."""
    n = len(inputs)
    x0 = inputs[0]
    M, A = x0.shape
    dev = x0.device
    for t in inputs:
        if t.dtype != torch.bfloat16 or t.stride(1) != 1 or t.shape != (M, A) or t.stride(0) != x0.stride(0):
            raise ValueError("rms_rope inputs must be bf16 [M, A] with a shared row stride and unit column stride.")
    for w in weights:
        _check(w, "weight", torch.bfloat16, device=dev)
    if rope is not None:
        _check(rope, "rope", torch.float32, device=dev)
        if rope.numel() != M * head_dim:
            raise ValueError("rope must be [M, head_dim/2, 2] fp32.")
    outs = outs if outs is not None else [torch.empty((M, A), dtype=torch.bfloat16, device=dev) for _ in range(n)]
    _lib.call("qi_b200_rms_rope", _ptr(inputs[0]), _ptr(inputs[-1]), x0.stride(0), _ptr(outs[0]), _ptr(outs[-1]),
              outs[0].stride(0), _ptr(weights[0]), _ptr(weights[-1]), _ptr(rope), int(head_dim), n, M, A,
              float(eps), _stream(dev))
    return outs


def attention_short(q: torch.Tensor, k: torch.Tensor, vt: torch.Tensor, heads: int,
                    scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(Q K^T * scale) V per head for at most 128 keys, head dim 128,
    on the tensor cores (``qi_b200_attention_short``).  ``q`` [Sq, H*128] and
    ``k`` [Sk, H*128] (row strides may exceed H*128), ``vt`` = V transposed,
    [H*128, Sk] (copied into a padded buffer when its row stride is not a
    multiple of 8 elements).  Returns
    [Sq, H*128] bf16 (or writes ``out``).  Default scale 1/sqrt(128), the
    default of torch's scaled_dot_product_attention."""
    for t, name in ((q, "q"), (k, "k"), (vt, "vt")):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or (t.stride(1) != 1 and t.shape[1] > 1) or not t.is_cuda:
            raise ValueError(f"attention_short: {name} must be a 2-D bf16 CUDA tensor with unit column stride.")
    width = heads * 128
    sq, sk = q.shape[0], k.shape[0]
    if q.shape[1] != width or k.shape[1] != width or vt.shape != (width, sk):
        raise ValueError(f"attention_short: q, k must be [S, {width}] and vt [{width}, Sk].")
    if vt.stride(0) % 8:  # TMA rows start on 16-byte boundaries: pad the key dimension
        padded = torch.zeros((width, (sk + 7) // 8 * 8), dtype=torch.bfloat16, device=vt.device)
        padded[:, :sk] = vt
        vt = padded[:, :sk]
    if out is None:
        out = torch.empty((sq, width), dtype=torch.bfloat16, device=q.device)
    elif out.dtype != torch.bfloat16 or out.shape != (sq, width) or out.stride(1) != 1:
        raise ValueError("attention_short: out must be bf16 [Sq, H*128] with unit column stride.")
    _lib.call("qi_b200_attention_short", _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(vt), vt.stride(0),
              _ptr(out), out.stride(0), sq, sk, int(heads), 128,
              float(128 ** -0.5 if scale is None else scale), _stream(q.device))
    return out


def rms_head_partials(inputs, head_dim: int) -> torch.Tensor:
    """Per-head sums of squares of one or two [M, A] bf16 row blocks (a
    rank's contiguous range of whole heads): fp32 [nparts, M, A / head_dim]."""
    x0 = inputs[0]
    M, A = x0.shape
    for t in inputs:
        if t.dtype != torch.bfloat16 or t.stride(1) != 1 or t.shape != (M, A) or t.stride(0) != x0.stride(0):
            raise ValueError("rms_head_partials inputs must be bf16 [M, A] with a shared row stride.")
    out = torch.empty((len(inputs), M, A // head_dim), dtype=torch.float32, device=x0.device)
    _lib.call("qi_b200_rms_head_partials", _ptr(inputs[0]), _ptr(inputs[-1]), x0.stride(0), _ptr(out),
              int(head_dim), len(inputs), M, A, _stream(x0.device))
    return out


def rms_rope_partials(inputs, weights, rope: torch.Tensor | None, head_dim: int, partials: torch.Tensor,
                      eps: float = 1e-6, outs=None):
    """``rms_rope`` of this rank's head columns with the row norm taken from
    every rank's per-head sums (``partials``: fp32 [ranks, nparts, M, heads],
    rank-major); bit-identical to ``rms_rope`` on the unsplit rows."""
    n = len(inputs)
    x0 = inputs[0]
    M, A = x0.shape
    _check(partials, "partials", torch.float32, 4, x0.device)
    if tuple(partials.shape[1:]) != (n, M, A // head_dim):
        raise ValueError(f"partials must be [ranks, {n}, {M}, {A // head_dim}], got {tuple(partials.shape)}.")
    outs = outs if outs is not None else [torch.empty((M, A), dtype=torch.bfloat16, device=x0.device)
                                          for _ in range(n)]
    _lib.call("qi_b200_rms_rope_partials", _ptr(inputs[0]), _ptr(inputs[-1]), x0.stride(0), _ptr(outs[0]),
              _ptr(outs[-1]), outs[0].stride(0), _ptr(weights[0]), _ptr(weights[-1]), _ptr(rope), int(head_dim), n,
              M, A, _ptr(partials), partials.shape[0], float(eps), _stream(x0.device))
    return outs


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


_WS_PLANS: dict = {}


def gemm_workspace_bytes(kind: int, M: int, N: int, K: int, tail_split: int = 0, tile_n: int = 0) -> int:
    """Workspace bytes ``qi_b200_gemm_ws`` needs for the CTA-pair kernel's
    split of its partial last wave (0: the launch for this problem does not
    split).  Host-side plan, cached per shape and device."""
    key = (kind, M, N, K, tail_split, tile_n, torch.cuda.current_device())
    v = _WS_PLANS.get(key)
    if v is None:
        import ctypes
        nb = ctypes.c_size_t(0)
        _lib.call("qi_b200_gemm_workspace_bytes", kind, M, N, K, tail_split << _lib.TAIL_SPLIT_SHIFT, tile_n,
                  ctypes.byref(nb))
        v = _WS_PLANS[key] = int(nb.value)
    return v


def gemm(kind: int, a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor | None,
         b_scale: torch.Tensor | None, bias: torch.Tensor | None = None, *, gelu: bool = False,
         raw_acc: bool = False, out: torch.Tensor | None = None, tile_n: int = 0,
         tail_split: int = 0) -> torch.Tensor:
    """D = epi(A[M,K] . B[N,K]^T); see ``qi_b200_gemm_ws`` in include/qi_b200.h.

    Scales of one element broadcast (per tensor); otherwise a_scale is [M]
    and b_scale is [N].  ``raw_acc`` returns the 32-bit accumulators (int32
    for INT8, fp32 otherwise) instead of bf16.  ``tail_split`` sets how the
    CTA-pair kernel spreads its partial last wave over idle pairs (0 the
    library's choice, 1 no split, S at most S splits per tile); the workspace
    that needs comes from torch's caching allocator (so it also works inside
    CUDA-graph capture).
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
    if not 0 <= tail_split <= 15:
        raise ValueError(f"tail_split must be in [0, 15], got {tail_split}.")
    ws_bytes = gemm_workspace_bytes(kind, M, N, K, tail_split, tile_n)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=a.device) if ws_bytes else None
    flags |= tail_split << _lib.TAIL_SPLIT_SHIFT
    _lib.call("qi_b200_gemm_ws", kind, _ptr(a), _ptr(b), _ptr(sa), sa_stride, _ptr(sb), sb_stride,
              _ptr(bias), _ptr(out), out.stride(0), M, N, K, flags, tile_n, _ptr(ws), ws_bytes, _stream(a.device))
    return out


# ---------------------------------------------------------------------------
# whole linears
# ---------------------------------------------------------------------------


def int8_linear(x_bf16_2d: torch.Tensor, qweight: torch.Tensor, weight_scales: torch.Tensor,
                bias: torch.Tensor | None = None, gelu: bool = False,
                input_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Same contract as the reference torch op
    ``qi_int8_w8a8::linear(Tensor x_bf16_2d, Tensor qweight, Tensor weight_scales, Tensor? bias)``
    (``bindings.cpp:87-165``); ``gelu`` additionally fuses GELU(tanh) into the epilogue, and
    ``input_scale`` the backend's SmoothQuant division into the activation quantizer."""
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
    if gelu or input_scale is not None or gemm_workspace_bytes(_lib.KIND_INT8, M, N, K):
        # the fused SmoothQuant division, the GELU epilogue or the tail split's
        # workspace: the quantizer and the GEMM as two calls
        quantize_int8_rowwise(x_bf16_2d, ws_q, ws_s, input_scale=input_scale)
        return gemm(_lib.KIND_INT8, ws_q, qweight, ws_s, weight_scales, bias, gelu=gelu)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _lib.call("qi_b200_int8_linear", _ptr(x_bf16_2d), _ptr(qweight), _ptr(weight_scales), _ptr(bias),
              _ptr(out), _ptr(ws_q), _ptr(ws_s), M, N, K, _stream(dev))
    return out


def w4a16_linear(x_bf16_2d: torch.Tensor, qweight_packed: torch.Tensor, scales_fp16: torch.Tensor,
                 zeros_packed: torch.Tensor, group_size: int, bias: torch.Tensor | None = None) -> torch.Tensor:
    """INT4 weight-only linear on the packed layout (see include/qi_b200.h,
    ``qi_b200_w4a16_linear``): y = bf16(x . bf16((q - z) s)^T + bias)."""
    _check(x_bf16_2d, "x_bf16_2d", torch.bfloat16, 2)
    dev = x_bf16_2d.device
    _check(qweight_packed, "qweight_packed", torch.int32, 2, dev)
    _check(scales_fp16, "scale_factors", torch.float16, 2, dev)
    _check(zeros_packed, "zeros", torch.int32, 2, dev)
    M, K = x_bf16_2d.shape
    N = qweight_packed.shape[0]
    if qweight_packed.shape[1] * 8 != K:
        raise ValueError(f"W4A16 K mismatch: activation K={K}, packed weight K={qweight_packed.shape[1] * 8}.")
    g = K if group_size <= 0 or group_size > K else group_size
    G = -(-K // g)
    if tuple(scales_fp16.shape) != (N, G) or tuple(zeros_packed.shape) != (N, -(-G // 8)):
        raise ValueError(f"W4A16 scales/zeros must be [{N},{G}] fp16 and [{N},{-(-G // 8)}] int32.")
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=dev)
        if bias.numel() != N:
            raise ValueError(f"bias must have {N} values.")
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    if M >= _lib.W4A16_DEQUANT_MIN_M:  # dequantize once into a workspace, then the bf16 GEMM
        ws = torch.empty((N * K * 2,), dtype=torch.uint8, device=dev)
        _lib.call("qi_b200_w4a16_linear_ws", _ptr(x_bf16_2d), _ptr(qweight_packed), _ptr(scales_fp16),
                  _ptr(zeros_packed), int(g), _ptr(bias), _ptr(out), M, N, K, _ptr(ws), ws.numel(), _stream(dev))
        return out
    _lib.call("qi_b200_w4a16_linear", _ptr(x_bf16_2d), _ptr(qweight_packed), _ptr(scales_fp16),
              _ptr(zeros_packed), int(g), _ptr(bias), _ptr(out), M, N, K, _stream(dev))
    return out


def weight_only_linear(x_bf16_2d: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                       zeros: torch.Tensor | None, group_size: int, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Weight-only linear on the reference's own buffers (``qweight`` int8
    codes [N, K], ``scales`` fp32 [N, G], ``zeros`` int16 [N, G] or None):
    the weights are dequantized exactly as the reference's dequantize_weight
    into a workspace, then multiplied with the bf16 tcgen05 GEMM
    (``qi_b200_wo_linear_ws``)."""
    _check(x_bf16_2d, "x_bf16_2d", torch.bfloat16, 2)
    dev = x_bf16_2d.device
    _check(qweight, "qweight", torch.int8, 2, dev)
    M, K = x_bf16_2d.shape
    N = qweight.shape[0]
    if qweight.shape[1] != K:
        raise ValueError(f"weight-only K mismatch: activation K={K}, weight K={qweight.shape[1]}.")
    g = K if group_size <= 0 or group_size > K else group_size
    G = -(-K // g)
    s = scales.reshape(N, -1).to(device=dev, dtype=torch.float32).contiguous()
    if s.shape[1] != G:
        raise ValueError(f"weight-only scales must be [{N}, {G}], got {tuple(scales.shape)}.")
    z = None
    if zeros is not None:
        z = zeros.reshape(N, -1).to(device=dev, dtype=torch.int16).contiguous()
        if z.shape[1] != G:
            raise ValueError(f"weight-only zeros must be [{N}, {G}], got {tuple(zeros.shape)}.")
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((N * K * 2,), dtype=torch.uint8, device=dev)
    _lib.call("qi_b200_wo_linear_ws", _ptr(x_bf16_2d), _ptr(qweight), _ptr(s), _ptr(z), int(g), _ptr(bias),
              _ptr(out), M, N, K, _ptr(ws), ws.numel(), _stream(dev))
    return out


def wo_dequant(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group_size: int):
    """Reference-layout weight-only codes -> bf16 [N, K] (``qi_b200_wo_dequant``)."""
    N, K = qweight.shape
    G = scales.reshape(N, -1).shape[1]
    out = torch.empty((N, K), dtype=torch.bfloat16, device=qweight.device)
    z = None if zeros is None else zeros.reshape(N, G).to(torch.int16).contiguous()
    _lib.call("qi_b200_wo_dequant", _ptr(qweight), _ptr(scales.reshape(N, G).float().contiguous()), _ptr(z),
              int(group_size), _ptr(out), N, K, _stream(qweight.device))
    return out


def w4a16_dequant(qweight_packed: torch.Tensor, scales_fp16: torch.Tensor, zeros_packed: torch.Tensor,
                  group_size: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed INT4 weights -> bf16 [N, K], exactly bf16((q - z) s) (``qi_b200_w4a16_dequant``)."""
    N = qweight_packed.shape[0]
    K = qweight_packed.shape[1] * 8
    if out is None:
        out = torch.empty((N, K), dtype=torch.bfloat16, device=qweight_packed.device)
    _lib.call("qi_b200_w4a16_dequant", _ptr(qweight_packed), _ptr(scales_fp16), _ptr(zeros_packed),
              int(group_size), _ptr(out), N, K, _stream(qweight_packed.device))
    return out


NVFP4_STATIC, NVFP4_DYNAMIC_TENSOR, NVFP4_DYNAMIC_ROW = 0, 1, 2


def nvfp4_sf_bytes(rows: int, cols: int) -> int:
    """Bytes of the scale-factor atom buffer for a [rows, cols] tensor."""
    return -(-rows // 128) * 128 * (cols // 16)


def quantize_nvfp4(x: torch.Tensor, mode: int = NVFP4_DYNAMIC_TENSOR, global_scale: torch.Tensor | None = None):
    """bf16 [M,K] -> (packed uint8 [M,K/2], scale atoms uint8, g fp32 [1] or [M])."""
    _check(x, "x", torch.bfloat16, 2)
    M, Kd = x.shape
    q = torch.empty((M, Kd // 2), dtype=_U8, device=x.device)
    sf = torch.empty((nvfp4_sf_bytes(M, Kd),), dtype=_U8, device=x.device)
    amax = torch.empty((1,), dtype=torch.int32, device=x.device) if mode == NVFP4_DYNAMIC_TENSOR else None
    if mode == NVFP4_STATIC:
        if global_scale is None:
            raise ValueError("static NVFP4 quantization needs global_scale")
        _check(global_scale, "global_scale", torch.float32, device=x.device)
        g = global_scale
    else:
        g = torch.empty((M if mode == NVFP4_DYNAMIC_ROW else 1,), dtype=torch.float32, device=x.device)
    _lib.call("qi_b200_quantize_nvfp4", _ptr(x), M, Kd, mode, _ptr(global_scale), _ptr(amax),
              None if mode == NVFP4_STATIC else _ptr(g), _ptr(q), _ptr(sf), _stream(x.device))
    return q, sf, g


def nvfp4_gemm(a_packed, a_sf, b_packed, b_sf, a_g, b_g, bias=None, out=None, raw_acc=False, tile: int = 0):
    """NVFP4 GEMM on packed operands and scale atoms.  ``tile``: 0 the
    library's choice, 1 single-CTA 128x128, 2 CTA pair 256x128, 3 CTA pair 256x256."""
    M, Kh = a_packed.shape
    N = b_packed.shape[0]
    if b_packed.shape[1] != Kh:
        raise ValueError("NVFP4 K mismatch")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32 if raw_acc else torch.bfloat16, device=a_packed.device)
    _lib.call("qi_b200_nvfp4_gemm", _ptr(a_packed), _ptr(a_sf), _ptr(b_packed), _ptr(b_sf), _ptr(a_g),
              int(a_g.numel() > 1), _ptr(b_g), _ptr(bias), _ptr(out), out.stride(0), M, N, 2 * Kh,
              (_lib.EPI_RAW_ACC if raw_acc else 0) | (tile << _lib.NVFP4_TILE_SHIFT), _stream(a_packed.device))
    return out


def nvfp4_linear(x_bf16_2d: torch.Tensor, weight_packed: torch.Tensor, weight_sf: torch.Tensor,
                 weight_global_scale: torch.Tensor, act_global_scale: torch.Tensor | None = None,
                 bias: torch.Tensor | None = None, per_row: bool = False, gelu: bool = False) -> torch.Tensor:
    """NVFP4 W4A4 linear.  ``act_global_scale`` (fp32 [1]) selects static
    activation quantization; otherwise dynamic per tensor (or per row)."""
    _check(x_bf16_2d, "x_bf16_2d", torch.bfloat16, 2)
    dev = x_bf16_2d.device
    _check(weight_packed, "qweight_packed", torch.uint8, 2, dev)
    _check(weight_sf, "scale_factors", torch.uint8, None, dev)
    _check(weight_global_scale, "weight_global_scale", torch.float32, None, dev)
    M, Kd = x_bf16_2d.shape
    N = weight_packed.shape[0]
    if weight_packed.shape[1] * 2 != Kd:
        raise ValueError(f"NVFP4 K mismatch: activation K={Kd}, weight K={weight_packed.shape[1] * 2}.")
    if weight_sf.numel() != nvfp4_sf_bytes(N, Kd):
        raise ValueError(f"NVFP4 weight scale atoms must have {nvfp4_sf_bytes(N, Kd)} bytes.")
    mode = NVFP4_STATIC if act_global_scale is not None else (NVFP4_DYNAMIC_ROW if per_row else NVFP4_DYNAMIC_TENSOR)
    if bias is not None:
        _check(bias, "bias", torch.bfloat16, device=dev)
    ws_q = torch.empty((M, Kd // 2), dtype=_U8, device=dev)
    ws_sf = torch.empty((nvfp4_sf_bytes(M, Kd),), dtype=_U8, device=dev)
    ws_g = torch.empty((M if per_row else 1,), dtype=torch.float32, device=dev)
    ws_amax = torch.empty((1,), dtype=torch.int32, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _lib.call("qi_b200_nvfp4_linear", _ptr(x_bf16_2d), _ptr(weight_packed), _ptr(weight_sf),
              _ptr(weight_global_scale), mode, _ptr(act_global_scale), _ptr(bias), _ptr(out), _ptr(ws_q),
              _ptr(ws_sf), _ptr(ws_g), _ptr(ws_amax), M, N, Kd, _lib.EPI_GELU if gelu else 0, _stream(dev))
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
