"""CPU oracle for the quantized-linear hot path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the arithmetic of hongzicong/qi's quantized
``nn.Linear`` path so that the CUDA kernels of ``qi_b200`` can be checked
against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` may use it; the product path never does.

Pinning: every function that has a counterpart in the reference is checked
against golden vectors produced by running the reference's own Python code
(``tests/golden/make_golden.py``; fixtures in ``tests/golden/``):

* ``quantize_weight_rtn``          <-> ``src/qi/quantization/quantize.py:32-78``   (bit-exact)
* ``dequantize_weight``            <-> ``src/qi/quantization/quantize.py:81-119``  (bit-exact)
* ``quantize_fp8_per_tensor``      <-> ``src/qi/quantization/backends/flashrt_fp8_ops.py:38-48`` (bit-exact)
* ``reference_linear`` (numpy)     <-> ``src/qi/quantization/backends/reference.py:48-91`` (tolerance)

Restatements of CUDA code that cannot run here (no GPU in the build
container):

* ``quantize_int8_rowwise``   <-> ``csrc/int8_w8a8/quantize_int8.cu:7-59`` (K1)
* ``int8_gemm_acc`` + ``int8_epilogue`` <-> ``csrc/int8_w8a8/cutlass_int8_rowwise.cu:43-71`` (K2)

Formats the reference does not implement (parity unpinned; restated from
their published definitions): per-token FP8-E4M3 (generalising
``flashrt_fp8_ops.py:38-48`` to one scale per row), NVFP4 (E2M1 values with
an E4M3 scale per 16 elements and an fp32 per-tensor scale) and the packed
INT4 layout (8 nibbles per int32, fp16 scales, packed uint4 zeros).

Number formats: bf16 tensors are carried as ``uint16`` bit patterns, fp8 and
packed fp4 as ``uint8`` codes, so comparisons against the GPU are bitwise.
All float arithmetic that the kernels do in fp32 is done here in numpy
float32 (one IEEE rounding per operation, as on the GPU).
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# bf16 / fp16 helpers
# ---------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bits, round to nearest even (NaN -> 0x7FC0)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    r = np.where(np.isnan(x), np.uint16(0x7FC0), r)
    return r.astype(np.uint16)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """float32 -> float16 with IEEE round to nearest even (numpy's cast)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16)


# ---------------------------------------------------------------------------
# minifloat formats (table-driven RNE so the rule is visible)
# ---------------------------------------------------------------------------


def _e4m3_table() -> np.ndarray:
    """Values of the positive E4M3 ("fn": no inf, 0x7F is NaN) codes 0x00..0x7E."""
    vals = []
    for code in range(0x7F):
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0:
            vals.append(m / 8.0 * 2.0 ** (-6))
        else:
            vals.append((1.0 + m / 8.0) * 2.0 ** (e - 7))
    return np.asarray(vals, dtype=np.float64)


def _e2m1_table() -> np.ndarray:
    """Values of the positive E2M1 codes 0..7: 0, .5, 1, 1.5, 2, 3, 4, 6."""
    return np.asarray([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


E4M3_VALUES = _e4m3_table()
E2M1_VALUES = _e2m1_table()
E4M3_MAX = 448.0
E2M1_MAX = 6.0


def _round_to_table(x: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Round |x| to the nearest entry of the ascending ``table`` (ties to the
    even code, i.e. the entry whose code has LSB 0); returns codes (no sign).
    Inputs must already be clamped to the table's range."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    hi = np.searchsorted(table, a, side="left")
    hi = np.clip(hi, 0, len(table) - 1)
    lo = np.clip(hi - 1, 0, len(table) - 1)
    d_lo = a - table[lo]
    d_hi = table[hi] - a
    pick_hi = d_hi < d_lo
    tie = d_hi == d_lo
    pick_hi = np.where(tie, (hi % 2) == 0, pick_hi)
    code = np.where(pick_hi, hi, lo)
    # exact hits
    code = np.where(table[hi] == a, hi, code)
    return code.astype(np.uint8)


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """float32 (|x| <= 448, finite) -> E4M3 code, RNE (matches torch's
    ``.to(torch.float8_e4m3fn)`` and PTX ``cvt.rn.satfinite.e4m3x2.f32``)."""
    x = np.asarray(x, dtype=np.float32)
    code = _round_to_table(x, E4M3_VALUES)
    # the sign bit is kept even when the magnitude rounds to zero (as torch
    # and the PTX conversion do)
    sign = np.where(np.signbit(x), np.uint8(0x80), np.uint8(0))
    return (code | sign).astype(np.uint8)


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    mag = E4M3_VALUES[np.minimum(c & 0x7F, 0x7E)].astype(np.float32)
    return np.where(c & 0x80, -mag, mag).astype(np.float32)


def f32_to_e2m1(x: np.ndarray) -> np.ndarray:
    """float32 (|x| <= 6) -> E2M1 nibble (sign in bit 3), RNE."""
    x = np.asarray(x, dtype=np.float32)
    code = _round_to_table(x, E2M1_VALUES)
    sign = np.where(np.signbit(x), np.uint8(0x8), np.uint8(0))
    return (code | sign).astype(np.uint8)


def e2m1_to_f32(nib: np.ndarray) -> np.ndarray:
    n = np.asarray(nib, dtype=np.uint8)
    mag = E2M1_VALUES[n & 0x7].astype(np.float32)
    return np.where(n & 0x8, -mag, mag).astype(np.float32)


# ---------------------------------------------------------------------------
# weight quantization (reference quantize.py)
# ---------------------------------------------------------------------------


def effective_group_size(group_size: int, in_features: int) -> int:
    """``quantize.py:26-29``: non-positive or oversized groups mean one group."""
    if group_size <= 0 or group_size > in_features:
        return in_features
    return int(group_size)


def quantize_weight_rtn(w: np.ndarray, bits: int, group_size: int, symmetric: bool):
    """Round-to-nearest weight quantization, ``quantize.py:32-78``.

    Returns (qweight int8 [N,K], scales float32 [N,G], zeros int16 [N,G] or None).
    Symmetric: s = max(amax, 1e-8) / (2^(b-1)-1), q = clamp(rint(w/s), +-qmax).
    Asymmetric: s = max((max-min)/(2^b-1), 1e-8), z = clamp(rint(-min/s), 0, 2^b-1),
    q = clamp(rint(w/s + z), 0, 2^b-1).  All arithmetic in float32.
    """
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    g = effective_group_size(group_size, K)
    G = math.ceil(K / g)
    q = np.empty((N, K), dtype=np.int8)
    scales = np.empty((N, G), dtype=np.float32)
    zeros = None if symmetric else np.empty((N, G), dtype=np.int16)
    for gi in range(G):
        blk = w[:, gi * g : min((gi + 1) * g, K)]
        if symmetric:
            qmax = 2 ** (bits - 1) - 1
            s = np.maximum(np.abs(blk).max(axis=1), F32(1e-8)) / F32(qmax)
            qq = np.clip(np.rint(blk / s[:, None]), -qmax, qmax)
        else:
            qmax = 2**bits - 1
            bmin = blk.min(axis=1)
            bmax = blk.max(axis=1)
            s = np.maximum((bmax - bmin) / F32(qmax), F32(1e-8))
            z = np.clip(np.rint(F32(0) - bmin / s), 0, qmax).astype(np.float32)
            qq = np.clip(np.rint(blk / s[:, None] + z[:, None]), 0, qmax)
            zeros[:, gi] = z.astype(np.int16)
        q[:, gi * g : min((gi + 1) * g, K)] = qq.astype(np.int8)
        scales[:, gi] = s.astype(np.float32)
    return q, scales, zeros


def dequantize_weight(q, scales, zeros, group_size: int, out: str = "bf16"):
    """``quantize.py:81-119``: w = (q - z) * s in float32, then cast.

    ``out`` = "bf16" returns uint16 bf16 bits, "f32" returns float32.
    """
    q = np.asarray(q)
    N, K = q.shape
    g = effective_group_size(group_size, K)
    G = math.ceil(K / g)
    s_full = np.repeat(np.asarray(scales, np.float32), g, axis=1)[:, :K]
    qf = q.astype(np.float32)
    if zeros is not None:
        z_full = np.repeat(np.asarray(zeros).astype(np.float32), g, axis=1)[:, :K]
        w = (qf - z_full) * s_full
    else:
        w = qf * s_full
    assert scales.shape == (N, G)
    return f32_to_bf16(w) if out == "bf16" else w.astype(np.float32)


# ---------------------------------------------------------------------------
# INT8 W8A8 (reference native K1 + K2)
# ---------------------------------------------------------------------------


def quantize_int8_rowwise(x_bf16: np.ndarray):
    """Per-token activation quantizer, ``quantize_int8.cu:7-59``.

    s = max(amax/127, 1e-10); q = clamp(rint(x * (1/s)), -127, 127), with a
    correctly rounded reciprocal (the reference build's ``--use_fast_math``
    approximate reciprocal is a build artefact; the kernels here are IEEE).
    Returns (q int8 [M,K], s float32 [M]).
    """
    s = int8_row_scales(x_bf16)
    return quantize_int8_rowwise_given(x_bf16, s), s


def int8_row_scales(x_bf16: np.ndarray) -> np.ndarray:
    """The scale half of ``quantize_int8.cu:7-59``: s = max(amax/127, 1e-10)."""
    x = bf16_to_f32(x_bf16)
    amax = np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32)
    return np.maximum(amax / F32(127.0), F32(1e-10)).astype(np.float32)


def quantize_int8_rowwise_given(x_bf16: np.ndarray, s: np.ndarray) -> np.ndarray:
    """The code half of ``quantize_int8.cu:7-59`` with given per-row scales:
    q = clamp(rint(x * (1/s)), -127, 127)."""
    x = bf16_to_f32(x_bf16)
    inv = (F32(1.0) / np.asarray(s, np.float32)).astype(np.float32)
    v = x * inv[:, None]
    return np.clip(np.rint(v), -127, 127).astype(np.int8)


def int8_gemm_acc(qa: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators sum_k qa[m,k]*qw[n,k] (float64 BLAS of
    integer values is exact below 2^53)."""
    acc = qa.astype(np.float64) @ qw.astype(np.float64).T
    return acc.astype(np.int64)


def int8_epilogue(acc: np.ndarray, sa: np.ndarray, sw: np.ndarray, bias_bf16=None) -> np.ndarray:
    """``cutlass_int8_rowwise.cu:43-71``: bf16(((float)acc * s_tok) * s_ch + bias),
    every step an fp32 round-to-nearest."""
    y = acc.astype(np.float32) * np.asarray(sa, np.float32)[:, None]
    y = y * np.asarray(sw, np.float32)[None, :]
    if bias_bf16 is not None:
        y = y + bf16_to_f32(bias_bf16)[None, :]
    return f32_to_bf16(y)


def int8_linear(x_bf16, qweight, wscale, bias_bf16=None):
    """Whole INT8 W8A8 linear as the native reference path computes it
    (``bindings.cpp:87-157``): K1 then K2.  Returns (y_bf16, acc, qa, sa)."""
    qa, sa = quantize_int8_rowwise(x_bf16)
    acc = int8_gemm_acc(qa, qweight)
    return int8_epilogue(acc, sa, wscale, bias_bf16), acc, qa, sa


# ---------------------------------------------------------------------------
# FP8 E4M3
# ---------------------------------------------------------------------------


def quantize_fp8_per_tensor(x_f32: np.ndarray):
    """``flashrt_fp8_ops.py:38-48``: s = max(amax/448, 1e-12);
    q = e4m3(clamp(x/s, +-448)).  Returns (codes uint8, s float32[1])."""
    x = np.asarray(x_f32, dtype=np.float32)
    amax = F32(np.abs(x).max()) if x.size else F32(0)
    s = np.maximum(F32(amax) / F32(448.0), F32(1e-12)).astype(np.float32)
    v = np.clip(x / s, -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return f32_to_e4m3(v), np.asarray([s], np.float32)


def quantize_fp8_rowwise(x_f32: np.ndarray):
    """Per-row generalisation of ``flashrt_fp8_ops.py:38-48`` (one scale per
    token / per output channel).  Returns (codes uint8 [R,C], s float32 [R])."""
    x = np.asarray(x_f32, dtype=np.float32)
    amax = np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32)
    s = np.maximum(amax / F32(448.0), F32(1e-12)).astype(np.float32)
    v = np.clip(x / s[:, None], -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return f32_to_e4m3(v), s


def quantize_fp8_static(x_f32: np.ndarray, scale: float):
    """Static per-tensor activation quantization with a calibrated scale
    (``flashrt_fp8_ops.py:207-216`` passes ``activation_scale``)."""
    x = np.asarray(x_f32, dtype=np.float32)
    v = np.clip(x / F32(scale), -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return f32_to_e4m3(v)


def gelu_tanh(y: np.ndarray) -> np.ndarray:
    """GELU, tanh form (``wan_video_dit.py:244-245``, ``nn.GELU(approximate='tanh')``),
    evaluated in float64 and rounded to float32."""
    y64 = np.asarray(y, np.float64)
    k = math.sqrt(2.0 / math.pi)
    return (0.5 * y64 * (1.0 + np.tanh(k * (y64 + 0.044715 * y64**3)))).astype(np.float32)


def fp8_linear(qa, sa, qw, sw, bias_bf16=None, gelu=False):
    """y = bf16(acc * s_a[m] * s_w[n] + bias); optional GELU applied to the
    bf16-rounded linear output, rounded to bf16 again (the unfused
    Linear -> GELU order of the model)."""
    acc = e4m3_to_f32(qa).astype(np.float64) @ e4m3_to_f32(qw).astype(np.float64).T
    y = acc.astype(np.float32) * np.asarray(sa, np.float32).reshape(-1, 1)
    y = y * np.asarray(sw, np.float32).reshape(1, -1)
    if bias_bf16 is not None:
        y = y + bf16_to_f32(bias_bf16)[None, :]
    yb = f32_to_bf16(y)
    if gelu:
        yb = f32_to_bf16(gelu_tanh(bf16_to_f32(yb)))
    return yb


# ---------------------------------------------------------------------------
# NVFP4 (E2M1 + E4M3 block-16 scales + fp32 tensor scale)
# ---------------------------------------------------------------------------

NVFP4_BLOCK = 16


def nvfp4_global_scale(amax: float) -> np.float32:
    """Per-tensor decode scale g = amax / (6 * 448) (fp32), floored so an
    all-zero tensor gives finite scales."""
    return np.maximum(F32(amax) / F32(6.0 * 448.0), F32(1e-12)).astype(np.float32)


def quantize_nvfp4(x_f32: np.ndarray, g: np.float32):
    """NVFP4 quantization of rows along K (K % 16 == 0).

    Block scale  sf = e4m3( amax_b / (6 * g) )  (|.| <= 448 by construction),
    element      q  = e2m1( clamp(x / (f32(sf) * g), +-6) ), sf == 0 -> q = 0.
    Returns (nibbles uint8 [R, K] one per element, sf codes uint8 [R, K/16]).
    """
    x = np.asarray(x_f32, dtype=np.float32)
    R, K = x.shape
    assert K % NVFP4_BLOCK == 0
    xb = x.reshape(R, K // NVFP4_BLOCK, NVFP4_BLOCK)
    amax_b = np.abs(xb).max(axis=2)
    sf_val = np.minimum(amax_b / (F32(6.0) * g), F32(E4M3_MAX)).astype(np.float32)
    sf = f32_to_e4m3(sf_val)
    denom = (e4m3_to_f32(sf) * g).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where(denom[:, :, None] > 0, xb / denom[:, :, None], F32(0)).astype(np.float32)
    v = np.clip(v, -E2M1_MAX, E2M1_MAX)
    q = f32_to_e2m1(v).reshape(R, K)
    return q, sf


def pack_fp4(nib: np.ndarray) -> np.ndarray:
    """Two E2M1 nibbles per byte along K: element 2j in the low nibble."""
    n = np.asarray(nib, np.uint8)
    return (n[:, 0::2] | (n[:, 1::2] << 4)).astype(np.uint8)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), np.uint8)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = p >> 4
    return out


def nvfp4_dequant(nib, sf, g) -> np.ndarray:
    """x_hat = e2m1(q) * e4m3(sf) * g in float64 (exact products)."""
    v = e2m1_to_f32(nib).astype(np.float64)
    s = e4m3_to_f32(sf).astype(np.float64)
    R, K = v.shape
    v = v.reshape(R, K // NVFP4_BLOCK, NVFP4_BLOCK) * s[:, :, None]
    return v.reshape(R, K) * float(g)


def nvfp4_linear(qa_nib, sfa, ga, qw_nib, sfw, gw, bias_bf16=None):
    """y = bf16( (acc * g_a) * g_w + bias ), acc = sum_blocks (sum q_a q_w) sf_a sf_w
    (exact in float64, rounded to fp32); g_a is one scale per tensor or per
    row, g_w per tensor; the epilogue multiplies in fp32 in that order."""
    a = nvfp4_dequant(qa_nib, sfa, 1.0)
    w = nvfp4_dequant(qw_nib, sfw, 1.0)
    acc = (a @ w.T).astype(np.float32)
    ga = np.asarray(ga, np.float32).reshape(-1, 1)
    y = (acc * ga) * np.asarray(gw, np.float32).reshape(1, -1)
    if bias_bf16 is not None:
        y = y + bf16_to_f32(bias_bf16)[None, :]
    return f32_to_bf16(y)


SF_ATOM_ROWS = 128
SF_ATOM_COLS = 4


def sf_to_atom_layout(sf: np.ndarray) -> np.ndarray:
    """Reorder a [R, K/16] block-scale matrix into the tensor-core scale-factor
    layout the NVFP4 kernels consume: 512-byte atoms covering 128 rows x 4
    scales, atoms ordered K-fastest then rows; inside an atom, row r = r0 +
    32*r1 sits at byte r0*16 + r1*4 + j (j = scale index).  Rows and scale
    columns are zero-padded to multiples of 128 and 4."""
    sf = np.asarray(sf, np.uint8)
    R, S = sf.shape
    Rp = -(-R // SF_ATOM_ROWS) * SF_ATOM_ROWS
    Sp = -(-S // SF_ATOM_COLS) * SF_ATOM_COLS
    pad = np.zeros((Rp, Sp), np.uint8)
    pad[:R, :S] = sf
    # [Rp/128, 128, Sp/4, 4] with row = ra*128 + r1*32 + r0
    t = pad.reshape(Rp // 128, 4, 32, Sp // 4, 4)  # ra, r1, r0, ka, j
    t = t.transpose(0, 3, 2, 1, 4)  # ra, ka, r0, r1, j
    return np.ascontiguousarray(t).reshape(-1)


def sf_from_atom_layout(flat: np.ndarray, R: int, S: int) -> np.ndarray:
    Rp = -(-R // SF_ATOM_ROWS) * SF_ATOM_ROWS
    Sp = -(-S // SF_ATOM_COLS) * SF_ATOM_COLS
    t = np.asarray(flat, np.uint8).reshape(Rp // 128, Sp // 4, 32, 4, 4)  # ra, ka, r0, r1, j
    t = t.transpose(0, 3, 2, 1, 4).reshape(Rp, Sp)
    return np.ascontiguousarray(t[:R, :S])


# ---------------------------------------------------------------------------
# INT4 W4A16 packed layout
# ---------------------------------------------------------------------------


def pack_int4_rows(q: np.ndarray) -> np.ndarray:
    """uint4 values [R, C] (C % 8 == 0) -> int32 [R, C/8]; element 8w+j in
    bits 4j..4j+3 of word w."""
    q = np.asarray(q).astype(np.uint32) & 0xF
    R, C = q.shape
    assert C % 8 == 0
    q = q.reshape(R, C // 8, 8)
    words = np.zeros((R, C // 8), np.uint32)
    for j in range(8):
        words |= q[:, :, j] << (4 * j)
    return words.view(np.int32)


def unpack_int4_rows(words: np.ndarray, C: int) -> np.ndarray:
    w = np.asarray(words).view(np.uint32)
    R = w.shape[0]
    out = np.empty((R, w.shape[1] * 8), np.uint8)
    for j in range(8):
        out[:, j::8] = (w >> (4 * j)) & 0xF
    return out[:, :C]


def pack_w4a16(qweight, scales, zeros):
    """Reference weight-only INT4 tensors (``quantize.py:32-78``: int8 values
    0..15, fp32 scales [N,G], int16 zeros [N,G]) -> packed layout
    (qweight_packed int32 [N,K/8], scales fp16 [N,G], zeros int32 [N,ceil(G/8)])."""
    N, K = qweight.shape
    G = scales.shape[1]
    qp = pack_int4_rows(np.asarray(qweight).astype(np.uint8))
    s16 = f32_to_f16(scales)
    Gp = -(-G // 8) * 8
    zpad = np.zeros((N, Gp), np.uint8)
    zpad[:, :G] = np.asarray(zeros).astype(np.uint8)
    zp = pack_int4_rows(zpad)
    return qp, s16, zp


def w4a16_dequant_bf16(qp, s16, zp, K: int, group_size: int) -> np.ndarray:
    """W_bf16 = bf16( f32(q - z) * f32(s16) ) -- the reference dequant
    (``quantize.py:110-117``) applied to the packed tensors."""
    q = unpack_int4_rows(qp, K).astype(np.float32)
    G = s16.shape[1]
    z = unpack_int4_rows(zp, G).astype(np.float32)
    g = effective_group_size(group_size, K)
    s_full = np.repeat(s16.astype(np.float32), g, axis=1)[:, :K]
    z_full = np.repeat(z, g, axis=1)[:, :K]
    return f32_to_bf16((q - z_full) * s_full)


def w4a16_linear(x_bf16, qp, s16, zp, group_size: int, bias_bf16=None):
    """y = bf16( x_bf16 @ W_bf16^T (exact accumulation) + bias )."""
    K = x_bf16.shape[1]
    wb = bf16_to_f32(w4a16_dequant_bf16(qp, s16, zp, K, group_size)).astype(np.float64)
    acc = bf16_to_f32(x_bf16).astype(np.float64) @ wb.T
    y = acc.astype(np.float32)
    if bias_bf16 is not None:
        y = y + bf16_to_f32(bias_bf16)[None, :]
    return f32_to_bf16(y)


# ---------------------------------------------------------------------------
# reference backend, restated (for parity reports and the CPU baseline)
# ---------------------------------------------------------------------------


def reference_linear_f32(x_f32, qweight, scales, zeros, group_size, bias_f32=None,
                         per_token_bits: int | None = None, input_scale=None):
    """``reference.py:48-91`` with float32 input (compute dtype float32):
    optional ``x / input_scale``; optional per-token fake quantization
    ts = max(amax, 1e-8)/qmax, x = clamp(rint(x/ts), +-qmax) * ts; then
    ``x @ dequant(W)^T + bias`` (float64 accumulation here)."""
    x = np.asarray(x_f32, np.float32)
    if input_scale is not None:
        x = x / np.asarray(input_scale, np.float32)[None, :]
    if per_token_bits is not None:
        qmax = 2 ** (per_token_bits - 1) - 1
        ts = np.maximum(np.abs(x).max(axis=1, keepdims=True), F32(1e-8)) / F32(qmax)
        x = np.clip(np.rint(x / ts), -qmax, qmax) * ts
    w = dequantize_weight(qweight, scales, zeros, group_size, out="f32")
    y = x.astype(np.float64) @ w.astype(np.float64).T
    if bias_f32 is not None:
        y = y + np.asarray(bias_f32, np.float64)[None, :]
    return y.astype(np.float32)


def rel_fro(a, b) -> float:
    """Relative Frobenius error ||a-b|| / ||b||."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(a - b)
    n = np.linalg.norm(b)
    return float(d / n) if n > 0 else float(d)
