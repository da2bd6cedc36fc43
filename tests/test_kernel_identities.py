"""CPU: the exact-arithmetic identities two kernels rely on, checked
exhaustively or on their whole input range.

- The NVFP4 codes pass (``k_quant_nvfp4_tensor``, quantize_nvfp4.cuh) finds a
  block's row as ``mulhi(t, m) >> (l - 1)`` with ``l = ceil(log2 bpr)`` and
  ``m = ceil(2^(31 + l) / bpr)`` instead of ``t / bpr``: exact for every
  ``0 <= t < 2^31`` and every blocks-per-row count the quantizer accepts
  (``bpr = cols / 16`` with ``cols % 64 == 0``).
- W4A16 dequantization (``dequant8``, gemm_w4a16.cuh) places a nibble ``q``
  in the mantissa of 0.5 (``0x3F00_0000 | q << 16`` is ``0.5 + q / 256``)
  and computes ``fma(0.5 + q / 256, 256 s, -(128 + z) s)``; the operands are
  exact in fp32 for every fp16 scale ``s`` and zero point ``z``, so the
  single rounding gives ``fp32((q - z) s)``, the reference's value.
"""

import random

import numpy as np


def _div_magic(bpr: int) -> tuple[int, int]:
    l = (bpr - 1).bit_length()
    return l, ((1 << (31 + l)) + bpr - 1) // bpr


def test_row_index_by_reciprocal_multiply():
    rng = random.Random(0)
    for bpr in list(range(4, 4097, 4)) + [8192, 65536, 131072, 2 ** 20]:
        l, m = _div_magic(bpr)
        assert l >= 2 and m < 2 ** 32
        ts = [0, 1, bpr - 1, bpr, 2 ** 31 - 1] + [rng.randrange(0, 2 ** 31) for _ in range(200)]
        for t in ts:
            assert ((t * m) >> 32) >> (l - 1) == t // bpr, (bpr, t)


def _f32_bits(v: float) -> int:
    return int(np.array([v], np.float32).view(np.uint32)[0])


def test_dequant_encoding_is_exact():
    # every nibble: the byte-permuted word is 0.5 + q / 256 exactly
    for q in range(16):
        w = np.array([0x3F000000 | (q << 16)], np.uint32).view(np.float32)[0]
        assert float(w) == 0.5 + q / 256
    # every finite positive fp16 scale, every zero point: 256 s and (128 + z) s
    # are exact in fp32, so the fma's exact value is (q - z) s
    s16 = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    s256 = (s16 * 256).astype(np.float32).astype(np.float64)
    assert np.array_equal(s256, s16 * 256)
    for z in range(16):
        c = (-(128 + z) * s16).astype(np.float32).astype(np.float64)
        assert np.array_equal(c, -(128 + z) * s16), z
        for q in (0, 7, 15):
            exact = (0.5 + q / 256) * (s16 * 256) + (-(128 + z) * s16)
            assert np.array_equal(exact, (q - z) * s16), (q, z)
