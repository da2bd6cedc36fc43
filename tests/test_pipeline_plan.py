"""CPU: row-chunk planning of ``HostLinearPipeline`` and which activation
formats may be chunked (rows independent)."""

from types import SimpleNamespace

import pytest
import torch

from qi_b200.pipeline import M_VARIANT_MIN_CHUNK, m_invariant, plan_chunks, rows_independent


def test_plan_chunks_cover_rows_in_order():
    for rows in (1, 255, 256, 257, 1000, 3120, 4096, 10000):
        for chunk in (None, 1, 64, 256, 5000):
            ch = plan_chunks(rows, chunk, True)
            assert ch[0][0] == 0 and ch[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
            assert all(r1 > r0 for r0, r1 in ch)
            if chunk is not None:
                assert all(r1 - r0 == chunk for r0, r1 in ch[:-1])


def test_plan_chunks_defaults():
    # BASELINE config 2 (bf16 in K = 3072, out N = 14336): 142 MB -> 8 chunks of 512 rows
    assert plan_chunks(4096, None, True, 2 * (3072 + 14336)) == [(i * 512, (i + 1) * 512) for i in range(8)]
    # config 1 (6 MB) and small M: one chunk
    assert plan_chunks(512, None, True, 2 * (3072 + 3072)) == [(0, 512)]
    assert plan_chunks(16, None, True, 2 * (3072 + 3072)) == [(0, 16)]
    # 4096 x (3072 + 3072) bf16 = 50 MB -> 3 chunks, multiples of 128 rows
    assert plan_chunks(4096, None, True, 2 * (3072 + 3072)) == [(0, 1408), (1408, 2816), (2816, 4096)]
    assert plan_chunks(4096, None, True) == [(0, 4096)]
    # the graph form: one chunk per 8 MiB, at most 16, >= 256 rows (config 2: 16 chunks of 256 rows; config 1: 1)
    assert plan_chunks(4096, None, True, 2 * (3072 + 14336), graph=True) == [(i * 256, (i + 1) * 256) for i in range(16)]
    assert plan_chunks(512, None, True, 2 * (3072 + 3072), graph=True) == [(0, 512)]
    assert plan_chunks(4096, 128, False) == [(0, 4096)]
    assert plan_chunks(0, None, True) == []
    with pytest.raises(ValueError):
        plan_chunks(10, 0, True)


def _fake(packed_dtype=None, sf=False, g=False, act_scale=None, gran=None):
    return SimpleNamespace(
        qweight_packed=None if packed_dtype is None else torch.zeros(1, dtype=packed_dtype),
        scale_factors=torch.zeros(1, dtype=torch.uint8) if sf else None,
        weight_global_scale=torch.ones(1) if g else None,
        activation_scale=act_scale, activation_granularity=gran)


def test_rows_independent_formats():
    assert rows_independent(_fake())                                  # INT8 / FP8 / weight-only
    assert rows_independent(_fake(torch.int32))                       # W4A16 packed
    assert rows_independent(_fake(torch.uint8))                       # FP8 stored in qweight_packed
    assert not rows_independent(_fake(torch.uint8, sf=True, g=True))  # NVFP4, dynamic per tensor
    assert rows_independent(_fake(torch.uint8, sf=True, g=True, gran="per_token"))
    assert rows_independent(_fake(torch.uint8, sf=True, g=True, act_scale=torch.ones(1)))


def test_min_chunk_for_weight_only_formats():
    m = M_VARIANT_MIN_CHUNK
    assert plan_chunks(1000, 256, True, min_chunk=m) == [(0, 384), (384, 1000)]  # short tail folded
    assert plan_chunks(300, 64, True, min_chunk=m) == [(0, 300)]
    assert plan_chunks(4096, 512, True, min_chunk=m) == [(i * 512, (i + 1) * 512) for i in range(8)]
    for rows in (385, 700, 1000, 3000):
        for chunk in (1, 100, 384, 500):
            ch = plan_chunks(rows, chunk, True, min_chunk=m)
            assert ch[0][0] == 0 and ch[-1][1] == rows and all(r1 - r0 >= m for r0, r1 in ch)


def test_m_invariant_formats():
    packed = SimpleNamespace(qweight_packed=torch.zeros(1, dtype=torch.int32), qweight=None, weight_fp8=None,
                             activation_granularity=None)
    assert not m_invariant(packed)                                         # W4A16
    wo = SimpleNamespace(qweight=torch.zeros(1, dtype=torch.int8), qweight_packed=None, weight_fp8=None,
                         activation_granularity=None)
    assert not m_invariant(wo)                                             # W8A16 / unpacked INT4
    w8a8 = SimpleNamespace(qweight=torch.zeros(1, dtype=torch.int8), qweight_packed=None, weight_fp8=None,
                           activation_granularity="per_token")
    assert m_invariant(w8a8)
    fp8 = SimpleNamespace(qweight=None, qweight_packed=None, weight_fp8=torch.zeros(1, dtype=torch.uint8),
                          activation_granularity="per_token")
    assert m_invariant(fp8)
