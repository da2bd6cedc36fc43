"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations of the quantized-linear path.

The reference publishes no dataset for this path; its configurations are
synthetic by definition (seeded ``torch.Generator().manual_seed(0)``, fp32
draws, then ``.bfloat16()``).  Everything here runs on the CPU so that the
same bytes are produced on every machine; callers move the tensors to the GPU.

Shapes follow the Wan2.2 MoT DiT the reference quantizes
(``configs/model/fastwam.yaml:12-45``: video hidden 3072 / FFN 14336, action
hidden 1024 / FFN 4096, 24 heads x 128).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LinearCase:
    """One quantized linear: X [M, K] bf16, W [N, K] fp32 master weight, bias [N] bf16."""

    name: str
    M: int
    N: int
    K: int
    outlier_frac: float = 0.0
    outlier_gain: float = 20.0
    w_std: float = 0.02
    bias_std: float = 0.01
    seed: int = 0


# The four single-linear configurations.
CFG_INT8 = LinearCase("int8_w8a8_M512_N3072_K3072", 512, 3072, 3072, outlier_frac=0.001)
CFG_FP8 = LinearCase("fp8_ffn_up_M4096_N14336_K3072", 4096, 14336, 3072)
CFG_NVFP4 = LinearCase("nvfp4_ffn_down_M4096_N3072_K14336", 4096, 3072, 14336)
CFG_W4A16 = {m: LinearCase(f"w4a16_g128_M{m}_N3072_K3072", m, 3072, 3072) for m in (1, 16, 256, 4096)}


def make_linear_inputs(case: LinearCase):
    """Return (x_bf16 [M,K], w_fp32 [N,K], bias_bf16 [N]) on the CPU.

    Draw order is fixed (x, outlier columns, w, bias) so the bytes are stable.
    Outliers: ``floor(outlier_frac * K)`` distinct random columns of X are
    multiplied by ``outlier_gain`` before the bf16 cast (
    0.1 % of columns x20).
    """
    g = torch.Generator().manual_seed(case.seed)
    x = torch.randn(case.M, case.K, generator=g, dtype=torch.float32)
    n_out = int(case.outlier_frac * case.K)
    if n_out > 0:
        cols = torch.randperm(case.K, generator=g)[:n_out]
        x[:, cols] *= case.outlier_gain
    w = torch.randn(case.N, case.K, generator=g, dtype=torch.float32) * case.w_std
    b = torch.randn(case.N, generator=g, dtype=torch.float32) * case.bias_std
    return x.bfloat16(), w, b.bfloat16()


def make_small_case(M: int, N: int, K: int, seed: int = 0, outlier_frac: float = 0.0):
    """Small parity case with the same distributions as the benchmark configs."""
    return make_linear_inputs(LinearCase(f"small_M{M}_N{N}_K{K}", M, N, K, outlier_frac=outlier_frac, seed=seed))
