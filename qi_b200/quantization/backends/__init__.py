"""Backend registry (reference ``src/qi/quantization/backends/__init__.py:8-17``).

Every native backend name of the reference is served by ``B200Backend``:
``"b200"``, ``"int8_w8a8"`` (CUTLASS INT8), ``"flashrt_fp8"`` (FlashRT FP8)
and ``"cuda_ext"`` (reserved weight-only kernel).  The reference's
``"reference"`` dequantise-then-matmul backend is deliberately not part of
this package: there is no CPU path here.
"""

from __future__ import annotations

from .b200 import B200Backend, B200Unavailable, load_b200_ops

_NATIVE = ("b200", "int8_w8a8", "flashrt_fp8", "cuda_ext")


def get_backend(name: str) -> B200Backend:
    if name in _NATIVE:
        return B200Backend()
    if name == "reference":
        raise ValueError(
            "qi_b200 has no dequantise-then-matmul CPU backend; pass backend='b200' "
            "(or load the checkpoint with prepare_model_for_quantized_checkpoint(..., backend='b200'))."
        )
    raise ValueError(f"Unknown quantization backend: {name}")


__all__ = ["B200Backend", "B200Unavailable", "get_backend", "load_b200_ops"]
