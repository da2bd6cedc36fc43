"""Torch operators over the C ABI: ``torch.ops.qi_int8_w8a8.linear`` with the
reference's schema (``src/qi/quantization/csrc/int8_w8a8/bindings.cpp:159-165``)
and ``torch.ops.qi_b200.{int8_linear, fp8_linear, w4a16_linear}``.

They live in the in-tree ``libqi_b200_torch.so`` (``qi_b200/csrc/torch_ops.cpp``,
built by ``python -m qi_b200.build``), which links the in-tree
``libqi_b200.so``.  ``load()`` registers them with torch once.
"""

from __future__ import annotations

import threading

from .build import TORCH_OPS_LIB

_lock = threading.Lock()
_loaded = False


def load() -> None:
    """Register the operators (idempotent).  Raises ``QiB200Unavailable``
    when the library has not been built."""
    global _loaded
    if _loaded:
        return
    with _lock:
        if _loaded:
            return
        import torch

        from ._lib import QiB200Unavailable, load as load_c_abi

        if not TORCH_OPS_LIB.exists():
            raise QiB200Unavailable(f"{TORCH_OPS_LIB} is missing; build it with `python -m qi_b200.build`.")
        load_c_abi()  # the C ABI library the operators call into
        torch.ops.load_library(str(TORCH_OPS_LIB))
        _loaded = True
