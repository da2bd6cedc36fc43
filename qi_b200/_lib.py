"""Loader for ``libqi_b200.so`` (the C ABI in ``include/qi_b200.h``).

The library is found next to this file (built in-tree by
``python -m qi_b200.build``).  There is no fallback: if the library is
missing or the device is not a B200, calls raise ``QiB200Unavailable``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqi_b200.so"

# status codes (include/qi_b200.h)
OK, EINVAL, ESHAPE, EALIGN, ECUDA, ETMAP, EARCH, ETOOBIG = range(8)
KIND_INT8, KIND_FP8_E4M3, KIND_BF16 = 0, 1, 2
EPI_GELU, EPI_RAW_ACC = 1, 2
W4A16_DEQUANT_MIN_M = 257  # QI_B200_W4A16_DEQUANT_MIN_M (measured crossover: M=512 26 us vs 43 us fused)
NVFP4_TILE_SHIFT = 8  # flags bits 8-9: 0 auto, 1 single-CTA 128x128, 2 pair 256x128, 3 pair 256x256
TAIL_SPLIT_SHIFT = 12  # flags bits 12-15 of qi_b200_gemm_ws: 0 auto, 1 no split, S = at most S splits per tail tile


class QiB200Unavailable(RuntimeError):
    """The native library is missing or cannot run on this device."""


class QiB200Error(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_F = ctypes.c_float

# name -> argtypes (restype is int unless listed in _RESTYPES)
SIGNATURES = {
    "qi_b200_abi_version": [],
    "qi_b200_error_string": [_I],
    "qi_b200_device_status": [_P, _I],
    "qi_b200_last_launch": [_P],
    "qi_b200_last_tail_split": [],
    "qi_b200_launch_count": [_P],
    "qi_b200_quantize_int8_rowwise_smooth": [_P, _P, _P, _P, _I, _I, _P],
    "qi_b200_w4a16_dequant": [_P, _P, _P, _I, _P, _I, _I, _P],
    "qi_b200_wo_dequant": [_P, _P, _P, _I, _P, _I, _I, _P],
    "qi_b200_wo_linear_ws": [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _P, ctypes.c_size_t, _P],
    "qi_b200_w4a16_linear_ws": [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _P, ctypes.c_size_t, _P],
    "qi_b200_quantize_int8_rowwise": [_P, _P, _P, _I, _I, _P],
    "qi_b200_quantize_int8_rowwise_given": [_P, _P, _P, _I, _I, _P],
    "qi_b200_int8_row_scales": [_P, _P, _I, _I, _P],
    "qi_b200_peer_alloc": [ctypes.c_size_t, _P, _P],
    "qi_b200_peer_open": [_P, _P],
    "qi_b200_peer_close": [_P],
    "qi_b200_peer_free": [_P],
    "qi_b200_peer_barrier": [_P, _I, _I, _P],
    "qi_b200_peer_barrier_timed": [_P, _I, _I, ctypes.c_ulonglong, _P],
    "qi_b200_gemm_csk": [_I, _P, _P, _P, _I, _P, _I, _P, _P, _LL, _I, _I, _I, _I, _I, _I, _P],
    "qi_b200_gemm_ws": [_I, _P, _P, _P, _I, _P, _I, _P, _P, _LL, _I, _I, _I, _I, _I, _P, ctypes.c_size_t, _P],
    "qi_b200_gemm_workspace_bytes": [_I, _I, _I, _I, _I, _I, _P],
    "qi_b200_gemm_gather": [_I, _P, _P, _P, _I, _P, _I, _P, _P, _I, _LL, _I, _I, _I, _I, _P],
    "qi_b200_resid_ln_quant": [_P, _P, _LL, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _F, _P],
    "qi_b200_rms_rope": [_P, _P, _LL, _P, _P, _LL, _P, _P, _P, _I, _I, _I, _I, _F, _P],
    "qi_b200_rms_head_partials": [_P, _P, _LL, _P, _I, _I, _I, _I, _P],
    "qi_b200_attention_short": [_P, _LL, _P, _LL, _P, _LL, _P, _LL, _I, _I, _I, _I, _F, _P],
    "qi_b200_rms_rope_partials": [_P, _P, _LL, _P, _P, _LL, _P, _P, _P, _I, _I, _I, _I, _P, _I, _F, _P],
    "qi_b200_int8_epilogue": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qi_b200_quantize_fp8_rowwise": [_P, _P, _P, _I, _I, _P],
    "qi_b200_quantize_fp8_static": [_P, _P, _P, _I, _I, _P],
    "qi_b200_int8_rowwise_bf16out": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qi_b200_int8_rowwise_bf16out_bias": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qi_b200_gemm": [_I, _P, _P, _P, _I, _P, _I, _P, _P, _LL, _I, _I, _I, _I, _I, _P],
    "qi_b200_int8_linear": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qi_b200_fp8_linear": [_P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qi_b200_int8_linear_noalloc": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qi_b200_w4a16_linear": [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _P],
    "qi_b200_quantize_nvfp4": [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P],
    "qi_b200_nvfp4_gemm": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _LL, _I, _I, _I, _I, _P],
    "qi_b200_nvfp4_linear": [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
}
_RESTYPES = {"qi_b200_error_string": ctypes.c_char_p}

_lock = threading.Lock()
_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the library once (thread-safe) and bind every declared symbol."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise QiB200Unavailable(
                f"{p} is missing; build it with `python -m qi_b200.build` (nvcc, sm_100a)."
            )
        lib = ctypes.CDLL(str(p))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        if lib.qi_b200_abi_version() != 1:
            raise QiB200Unavailable("libqi_b200 ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


def check(fn_name: str, rc: int) -> None:
    if rc != OK:
        msg = load().qi_b200_error_string(rc).decode()
        if rc == EARCH:
            raise QiB200Unavailable(f"{fn_name}: {msg}")
        raise QiB200Error(fn_name, rc, msg)


def call(fn_name: str, *args) -> None:
    """Call a C-ABI entry point and raise on a non-zero status."""
    check(fn_name, getattr(load(), fn_name)(*args))


def launch_count() -> int:
    """Kernels this library has launched in this process (graph captures count once)."""
    n = ctypes.c_ulonglong(0)
    check("qi_b200_launch_count", load().qi_b200_launch_count(ctypes.byref(n)))
    return n.value


def last_launch() -> dict:
    """Plan of this thread's most recent GEMM launch (see qi_b200_last_launch)."""
    buf = (ctypes.c_int * 6)()
    check("qi_b200_last_launch", load().qi_b200_last_launch(ctypes.cast(buf, _P)))
    names = {1: "gemm_int8", 2: "gemm_fp8", 3: "gemm_bf16", 4: "gemm_nvfp4", 6: "w4a16_splitk",
             7: "w4a16_small", 8: "gemm_int8_pair", 9: "gemm_fp8_pair", 10: "gemm_bf16_pair",
             11: "gemm_nvfp4_pair", 12: "gemm_int8_csk", 13: "gemm_fp8_csk", 14: "gemm_bf16_csk"}
    v = list(buf)
    return {"kernel": names.get(v[0], "none"), "grid": v[1], "cluster": v[2], "tile_n": v[3], "stages": v[4],
            "smem": v[5]}


def last_tail_split() -> int:
    """Splits per tail tile of this thread's most recent CTA-pair GEMM (1 = none)."""
    return int(load().qi_b200_last_tail_split())


def device_status(clear: bool = False) -> tuple[int, int, int, int]:
    buf = (ctypes.c_uint * 4)()
    check("qi_b200_device_status", load().qi_b200_device_status(ctypes.cast(buf, _P), int(clear)))
    return tuple(int(v) for v in buf)


class QiB200DeviceError(RuntimeError):
    """A kernel of this library gave up a bounded wait (device status word set).

    The kernel returned early, so the outputs of the launch that set the word
    (and of every launch after it on that device) are incomplete."""

    def __init__(self, status: tuple):
        self.status = tuple(status)
        super().__init__(
            "qi_b200: a bounded device wait timed out (kernel tag 0x%x, wait site %d, block %d); outputs of the "
            "launches since the last status check are incomplete" % (status[1], status[2], status[3]))


def raise_on_device_error(clear: bool = True) -> None:
    """Read the current device's status word (synchronous: the host waits for
    the device) and raise ``QiB200DeviceError`` if a bounded wait timed out.
    ``clear`` resets the word (and the counters an aborted launch may have
    left) so the context can run again.  Call it at a point where the caller
    synchronizes anyway: after a step, between graph replays, at shutdown."""
    st = device_status(clear=False)
    if st[0] != 0:
        if clear:
            device_status(clear=True)
        raise QiB200DeviceError(st)
