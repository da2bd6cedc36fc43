"""The C ABI on CPU: the library loads, exports every symbol the header
declares, and the Python bindings match the declarations.  No compute call
runs here (there is no GPU in the build container).  The product path fails
loudly without the library or a B200."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from qi_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qi_b200.h"


def declared():
    """{name: number of parameters} of every function in include/qi_b200.h."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int|const char\s*\*)\s+(qi_b200_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p for p in m.group(2).split(",") if p.strip() and p.strip() != "void"]
        out[m.group(1)] = len(params)
    return out


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from qi_b200 import build
        build.build()
    return _lib.load()


def test_header_declares_the_abi():
    d = declared()
    assert len(d) >= 20
    for name in ("qi_b200_int8_linear", "qi_b200_gemm", "qi_b200_fp8_linear", "qi_b200_w4a16_linear",
                 "qi_b200_nvfp4_linear", "qi_b200_quantize_int8_rowwise", "qi_b200_int8_linear_noalloc"):
        assert name in d, name


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared():
        assert hasattr(raw, name), f"{name} declared in qi_b200.h but not exported"


def test_bindings_match_declarations(lib):
    d = declared()
    assert set(_lib.SIGNATURES) | {"qi_b200_abi_version", "qi_b200_error_string"} >= set(d)
    for name, nparams in d.items():
        if name in _lib.SIGNATURES:
            assert len(_lib.SIGNATURES[name]) == nparams, (name, len(_lib.SIGNATURES[name]), nparams)


def test_version_and_error_strings(lib):
    assert lib.qi_b200_abi_version() == 1
    for code in range(8):
        assert lib.qi_b200_error_string(code)
    assert b"ok" in lib.qi_b200_error_string(0).lower() or lib.qi_b200_error_string(0)


def test_missing_library_raises(tmp_path):
    with pytest.raises(_lib.QiB200Unavailable):
        _lib.load(tmp_path / "nope.so")


def test_backend_refuses_cpu_tensors():
    from qi_b200.quantization.backends import B200Backend, get_backend

    be = get_backend("b200")
    assert isinstance(be, B200Backend)
    with pytest.raises((ValueError, RuntimeError)):
        be.linear(x=torch.zeros(2, 16, dtype=torch.bfloat16), qweight=torch.zeros(8, 16, dtype=torch.int8),
                  scales=torch.ones(8, 1), zeros=None, bias=None, bits=8, group_size=-1, symmetric=True,
                  input_scale=None, keep_output_dtype="input", activation_granularity="per_token",
                  weight_granularity="per_channel")
    with pytest.raises(ValueError):
        get_backend("reference")


def test_torch_ops_library_registers_reference_schema():
    """The compiled torch-operator library loads on the CPU (no kernel runs)
    and registers qi_int8_w8a8::linear with the reference's schema
    (bindings.cpp:159-165) and the qi_b200 operators."""
    import torch

    from qi_b200 import build as B, torch_ops

    B.build_torch_ops()
    torch_ops.load()
    schema = str(torch.ops.qi_int8_w8a8.linear.default._schema)
    assert schema == ("qi_int8_w8a8::linear(Tensor x_bf16_2d, Tensor qweight, Tensor weight_scales, "
                      "Tensor? bias=None) -> Tensor"), schema
    for op in ("int8_linear", "fp8_linear", "w4a16_linear"):
        assert hasattr(torch.ops.qi_b200, op)
