"""GPU parity of the weight-only path on the reference's own buffers
(``cuda_ext``: W8A16 and INT4 stored one value per int8), through the C ABI.

* ``qi_b200_wo_dequant`` gives the reference's dequantize_weight bytes
  (bf16), bit for bit, on the reference-generated fixtures: INT8 symmetric
  per channel, INT8 asymmetric g32, INT4 symmetric g64, INT4 asymmetric g128
  and ragged groups;
* the linear (dequantize + bf16 tcgen05 GEMM) within 5e-3 of the
  reference's ReferenceBackend.linear output (fixture) and within 2e-3 of an
  fp64 matmul of the same dequantized weights;
* the module path: WeightOnlyQuantConfig's defaults (bits 8, group 128,
  symmetric) with backend "cuda_ext" through replace_linear_with_weight_only.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qi_oracle as O
from qi_b200 import _lib, kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    torch.cuda.set_device(0)
    yield
    torch.cuda.synchronize()
    st = _lib.device_status(clear=True)
    assert st[0] == 0, f"device status word reports a timed-out wait: {st}"


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("name", ["rtn_int8_sym_pc", "rtn_int8_asym_g32", "rtn_int4_sym_g64", "rtn_int4_asym_g128"])
def test_wo_dequant_matches_reference_bytes(name):
    f = dict(np.load(GOLD / f"{name}.npz"))
    N, Kd, nbits, group, sym = (int(v) for v in f["meta"])
    q = torch.from_numpy(f["qweight"]).to(DEV)
    s = torch.from_numpy(f["scales"]).to(DEV)
    z = None if sym else torch.from_numpy(f["zeros"]).to(DEV)
    w = K.wo_dequant(q, s, z, group)
    np.testing.assert_array_equal(bits(w), f["deq_bf16"])


def test_wo_linear_vs_reference_backend_fixture():
    f = dict(np.load(GOLD / "linear_w4a16_M9_N128_K384.npz"))
    x, b = from_bits(f["x"]).to(DEV), from_bits(f["bias"]).to(DEV)
    q = torch.from_numpy(f["qweight"]).to(DEV)
    s = torch.from_numpy(f["scales"]).to(DEV)
    z = torch.from_numpy(f["zeros"]).to(DEV)
    y = K.weight_only_linear(x, q, s, z, 128, b)
    e = O.rel_fro(O.bf16_to_f32(bits(y)), O.bf16_to_f32(f["y_ref_bf16in"]))
    assert e <= 5e-3, e
    wd = O.bf16_to_f32(bits(K.wo_dequant(q, s, z, 128))).astype(np.float64)
    ref = O.bf16_to_f32(f["x"]).astype(np.float64) @ wd.T + O.bf16_to_f32(f["bias"])
    assert O.rel_fro(O.bf16_to_f32(bits(y)), ref) <= 2e-3


@pytest.mark.parametrize("M", [1, 16, 300])
def test_w8a16_default_config_through_cuda_ext(M):
    from qi_b200.quantization import WeightOnlyQuantConfig, replace_linear_with_weight_only
    from qi_b200.quantization.quantize import dequantize_weight

    g = torch.Generator().manual_seed(M)
    N, Kd = 384, 1024
    lin = torch.nn.Linear(Kd, N)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, Kd, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(N, generator=g) * 0.01)
    model = torch.nn.Module()
    model.ffn = torch.nn.Sequential(lin)
    cfg = WeightOnlyQuantConfig(enabled=True, algo="rtn", backend="cuda_ext")  # defaults: bits 8, group 128, symmetric
    replace_linear_with_weight_only(model, cfg)
    layer = model.ffn[0]
    assert layer.qweight.dtype == torch.int8 and layer.bits == 8 and layer.group_size == 128
    wd = dequantize_weight(layer.qweight, layer.scales, layer.zeros, 8, 128, True, dtype=torch.bfloat16)
    model.to(DEV)
    x = (torch.randn(M, Kd, generator=g)).to(torch.bfloat16)
    y = layer(x.to(DEV))
    ref = x.double() @ wd.double().T + layer.bias.double().cpu()
    e = O.rel_fro(y.float().cpu().numpy(), ref.numpy())
    assert e <= 2e-3, e


@pytest.mark.parametrize("sym", [False, True])
def test_reference_int4_checkpoint_runs_on_b200(sym):
    """A weight-only INT4 checkpoint written by the reference's own
    save_quantized_checkpoint, loaded for the B200 backend (repacked at
    load), runs the reference model's FFN within the INT4 bound (5e-3) of the
    reference's own output on the same input."""
    import torch.nn as nn

    from qi_b200.quantization import load_checkpoint_payload, load_quantized_checkpoint

    name = f"ckpt_ref_int4_{'sym' if sym else 'asym'}_g64"
    payload = load_checkpoint_payload(GOLD / f"{name}.pt")
    io = np.load(GOLD / f"{name}_io.npz")
    model = nn.Module()
    model.mot = nn.Module()
    model.mot.ffn = nn.Sequential(nn.Linear(128, 64), nn.GELU(approximate="tanh"), nn.Linear(64, 128))
    load_quantized_checkpoint(model, payload, backend="b200")
    model.to(DEV)
    for m in model.mot.ffn:
        if getattr(m, "bias", None) is not None:
            m.bias = m.bias.to(torch.bfloat16)
    with torch.no_grad():
        y = model.mot.ffn(from_bits(io["x"]).to(DEV))
    e = O.rel_fro(O.bf16_to_f32(bits(y)), O.bf16_to_f32(io["y"]))
    assert e <= 5e-3, e
