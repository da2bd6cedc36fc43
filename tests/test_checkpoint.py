"""Quantized checkpoints (``qi_b200.quantization.checkpoint``) on the CPU.

* A checkpoint written by the reference's own save_quantized_checkpoint
  (tests/golden/ckpt_ref_int4_*.pt, weight-only INT4, asymmetric and
  symmetric) loads for the B200 backend with its INT4 layers repacked into the
  kernels' layout, dequantizing to the reference's dequantize_weight values.
* Models that hold packed buffers (W4A16, NVFP4) save in the packed v2 format
  with its layout names, and load back byte for byte with no repack.
* INT8 W8A8 saves in the reference's v1 format with the reference's keys.
* Unknown formats and packed checkpoints with other layouts are refused.
"""

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import qi_oracle as O
from qi_b200.quantization import (WeightActivationQuantConfig, WeightOnlyQuantConfig, checkpoint_format,
                                  load_checkpoint_payload, load_quantized_checkpoint, replace_linear_with_weight_only,
                                  save_quantized_checkpoint)
from qi_b200.quantization import checkpoint as C
from qi_b200.quantization.quantize import dequantize_weight

GOLD = Path(__file__).resolve().parent / "golden"


def skeleton(d_in=128, d_hid=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    model = nn.Module()
    model.mot = nn.Module()
    model.mot.ffn = nn.Sequential(nn.Linear(d_in, d_hid), nn.GELU(approximate="tanh"), nn.Linear(d_hid, d_in))
    with torch.no_grad():
        for p in model.mot.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return model


@pytest.mark.parametrize("sym", [False, True])
def test_reference_int4_checkpoint_loads_repacked(sym):
    payload = load_checkpoint_payload(GOLD / f"ckpt_ref_int4_{'sym' if sym else 'asym'}_g64.pt")
    ref_state = {k: v.clone() for k, v in payload["mot"].items()}
    assert checkpoint_format(payload) == C.FORMAT_WEIGHT_ONLY
    model = skeleton()
    cfg = load_quantized_checkpoint(model, payload, backend="b200")
    assert cfg.bits == 4 and cfg.group_size == 64 and cfg.symmetric == sym and cfg.backend == "b200"
    for name in ("ffn.0", "ffn.2"):
        layer = model.mot.get_submodule(name)
        assert layer.qweight is None and layer.qweight_packed.dtype == torch.int32
        q, s = ref_state[name + ".qweight"], ref_state[name + ".scales"].float()
        z = None if sym else ref_state[name + ".zeros"]
        want = dequantize_weight(q, s, z, 4, 64, sym, dtype=torch.bfloat16)
        got = O.w4a16_dequant_bf16(layer.qweight_packed.numpy(), layer.scale_factors.numpy(), layer.zeros.numpy(),
                                   q.shape[1], 64)
        np.testing.assert_array_equal(got, want.view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("kind", ["w4a16", "nvfp4"])
def test_packed_checkpoint_round_trip(kind, tmp_path):
    if kind == "w4a16":
        cfg = WeightOnlyQuantConfig(enabled=True, algo="rtn", bits=4, group_size=64, symmetric=False, backend="b200")
        fmt = C.FORMAT_PACKED_WEIGHT_ONLY
    else:
        cfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="nvfp4", bits=4, activation_bits=4,
                                          backend="b200")
        fmt = C.FORMAT_PACKED_WEIGHT_ACTIVATION
    model = skeleton(256, 128)
    replace_linear_with_weight_only(model.mot, cfg)
    path = tmp_path / "q.pt"
    assert save_quantized_checkpoint(model, path, cfg, source_payload={"optimizer": {"lr": 1.0}, "step": 7},
                                     source_checkpoint="src.pt") == fmt
    payload = load_checkpoint_payload(path)
    assert "optimizer" not in payload and payload["step"] == 7
    meta = payload[C.METADATA_KEY]
    assert meta["format"] == fmt and meta["layouts"] == C.LAYOUTS and meta["source_checkpoint"] == "src.pt"
    fresh = skeleton(256, 128, seed=1)
    load_quantized_checkpoint(fresh, payload)
    for (k, a), (k2, b) in zip(sorted(model.mot.state_dict().items()), sorted(fresh.mot.state_dict().items())):
        assert k == k2 and a.dtype == b.dtype and torch.equal(a, b), k


def test_int8_w8a8_checkpoint_is_reference_format(tmp_path):
    cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="int", backend="b200",
                                      activation_granularity="per_token", weight_granularity="per_channel")
    model = skeleton()
    replace_linear_with_weight_only(model.mot, cfg)
    path = tmp_path / "q.pt"
    assert save_quantized_checkpoint(model, path, cfg) == C.FORMAT_WEIGHT_ACTIVATION
    payload = load_checkpoint_payload(path)
    assert set(payload[C.METADATA_KEY]) == {"format", "config", "source_checkpoint"}
    assert set(payload["mot"]) == {f"ffn.{i}.{b}" for i in (0, 2) for b in ("qweight", "scales", "bias")}
    fresh = skeleton(seed=2)
    load_quantized_checkpoint(fresh, payload)
    for k, v in model.mot.state_dict().items():
        assert torch.equal(v, fresh.mot.state_dict()[k]), k


def test_unknown_formats_are_refused(tmp_path):
    payload = load_checkpoint_payload(GOLD / "ckpt_ref_int4_asym_g64.pt")
    bad = dict(payload)
    bad[C.METADATA_KEY] = dict(payload[C.METADATA_KEY], format="qi_b200.weight_only.packed.v3")
    with pytest.raises(ValueError, match="Unsupported"):
        load_quantized_checkpoint(skeleton(), bad, backend="b200")
    other = dict(payload)
    other[C.METADATA_KEY] = dict(payload[C.METADATA_KEY], format=C.FORMAT_PACKED_WEIGHT_ONLY,
                                 layouts={"w4a16": "something else"})
    with pytest.raises(ValueError, match="layout"):
        checkpoint_format(other)
    with pytest.raises(ValueError, match="metadata"):
        checkpoint_format({"mot": {}})
