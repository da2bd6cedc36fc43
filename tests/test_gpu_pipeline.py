"""GPU: ``HostLinearPipeline`` (pinned host rows in chunks; host-to-device
copies, the linear and device-to-host copies on three streams) gives the
device module's result, for every format.

INT8 outputs are compared bit for bit (exact integer accumulation).  FP8
and NVFP4 are compared bit for bit too at these shapes (K = 1024: no K
split of the last wave, so each output element's arithmetic does not depend
on M); W4A16 picks its kernel by M, so its chunks stay above the small-M
kernels' 256 rows and match bit for bit as well.  Ragged last chunks, a
single chunk, and dynamic per-tensor NVFP4 (always one chunk: its global
scale is the amax of all rows) included.
"""

import pytest
import torch

from qi_b200 import _lib
from qi_b200.pipeline import M_VARIANT_MIN_CHUNK, HostLinearPipeline, m_invariant, plan_chunks, rows_independent
from qi_b200.quantization import WeightActivationQuantConfig, WeightOnlyLinear, WeightOnlyQuantConfig
from qi_b200.quantization.backends import get_backend
from qi_b200.quantization.quantize import quantize_linear_weight

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


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


def _layer(kind: str, N: int, K: int, gelu: bool, seed: int):
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * K ** -0.5)
        lin.bias.copy_(torch.randn(N, generator=g) * 0.1)
    if kind == "int8":
        cfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="int", backend="b200",
                                          activation_granularity="per_token", weight_granularity="per_channel")
    elif kind == "fp8":
        cfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="fp8", backend="b200",
                                          activation_granularity="per_token", weight_granularity="per_channel")
    elif kind == "w4a16":
        cfg = WeightOnlyQuantConfig(enabled=True, algo="rtn", bits=4, group_size=128, symmetric=False,
                                    backend="b200")
    else:
        cfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="nvfp4", bits=4,
                                          activation_bits=4, backend="b200")
    q = quantize_linear_weight(lin.weight.detach().to(DEV), cfg)
    layer = WeightOnlyLinear.from_linear(lin, q, cfg, get_backend("b200")).to(DEV)
    layer.bias = layer.bias.to(torch.bfloat16)
    layer.fuse_gelu = gelu and kind != "w4a16"
    return layer


@pytest.mark.parametrize("kind", ["int8", "fp8", "w4a16", "nvfp4"])
@pytest.mark.parametrize("rows,chunk", [(1000, 256), (1000, None), (77, 32), (300, 4096)])
def test_pipeline_matches_device_forward(kind, rows, chunk):
    N, K = 768, 1024
    layer = _layer(kind, N, K, gelu=kind in ("int8", "fp8"), seed=rows)
    g = torch.Generator().manual_seed(7 + rows)
    x = (torch.randn(rows, K, generator=g) * 2).to(torch.bfloat16)
    want = layer(x.to(DEV)).cpu()
    pipe = HostLinearPipeline(layer, chunk_rows=chunk)
    xh = x.pin_memory()
    out = pipe(xh)
    torch.cuda.current_stream().synchronize()
    assert out.shape == (rows, N) and out.dtype == torch.bfloat16
    assert torch.equal(out, want), (kind, rows, chunk, (out.float() - want.float()).abs().max().item())
    # twice more into the same pinned output (staging slots reused across calls)
    out2 = torch.empty_like(out).pin_memory()
    for _ in range(2):
        pipe(xh, out=out2)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out2, want)
    min_chunk = 1 if m_invariant(layer) else M_VARIANT_MIN_CHUNK
    n_chunks = len(plan_chunks(rows, chunk, rows_independent(layer), min_chunk=min_chunk))
    if kind == "nvfp4":
        assert n_chunks == 1  # dynamic per-tensor activations
    elif kind == "w4a16":
        assert not m_invariant(layer)  # chunks stay above the small-M kernels' 256 rows
        assert n_chunks == (2 if (rows, chunk) == (1000, 256) else 1)
    elif chunk is not None:
        assert n_chunks == -(-rows // chunk)


@pytest.mark.parametrize("kind", ["int8", "fp8", "w4a16"])
def test_pipeline_graph_replay(kind):
    """capture() records the chunked call as a CUDA graph on fixed pinned
    buffers; replay() with new input contents gives the device forward."""
    N, K, rows = 768, 1024, 3000
    layer = _layer(kind, N, K, gelu=kind != "w4a16", seed=11)
    pipe = HostLinearPipeline(layer, chunk_rows=512)
    xh = torch.empty(rows, K, dtype=torch.bfloat16).pin_memory()
    g = torch.Generator().manual_seed(3)
    xh.copy_((torch.randn(rows, K, generator=g) * 2).to(torch.bfloat16))
    out = pipe.capture(xh)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, layer(xh.to(DEV)).cpu())
    for seed in (4, 5):
        xh.copy_((torch.randn(rows, K, generator=torch.Generator().manual_seed(seed)) * 2).to(torch.bfloat16))
        y = pipe.replay()
        torch.cuda.current_stream().synchronize()
        assert y is out and torch.equal(out, layer(xh.to(DEV)).cpu()), seed


def test_pipeline_3d_input_and_errors():
    layer = _layer("int8", 256, 512, gelu=False, seed=3)
    x = torch.randn(2, 90, 512).to(torch.bfloat16)
    want = layer(x.to(DEV)).cpu()
    out = HostLinearPipeline(layer, chunk_rows=64)(x.pin_memory())
    torch.cuda.current_stream().synchronize()
    assert out.shape == (2, 90, 256) and torch.equal(out, want)
    pipe = HostLinearPipeline(layer)
    with pytest.raises(ValueError):
        pipe(x)  # not pinned
    with pytest.raises(ValueError):
        pipe(x.to(DEV))
    with pytest.raises(ValueError):
        pipe(torch.randn(4, 100).to(torch.bfloat16).pin_memory())
