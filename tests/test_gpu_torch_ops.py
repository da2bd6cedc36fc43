"""The compiled torch operators on the GPU.

``torch.ops.qi_int8_w8a8.linear`` is called exactly as the reference's
Int8W8A8Backend calls its own extension (backends/int8_w8a8_ops.py:176:
``self._custom_linear(x_2d, qweight_2d, weight_scales, bias_kernel)``), with
and without bias, and must give the oracle's bytes (INT8 is bit-exact),
including at a size where the CTA-pair kernel splits its last wave through
the operator's workspace.  The qi_b200 operators give the same bytes as the
Python front end, and bad arguments raise torch errors.
"""

import numpy as np
import pytest
import torch

from oracle import qi_oracle as O
from qi_b200 import _lib, kernels as K, torch_ops
from qi_b200.synthetic import make_small_case

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    torch_ops.load()
    torch.cuda.set_device(0)
    yield
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True)[0] == 0


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("M,N,Kd", [(17, 192, 256), (512, 3072, 3072), (3120, 3072, 14336)])
@pytest.mark.parametrize("with_bias", [True, False])
def test_reference_schema_linear_bit_exact(M, N, Kd, with_bias):
    x, w, b = make_small_case(M, N, Kd, seed=M + N, outlier_frac=0.002)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    x_2d, qweight_2d = x.to(DEV), torch.from_numpy(qw).to(DEV)
    weight_scales = torch.from_numpy(sw[:, 0]).contiguous().to(DEV)
    bias_kernel = b.to(DEV) if with_bias else None
    out = torch.ops.qi_int8_w8a8.linear(x_2d, qweight_2d, weight_scales, bias_kernel)
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == (M, N)
    if Kd == 14336:  # the long-K case: same bytes as the Python front end, which splits the tail
        ref = K.int8_linear(x_2d, qweight_2d, weight_scales, bias_kernel)
        assert torch.equal(out, ref)
        rows = np.r_[0:8, 1500:1508, M - 8:M]
        yo, _, _, _ = O.int8_linear(bits(x)[rows], qw, sw[:, 0], bits(b) if with_bias else None)
        np.testing.assert_array_equal(bits(out)[rows], yo)
    else:
        yo, _, _, _ = O.int8_linear(bits(x), qw, sw[:, 0], bits(b) if with_bias else None)
        np.testing.assert_array_equal(bits(out), yo)


def test_qi_b200_ops_match_front_end():
    x, w, b = make_small_case(64, 256, 512, seed=9)
    xd, bd = x.to(DEV), b.to(DEV)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    q8, s8 = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).contiguous().to(DEV)
    assert torch.equal(torch.ops.qi_b200.int8_linear(xd, q8, s8, bd, True), K.int8_linear(xd, q8, s8, bd, gelu=True))
    wf, sf = O.quantize_fp8_rowwise(w.numpy())
    wfd, sfd = torch.from_numpy(wf).to(DEV), torch.from_numpy(sf).to(DEV)
    assert torch.equal(torch.ops.qi_b200.fp8_linear(xd, wfd, sfd, None, bd, True),
                       K.fp8_linear(xd, wfd, sfd, None, bd, gelu=True))
    act = torch.tensor([0.02], device=DEV)
    assert torch.equal(torch.ops.qi_b200.fp8_linear(xd, wfd, sfd, act, bd, False), K.fp8_linear(xd, wfd, sfd, act, bd))
    q4, s4, z4 = O.quantize_weight_rtn(w.numpy(), 4, 128, False)
    qp, s16, zp = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in O.pack_w4a16(q4, s4, z4))
    for m in (1, 300):
        xm = torch.randn(m, 512, device=DEV).to(torch.bfloat16)
        assert torch.equal(torch.ops.qi_b200.w4a16_linear(xm, qp, s16, zp, 128, bd),
                           K.w4a16_linear(xm, qp, s16, zp, 128, bd))


def test_errors_are_torch_errors():
    x = torch.randn(4, 64, device=DEV).to(torch.bfloat16)
    qw = torch.zeros(32, 64, dtype=torch.int8, device=DEV)
    ws = torch.ones(32, device=DEV)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        torch.ops.qi_int8_w8a8.linear(x.cpu(), qw, ws, None)
    with pytest.raises(RuntimeError, match="K dimension"):
        torch.ops.qi_int8_w8a8.linear(x, qw[:, :32].contiguous(), ws, None)
    with pytest.raises(RuntimeError, match="int8"):
        torch.ops.qi_int8_w8a8.linear(x, qw.float(), ws, None)
