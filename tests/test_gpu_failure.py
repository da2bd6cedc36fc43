"""Failure detection on one GPU without a fault: a bounded device wait that
runs out of time reports itself through the device status word, the host
turns that into an exception at its next check, and the context stays usable.

The wait that runs out is the cross-GPU barrier's, given a peer flag block
that nothing writes (a second buffer on the same GPU standing in for a rank
that never arrives) and a 20 ms limit.  No kernel traps, faults or hangs:
the barrier kernel gives up after its limit, records the rank it waited for
and returns.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import qi_oracle as O
from qi_b200 import _lib, kernels as K
from qi_b200.synthetic import make_small_case

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True)[0] == 0


def test_barrier_timeout_is_reported_and_context_survives():
    lib = _lib.load()
    own = torch.zeros(64, dtype=torch.int32, device=DEV)     # this rank's flag block
    ghost = torch.zeros(64, dtype=torch.int32, device=DEV)   # "rank 1": never arrives
    flags = (ctypes.c_void_p * 2)(own.data_ptr(), ghost.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    # a limit outside (0, 2 s] is refused on the host
    assert lib.qi_b200_peer_barrier_timed(flags, 2, 0, 0, st) == _lib.EINVAL
    assert lib.qi_b200_peer_barrier_timed(flags, 2, 0, 3_000_000_000, st) == _lib.EINVAL
    _lib.call("qi_b200_peer_barrier_timed", flags, 2, 0, 20_000_000, st)
    torch.cuda.synchronize()
    with pytest.raises(_lib.QiB200DeviceError) as err:
        _lib.raise_on_device_error()
    code, tag, site, _ = err.value.status
    assert (code, tag, site) == (1, 0x300, 1)
    assert ghost[0].item() == 1          # this rank did publish its epoch to the absent peer
    assert _lib.device_status()[0] == 0  # cleared by raise_on_device_error

    # the context still runs kernels correctly
    x, w, b = make_small_case(64, 256, 512, seed=5)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    y = K.int8_linear(x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV))
    yo, _, _, _ = O.int8_linear(x.contiguous().view(torch.int16).numpy().view(np.uint16), qw, sw[:, 0],
                                b.contiguous().view(torch.int16).numpy().view(np.uint16))
    np.testing.assert_array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), yo)
    _lib.raise_on_device_error()


def test_backend_status_check_raises():
    """``B200Backend(check_errors=True)`` checks the status word after every
    call: a timeout left by an earlier launch surfaces at the next linear."""
    from qi_b200.quantization.backends import B200Backend
    from qi_b200.quantization import WeightActivationQuantConfig
    from qi_b200.quantization.quantize import quantize_linear_weight
    from qi_b200.quantization.modules import WeightOnlyLinear

    lib = _lib.load()
    cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="int", backend="b200",
                                      activation_granularity="per_token", weight_granularity="per_channel")
    lin = torch.nn.Linear(256, 128)
    layer = WeightOnlyLinear.from_linear(lin, quantize_linear_weight(lin.weight.detach(), cfg), cfg,
                                         B200Backend(check_errors=True)).to(DEV)
    x = torch.randn(8, 256).to(torch.bfloat16).to(DEV)
    layer.bias = layer.bias.to(torch.bfloat16)
    layer(x)  # clean
    own = torch.zeros(64, dtype=torch.int32, device=DEV)
    ghost = torch.zeros(64, dtype=torch.int32, device=DEV)
    flags = (ctypes.c_void_p * 2)(own.data_ptr(), ghost.data_ptr())
    _lib.call("qi_b200_peer_barrier_timed", flags, 2, 0, 10_000_000, torch.cuda.current_stream().cuda_stream)
    with pytest.raises(_lib.QiB200DeviceError):
        layer(x)
    layer(x)  # the check cleared the word
