"""The INT8 linear entry point that allocates nothing
(``qi_b200_int8_linear_noalloc``), called through the C ABI.

It exists for callers that cannot allocate or be handed scratch memory (an
FFI plugin whose host runtime owns all device memory, a real-time loop that
may not call cudaMalloc); its activation scratch is a fixed array inside the
library.  Checked here:

* its output is identical (bit for bit, the bar of the INT8 tests) to the
  allocating entry point ``qi_b200_int8_linear`` given caller workspace, on
  two calls in a row with different inputs (the second call reuses the
  scratch the first one left behind), for a small problem and for one large
  enough to run on the CTA-pair kernel;
* a call allocates nothing: the device's free memory is the same before and
  after it (measured on the second call of each shape, so the first call's
  one-time set-up and lazy loading of kernel code are not counted), and the
  CTA-pair launch ran without the tail split, whose partial accumulators
  would need a workspace;
* oversized calls are refused before anything is launched.

Everything runs on a fresh stream, so no workspace or slot that an earlier
test registered for torch's default stream can stand in for anything.
This file is named so pytest collects it last.
"""

import numpy as np
import pytest
import torch

from oracle import qi_oracle as O
from qi_b200 import _lib
from qi_b200.synthetic import make_small_case

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _case(M, N, K, seed):
    x, w, b = make_small_case(M, N, K, seed=seed, outlier_frac=0.002)
    x2 = (x.float() * -0.75).to(torch.bfloat16)  # a second input for the second call
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    return ([x.to(DEV), x2.to(DEV)], torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).contiguous().to(DEV),
            b.to(DEV))


@pytest.mark.parametrize("M,N,K,kernel", [(1024, 9216, 8192, "gemm_int8_pair"), (17, 192, 256, None)])
def test_int8_linear_noalloc_matches_allocating_entry_point(M, N, K, kernel):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    lib = _lib.load()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        st = side.cuda_stream
        xs, qw, sw, b = _case(M, N, K, seed=M + N)
        ws_q = torch.empty((M, K), dtype=torch.int8, device=DEV)
        ws_s = torch.empty((M,), dtype=torch.float32, device=DEV)
        y_ref = [torch.empty((M, N), dtype=torch.bfloat16, device=DEV) for _ in xs]
        y_na = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in xs]
        for x, y in zip(xs, y_ref):
            _lib.check("qi_b200_int8_linear", lib.qi_b200_int8_linear(
                x.data_ptr(), qw.data_ptr(), sw.data_ptr(), b.data_ptr(), y.data_ptr(), ws_q.data_ptr(),
                ws_s.data_ptr(), M, N, K, st))
        for i, (x, y) in enumerate(zip(xs, y_na)):
            side.synchronize()
            free0 = torch.cuda.mem_get_info(0)[0]
            _lib.check("qi_b200_int8_linear_noalloc", lib.qi_b200_int8_linear_noalloc(
                x.data_ptr(), qw.data_ptr(), sw.data_ptr(), b.data_ptr(), y.data_ptr(), M, N, K, st))
            if kernel is not None:
                assert _lib.last_launch()["kernel"] == kernel
                assert _lib.last_tail_split() == 1
            side.synchronize()
            if i == 1:
                assert torch.cuda.mem_get_info(0)[0] == free0, "the call changed the device's free memory"
        side.synchronize()
        for a, r in zip(y_na, y_ref):
            np.testing.assert_array_equal(_bits(a), _bits(r))

        # sizes beyond the fixed scratch are refused on the host (nothing launched)
        rows = 16384 + 1
        assert lib.qi_b200_int8_linear_noalloc(1, 1, 1, None, 1, rows, 64, 64, st) == _lib.ETOOBIG
        assert lib.qi_b200_int8_linear_noalloc(1, 1, 1, None, 1, 1024, 64, 8192 + 16, st) == _lib.ETOOBIG
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
