"""The INT8 linear entry point that allocates nothing
(``qi_b200_int8_linear_noalloc``), called through the C ABI.

It exists for callers that cannot allocate or be handed scratch memory (an
FFI plugin whose host runtime owns all device memory, a real-time loop that
may not call cudaMalloc); its activation scratch is a fixed array inside the
library.  Its output must be identical (bit for bit, the bar of the INT8
tests) to the allocating entry point ``qi_b200_int8_linear`` given caller
workspace, on two calls in a row with different inputs and shapes (the
second call reuses the scratch the first one left behind), and oversized
calls must be refused before anything is launched.

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
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    return (x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).contiguous().to(DEV), b.to(DEV))


def test_int8_linear_noalloc_matches_allocating_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # a large call, then a small one reusing (and only partly overwriting) the scratch
    for (M, N, K), seed in (((512, 3072, 3072), 1), ((17, 192, 256), 2)):
        x, qw, sw, b = _case(M, N, K, seed)
        ws_q = torch.empty((M, K), dtype=torch.int8, device=DEV)
        ws_s = torch.empty((M,), dtype=torch.float32, device=DEV)
        y_ref = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
        y_na = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        _lib.check("qi_b200_int8_linear", lib.qi_b200_int8_linear(
            x.data_ptr(), qw.data_ptr(), sw.data_ptr(), b.data_ptr(), y_ref.data_ptr(), ws_q.data_ptr(),
            ws_s.data_ptr(), M, N, K, stream))
        _lib.check("qi_b200_int8_linear_noalloc", lib.qi_b200_int8_linear_noalloc(
            x.data_ptr(), qw.data_ptr(), sw.data_ptr(), b.data_ptr(), y_na.data_ptr(), M, N, K, stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(_bits(y_na), _bits(y_ref))

    # sizes beyond the fixed scratch are refused on the host (nothing launched)
    rows = 16384 + 1
    assert lib.qi_b200_int8_linear_noalloc(1, 1, 1, None, 1, rows, 64, 64, stream) == _lib.ETOOBIG
    assert lib.qi_b200_int8_linear_noalloc(1, 1, 1, None, 1, 1024, 64, 8192 + 16, stream) == _lib.ETOOBIG
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
