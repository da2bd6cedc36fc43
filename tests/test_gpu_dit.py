"""GPU checks of the DiT step: the B200 execution plan (``DiTStepRunner``:
fused QKV / context-KV GEMMs, CUDA graph) against the module-structured
forward through ``WeightOnlyLinear`` on the same INT8 weights.

* Both paths use the block form of the joint mask.  They then run the same
  kernels on the same bytes, so their outputs are bit-identical.  This holds
  because fusing q/k/v along N leaves every INT8 output element unchanged.
* The reference's masked single-SDPA form agrees within a stated bound.
  Attention differs only in summation order, and INT8 re-quantization of
  later layers amplifies that slightly.
* A graph replay reproduces the eager step bit for bit.
* One layer at the full config-5 sizes (3120 video tokens, QKV N = 9216,
  FFN 14336) runs through both paths.
"""

import pytest
import torch

from qi_b200 import _lib
from qi_b200 import dit as D

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

SMALL = D.DiTConfig(layers=2, heads=4, head_dim=128, ctx_tokens=128, tokens_per_frame=120,
                    experts=(D.ExpertSpec("video", 512, 1024, 240), D.ExpertSpec("action", 256, 512, 32)))


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


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("cfg", [SMALL, D.DiTConfig(layers=1)], ids=["small", "cfg5_one_layer"])
def test_runner_matches_module_forward(cfg):
    model = D.build_mot_dit(cfg, device=DEV, seed=0)
    tokens, rope, ctx, t_mod, mask = D.make_step_inputs(cfg, DEV, seed=0)
    with torch.no_grad():
        ref = model(tokens, rope, ctx, t_mod)
        runner = D.DiTStepRunner(model)
        out = runner.step(tokens, rope, ctx, t_mod)
        for n in ref:
            assert torch.equal(out[n], ref[n]), (n, rel(out[n], ref[n]))
        masked = model(tokens, rope, ctx, t_mod, mask)
        for n in ref:
            assert rel(masked[n], ref[n]) < 2e-2, (n, rel(masked[n], ref[n]))


def test_graph_replay_bit_exact():
    model = D.build_mot_dit(SMALL, device=DEV, seed=1)
    tokens, rope, ctx, t_mod, _ = D.make_step_inputs(SMALL, DEV, seed=1)
    with torch.no_grad():
        runner = D.DiTStepRunner(model)
        eager = runner.step(tokens, rope, ctx, t_mod)
        runner.capture(tokens, rope, ctx, t_mod)
        for n, x in tokens.items():
            runner.static_in[0][n].copy_(x)
        out = runner.replay()
        torch.cuda.synchronize()
        for n in eager:
            assert torch.equal(out[n], eager[n]), n
