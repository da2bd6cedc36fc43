"""Head-parallel (tensor-parallel) DiT step on CPU ranks (``gloo``, world
sizes 2 and 4): ``DiTStepRunner(partition="heads")`` with the CPU kernel
stand-ins of ``tests/cpu_kernels.py``.  Every rank's output tokens must be
bit-identical to the same step run by one rank, which checks the weight
slicing (q/k/v, cross-q, cross-k/v and ffn.0 by rows; o, cross-o and ffn.2
by input columns), the per-head RMS-sum gathers, and the exact row-parallel
reductions (MAX of the per-token INT8 scales, SUM of int32 partial sums).
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qi_b200 import dit as D

CFG = D.DiTConfig(layers=2, heads=4, head_dim=32, ctx_tokens=8, tokens_per_frame=24,
                  experts=(D.ExpertSpec("video", 128, 256, 48), D.ExpertSpec("action", 64, 128, 4)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(group):
    import cpu_kernels

    model = D.build_mot_dit(CFG, device="cpu", seed=3)
    tokens, rope, ctx, t_mod, _ = D.make_step_inputs(CFG, "cpu", seed=3)
    runner = D.DiTStepRunner(model, group=group, partition="heads", kernels=cpu_kernels)
    return runner.step(tokens, rope, ctx, t_mod)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = _step(dist.group.WORLD)
        torch.save({n: v.clone() for n, v in out.items()}, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_parallel_step_bit_identical_to_one_rank(world, tmp_path):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    torch.set_num_threads(1)
    ref = _step(None)
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        got = torch.load(tmp_path / f"rank{r}.pt")
        for n in ref:
            assert torch.equal(got[n], ref[n]), (r, n, (got[n].float() - ref[n].float()).abs().max().item())
