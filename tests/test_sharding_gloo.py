"""Tensor-parallel sharding on CPU ranks (``gloo``, world sizes 2 and 4).

The exchange logic of ``qi_b200.sharding`` runs unchanged.  The CPU oracle
stands in for the sm_100a kernels: a test backend for the column-parallel
local linear and a test ``ops`` object for the row-parallel one.  Every check
is bit-exact against the unsharded oracle linear:

* column parallel, INT8 W8A8, all three gather layouts;
* row parallel, INT8 W8A8, with and without a SmoothQuant ``input_scale``,
  on rows whose amax sits on one rank only (the MAX all-reduce of scales);
* a column-parallel FFN-up feeding a row-parallel FFN-down with GELU between
  them (the Megatron layout), against the single-rank FFN;
* the per-format weight slicing (INT8, FP8, W4A16, NVFP4 atoms), against
  quantizing the weight slice on its own.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from oracle import qi_oracle as O
from qi_b200 import sharding as S
from qi_b200.quantization.config import WeightActivationQuantConfig, WeightOnlyQuantConfig
from qi_b200.quantization.modules import WeightOnlyLinear
from qi_b200.quantization.quantize import quantize_linear_weight, quantize_nvfp4, sf_atom_layout


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


class OracleInt8Backend:
    """CPU stand-in for ``B200Backend.linear`` on INT8 W8A8 buffers."""

    def linear(self, x, qweight, scales, bias, gelu=False, **_):
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16)
        y, _, _, _ = O.int8_linear(bits(x2), qweight.numpy(), scales.reshape(-1).numpy(),
                                   None if bias is None else bits(bias.to(torch.bfloat16)))
        out = from_bits(y)
        if gelu:
            out = from_bits(O.f32_to_bf16(O.gelu_tanh(O.bf16_to_f32(y))))
        return out.reshape(*x.shape[:-1], out.shape[-1])


class OracleOps:
    """CPU stand-in for ``sharding.KernelOps``."""

    def row_scales(self, x):
        return torch.from_numpy(O.int8_row_scales(bits(x)))

    def quantize_given(self, x, s):
        return torch.from_numpy(O.quantize_int8_rowwise_given(bits(x), s.numpy()))

    def gemm_acc(self, q, w):
        return torch.from_numpy(O.int8_gemm_acc(q.numpy(), w.numpy()).astype(np.int32))

    def epilogue(self, acc, s, ws, bias, gelu):
        y = O.int8_epilogue(acc.numpy().astype(np.int64), s.numpy(), ws.numpy(),
                            None if bias is None else bits(bias))
        if gelu:
            y = O.f32_to_bf16(O.gelu_tanh(O.bf16_to_f32(y)))
        return from_bits(y)


INT8_CFG = WeightActivationQuantConfig(enabled=True, quant_dtype="int", backend="b200",
                                       activation_granularity="per_token", weight_granularity="per_channel")


def int8_layer(N, K, seed, bias=True, input_scale=False, gelu=False):
    g = torch.Generator().manual_seed(seed)
    lin = nn.Linear(K, N, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        if bias:
            lin.bias.copy_(torch.randn(N, generator=g) * 0.01)
    q = quantize_linear_weight(lin.weight.detach(), INT8_CFG)
    layer = WeightOnlyLinear.from_linear(lin, q, INT8_CFG, OracleInt8Backend())
    layer.bias = None if layer.bias is None else layer.bias.to(torch.bfloat16)
    if input_scale:
        layer.input_scale = (torch.rand(K, generator=g) + 0.5).float()
    layer.fuse_gelu = gelu
    return layer


def activations(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    x[::3, 5] *= 40.0          # row amax on the first rank's slice
    x[1::3, K - 7] *= 40.0     # row amax on the last rank's slice
    return x.to(torch.bfloat16)


def unsharded(layer, x):
    xs = x if layer.input_scale is None else x / layer.input_scale.to(x.dtype)
    y, _, _, _ = O.int8_linear(bits(xs), layer.qweight.numpy(), layer.scales.reshape(-1).numpy(),
                               None if layer.bias is None else bits(layer.bias))
    if layer.fuse_gelu:
        y = O.f32_to_bf16(O.gelu_tanh(O.bf16_to_f32(y)))
    return y


# ---------------------------------------------------------------------------
# distributed workers
# ---------------------------------------------------------------------------


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _column_worker(rank, world, port):
    _init(rank, world, port)
    try:
        M, N, K = 37, 64 * world, 96
        layer = int8_layer(N, K, seed=1)
        x = activations(M, K, seed=2)
        ref = unsharded(layer, x)
        full = S.ColumnShardedLinear(layer, gather=S.GATHER_FULL)
        np.testing.assert_array_equal(bits(full(x)), ref)
        x3 = x.reshape(1, M, K)
        np.testing.assert_array_equal(bits(full(x3)).reshape(M, N), ref)
        rank_major = S.ColumnShardedLinear(layer, gather=S.GATHER_RANK_MAJOR)(x)
        assert rank_major.shape == (world, M, N // world)
        np.testing.assert_array_equal(bits(rank_major.permute(1, 0, 2).reshape(M, N)), ref)
        local = S.ColumnShardedLinear(layer, gather=S.GATHER_NONE)(x)
        n = N // world
        np.testing.assert_array_equal(bits(local), ref[:, rank * n:(rank + 1) * n])
    finally:
        dist.destroy_process_group()


def _row_worker(rank, world, port):
    _init(rank, world, port)
    try:
        for input_scale in (False, True):
            M, N, K = 29, 48, 64 * world
            layer = int8_layer(N, K, seed=3 + input_scale, input_scale=input_scale)
            x = activations(M, K, seed=4)
            ref = unsharded(layer, x)
            row = S.RowShardedInt8Linear(layer, ops=OracleOps())
            y = row(S.local_k_slice(x))
            np.testing.assert_array_equal(bits(y), ref)
        # empty batch: the collectives still run with zero-size tensors
        y0 = row(S.local_k_slice(x[:0]))
        assert y0.shape == (0, N)
    finally:
        dist.destroy_process_group()


def _ffn_worker(rank, world, port):
    _init(rank, world, port)
    try:
        M, D, F = 21, 64, 32 * world * 2
        up = int8_layer(F, D, seed=5, gelu=True)
        down = int8_layer(D, F, seed=6)
        x = activations(M, D, seed=7)
        h_ref = unsharded(up, x)
        y_ref = unsharded(down, from_bits(h_ref))
        up_tp = S.ColumnShardedLinear(up, gather=S.GATHER_NONE)
        down_tp = S.RowShardedInt8Linear(down, ops=OracleOps())
        y = down_tp(up_tp(x))
        np.testing.assert_array_equal(bits(y), y_ref)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("worker", [_column_worker, _row_worker, _ffn_worker],
                         ids=["column", "row", "ffn"])
def test_tensor_parallel_gloo(worker, world):
    mp.spawn(worker, args=(world, _free_port()), nprocs=world, join=True)


# ---------------------------------------------------------------------------
# weight slicing per format (no process group needed)
# ---------------------------------------------------------------------------


def _linear(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    lin = nn.Linear(K, N)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(N, generator=g) * 0.01)
    return lin


def _sub_linear(lin, lo, hi):
    sub = nn.Linear(lin.in_features, hi - lo)
    with torch.no_grad():
        sub.weight.copy_(lin.weight[lo:hi])
        sub.bias.copy_(lin.bias[lo:hi])
    return sub


def _assert_same_buffers(a: WeightOnlyLinear, b: WeightOnlyLinear):
    for name in ("qweight", "scales", "zeros", "qweight_packed", "scale_factors", "weight_global_scale",
                 "weight_scale", "weight_fp8", "bias"):
        ta, tb = getattr(a, name), getattr(b, name)
        assert (ta is None) == (tb is None), name
        if ta is not None:
            assert ta.shape == tb.shape, (name, ta.shape, tb.shape)
            assert torch.equal(ta, tb), name


@pytest.mark.parametrize("fmt", ["int8", "fp8", "w4a16", "nvfp4"])
@pytest.mark.parametrize("world", [2, 4])
def test_column_shard_buffers_match_slice_quantization(fmt, world):
    N, K = 512, 256
    lin = _linear(N, K, seed=11)
    if fmt == "int8":
        cfg = INT8_CFG
    elif fmt == "fp8":
        cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="fp8", backend="b200",
                                          activation_granularity="per_token", weight_granularity="per_channel")
    elif fmt == "w4a16":
        cfg = WeightOnlyQuantConfig(enabled=True, algo="rtn", bits=4, group_size=128, symmetric=False,
                                    backend="b200")
    else:
        cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="nvfp4", bits=4, activation_bits=4,
                                          backend="b200", activation_granularity="per_token")
    full = WeightOnlyLinear.from_linear(lin, quantize_linear_weight(lin.weight.detach(), cfg), cfg, None)
    n = N // world
    for r in range(world):
        shard = S.column_shard_buffers(full, r, world)
        sub = _sub_linear(lin, r * n, (r + 1) * n)
        if fmt == "nvfp4":
            # the global scale is per tensor: quantize the slice with the full tensor's g
            packed, sf, g = quantize_nvfp4(sub.weight.detach(), global_scale=full.weight_global_scale)
            assert torch.equal(shard.qweight_packed, packed)
            assert torch.equal(shard.scale_factors, sf_atom_layout(sf))
            assert torch.equal(shard.weight_global_scale, full.weight_global_scale)
            continue
        expect = WeightOnlyLinear.from_linear(sub, quantize_linear_weight(sub.weight.detach(), cfg), cfg, None)
        _assert_same_buffers(shard, expect)
        assert shard.out_features == n and shard.in_features == K


def test_shard_shape_errors():
    lin = _linear(96, 64, seed=12)
    full = WeightOnlyLinear.from_linear(lin, quantize_linear_weight(lin.weight.detach(), INT8_CFG), INT8_CFG, None)
    with pytest.raises(ValueError):
        S.column_shard_buffers(full, 0, 5)  # 96 % 5
    cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="nvfp4", bits=4, activation_bits=4,
                                      backend="b200", activation_granularity="per_token")
    nv = WeightOnlyLinear.from_linear(lin, quantize_linear_weight(lin.weight.detach(), cfg), cfg, None)
    with pytest.raises(ValueError):
        S.column_shard_buffers(nv, 0, 2)  # 48 rows per rank: not whole 128-row scale atoms


# ---------------------------------------------------------------------------
# sequence-parallel DiT step (video tokens sharded, K/V all-gathered)
# ---------------------------------------------------------------------------


class OracleKernels:
    """CPU stand-in for ``qi_b200.kernels`` in ``DiTStepRunner``."""

    @staticmethod
    def int8_linear(x2, w, s, b, gelu=False):
        y, _, _, _ = O.int8_linear(bits(x2), w.numpy(), s.numpy(), bits(b))
        if gelu:
            y = O.f32_to_bf16(O.gelu_tanh(O.bf16_to_f32(y)))
        return from_bits(y)


def _dit_worker(rank, world, port, out_dir):
    from qi_b200 import dit as D

    _init(rank, world, port)
    try:
        cfg = D.DiTConfig(layers=2, heads=2, head_dim=24, ctx_tokens=8, tokens_per_frame=24,
                          experts=(D.ExpertSpec("video", 32, 64, 96), D.ExpertSpec("action", 16, 32, 4)))
        model = D.build_mot_dit(cfg, device="cpu", seed=3)
        tokens, rope, ctx, t_mod, _ = D.make_step_inputs(cfg, "cpu", seed=3)
        # the tensor-op form of the step (the fused form needs CUDA streams)
        single = D.DiTStepRunner(model, fused=False)
        single.K = OracleKernels
        ref = single.step(tokens, rope, ctx, t_mod)
        tp = D.DiTStepRunner(model, group=dist.group.WORLD, fused=False)
        tp.K = OracleKernels
        tok, rp = tp.shard(tokens, rope)
        out = tp.step(tok, rp, ctx, t_mod)
        lo, hi = tp.video_offset, tp.video_offset + tp.video_local
        torch.save({"video": out["video"], "video_ref": ref["video"][:, lo:hi], "action": out["action"],
                    "action_ref": ref["action"]}, os.path.join(out_dir, f"dit{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_dit_sequence_parallel_gloo(world, tmp_path):
    """Each rank's video rows (and the replicated action rows) match the
    single-process step.  Token shards cross the first-frame boundary at
    world 4 (24 first-frame tokens, 24 tokens per rank)."""
    mp.spawn(_dit_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        d = torch.load(tmp_path / f"dit{r}.pt")
        for n in ("video", "action"):
            a, b = d[n].float(), d[n + "_ref"].float()
            assert a.shape == b.shape
            err = ((a - b).norm() / b.norm()).item()
            assert err < 1e-2, (r, n, err)
