"""DiT-step harness on CPU: structure, op count, mask and RoPE semantics.

The quantized GEMMs need a B200 (``tests/test_gpu_dit.py``).  These checks
run on CPU with plain fp32 layers:

* the op count of BASELINE config 5 (2.733e13 INT8 ops per step);
* the INT8 swap selects exactly the 10 target Linears of every block and
  expert (``config.py:7-18``, ``swap.py:49-102`` of the reference);
* the block form of the first_frame_causal joint attention equals SDPA over
  the concatenated tokens with the boolean mask of ``fastwam.py:914-935``;
* RoPE in fp32 matches the reference's fp64 complex product
  (``wan_video_dit.py:55-61``) to bf16 rounding;
* the module-structured forward runs and keeps token shapes.
"""

import pytest
import torch

from qi_b200 import dit as D

TINY = D.DiTConfig(layers=2, heads=2, head_dim=24, ctx_tokens=8, tokens_per_frame=24,
                   experts=(D.ExpertSpec("video", 32, 64, 48), D.ExpertSpec("action", 16, 32, 4)))


def test_cfg5_op_count():
    assert abs(D.CFG5.linear_ops() - 2.733e13) / 2.733e13 < 1e-3
    assert D.CFG5.attn_dim == 3072


def test_int8_swap_selects_ten_linears_per_block():
    m = D.build_mot_dit(TINY, device="cpu", quantize=True)
    assert D.count_quantized_linears(m) == 10 * 2 * TINY.layers
    names = {n.split(".", 4)[-1] for n, mod in m.named_modules() if type(mod).__name__ == "WeightOnlyLinear"}
    assert names == {"self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o", "cross_attn.q", "cross_attn.k",
                     "cross_attn.v", "cross_attn.o", "ffn.0", "ffn.2"}
    # ffn.0 carries the GELU in its epilogue; the model's GELU became an identity
    blk = m.mixtures["video"].blocks[0]
    assert blk.ffn[0].fuse_gelu and isinstance(blk.ffn[1], torch.nn.Identity)


@pytest.mark.parametrize("sv,t", [(48, 24), (24, 24), (60, 12)])
def test_block_attention_equals_masked(sv, t):
    cfg = D.DiTConfig(layers=1, heads=2, head_dim=16, tokens_per_frame=t,
                      experts=(D.ExpertSpec("video", 32, 64, sv), D.ExpertSpec("action", 16, 32, 5)))
    g = torch.Generator().manual_seed(sv + t)
    q = {n: torch.randn(1, e.tokens, 32, generator=g, dtype=torch.float64) for n, e in
         zip(("video", "action"), cfg.experts)}
    k = {n: torch.randn_like(x) for n, x in q.items()}
    v = {n: torch.randn_like(x) for n, x in q.items()}
    out = D.joint_attention_blocks(q, k, v, cfg)
    mask = D.first_frame_causal_mask(cfg, sv, 5, "cpu")
    ref = D.attention(torch.cat([q["video"], q["action"]], 1), torch.cat([k["video"], k["action"]], 1),
                      torch.cat([v["video"], v["action"]], 1), 2, mask)
    torch.testing.assert_close(torch.cat([out["video"], out["action"]], 1), ref, rtol=1e-12, atol=1e-12)


def test_rope_matches_complex_product():
    spec = TINY.experts[0]
    tab = D.rope_tables(TINY, spec, "cpu")
    x = torch.randn(1, spec.tokens, TINY.attn_dim).to(torch.bfloat16)
    got = D.rope_apply(x, tab, TINY.heads)
    # reference form: complex fp64 product of (even, odd) pairs with polar(1, angle)
    ang = torch.atan2(tab[..., 1].double(), tab[..., 0].double())
    xc = torch.view_as_complex(x.double().view(1, spec.tokens, TINY.heads, -1, 2).contiguous())
    ref = torch.view_as_real(xc * torch.polar(torch.ones_like(ang), ang)[None, :, None]).flatten(2)
    assert (got.float() - ref.to(torch.bfloat16).float()).abs().max() <= 2 ** -7 * ref.abs().max()


def test_module_forward_shapes():
    m = D.build_mot_dit(TINY, device="cpu", quantize=False, dtype=torch.float32)
    tokens, rope, ctx, t_mod, mask = D.make_step_inputs(TINY, "cpu", dtype=torch.float32)
    out = m(tokens, rope, ctx, t_mod, mask)
    for n, x in tokens.items():
        assert out[n].shape == x.shape and torch.isfinite(out[n]).all()
