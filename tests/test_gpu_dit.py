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
        out = D.DiTStepRunner(model, fused=False).step(tokens, rope, ctx, t_mod)
        for n in ref:
            assert torch.equal(out[n], ref[n]), (n, rel(out[n], ref[n]))
        # fused row kernels: LayerNorm / RMSNorm reductions in another order
        # (an occasional 1-ulp bf16 difference, then INT8 re-quantization)
        fused = D.DiTStepRunner(model).step(tokens, rope, ctx, t_mod)
        for n in ref:
            assert rel(fused[n], ref[n]) < 2e-2, (n, rel(fused[n], ref[n]))
        masked = model(tokens, rope, ctx, t_mod, mask)
        for n in ref:
            assert rel(masked[n], ref[n]) < 2e-2, (n, rel(masked[n], ref[n]))


def _mot_fixture():
    """The reference MoT step fixture (tests/golden/mot_step_small_int8.npz):
    config, unquantized weights, inputs, joint mask and the reference's
    outputs in fp32 and bf16."""
    import json
    from pathlib import Path

    import numpy as np

    f = np.load(Path(__file__).resolve().parent / "golden" / "mot_step_small_int8.npz")
    c = json.loads(bytes(f["meta"]).decode())
    cfg = D.DiTConfig(layers=c["layers"], heads=c["heads"], head_dim=c["head_dim"], ctx_tokens=c["ctx"],
                      tokens_per_frame=c["tokens_per_frame"],
                      experts=tuple(D.ExpertSpec(n, h, ff, t) for n, h, ff, t in c["experts"]))

    def bf(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)

    state = {k[3:]: bf(f[k]).float() for k in f.files if k.startswith("w::")}
    names = [e.name for e in cfg.experts]
    inputs = ({n: bf(f["tok_" + n]).to(DEV) for n in names}, {n: torch.from_numpy(f["rope_" + n]).to(DEV) for n in names},
              {n: bf(f["ctx_" + n]).to(DEV) for n in names}, {n: bf(f["tmod_" + n]).to(DEV) for n in names})
    ref32 = {n: torch.from_numpy(f["y_f32_" + n]).to(DEV) for n in names}
    ref16 = {n: bf(f["y_bf16_" + n]).to(DEV) for n in names}
    return cfg, state, inputs, torch.from_numpy(f["mask"]).to(DEV), ref32, ref16


def test_step_vs_reference_mot_forward():
    """The DiT step against the reference's own MoT.forward (mot.py:465-574,
    blocks wan_video_dit.py:147-268) on the same weights and inputs, with the
    reference's INT8 W8A8 ReferenceBackend behind every Linear.  Module path,
    unfused runner and fused runner (row kernels, CUDA graph) all stay within
    2.5e-2 rel-Frobenius of the reference in fp32 and in bf16; the reference's
    own bf16 and fp32 runs differ by about 1.2e-2 (measured), the noise floor
    of bf16 activations, and a CPU emulation of this path with the INT8 kernel
    semantics lands 1.1e-2 from the fp32 reference.  Each sublayer moves the
    residual visibly (weights 1/sqrt(fan_in)), so a wiring error (a wrong
    modulation chunk, gate, norm or mask block) shows as an O(1) error; the
    same bound is also asserted on the residual update alone (y - x)."""
    cfg, state, inputs, mask, ref32, ref16 = _mot_fixture()
    model = D.build_mot_dit(cfg, device=DEV, state_dict=state)
    tok = inputs[0]
    with torch.no_grad():
        outs = {"module": model(*inputs), "module_masked": model(*inputs, mask),
                "runner": D.DiTStepRunner(model, fused=False).step(*inputs)}
        r = D.DiTStepRunner(model)
        outs["runner_fused"] = r.step(*inputs)
        r.capture(*inputs, warmup=1)
        outs["runner_graph"] = {n: v.clone() for n, v in r.replay().items()}
    report = {}
    for path, y in outs.items():
        for n in y:
            yf = y[n].float().reshape(ref32[n].shape)
            upd = yf - tok[n].float()
            e = (rel(yf, ref32[n]), rel(yf, ref16[n]), rel(upd, ref32[n] - tok[n].float()))
            report[(path, n)] = e
            assert max(e) < 2.5e-2, (path, n, e)
    print("MoT fixture (vs ref fp32, vs ref bf16, update vs ref fp32):",
          {f"{p}/{n}": tuple(round(v, 4) for v in e) for (p, n), e in report.items()})


def _bf16_chain(x, y, gate, ln_w, ln_b, s1, sh, eps):
    """The reference's bf16 tensor ops (GateModule, LayerNorm, modulate)."""
    if y is not None:
        x = x + (gate * y if gate is not None else y)
    n = torch.nn.functional.layer_norm(x, (x.shape[-1],), ln_w, ln_b, eps)
    if s1 is not None:
        n = n * s1 + sh
    return x, n


@pytest.mark.parametrize("D_,gated,affine,mod", [(3072, True, False, True), (3072, False, True, False),
                                                 (1024, False, False, True), (4096, True, True, True)])
def test_resid_ln_quant_matches_tensor_ops(D_, gated, affine, mod):
    from qi_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(D_)
    M = 257
    bf = torch.bfloat16
    x = (torch.randn(M, D_, generator=g, device=DEV) * 2).to(bf)
    y = torch.randn(M, D_, generator=g, device=DEV).to(bf)
    gate = (torch.randn(D_, generator=g, device=DEV) * 0.5).to(bf) if gated else None
    w = (1 + 0.1 * torch.randn(D_, generator=g, device=DEV)).to(bf) if affine else None
    b = (0.1 * torch.randn(D_, generator=g, device=DEV)).to(bf) if affine else None
    s1 = (1 + 0.2 * torch.randn(D_, generator=g, device=DEV)).to(bf) if mod else None
    sh = (0.2 * torch.randn(D_, generator=g, device=DEV)).to(bf) if mod else None
    x_ref, n_ref = _bf16_chain(x, y, gate, w, b, s1, sh, 1e-6)
    xk = x.clone()
    xn = torch.empty_like(x)
    q, s = K.resid_ln_quant(xk, y, gate=gate, ln_w=w, ln_b=b, mod_scale1=s1, mod_shift=sh, xn=xn)
    assert torch.equal(xk, x_ref)                        # residual update: elementwise, bit-exact
    # LayerNorm statistics reduce in another order: a few elements differ by
    # an ulp or two of bf16 (after modulate, relative to the operands' size)
    diff = (xn.float() - n_ref.float()).abs()
    assert (diff <= n_ref.float().abs() * 2 ** -6 + 2 ** -8).all()
    assert (diff > 0).float().mean() < 0.02
    q_ref, s_ref = K.quantize_int8_rowwise(xn)        # codes from the kernel's own bf16 row
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)


def test_rms_rope_matches_tensor_ops():
    from qi_b200 import kernels as K

    cfg = D.CFG5
    spec = cfg.experts[0]
    g = torch.Generator(device=DEV).manual_seed(5)
    M, a = spec.tokens, cfg.attn_dim
    qkv = torch.randn(M, 3 * a, generator=g, device=DEV).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(a, generator=g, device=DEV)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(a, generator=g, device=DEV)).to(torch.bfloat16)
    rope = D.rope_tables(cfg, spec, DEV)
    qn, kn = K.rms_rope([qkv[:, :a], qkv[:, a:2 * a]], [wq, wk], rope, cfg.head_dim, cfg.eps)
    for got, src, w in ((qn, qkv[:, :a], wq), (kn, qkv[:, a:2 * a], wk)):
        norm = D.RMSNorm(a, cfg.eps).to(DEV)
        norm.weight.data = w
        ref = D.rope_apply(norm(src.unsqueeze(0)), rope, cfg.heads)[0]
        # the RMS reduction runs in another order: an occasional 1-ulp bf16
        # difference before RoPE, which the rotation mixes into both outputs
        # of the pair (absolute bound, outputs are O(1) after the norm)
        diff = (got.float() - ref.float()).abs()
        assert diff.max().item() <= 2 ** -5, diff.max().item()
        assert (diff > 0).float().mean().item() < 0.05


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
@pytest.mark.parametrize("a,head_dim,rope", [(3072, 128, True), (3072, 128, False), (1024, 128, True),
                                             (128, 32, True)])
def test_rms_head_partials_bit_identical_to_unsplit(ranks, a, head_dim, rope):
    """Head-parallel RMSNorm: each of `ranks` emulated ranks (a contiguous
    slice of whole heads) computes its per-head sums, the sums are gathered
    rank-major, and each rank normalizes its slice.  The result is the same
    bytes as the unsplit kernel's, for q and k together, with and without
    RoPE."""
    from qi_b200 import kernels as K

    heads = a // head_dim
    if heads % ranks:
        pytest.skip("heads do not split")
    g = torch.Generator(device=DEV).manual_seed(a + ranks)
    M = 777
    qk = torch.randn(M, 2 * a, generator=g, device=DEV).to(torch.bfloat16) * 3
    w = [(1 + 0.1 * torch.randn(a, generator=g, device=DEV)).to(torch.bfloat16) for _ in range(2)]
    tab = None
    if rope:
        ang = torch.rand(M, head_dim // 2, generator=g, device=DEV) * 6.28
        tab = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    full = K.rms_rope([qk[:, :a], qk[:, a:]], w, tab, head_dim)
    al = a // ranks
    parts = torch.cat([K.rms_head_partials([qk[:, r * al:(r + 1) * al], qk[:, a + r * al:a + (r + 1) * al]],
                                           head_dim).unsqueeze(0) for r in range(ranks)], 0)
    for r in range(ranks):
        sl = slice(r * al, (r + 1) * al)
        got = K.rms_rope_partials([qk[:, r * al:(r + 1) * al], qk[:, a + r * al:a + (r + 1) * al]],
                                  [w[0][sl].contiguous(), w[1][sl].contiguous()], tab, head_dim, parts)
        for i in range(2):
            assert torch.equal(got[i], full[i][:, sl]), (r, i)


def test_head_parallel_plan_on_one_gpu_matches_fused():
    """The head-parallel plan (row-parallel o / cross-o / ffn.2 through raw
    int32 accumulators and the standalone epilogue, RMSNorm from per-head
    sums) run with one rank gives the fused single-GPU step's bytes."""
    model = D.build_mot_dit(SMALL, device=DEV, seed=2)
    tokens, rope, ctx, t_mod, _ = D.make_step_inputs(SMALL, DEV, seed=2)
    with torch.no_grad():
        ref = D.DiTStepRunner(model).step(tokens, rope, ctx, t_mod)
        tp = D.DiTStepRunner(model, partition="heads").step(tokens, rope, ctx, t_mod)
    for n in ref:
        assert torch.equal(tp[n], ref[n]), (n, rel(tp[n], ref[n]))


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
