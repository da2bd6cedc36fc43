"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs hongzicong/qi's own quantization code (its Python package, imported
from a source checkout) on seeded inputs and stores inputs + outputs as
small ``.npz`` files next to this script.  The reference's package
``qi/__init__.py`` imports hydra (absent here), so a bare ``qi`` package
whose ``__path__`` points at ``src/qi`` is registered first and only
``qi.quantization`` is imported.

Usage:  python tests/golden/make_golden.py --reference <path to qi checkout>

Reference functions exercised (paths inside the reference project):
  quantize_weight_rtn      src/qi/quantization/quantize.py:32-78
  dequantize_weight        src/qi/quantization/quantize.py:81-119
  quantize_to_fp8_e4m3     src/qi/quantization/backends/flashrt_fp8_ops.py:43-48
                           (also applied to one row at a time: per-token / per-channel FP8)
  dequantize_fp8_e4m3      src/qi/quantization/backends/flashrt_fp8_ops.py:51-53
  ReferenceBackend.linear  src/qi/quantization/backends/reference.py:48-91
  WeightOnlyLinear         src/qi/quantization/modules.py:7-133
  replace_linear_with_weight_only src/qi/quantization/swap.py:126-150
  MoT.forward              src/qi/models/wan22/mot.py:465-574 (blocks: wan_video_dit.py:147-268)

The MoT step fixture needs ``qi.models.wan22`` too: bare ``qi.utils``,
``qi.models``, ``qi.models.wan22`` and ``qi.models.wan22.helpers`` packages
are registered so that only the modules the step needs are imported.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
import types
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from qi_b200.synthetic import CFG_INT8, CFG_W4A16, make_linear_inputs, make_small_case  # noqa: E402


def import_reference(ref_root: Path):
    src = ref_root / "src" / "qi"
    for name, sub in (("qi", ""), ("qi.utils", "utils"), ("qi.models", "models"), ("qi.models.wan22", "models/wan22"),
                      ("qi.models.wan22.helpers", "models/wan22/helpers")):
        pkg = types.ModuleType(name)
        pkg.__path__ = [str(src / sub) if sub else str(src)]
        sys.modules[name] = pkg
    import qi.quantization as qq  # noqa: F401
    from qi.quantization import quantize as Q
    from qi.quantization.backends import flashrt_fp8_ops as F8
    from qi.quantization.backends.reference import ReferenceBackend
    from qi.quantization.config import WeightActivationQuantConfig, WeightOnlyQuantConfig
    from qi.quantization.swap import replace_linear_with_weight_only  # noqa: F401

    return types.SimpleNamespace(
        Q=Q, F8=F8, ReferenceBackend=ReferenceBackend,
        WAQ=WeightActivationQuantConfig, WOQ=WeightOnlyQuantConfig,
        swap=replace_linear_with_weight_only,
    )


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_linear(R, x, qweight, scales, zeros, bits, group, sym, bias, per_token):
    be = R.ReferenceBackend()
    return be.linear(
        x=x, qweight=qweight, scales=scales, zeros=zeros, bias=bias, bits=bits,
        group_size=group, symmetric=sym, input_scale=None, keep_output_dtype="input",
        activation_granularity="per_token" if per_token else None,
        weight_granularity="per_channel" if per_token else None,
    )


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    R = import_reference(args.reference)
    out = {}

    # ---- weight RTN: int8 symmetric per-channel, int4 asymmetric g128, ragged groups
    for name, (N, K, bits, group, sym) in {
        "rtn_int8_sym_pc": (96, 256, 8, -1, True),
        "rtn_int4_asym_g128": (96, 512, 4, 128, False),
        "rtn_int4_sym_g64": (64, 256, 4, 64, True),
        "rtn_int4_asym_ragged": (48, 200, 4, 128, False),
        "rtn_int8_asym_g32": (32, 96, 8, 32, False),
    }.items():
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 1000)
        w = torch.randn(N, K, generator=g) * 0.02
        if name == "rtn_int4_asym_ragged":
            w[3] = 0.0  # constant row: exercises the 1e-8 scale floor
        q, s, z = R.Q.quantize_weight_rtn(w, bits=bits, group_size=group, symmetric=sym)
        deq_bf16 = R.Q.dequantize_weight(q, s, z, bits, group, sym, dtype=torch.bfloat16)
        deq_f32 = R.Q.dequantize_weight(q, s, z, bits, group, sym, dtype=torch.float32)
        rec = dict(w=w.numpy(), qweight=q.numpy(), scales=s.numpy(),
                   deq_bf16=bf16_bits(deq_bf16), deq_f32=deq_f32.numpy(),
                   meta=np.array([N, K, bits, group, int(sym)], np.int64))
        if z is not None:
            rec["zeros"] = z.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **rec)

    # ---- FP8 per-tensor quantizer
    g = torch.Generator().manual_seed(7)
    xf = torch.randn(64, 256, generator=g) * 3.0
    xf[0, :5] = torch.tensor([0.0, -0.0, 1e-9, -1e-9, 5.0])
    qb, sc = R.F8.quantize_to_fp8_e4m3(xf)
    np.savez_compressed(HERE / "fp8_per_tensor.npz", x=xf.numpy(), q=qb.numpy(), s=sc.numpy())

    # ---- ReferenceBackend.linear: INT8 W8A8 (fp32 and bf16 inputs), with an
    #      all-zero token row and outlier columns, and INT4 weight-only.
    for name, (M, N, K) in {"linear_int8_M17_N192_K256": (17, 192, 256),
                            "linear_int8_M1_N64_K128": (1, 64, 128)}.items():
        x, w, b = make_small_case(M, N, K, seed=3, outlier_frac=0.02)
        x = x.clone()
        if M > 2:
            x[2] = 0
        q, s, _ = R.Q.quantize_weight_rtn(w, bits=8, group_size=-1, symmetric=True)
        y32 = ref_linear(R, x.float(), q, s, None, 8, -1, True, b.float(), True)
        y16 = ref_linear(R, x, q, s, None, 8, -1, True, b, True)
        np.savez_compressed(HERE / f"{name}.npz", x=bf16_bits(x), w=w.numpy(), bias=bf16_bits(b),
                            qweight=q.numpy(), scales=s.numpy(),
                            y_ref_f32in=y32.numpy(), y_ref_bf16in=bf16_bits(y16))

    x, w, b = make_small_case(9, 128, 384, seed=5)
    q, s, z = R.Q.quantize_weight_rtn(w, bits=4, group_size=128, symmetric=False)
    y16 = ref_linear(R, x, q, s, z, 4, 128, False, b, False)
    np.savez_compressed(HERE / "linear_w4a16_M9_N128_K384.npz", x=bf16_bits(x), w=w.numpy(),
                        bias=bf16_bits(b), qweight=q.numpy(), scales=s.numpy(), zeros=z.numpy(),
                        y_ref_bf16in=bf16_bits(y16))

    # ---- module swap through the reference's own API (WeightOnlyLinear)
    lin = torch.nn.Linear(128, 64)
    with torch.no_grad():
        g = torch.Generator().manual_seed(11)
        lin.weight.copy_(torch.randn(64, 128, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(64, generator=g) * 0.01)
    model = torch.nn.Module()
    model.ffn = torch.nn.Sequential(lin)
    cfg = R.WAQ(enabled=True, algo="rtn", quant_dtype="int", backend="reference",
                activation_granularity="per_token", weight_granularity="per_channel")
    R.swap(model, cfg)
    xm = torch.randn(5, 128, generator=g)
    ym = model.ffn[0](xm)
    np.savez_compressed(HERE / "module_int8_swap.npz", w=lin.weight.detach().numpy(),
                        bias=lin.bias.detach().numpy(), x=xm.numpy(), y=ym.detach().numpy(),
                        qweight=model.ffn[0].qweight.numpy(), scales=model.ffn[0].scales.numpy())

    fp8_per_token(R)
    w4a16_cfg3(R)
    mot_step(R)
    reference_checkpoints(R)

    # ---- hashes of the reference quantizer at the full BASELINE sizes
    _, w1, _ = make_linear_inputs(CFG_INT8)
    q1, s1, _ = R.Q.quantize_weight_rtn(w1, bits=8, group_size=-1, symmetric=True)
    _, w3, _ = make_linear_inputs(CFG_W4A16[1])
    q3, s3, z3 = R.Q.quantize_weight_rtn(w3, bits=4, group_size=128, symmetric=False)
    out["cfg1_int8_qweight"] = sha(q1.numpy())
    out["cfg1_int8_scales"] = sha(s1.numpy())
    out["cfg3_int4_qweight"] = sha(q3.numpy())
    out["cfg3_int4_scales"] = sha(s3.numpy())
    out["cfg3_int4_zeros"] = sha(z3.numpy())
    (HERE / "baseline_hashes.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote fixtures to", HERE)


def reference_checkpoints(R) -> None:
    """Quantized checkpoints written by the reference's own
    save_quantized_checkpoint (checkpoint.py:71-98): a model with a ``mot``
    whose FFN is weight-only INT4 (asymmetric g64, and symmetric g64), plus
    an input and the reference model's output (ReferenceBackend)."""
    from qi.quantization.checkpoint import save_quantized_checkpoint

    for sym in (False, True):
        g = torch.Generator().manual_seed(31 + sym)
        model = torch.nn.Module()
        model.mot = torch.nn.Module()
        model.mot.ffn = torch.nn.Sequential(torch.nn.Linear(128, 64), torch.nn.GELU(approximate="tanh"),
                                            torch.nn.Linear(64, 128))
        with torch.no_grad():
            for p in model.mot.parameters():
                p.copy_(torch.randn(p.shape, generator=g) * (0.05 if p.dim() == 2 else 0.01))
        cfg = R.WOQ(enabled=True, algo="rtn", bits=4, group_size=64, symmetric=sym, backend="reference")
        R.swap(model.mot, cfg)
        model.mot.to(torch.bfloat16)
        x = torch.randn(5, 128, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            y = model.mot.ffn(x)
        name = f"ckpt_ref_int4_{'sym' if sym else 'asym'}_g64"
        save_quantized_checkpoint(model, HERE / f"{name}.pt", cfg, source_payload={"optimizer": {"step": 1}},
                                  source_checkpoint="synthetic")
        np.savez_compressed(HERE / f"{name}_io.npz", x=bf16_bits(x), y=bf16_bits(y))


def fp8_rows(R, t: torch.Tensor):
    """The reference's per-tensor FP8 quantizer applied to each row as a
    one-row tensor: per-token (activations) / per-channel (weights) codes."""
    qs, ss = zip(*(R.F8.quantize_to_fp8_e4m3(t[i:i + 1]) for i in range(t.shape[0])))
    return torch.cat(qs, 0), torch.cat(ss, 0)


def fp8_per_token(R) -> None:
    """Per-token / per-channel FP8 W8A8 (BASELINE config 2's scheme) from the
    reference's own quantizer, and the reference-style dequantise-then-matmul
    output (reference.py:48-91's structure: dequantise both operands with
    dequantize_fp8_e4m3, F.linear in fp32, output in the input dtype), with
    and without the FFN's GELU(tanh) (wan_video_dit.py:244-245)."""
    M, N, K = 33, 256, 512
    x, w, b = make_small_case(M, N, K, seed=13, outlier_frac=0.01)
    x = x.clone()
    x[4] = 0  # all-zero token -> the 1e-12 scale floor
    qx, sx = fp8_rows(R, x)
    qw, sw = fp8_rows(R, w)
    xd = torch.cat([R.F8.dequantize_fp8_e4m3(qx[i], sx[i]).reshape(1, -1) for i in range(M)], 0)
    wd = torch.cat([R.F8.dequantize_fp8_e4m3(qw[i], sw[i]).reshape(1, -1) for i in range(N)], 0)
    y = torch.nn.functional.linear(xd, wd, b.float())
    yb = y.to(torch.bfloat16)
    yg = torch.nn.functional.gelu(yb.float(), approximate="tanh").to(torch.bfloat16)
    np.savez_compressed(HERE / "fp8_per_token_M33_N256_K512.npz", x=bf16_bits(x), w=w.numpy(), bias=bf16_bits(b),
                        qx=qx.numpy(), sx=sx.numpy(), qw=qw.numpy(), sw=sw.numpy(), y_ref=bf16_bits(yb),
                        y_ref_gelu=bf16_bits(yg))


def w4a16_cfg3(R) -> None:
    """ReferenceBackend.linear (bf16 input, INT4 asym g128) at BASELINE
    config 3's full weight (3072 x 3072) for M = 1 and M = 16.  Only the
    outputs are stored; the inputs are regenerated by qi_b200.synthetic
    (their hashes are stored to prove it)."""
    rec = {}
    for m in (1, 16):
        x, w, b = make_linear_inputs(CFG_W4A16[m])
        q, s, z = R.Q.quantize_weight_rtn(w, bits=4, group_size=128, symmetric=False)
        y = ref_linear(R, x, q, s, z, 4, 128, False, b, False)
        rec[f"y_M{m}"] = bf16_bits(y)
        rec[f"x_sha_M{m}"] = np.frombuffer(sha(bf16_bits(x)).encode(), np.uint8)
        rec[f"q_sha_M{m}"] = np.frombuffer(sha(q.numpy()).encode(), np.uint8)
    np.savez_compressed(HERE / "linear_w4a16_cfg3_M1_M16.npz", **rec)


# the small MoT used for the step fixture: 2 layers, 2 heads x 32, video 3
# frames x 8 tokens at hidden 128 / FFN 256, action 4 tokens at hidden 64 /
# FFN 128, 8 context tokens
MOT_SMALL = dict(layers=2, heads=2, head_dim=32, ctx=8, tokens_per_frame=8,
                 experts=(("video", 128, 256, 24), ("action", 64, 128, 4)))


def mot_step(R) -> None:
    """One MoT.forward of the reference (mot.py:465-574) with every target
    Linear swapped for the reference's INT8 W8A8 WeightOnlyLinear
    (ReferenceBackend, per-token activations), run on the CPU in bf16 and in
    fp32, on seeded weights and inputs.  Stores the unquantized weights, the
    inputs (RoPE as cos/sin of the reference's complex frequencies), the
    joint first_frame_causal mask and both outputs."""
    from qi.models.wan22.mot import MoT
    from qi.models.wan22.wan_video_dit import DiTBlock, precompute_freqs_cis

    c = MOT_SMALL
    g = torch.Generator().manual_seed(2024)

    class Expert(torch.nn.Module):
        def __init__(self, hidden, ffn):
            super().__init__()
            self.num_heads, self.attn_head_dim = c["heads"], c["head_dim"]
            self.blocks = torch.nn.ModuleList(
                DiTBlock(hidden, c["head_dim"], c["heads"], ffn, 1e-6) for _ in range(c["layers"]))

    mot = MoT({n: Expert(h, f) for n, h, f, _ in c["experts"]}, mot_checkpoint_mixed_attn=False)
    with torch.no_grad():   # bf16-valued master weights (stored as bf16 bits)
        for name, p in mot.named_parameters():
            if name.endswith("modulation"):
                v = torch.randn(p.shape, generator=g) / p.shape[-1] ** 0.5
            elif "norm" in name:   # RMSNorm / affine LayerNorm: near 1 (weights) and 0 (biases)
                v = (1.0 if name.endswith("weight") else 0.0) + 0.1 * torch.randn(p.shape, generator=g)
            elif name.endswith("weight"):   # 1/sqrt(fan_in): every sublayer changes the residual visibly
                v = torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5
            else:
                v = torch.randn(p.shape, generator=g) * 0.1
            p.copy_(v.bfloat16().float())
    state = {k: v.clone() for k, v in mot.state_dict().items()}
    cfg = R.WAQ(enabled=True, algo="rtn", quant_dtype="int", backend="reference",
                activation_granularity="per_token", weight_granularity="per_channel")
    R.swap(mot, cfg)
    n_q = sum(type(m).__name__ == "WeightOnlyLinear" for m in mot.modules())
    assert n_q == 10 * c["layers"] * len(c["experts"]), n_q
    mot.eval()

    sv, sa = c["experts"][0][3], c["experts"][1][3]
    t = min(c["tokens_per_frame"], sv)
    mask = torch.zeros((sv + sa, sv + sa), dtype=torch.bool)   # fastwam.py:914-935, first_frame_causal
    mask[:sv, :sv] = True
    mask[:t, t:sv] = False
    mask[sv:, sv:] = True
    mask[sv:, :t] = True
    fr = precompute_freqs_cis(c["head_dim"], 64)
    tok, ctx, tmod, freqs, rope = {}, {}, {}, {}, {}
    for name, hidden, _, n in c["experts"]:
        # inputs are bf16 values, so the fp32 and bf16 runs see the same numbers
        tok[name] = torch.randn(1, n, hidden, generator=g).bfloat16().float()
        ctx[name] = torch.randn(1, c["ctx"], hidden, generator=g).bfloat16().float()
        tmod[name] = (torch.randn(1, 6, hidden, generator=g) * 0.5).bfloat16().float()
        off = 0 if name == "video" else 7   # action positions differ from video's
        freqs[name] = fr[off:off + n].unsqueeze(1)
        rope[name] = torch.stack([freqs[name].real, freqs[name].imag], -1).reshape(n, -1, 2).double()

    out = {}
    # fp32 first: casting the model to bf16 also rounds its fp32 scale buffers
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        m = mot.to(dt)
        with torch.no_grad():
            y = m({k: v.to(dt) for k, v in tok.items()}, mask, freqs,
                  {k: {"context": v.to(dt), "mask": None} for k, v in ctx.items()},
                  {k: v.to(dt) for k, v in tmod.items()})
        for k, v in y.items():
            out[f"y_{tag}_{k}"] = bf16_bits(v) if dt == torch.bfloat16 else v.float().numpy()
    rec = {f"w::{k}": bf16_bits(v.bfloat16()) for k, v in state.items()}
    for k in tok:
        rec[f"tok_{k}"] = bf16_bits(tok[k].to(torch.bfloat16))
        rec[f"ctx_{k}"] = bf16_bits(ctx[k].to(torch.bfloat16))
        rec[f"tmod_{k}"] = bf16_bits(tmod[k].to(torch.bfloat16))
        rec[f"rope_{k}"] = rope[k].float().numpy()
    rec["mask"] = mask.numpy()
    rec["meta"] = np.frombuffer(json.dumps(c).encode(), np.uint8)
    np.savez_compressed(HERE / "mot_step_small_int8.npz", **rec, **out)


if __name__ == "__main__":
    main()
