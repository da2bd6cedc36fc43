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
  ReferenceBackend.linear  src/qi/quantization/backends/reference.py:48-91
  WeightOnlyLinear         src/qi/quantization/modules.py:7-133
  replace_linear_with_weight_only src/qi/quantization/swap.py:126-150
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
    pkg = types.ModuleType("qi")
    pkg.__path__ = [str(ref_root / "src" / "qi")]
    sys.modules["qi"] = pkg
    import qi.quantization as qq  # noqa: F401
    from qi.quantization import quantize as Q
    from qi.quantization.backends import flashrt_fp8_ops as F8
    from qi.quantization.backends.reference import ReferenceBackend
    from qi.quantization.config import WeightActivationQuantConfig, WeightOnlyQuantConfig
    from qi.quantization.swap import replace_linear_with_weight_only

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


if __name__ == "__main__":
    main()
