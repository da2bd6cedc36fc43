"""CPU stand-ins for the ``qi_b200.kernels`` functions the DiT step calls
(TEST INFRASTRUCTURE ONLY).

They let the multi-rank logic of ``DiTStepRunner`` (which tensors are sliced,
gathered and reduced, in which order) run on ``gloo`` CPU ranks.  Each one
follows the arithmetic of its kernel closely enough for the step to be
meaningful, and has the one property the checks rely on: per token and per
column it gives the same bytes whether it sees all heads / columns or a
rank's share of them.  Exact integer GEMMs (float64 products of int8 codes),
per-head sums of squares in float64 (exact for these values, so independent
of summation order), and row reductions only over whole rows, which every
rank holds.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

KIND_INT8 = 0


def _q8(x, s):
    inv = 1.0 / s
    return torch.round(x.float() * inv[:, None]).clamp(-127, 127).to(torch.int8)


def int8_row_scales(x):
    return (x.float().abs().amax(dim=1) / 127.0).clamp(min=1e-10)


def quantize_int8_rowwise(x, out=None, scales=None, input_scale=None):
    s = int8_row_scales(x)
    return _q8(x, s), s


def quantize_int8_rowwise_given(x, scales):
    return _q8(x, scales)


def _epilogue(acc, sa, sb, bias, gelu):
    y = acc.float()
    if sa is not None:
        y = y * (sa.reshape(-1, 1) if sa.numel() > 1 else sa.reshape(1, 1))
    if sb is not None:
        y = y * (sb.reshape(1, -1) if sb.numel() > 1 else sb.reshape(1, 1))
    if bias is not None:
        y = y + bias.float().reshape(1, -1)
    y = y.to(torch.bfloat16)
    if gelu:
        y = F.gelu(y.float(), approximate="tanh").to(torch.bfloat16)
    return y


def gemm(kind, a, b, a_scale, b_scale, bias=None, *, gelu=False, raw_acc=False, out=None, tile_n=0, tail_split=0):
    assert kind == KIND_INT8
    acc = (a.double() @ b.double().T).to(torch.int32)   # exact: |acc| < 2^53
    return acc if raw_acc else _epilogue(acc, a_scale, b_scale, bias, gelu)


def int8_epilogue(acc, act_scale, weight_scale, bias=None, gelu=False):
    return _epilogue(acc, act_scale, weight_scale, bias, gelu)


def int8_linear(x, qweight, weight_scales, bias=None, gelu=False, input_scale=None):
    q, s = quantize_int8_rowwise(x)
    return gemm(KIND_INT8, q, qweight, s, weight_scales, bias, gelu=gelu)


def resid_ln_quant(x, y=None, gate=None, ln_w=None, ln_b=None, mod_scale1=None, mod_shift=None, eps=1e-6,
                   quant=True, q=None, s=None, xn=None):
    if y is not None:
        upd = y if gate is None else (gate.reshape(1, -1) * y).to(torch.bfloat16)
        x.copy_((x + upd).to(torch.bfloat16))
    if not quant:
        return None, None
    n = F.layer_norm(x.float(), (x.shape[-1],), None if ln_w is None else ln_w.float(),
                     None if ln_b is None else ln_b.float(), eps).to(torch.bfloat16)
    if mod_scale1 is not None:
        n = ((n * mod_scale1.reshape(1, -1)).to(torch.bfloat16) + mod_shift.reshape(1, -1)).to(torch.bfloat16)
    return quantize_int8_rowwise(n)


def rms_head_partials(inputs, head_dim):
    return torch.stack([x.float().reshape(x.shape[0], -1, head_dim).double().pow(2).sum(-1).float()
                        for x in inputs], 0)


def rms_rope_partials(inputs, weights, rope, head_dim, partials, eps=1e-6, outs=None):
    ranks = partials.shape[0]
    outs = []
    for i, (x, w) in enumerate(zip(inputs, weights)):
        tot = partials[:, i].permute(1, 0, 2).reshape(x.shape[0], -1).double().sum(-1).float()
        a_total = x.shape[1] * ranks
        r = torch.rsqrt(tot / a_total + eps)
        v = ((x.float() * r[:, None]).to(torch.bfloat16).float() * w.float()).to(torch.bfloat16).float()
        if rope is not None:
            m = x.shape[0]
            vp = v.reshape(m, -1, head_dim // 2, 2)
            c, sn = rope[:, None, :, 0], rope[:, None, :, 1]
            e, o = vp[..., 0], vp[..., 1]
            v = torch.stack([e * c - o * sn, e * sn + o * c], -1).reshape(m, -1)
        outs.append(v.to(torch.bfloat16))
    return outs


def attention_short(q, k, vt, heads, scale=None, out=None):
    """CPU stand-in of the short-key attention: fp32 scores, row max, exp,
    probabilities rounded to bf16, their fp32 sum, P V / sum -> bf16."""
    sq, sk = q.shape[0], k.shape[0]
    hd = q.shape[1] // heads
    scale = hd ** -0.5 if scale is None else scale
    qh = q.float().view(sq, heads, hd).transpose(0, 1)
    kh = k.float().view(sk, heads, hd).transpose(0, 1)
    vh = vt.float().reshape(heads, hd, sk).transpose(1, 2)
    s = torch.bmm(qh, kh.transpose(1, 2)) * scale
    p = torch.exp(s - s.amax(-1, keepdim=True)).to(torch.bfloat16).float()
    o = (torch.bmm(p, vh) / p.sum(-1, keepdim=True)).transpose(0, 1).reshape(sq, heads * hd).to(torch.bfloat16)
    if out is not None:
        out.copy_(o)
        return out
    return o
