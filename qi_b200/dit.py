"""The MoT DiT denoising step that drives the quantized linears.

This is the BASELINE "DiT step" workload.  It has 30 blocks and two experts
that share one joint self-attention.  Every block of every expert runs 10
quantized Linears: self-attn q/k/v/o, cross-attn q/k/v/o, ffn.0 and ffn.2.

Two forms, on the same weights:

* ``MoTDiT`` follows the reference's module structure, with the same
  names, so ``replace_linear_with_weight_only`` selects the same layers.
  The block math restates ``src/qi/models/wan22/wan_video_dit.py:147-268``:
  LayerNorm, modulate, RMSNorm of q/k over all heads, RoPE, SDPA,
  gate-residual, and an FFN with GELU(tanh).  The joint MoT layer loop
  restates ``src/qi/models/wan22/mot.py:465-574``: per-expert q/k/v, one
  attention over the concatenated tokens under a boolean mask, then the
  per-expert post block.  Each quantized Linear goes through
  ``WeightOnlyLinear.forward`` -> ``B200Backend.linear``.
* ``DiTStepRunner`` is the B200 execution plan of the same step:
  - q, k and v of an expert share one activation.  Their INT8 weights are
    concatenated, so one quantization and one GEMM (N = 3 x 3072) replace
    three of each.  The context's cross-attn k and v are fused the same
    way.  INT8 outputs are per-element, so this is bit-identical to
    separate layers.
  - The joint mask of ``fastwam.py:914-935`` ("first_frame_causal") has
    block structure.  The runner runs it as three unmasked attention calls:
    first-frame video queries over first-frame keys; the other video
    queries over all video keys; action queries over first-frame video
    keys plus action keys.  These give the same result as the masked
    attention but can use the fused (flash) kernels.
  - The whole step is captured once in a CUDA graph and replayed, so about
    1,200 launches per step cost no host time.

RoPE is computed in fp32 here.  The reference uses fp64 complex numbers
(``wan_video_dit.py:55-61``).  Both round to bf16 at the end; fp32 keeps
about 1e-7 relative error before that rounding.  Attention is bf16 SDPA
(library code, not the quantized hot path).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class ExpertSpec:
    name: str
    hidden: int
    ffn: int
    tokens: int


@dataclass(frozen=True)
class DiTConfig:
    """BASELINE config 5.  The action expert uses 24 heads x 128.  The
    reference MoT requires every expert to share ``num_heads`` and
    ``attn_head_dim`` (``mot.py:43-51``, ``configs/model/fastwam.yaml:39-40``)."""

    layers: int = 30
    heads: int = 24
    head_dim: int = 128
    ctx_tokens: int = 128
    tokens_per_frame: int = 120          # 12 x 10 latent patches per frame
    eps: float = 1e-6
    experts: tuple = field(default_factory=lambda: (ExpertSpec("video", 3072, 14336, 3120),
                                                    ExpertSpec("action", 1024, 4096, 32)))

    @property
    def attn_dim(self) -> int:
        return self.heads * self.head_dim

    def linear_ops(self) -> float:
        """2*M*N*K over the 10 Linears of every block and expert."""
        a = self.attn_dim
        tot = 0.0
        for e in self.experts:
            m, d, f, c = e.tokens, e.hidden, e.ffn, self.ctx_tokens
            tot += 2 * m * d * a * 3 + 2 * m * a * d          # self q,k,v + o
            tot += 2 * m * d * a + 2 * c * d * a * 2 + 2 * m * a * d   # cross q + k,v (context) + o
            tot += 2 * m * d * f * 2                          # ffn.0 + ffn.2
        return tot * self.layers


CFG5 = DiTConfig()


# ---------------------------------------------------------------------------
# block modules (reference structure and names)
# ---------------------------------------------------------------------------


class RMSNorm(nn.Module):
    """``wan_video_dit.py:147-158``: fp32 normalisation, cast back, times weight."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


class _Attn(nn.Module):
    def __init__(self, hidden: int, heads: int, head_dim: int, eps: float):
        super().__init__()
        a = heads * head_dim
        self.num_heads = heads
        self.q = nn.Linear(hidden, a)
        self.k = nn.Linear(hidden, a)
        self.v = nn.Linear(hidden, a)
        self.o = nn.Linear(a, hidden)
        self.norm_q = RMSNorm(a, eps)
        self.norm_k = RMSNorm(a, eps)


class SelfAttention(_Attn):
    pass


class CrossAttention(_Attn):
    def forward(self, x, ctx):
        q = self.norm_q(self.q(x))
        k = self.norm_k(self.k(ctx))
        v = self.v(ctx)
        return self.o(attention(q, k, v, self.num_heads))


class DiTBlock(nn.Module):
    def __init__(self, hidden: int, ffn: int, heads: int, head_dim: int, eps: float):
        super().__init__()
        self.num_heads = heads
        self.self_attn = SelfAttention(hidden, heads, head_dim, eps)
        self.cross_attn = CrossAttention(hidden, heads, head_dim, eps)
        self.norm1 = nn.LayerNorm(hidden, eps=eps, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(hidden, eps=eps, elementwise_affine=False)
        self.norm3 = nn.LayerNorm(hidden, eps=eps)
        self.ffn = nn.Sequential(nn.Linear(hidden, ffn), nn.GELU(approximate="tanh"), nn.Linear(ffn, hidden))
        self.modulation = nn.Parameter(torch.randn(1, 6, hidden) / hidden ** 0.5)


class Expert(nn.Module):
    def __init__(self, spec: ExpertSpec, cfg: DiTConfig):
        super().__init__()
        self.spec = spec
        self.num_heads = cfg.heads
        self.attn_head_dim = cfg.head_dim
        self.blocks = nn.ModuleList()


def attention(q, k, v, heads: int, mask=None):
    """``wan_video_dit.py:14-23``: [B, S, H*D] -> SDPA over heads -> [B, S, H*D]."""
    b, sq, hd = q.shape
    d = hd // heads
    qh = q.view(b, sq, heads, d).transpose(1, 2)
    kh = k.view(b, k.shape[1], heads, d).transpose(1, 2)
    vh = v.view(b, v.shape[1], heads, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask)
    return o.transpose(1, 2).reshape(b, sq, hd)


def modulate(x, shift, scale):
    return x * (1 + scale) + shift


def rope_tables(cfg: DiTConfig, spec: ExpertSpec, device) -> torch.Tensor:
    """[S, D/2, 2] fp32 (cos, sin).  Video tokens use the 3-D (frame, h, w)
    split of ``precompute_freqs_cis_3d`` (``wan_video_dit.py:38-52``).  The
    frame axis gets D - 2*(D//3) dims and h and w get D//3 each.  The grid
    is frames x 12 x 10.  Action tokens use the 1-D table over the whole
    head dimension."""
    d = cfg.head_dim

    def freqs(dim, pos):
        inv = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64)[: dim // 2] / dim))
        return torch.outer(pos.double(), inv)

    s = spec.tokens
    if spec.name == "video" and s % cfg.tokens_per_frame == 0:
        hgt, wid = 12, cfg.tokens_per_frame // 12
        t = torch.arange(s)
        f_i, h_i, w_i = t // cfg.tokens_per_frame, (t % cfg.tokens_per_frame) // wid, t % wid
        df = d - 2 * (d // 3)
        ang = torch.cat([freqs(df, f_i), freqs(d // 3, h_i), freqs(d // 3, w_i)], dim=1)
        assert hgt * wid == cfg.tokens_per_frame
    else:
        ang = freqs(d, torch.arange(s))
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).float().to(device)


def rope_apply(x, table, heads: int):
    """Rotate (even, odd) pairs of every head: the complex product of
    ``wan_video_dit.py:55-61``, in fp32, rounded to x's dtype."""
    b, s, hd = x.shape
    xf = x.float().view(b, s, heads, -1, 2)
    c, sn = table[None, :, None, :, 0], table[None, :, None, :, 1]
    xe, xo = xf[..., 0], xf[..., 1]
    out = torch.stack([xe * c - xo * sn, xe * sn + xo * c], dim=-1)
    return out.view(b, s, hd).to(x.dtype)


def first_frame_causal_mask(cfg: DiTConfig, sv: int, sa: int, device) -> torch.Tensor:
    """The joint [video+action] bool mask of ``fastwam.py:914-935`` with the
    ``first_frame_causal`` video mode (``wan_video_dit.py:501-505``)."""
    t = min(cfg.tokens_per_frame, sv)
    m = torch.zeros((sv + sa, sv + sa), dtype=torch.bool, device=device)
    m[:sv, :sv] = True
    m[:t, t:sv] = False
    m[sv:, sv:] = True
    m[sv:, :t] = True
    return m


def joint_attention_blocks(q: dict, k: dict, v: dict, cfg: DiTConfig, q_offset: int = 0) -> dict:
    """Attention under the first_frame_causal joint mask, as unmasked calls
    over the mask's blocks (same result as ``attention`` over the
    concatenated tokens with ``first_frame_causal_mask``).

    ``k``/``v`` hold every video token; ``q["video"]`` may be a contiguous
    run of video queries starting at token ``q_offset`` (a token shard)."""
    h = cfg.heads
    qv, kv, vv = q["video"], k["video"], v["video"]
    sv = kv.shape[1]
    t = min(cfg.tokens_per_frame, sv)
    nf = max(0, min(t - q_offset, qv.shape[1]))   # local queries inside the first frame
    parts = []
    if nf > 0:
        parts.append(attention(qv[:, :nf], kv[:, :t], vv[:, :t], h))
    if nf < qv.shape[1]:
        parts.append(attention(qv[:, nf:], kv, vv, h))
    out_v = parts[0] if len(parts) == 1 else torch.cat(parts, dim=1)
    out_a = attention(q["action"], torch.cat([kv[:, :t], k["action"]], 1),
                      torch.cat([vv[:, :t], v["action"]], 1), h)
    return {"video": out_v, "action": out_a}


class MoTDiT(nn.Module):
    """Random-init MoT DiT blocks with the reference's module names
    (``mixtures.<expert>.blocks.<i>.self_attn.q`` and so on)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        self.mixtures = nn.ModuleDict({e.name: Expert(e, cfg) for e in cfg.experts})
        self.expert_order = [e.name for e in cfg.experts]

    def forward(self, tokens: dict, rope: dict, ctx: dict, t_mod: dict, mask: torch.Tensor | None = None) -> dict:
        """``mot.py:465-574``, one call per Linear through the module API.
        With ``mask`` the joint attention is one SDPA over the concatenated
        tokens under that boolean mask (the reference's form); without it,
        the block form of the first_frame_causal mask."""
        cfg = self.cfg
        h = cfg.heads
        tokens = dict(tokens)
        for li in range(cfg.layers):
            q, k, v, post = {}, {}, {}, {}
            for name in self.expert_order:
                blk = self.mixtures[name].blocks[li]
                x = tokens[name]
                sm, cm, gm, s2, c2, g2 = (blk.modulation.to(t_mod[name].dtype) + t_mod[name]).chunk(6, dim=1)
                a_in = modulate(blk.norm1(x), sm, cm)
                sa = blk.self_attn
                q[name] = rope_apply(sa.norm_q(sa.q(a_in)), rope[name], h)
                k[name] = rope_apply(sa.norm_k(sa.k(a_in)), rope[name], h)
                v[name] = sa.v(a_in)
                post[name] = (blk, x, gm, s2, c2, g2)
            if mask is None:
                att = joint_attention_blocks(q, k, v, cfg)
            else:
                cat = [torch.cat([d[n] for n in self.expert_order], 1) for d in (q, k, v)]
                mixed = attention(*cat, h, mask)
                att, start = {}, 0
                for name in self.expert_order:
                    n = tokens[name].shape[1]
                    att[name] = mixed[:, start:start + n]
                    start += n
            for name in self.expert_order:
                blk, x, gm, s2, c2, g2 = post[name]
                x = x + gm * blk.self_attn.o(att[name])
                x = x + blk.cross_attn(blk.norm3(x), ctx[name])
                x = x + g2 * blk.ffn(modulate(blk.norm2(x), s2, c2))
                tokens[name] = x
        return tokens


# ---------------------------------------------------------------------------
# construction (random init, quantized block by block)
# ---------------------------------------------------------------------------


INT8_DIT_CFG = dict(enabled=True, quant_dtype="int", backend="b200", activation_granularity="per_token",
                    weight_granularity="per_channel")


def _init_block(blk: DiTBlock, gen: torch.Generator):
    with torch.no_grad():
        for mod in blk.modules():
            if isinstance(mod, nn.Linear):
                mod.weight.normal_(0.0, 0.02, generator=gen)
                mod.bias.normal_(0.0, 0.01, generator=gen)
            elif isinstance(mod, nn.LayerNorm) and mod.weight is not None:
                mod.weight.fill_(1.0)
                mod.bias.zero_()
        blk.modulation.normal_(0.0, 1.0, generator=gen).div_(blk.modulation.shape[-1] ** 0.5)


def build_mot_dit(cfg: DiTConfig = CFG5, device="cuda", seed: int = 0, quantize: bool = True,
                  dtype=torch.bfloat16, state_dict=None) -> MoTDiT:
    """MoT DiT with every target Linear swapped for an INT8 W8A8
    ``WeightOnlyLinear`` as each block is built.  Weights are random (seeded)
    or, with ``state_dict``, an unquantized checkpoint of the reference's MoT
    (same parameter names: ``mixtures.<expert>.blocks.<i>.<module>``).  The
    fp32 weights of one block at a time are resident, so peak memory is the
    INT8 model plus one block."""
    from .quantization import WeightActivationQuantConfig, fuse_ffn_gelu, replace_linear_with_weight_only

    qcfg = WeightActivationQuantConfig(**INT8_DIT_CFG)
    model = MoTDiT(cfg)
    gen = torch.Generator(device=device).manual_seed(seed)
    for spec in cfg.experts:
        ex = model.mixtures[spec.name]
        for li in range(cfg.layers):
            blk = DiTBlock(spec.hidden, spec.ffn, cfg.heads, cfg.head_dim, cfg.eps).to(device)
            if state_dict is None:
                _init_block(blk, gen)
            else:
                pre = f"mixtures.{spec.name}.blocks.{li}."
                blk.load_state_dict({k[len(pre):]: v for k, v in state_dict.items() if k.startswith(pre)})
            if quantize:
                replace_linear_with_weight_only(blk, qcfg)
                fuse_ffn_gelu(blk)
                for mod in blk.modules():
                    if hasattr(mod, "qweight") and getattr(mod, "bias", None) is not None:
                        mod.bias = mod.bias.to(dtype)
            blk.to(dtype)
            ex.blocks.append(blk)
    return model


def make_step_inputs(cfg: DiTConfig, device, seed: int = 0, dtype=torch.bfloat16):
    """Seeded synthetic step inputs: tokens, context (already at each
    expert's width), time modulation [1, 6, D], RoPE tables, joint mask."""
    g = torch.Generator(device=device).manual_seed(seed + 1)
    tokens, ctx, t_mod, rope = {}, {}, {}, {}
    for e in cfg.experts:
        tokens[e.name] = torch.randn(1, e.tokens, e.hidden, generator=g, device=device).to(dtype)
        ctx[e.name] = torch.randn(1, cfg.ctx_tokens, e.hidden, generator=g, device=device).to(dtype)
        t_mod[e.name] = (torch.randn(1, 6, e.hidden, generator=g, device=device) * 0.1).to(dtype)
        rope[e.name] = rope_tables(cfg, e, device)
    sv, sa = cfg.experts[0].tokens, cfg.experts[1].tokens
    return tokens, rope, ctx, t_mod, first_frame_causal_mask(cfg, sv, sa, device)


# ---------------------------------------------------------------------------
# the B200 execution plan
# ---------------------------------------------------------------------------


def _cat_int8(layers):
    """Concatenate INT8 W8A8 ``WeightOnlyLinear`` layers along N."""
    w = torch.cat([l.qweight for l in layers], 0).contiguous()
    s = torch.cat([l.scales.reshape(-1) for l in layers], 0).float().contiguous()
    b = torch.cat([l.bias.reshape(-1) for l in layers], 0).to(torch.bfloat16).contiguous()
    return w, s, b


def _int8(layer):
    return layer.qweight, layer.scales.reshape(-1).float().contiguous(), layer.bias.to(torch.bfloat16).contiguous()


class _BlockPlan:
    def __init__(self, blk: DiTBlock):
        sa, ca = blk.self_attn, blk.cross_attn
        self.qkv = _cat_int8([sa.q, sa.k, sa.v])
        self.o = _int8(sa.o)
        self.cq = _int8(ca.q)
        self.ckv = _cat_int8([ca.k, ca.v])
        self.co = _int8(ca.o)
        self.f0 = _int8(blk.ffn[0])
        self.f2 = _int8(blk.ffn[2])
        self.nq, self.nk = sa.norm_q, sa.norm_k
        self.cnq, self.cnk = ca.norm_q, ca.norm_k
        self.norm1, self.norm2, self.norm3 = blk.norm1, blk.norm2, blk.norm3
        self.modulation = blk.modulation


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


class _TPBlockPlan:
    """One rank's shard of a block for the head-parallel step: rows of the
    fused q/k/v, cross-q, cross-k/v and ffn.0 weights for this rank's heads /
    FFN columns (column parallel), and the matching input columns of o,
    cross-o and ffn.2 (row parallel; their per-channel scales and bias stay
    whole and are applied once after the int32 sum).  INT8 per-channel rows
    slice exactly, so every output element is the single-GPU one."""

    def __init__(self, p: _BlockPlan, cfg: DiTConfig, spec: ExpertSpec, rank: int, world: int):
        if cfg.heads % world or spec.ffn % (8 * world):
            raise ValueError(f"{cfg.heads} heads / FFN {spec.ffn} do not split over {world} ranks.")
        a = cfg.attn_dim
        self.heads = cfg.heads // world
        self.al = al = a // world
        fl = spec.ffn // world
        lo, hi = rank * al, (rank + 1) * al

        def rows(wsb, ranges):
            return tuple(torch.cat([t[r0:r1] for r0, r1 in ranges], 0).contiguous() for t in wsb)

        def cols(wsb, c0, c1):
            return wsb[0][:, c0:c1].contiguous(), wsb[1], wsb[2]

        self.qkv = rows(p.qkv, [(lo, hi), (a + lo, a + hi), (2 * a + lo, 2 * a + hi)])
        self.cq = rows(p.cq, [(lo, hi)])
        self.ckv = rows(p.ckv, [(lo, hi), (a + lo, a + hi)])
        self.f0 = rows(p.f0, [(rank * fl, (rank + 1) * fl)])
        self.o = cols(p.o, lo, hi)
        self.co = cols(p.co, lo, hi)
        self.f2 = cols(p.f2, rank * fl, (rank + 1) * fl)
        self.nq, self.nk = p.nq.weight[lo:hi].contiguous(), p.nk.weight[lo:hi].contiguous()
        self.cnq, self.cnk = p.cnq.weight[lo:hi].contiguous(), p.cnk.weight[lo:hi].contiguous()
        self.norm3 = p.norm3


class DiTStepRunner:
    """One MoT DiT step on B200 (INT8 tcgen05 GEMMs, fused QKV, block-mask
    attention), optionally captured as a CUDA graph.

    With ``group`` (a process group of P ranks, one per GPU) the video
    tokens are sharded by sequence.  Rank r owns tokens
    ``[r*Sv/P, (r+1)*Sv/P)`` and runs all of their Linears locally with
    replicated weights.  Per-token quantization makes those rows
    bit-identical to one GPU.  The only exchange is one NCCL all-gather per
    layer of the video K and V (``2*Sv*3072`` bf16), which the joint
    attention needs.  The 32 action tokens are replicated: their GEMMs are
    bound by weight bandwidth, so splitting them would not shorten the step.
    """

    def __init__(self, model: MoTDiT, group=None, fused: bool = True, partition: str = "sequence", kernels=None):
        from . import _lib

        if kernels is None:
            from . import kernels as K
        else:
            K = kernels  # a stand-in with the same functions (CPU tests of the multi-rank logic)
        if partition not in ("sequence", "heads"):
            raise ValueError("partition must be 'sequence' or 'heads'")
        self.K = K
        self.kind_int8 = _lib.KIND_INT8
        self.cfg = model.cfg
        self.names = model.expert_order
        self.partition = partition
        self.plans = {n: [_BlockPlan(b) for b in model.mixtures[n].blocks] for n in self.names}
        # all layers' modulation tables of an expert, [L, 6, D]: one add per step
        self.mod_tables = {n: torch.cat([p.modulation for p in self.plans[n]], 0).contiguous() for n in self.names}
        self.fused = fused
        self.graph = None
        self.group = group
        if group is not None:
            import torch.distributed as dist

            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        sv = self.cfg.experts[0].tokens
        if partition == "heads":
            # tensor parallel: every rank holds all tokens and a contiguous range of heads / FFN columns
            self.video_local, self.video_offset = sv, 0
            self.tp = {n: [_TPBlockPlan(p, self.cfg, spec, self.rank, self.world)
                           for p in self.plans[n]] for n, spec in zip(self.names, self.cfg.experts)}
            self.tp_groups = {self.names[0]: group}
            if group is not None:
                import torch.distributed as dist

                # the action expert's collectives run on a side stream: a communicator of its own
                self.tp_groups[self.names[1]] = dist.new_group(dist.get_process_group_ranks(group))
            else:
                self.tp_groups[self.names[1]] = None
            return
        if sv % self.world:
            raise ValueError(f"{sv} video tokens do not split over {self.world} ranks.")
        self.video_local = sv // self.world
        self.video_offset = self.rank * self.video_local

    def shard(self, tokens: dict, rope: dict):
        """This rank's video tokens and RoPE rows (action replicated)."""
        lo, hi = self.video_offset, self.video_offset + self.video_local
        tok = {n: (x[:, lo:hi].contiguous() if n == "video" else x) for n, x in tokens.items()}
        rp = {n: (r[lo:hi].contiguous() if n == "video" else r) for n, r in rope.items()}
        return tok, rp

    def _gather_video_kv(self, k, v):
        import torch.distributed as dist

        a = self.cfg.attn_dim
        n = k.shape[1]
        kv = torch.cat([k.reshape(n, a), v.reshape(n, a)], dim=1)
        out = torch.empty((self.world * n, 2 * a), dtype=kv.dtype, device=kv.device)
        dist.all_gather_into_tensor(out, kv, group=self.group)
        return out[:, :a].unsqueeze(0), out[:, a:].unsqueeze(0)

    def _lin(self, x, wsb, gelu=False):
        w, s, b = wsb
        x2 = x.reshape(-1, x.shape[-1])
        y = self.K.int8_linear(x2, w, s, b, gelu=gelu)
        return y.view(*x.shape[:-1], w.shape[0])

    def _joint_attention(self, q, k, v):
        if self.world > 1:
            k, v = dict(k), dict(v)
            k["video"], v["video"] = self._gather_video_kv(k["video"], v["video"])
        return joint_attention_blocks(q, k, v, self.cfg, q_offset=self.video_offset)

    @torch.no_grad()
    def step(self, tokens: dict, rope: dict, ctx: dict, t_mod: dict) -> dict:
        if self.partition == "heads":
            return self._step_tp(tokens, rope, ctx, t_mod)
        if self.fused:
            return self._step_fused(tokens, rope, ctx, t_mod)
        return self._step_unfused(tokens, rope, ctx, t_mod)

    # -- tensor parallel (heads) ---------------------------------------------

    def _all_gather(self, t, group):
        if group is None:
            return t.unsqueeze(0)
        import torch.distributed as dist

        out = torch.empty((self.world * t.numel(),), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous().reshape(-1), group=group)
        return out.view((self.world,) + tuple(t.shape))

    def _all_reduce(self, t, group, op):
        if group is not None:
            import torch.distributed as dist

            dist.all_reduce(t, op=op, group=group)
        return t

    def _row_parallel(self, x_l, wsb, group):
        """Row-parallel INT8 linear, exact: per-token scales reduced with MAX
        (the scale of the whole row), int32 partial sums reduced with SUM,
        then the epilogue.  Bit-identical to the single-GPU INT8 linear."""
        import torch.distributed as dist

        K = self.K
        w, sw, b = wsb
        s = self._all_reduce(K.int8_row_scales(x_l), group, dist.ReduceOp.MAX if group is not None else None)
        q = K.quantize_int8_rowwise_given(x_l, s)
        acc = K.gemm(self.kind_int8, q, w, None, None, raw_acc=True)
        acc = self._all_reduce(acc, group, dist.ReduceOp.SUM if group is not None else None)
        return K.int8_epilogue(acc, s, sw, b)

    def _norm_heads(self, parts, weights, rope, group, eps):
        """RMSNorm (+ RoPE) of this rank's head columns with the row norm over
        all heads: per-head sums gathered from every rank (head order)."""
        K, hd = self.K, self.cfg.head_dim
        sums = self._all_gather(K.rms_head_partials(parts, hd), group)
        return K.rms_rope_partials(parts, weights, rope, hd, sums, eps)

    def _tp_pre(self, n, li, x, y_ffn, mods, sc1, rope):
        """Residual + norm1 + modulate + INT8 (all rows, every rank) -> this
        rank's heads of q, k, v -> RMSNorm over all heads + RoPE."""
        K, cfg = self.K, self.cfg
        tp, m, g = self.tp[n][li], mods[n][li], self.tp_groups[n]
        if li == 0:
            q8, s8 = K.resid_ln_quant(x[n], mod_scale1=sc1[n][li, 0], mod_shift=m[0], eps=cfg.eps)
        else:
            q8, s8 = K.resid_ln_quant(x[n], y_ffn[n], gate=mods[n][li - 1][5], mod_scale1=sc1[n][li, 0],
                                      mod_shift=m[0], eps=cfg.eps)
        qkv = self._gemm(q8, s8, tp.qkv)
        al = tp.al
        qn, kn = self._norm_heads([qkv[:, :al], qkv[:, al:2 * al]], [tp.nq, tp.nk], rope[n], g, cfg.eps)
        return qn.unsqueeze(0), kn.unsqueeze(0), qkv[:, 2 * al:].unsqueeze(0)

    def _tp_post(self, n, li, att, x, y_ffn, mods, sc1, ctxq):
        """Row-parallel o -> gate-residual + norm3 -> cross-attention over this
        rank's heads -> row-parallel cross-o -> norm2 + modulate -> ffn.0 on
        this rank's FFN columns (GELU fused) -> row-parallel ffn.2."""
        K, cfg = self.K, self.cfg
        tp, m, g = self.tp[n][li], mods[n][li], self.tp_groups[n]
        al, hl, eps = tp.al, tp.heads, cfg.eps
        y_o = self._row_parallel(att.reshape(-1, al), tp.o, g)
        q8, s8 = K.resid_ln_quant(x[n], y_o, gate=m[2], ln_w=tp.norm3.weight, ln_b=tp.norm3.bias, eps=eps)
        cq = self._gemm(q8, s8, tp.cq)
        ckv = self._gemm(*ctxq[n], tp.ckv)
        cqn = self._norm_heads([cq], [tp.cnq], None, g, eps)[0]
        ckn = self._norm_heads([ckv[:, :al]], [tp.cnk], None, g, eps)[0]
        ca = self._attn_short(cqn, ckn, ckv[:, al:], heads=hl)
        y_co = self._row_parallel(ca.reshape(-1, al), tp.co, g)
        q8, s8 = K.resid_ln_quant(x[n], y_co, mod_scale1=sc1[n][li, 1], mod_shift=m[3], eps=eps)
        f = self._gemm(q8, s8, tp.f0, gelu=True)
        y_ffn[n] = self._row_parallel(f, tp.f2, g)

    def _step_tp(self, tokens, rope, ctx, t_mod):
        """The step with heads and FFN columns split over the ranks (config 5's
        N-sharded QKV / FFN, completed Megatron-style so attention is head-local):
        per expert and layer 2 all-gathers of per-head RMS sums and 3 exact
        row-parallel reductions (MAX of [M] scales, SUM of int32 [M, D]).  Every
        rank ends with all tokens, bit-identical to one GPU."""
        K, cfg = self.K, self.cfg
        x = {n: t.reshape(-1, t.shape[-1]).clone() for n, t in tokens.items()}
        mods, sc1, ctxq = {}, {}, {}
        for n in self.names:
            mods[n] = self.mod_tables[n] + t_mod[n]
            sc1[n] = 1 + mods[n][:, 1::3]
            ctxq[n] = K.quantize_int8_rowwise(ctx[n].reshape(-1, ctx[n].shape[-1]).contiguous())
        cuda = x[self.names[0]].is_cuda
        main = torch.cuda.current_stream() if cuda else None
        side = self._side_stream() if cuda else None
        if cuda:
            side.wait_stream(main)
        t = min(cfg.tokens_per_frame, cfg.experts[0].tokens)
        hl = cfg.heads // self.world
        y_ffn = {}
        va_name, ac_name = self.names
        for li in range(cfg.layers):
            qv, kv, vv = self._tp_pre(va_name, li, x, y_ffn, mods, sc1, rope)
            kf, vf = kv[:, :t].contiguous(), vv[:, :t].contiguous()
            if cuda:
                side.wait_stream(main)
            with (torch.cuda.stream(side) if cuda else _nullctx()):
                qa, ka, va = self._tp_pre(ac_name, li, x, y_ffn, mods, sc1, rope)
                att_a = attention(qa, torch.cat([kf, ka], 1), torch.cat([vf, va], 1), hl)
                self._tp_post(ac_name, li, att_a, x, y_ffn, mods, sc1, ctxq)
            if cuda:
                kf.record_stream(side)
                vf.record_stream(side)
            att_v = self._video_attention(qv, kv, vv, heads=hl)
            self._tp_post(va_name, li, att_v, x, y_ffn, mods, sc1, ctxq)
        with (torch.cuda.stream(side) if cuda else _nullctx()):
            K.resid_ln_quant(x[ac_name], y_ffn[ac_name], gate=mods[ac_name][cfg.layers - 1][5], quant=False)
        K.resid_ln_quant(x[va_name], y_ffn[va_name], gate=mods[va_name][cfg.layers - 1][5], quant=False)
        if cuda:
            main.wait_stream(side)
            for n in self.names:
                x[n].record_stream(side)
        return {n: x[n].view(tokens[n].shape) for n in self.names}

    def _gemm(self, q8, s8, wsb, gelu=False):
        w, sw, b = wsb
        return self.K.gemm(self.kind_int8, q8, w, s8, sw, b, gelu=gelu)

    def _pre(self, n, li, x, y_ffn, mods, sc1, rope):
        """Residual + norm1 + modulate + INT8 -> fused QKV GEMM -> RMSNorm+RoPE."""
        K, cfg = self.K, self.cfg
        a, hd, eps = cfg.attn_dim, cfg.head_dim, cfg.eps
        p, m = self.plans[n][li], mods[n][li]
        if li == 0:
            q8, s8 = K.resid_ln_quant(x[n], mod_scale1=sc1[n][li, 0], mod_shift=m[0], eps=eps)
        else:
            q8, s8 = K.resid_ln_quant(x[n], y_ffn[n], gate=mods[n][li - 1][5], mod_scale1=sc1[n][li, 0],
                                      mod_shift=m[0], eps=eps)
        qkv = self._gemm(q8, s8, p.qkv)
        qn, kn = K.rms_rope([qkv[:, :a], qkv[:, a:2 * a]], [p.nq.weight, p.nk.weight], rope[n], hd, eps)
        return qn.unsqueeze(0), kn.unsqueeze(0), qkv[:, 2 * a:].unsqueeze(0), qkv

    def _ctx_kv(self, n, li, ctxq):
        """Cross-attention K (RMSNorm) and V^T of layer ``li``: they depend on
        the context tokens only, so they run ahead of the layer on the side
        stream."""
        K, cfg = self.K, self.cfg
        a = cfg.attn_dim
        ckv = self._gemm(*ctxq[n], self.plans[n][li].ckv)
        ck = K.rms_rope([ckv[:, :a]], [self.plans[n][li].cnk.weight], None, cfg.head_dim, cfg.eps)[0]
        return ck, ckv[:, a:].t().contiguous()

    def _attn_short(self, q, k, v=None, heads=None, vt=None):
        """Cross-attention over the (at most 128) context tokens on the tensor
        cores (``attention_short``; cuDNN's SDPA runs an sm80 kernel there, 34
        against 21 us per video layer).  q [.., Sq, W], k [.., Sk, W],
        v [.., Sk, W] (or vt = V^T [W, Sk]); rows may be strided."""
        h = self.cfg.heads if heads is None else heads
        w = q.shape[-1]
        if self.cfg.head_dim != 128:  # the kernel's head dim; other configs (small tests) use SDPA
            v2 = v.reshape(-1, w) if v is not None else vt.t()
            o = attention(q.reshape(1, -1, w), k.reshape(1, -1, w), v2.unsqueeze(0), h)[0]
        else:
            if vt is None:
                vt = v.reshape(-1, w).t().contiguous()
            o = self.K.attention_short(q.reshape(-1, w), k.reshape(-1, w), vt, h)
        return o.unsqueeze(0) if q.dim() == 3 else o

    def _post(self, n, li, att, x, y_ffn, mods, sc1, ctxq, ctx_kv=None):
        """o GEMM + gate-residual + norm3 -> cross-attention -> norm2 + FFN."""
        K, cfg = self.K, self.cfg
        h, a, hd, eps = cfg.heads, cfg.attn_dim, cfg.head_dim, cfg.eps
        p, m = self.plans[n][li], mods[n][li]
        y_o = K.int8_linear(att.reshape(-1, a), *p.o)
        q8, s8 = K.resid_ln_quant(x[n], y_o, gate=m[2], ln_w=p.norm3.weight, ln_b=p.norm3.bias, eps=eps)
        cq = K.rms_rope([self._gemm(q8, s8, p.cq)], [p.cnq.weight], None, hd, eps)[0]
        ck, cvt = self._ctx_kv(n, li, ctxq) if ctx_kv is None else ctx_kv
        ca = self._attn_short(cq, ck, vt=cvt)
        y_co = K.int8_linear(ca.reshape(-1, a), *p.co)
        q8, s8 = K.resid_ln_quant(x[n], y_co, mod_scale1=sc1[n][li, 1], mod_shift=m[3], eps=eps)
        f = self._gemm(q8, s8, p.f0, gelu=True)
        y_ffn[n] = K.int8_linear(f, *p.f2)

    def _video_attention(self, q, k, v, heads=None):
        """Video queries of this rank under the first_frame_causal mask: all
        video keys, except first-frame queries, which see first-frame keys
        only (recomputed for those rows and written over them, so the bulk
        attention output needs no concatenation)."""
        h = self.cfg.heads if heads is None else heads
        sv = k.shape[1]
        t = min(self.cfg.tokens_per_frame, sv)
        nf = max(0, min(t - self.video_offset, q.shape[1]))
        out = attention(q, k, v, h)
        if nf > 0 and sv > t:
            out[:, :nf] = attention(q[:, :nf], k[:, :t], v[:, :t], h)
        return out

    def _step_fused(self, tokens, rope, ctx, t_mod):
        """The step with the elementwise chains fused into row kernels:
        ``resid_ln_quant`` (gate-residual + LayerNorm + modulate + INT8
        quantization, feeding the next GEMM directly) and ``rms_rope``.
        Per expert and layer: 3 row kernels, 3 RMSNorm(+RoPE) kernels, 7
        GEMMs, 3 activation quantizers (attention outputs, FFN hidden).

        The action expert runs on a second stream.  It joins the video
        stream once per layer, after the video K/V exist, because action
        queries attend first-frame video keys; video never attends action
        tokens.  Its small launches then overlap the video GEMMs.  The side
        stream also computes both experts' cross-attention K / V one layer
        ahead (they depend on the context tokens only), so the video stream
        only waits on an event for them."""
        K, cfg = self.K, self.cfg
        x = {n: t.reshape(-1, t.shape[-1]).clone() for n, t in tokens.items()}
        mods, sc1, ctxq = {}, {}, {}
        for n in self.names:
            mods[n] = self.mod_tables[n] + t_mod[n]              # [L, 6, D] bf16 (mot.py:56-75)
            sc1[n] = 1 + mods[n][:, 1::3]                        # bf16(1 + scale) for msa / mlp
            ctxq[n] = K.quantize_int8_rowwise(ctx[n].reshape(-1, ctx[n].shape[-1]).contiguous())
        main = torch.cuda.current_stream()
        side = self._side_stream()
        side.wait_stream(main)
        t = min(cfg.tokens_per_frame, cfg.experts[0].tokens)
        y_ffn = {}
        ckv, ckv_ready = {}, {}

        def ctx_kv_ahead(li):  # on the side stream
            for n in self.names:
                ckv[n, li] = self._ctx_kv(n, li, ctxq)
            ckv_ready[li] = torch.cuda.Event()
            ckv_ready[li].record(side)

        with torch.cuda.stream(side):
            ctx_kv_ahead(0)
        for li in range(cfg.layers):
            qv, kv, vv, qkv_v = self._pre("video", li, x, y_ffn, mods, sc1, rope)
            if self.world > 1:
                kv, vv = self._gather_video_kv(kv, vv)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                # the action queries attend the first-frame video keys and their own;
                # the copies that join them run here, off the video stream
                qa, ka, va, _ = self._pre("action", li, x, y_ffn, mods, sc1, rope)
                att_a = attention(qa, torch.cat([kv[:, :t], ka], 1), torch.cat([vv[:, :t], va], 1), cfg.heads)
                self._post("action", li, att_a, x, y_ffn, mods, sc1, ctxq, ckv.pop(("action", li)))
                if li + 1 < cfg.layers:
                    ctx_kv_ahead(li + 1)
            kv.record_stream(side)
            vv.record_stream(side)  # a view: records the fused QKV output (or the gathered K/V) it lives in
            att_v = self._video_attention(qv, kv, vv)
            main.wait_event(ckv_ready.pop(li))
            ck, cvt = ckv.pop(("video", li))
            ck.record_stream(main)
            cvt.record_stream(main)
            self._post("video", li, att_v, x, y_ffn, mods, sc1, ctxq, (ck, cvt))
        with torch.cuda.stream(side):
            K.resid_ln_quant(x["action"], y_ffn["action"], gate=mods["action"][cfg.layers - 1][5], quant=False)
        K.resid_ln_quant(x["video"], y_ffn["video"], gate=mods["video"][cfg.layers - 1][5], quant=False)
        main.wait_stream(side)
        for n in self.names:
            x[n].record_stream(side)
        return {n: x[n].view(tokens[n].shape) for n in self.names}

    def _side_stream(self):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream()
        return self._side

    def _step_unfused(self, tokens, rope, ctx, t_mod):
        """The step as the reference's tensor-op chain (fused QKV GEMM only)."""
        cfg, h = self.cfg, self.cfg.heads
        a = cfg.attn_dim
        x = dict(tokens)
        for li in range(cfg.layers):
            q, k, v, post = {}, {}, {}, {}
            for n in self.names:
                p = self.plans[n][li]
                sm, cm, gm, s2, c2, g2 = (p.modulation + t_mod[n]).chunk(6, dim=1)
                qkv = self._lin(modulate(p.norm1(x[n]), sm, cm), p.qkv)
                q[n] = rope_apply(p.nq(qkv[..., :a]), rope[n], h)
                k[n] = rope_apply(p.nk(qkv[..., a:2 * a]), rope[n], h)
                v[n] = qkv[..., 2 * a:]
                post[n] = (gm, s2, c2, g2)
            att = self._joint_attention(q, k, v)
            for n in self.names:
                p = self.plans[n][li]
                gm, s2, c2, g2 = post[n]
                xn = x[n] + gm * self._lin(att[n], p.o)
                cq = p.cnq(self._lin(p.norm3(xn), p.cq))
                ckv = self._lin(ctx[n], p.ckv)
                ck, cv = p.cnk(ckv[..., :a]), ckv[..., a:]
                xn = xn + self._lin(attention(cq, ck, cv, h), p.co)
                f = self._lin(modulate(p.norm2(xn), s2, c2), p.f0, gelu=True)
                x[n] = xn + g2 * self._lin(f, p.f2)
        return x

    # -- CUDA graph ---------------------------------------------------------

    def check(self) -> None:
        """Raise ``QiB200DeviceError`` if a kernel of the step gave up a
        bounded wait since the last check (its outputs are then incomplete).
        Synchronizes the host with the device: call it between steps."""
        from . import _lib

        _lib.raise_on_device_error()

    def capture(self, tokens: dict, rope: dict, ctx: dict, t_mod: dict, warmup: int = 2):
        """Capture one step on static input buffers; ``replay()`` reruns it."""
        self.static_in = ({n: t.clone() for n, t in tokens.items()}, rope, ctx, t_mod)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(*self.static_in)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.check()  # the eager warm-up steps ran clean before they are captured
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_out = self.step(*self.static_in)
        return self.static_out

    def replay(self):
        self.graph.replay()
        return self.static_out


def count_quantized_linears(model: nn.Module) -> int:
    from .quantization import WeightOnlyLinear

    return sum(isinstance(m, WeightOnlyLinear) for m in model.modules())


def step_flops_attention(cfg: DiTConfig) -> float:
    """bf16 attention FLOPs of one step under the first_frame_causal mask
    (QK^T and PV, 4*Sq*Sk*H*D per pair of blocks)."""
    sv, sa = cfg.experts[0].tokens, cfg.experts[1].tokens
    t = min(cfg.tokens_per_frame, sv)
    hd = cfg.attn_dim
    pairs = t * t + (sv - t) * sv + sa * (t + sa)
    cross = sum(e.tokens for e in cfg.experts) * cfg.ctx_tokens
    return 4.0 * (pairs + cross) * hd * cfg.layers


__all__ = ["CFG5", "DiTConfig", "DiTStepRunner", "ExpertSpec", "MoTDiT", "build_mot_dit", "count_quantized_linears",
           "first_frame_causal_mask", "joint_attention_blocks", "make_step_inputs", "rope_tables",
           "step_flops_attention"]
