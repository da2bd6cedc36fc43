#!/usr/bin/env python
"""Benchmark of the B200 quantized-linear hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config fp8|int8|...] [--only] [--impl ours|reference]

One step = one quantized linear forward over one batch of synthetic input
(activation quantization kernel + tcgen05 GEMM with fused epilogue; for N > 1
also the all-gather of the column-sharded outputs).  The headline config is
BASELINE config 2 (FP8-E4M3 FFN up-projection, M=4096 N=14336 K=3072,
per-token activations, per-channel weights, bias + GELU).

Prints ONE JSON line on rank 0.  ``value`` = whole-job TOPS (2*M*N*K per
step / max-over-ranks device time), inputs resident in HBM; ``e2e`` = the
same through the public module API (``WeightOnlyLinear.forward``) with the
activations copied in from pinned host memory and the output copied back
every step.  Without ``--only`` the same line carries a ``configs`` map with
every other BASELINE config measured the same way in the same process
(N = 1: configs 1, 3 at M = 1/16/256/4096, 4 and 5; N > 1: the DiT step of
config 5 on N GPUs).  ``--impl reference`` times the reference's own CPU
algorithm (the dequantise-then-matmul port in ``oracle/reference_port.py``)
on this host's cores instead, on the full config.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from qi_b200.synthetic import CFG_FP8, CFG_INT8, CFG_NVFP4, CFG_W4A16, make_linear_inputs  # noqa: E402

CONFIGS = {
    "fp8": dict(case=CFG_FP8, kind="fp8", gelu=True, dtype="fp8_e4m3 (fp32 accumulate)"),
    "int8": dict(case=CFG_INT8, kind="int8", gelu=False, dtype="int8 (int32 accumulate)"),
    "nvfp4": dict(case=CFG_NVFP4, kind="nvfp4", gelu=False,
                  dtype="nvfp4 e2m1 + e4m3 block16 scales (fp32 accumulate)"),
}
for _m in (1, 16, 256, 4096):
    CONFIGS[f"w4a16_m{_m}"] = dict(case=CFG_W4A16[_m], kind="w4a16", gelu=False, group=128,
                                   dtype="bf16 x int4-g128 (fp32 accumulate)")
CONFIGS["dit"] = dict(case=None, kind="dit", gelu=True, dtype="int8 (int32 accumulate) linears, bf16 attention",
                      partition="sequence")
# config 5 with the partition BASELINE names (QKV / FFN N-sharded; o / ffn.2
# row-parallel so attention stays head-local); the same as "dit" on one GPU
CONFIGS["dit_tp"] = dict(case=None, kind="dit", gelu=True, dtype="int8 (int32 accumulate) linears, bf16 attention",
                         partition="heads")
L2_BYTES = 126 * 2**20


def peaks():
    """Roofline denominators: MEASURED_PEAKS.json (driver-measured on this
    pool), else the profiling recipe's fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json)"
    except Exception:
        return 6650.0, 1590.0, "fallback (profiling recipe)"


# --------------------------------------------------------------------------
# clocks sampled during the timed region (NVML, background thread)
# --------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int):
        self.samples, self.reasons, self.ok, self.power = [], 0, False, []
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _poll(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.power.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._poll, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for b, n in _REASONS.items() if self.reasons & b and n != "gpu_idle"]
        out = {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
               "samples": len(self.samples)}
        if self.power:
            out["power_w"] = round(statistics.median(self.power), 1)
        return out


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------
# workload
# --------------------------------------------------------------------------


def build_layer(cfg_name: str, w_shard: torch.Tensor, b_shard: torch.Tensor, device, nvfp4_global=None):
    """One WeightOnlyLinear (the public module API) for this rank's column shard.
    ``nvfp4_global``: the per-tensor NVFP4 scale of the WHOLE weight, so every
    shard quantizes exactly as the unsharded weight would."""
    from qi_b200.quantization import WeightActivationQuantConfig, WeightOnlyLinear
    from qi_b200.quantization.backends import get_backend
    from qi_b200.quantization.quantize import quantize_linear_weight

    from qi_b200.quantization import WeightOnlyQuantConfig

    c = CONFIGS[cfg_name]
    if c["kind"] == "fp8":
        qcfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="fp8", backend="b200",
                                           activation_granularity="per_token", weight_granularity="per_channel")
    elif c["kind"] == "w4a16":
        qcfg = WeightOnlyQuantConfig(enabled=True, algo="rtn", bits=4, group_size=c["group"], symmetric=False,
                                     backend="b200")
    elif c["kind"] == "nvfp4":
        qcfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="nvfp4", bits=4,
                                           activation_bits=4, backend="b200")
    else:
        qcfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="int", backend="b200",
                                           activation_granularity="per_token", weight_granularity="per_channel")
    if c["kind"] == "nvfp4" and nvfp4_global is not None:
        from qi_b200.quantization.quantize import QuantizedLinearWeight, quantize_nvfp4, sf_atom_layout
        packed, sf, g = quantize_nvfp4(w_shard.to(device), global_scale=nvfp4_global.to(device))
        q = QuantizedLinearWeight(qweight=None, scales=None, zeros=None, qweight_packed=packed,
                                  scale_factors=sf_atom_layout(sf), weight_global_scale=g)
    else:
        q = quantize_linear_weight(w_shard.to(device), qcfg)
    lin = torch.nn.Linear(w_shard.shape[1], w_shard.shape[0], bias=True)
    with torch.no_grad():
        lin.bias.copy_(b_shard.float())
    layer = WeightOnlyLinear.from_linear(lin, q, qcfg, get_backend("b200")).to(device)
    layer.bias = layer.bias.to(torch.bfloat16)
    layer.fuse_gelu = c["gelu"]
    return layer


def linear_config(cfg_name: str) -> dict:
    """The workload keys of a single-linear config (the same in both arms)."""
    c = CONFIGS[cfg_name]
    case = c["case"]
    return {"workload": case.name, "M": case.M, "N": case.N, "K": case.K, "bias": True, "gelu": c["gelu"],
            "act_quant": {"w4a16": "none (bf16)",
                          "nvfp4": "nvfp4 block16, dynamic per-tensor global scale"}.get(c["kind"], "per_token"),
            "weight_quant": {"w4a16": "int4 asym g128 packed",
                             "nvfp4": "nvfp4 block16 + per-tensor global scale"}.get(c["kind"], "per_channel")}


_KERNEL_NAMES = {"gemm_int8": "k_gemm_tc<int8>", "gemm_fp8": "k_gemm_tc<fp8>", "gemm_bf16": "k_gemm_tc<bf16>",
                 "gemm_nvfp4": "k_gemm_tc<nvfp4>", "gemm_int8_pair": "k_gemm_tc2<int8>",
                 "gemm_fp8_pair": "k_gemm_tc2<fp8>", "gemm_bf16_pair": "k_gemm_tc2<bf16>",
                 "gemm_nvfp4_pair": "k_gemm_tc2<nvfp4>", "gemm_int8_csk": "k_gemm_csk<int8>",
                 "gemm_fp8_csk": "k_gemm_csk<fp8>", "gemm_bf16_csk": "k_gemm_csk<bf16>",
                 "w4a16_small": "k_gemm_w4a16_small", "w4a16_splitk": "k_gemm_w4a16_skinny"}


def kernel_label(plan: dict) -> str:
    """Name and tile of the kernel the library launched last (qi_b200_last_launch)."""
    k = plan["kernel"]
    name = _KERNEL_NAMES.get(k, k)
    if k.endswith("_pair"):
        return f"{name} (CTA pair, 256 x {plan['tile_n']} tiles, grid {plan['grid']})"
    if k.startswith("gemm_"):
        return f"{name} (128 x {plan['tile_n']} tiles, grid {plan['grid']}, cluster {plan['cluster']})"
    return f"{name} (grid {plan['grid']}, cluster {plan['cluster']})"


def measure_linear(cfg_name: str, args, world: int, rank: int, local: int, device) -> dict:
    """One single-linear config: the device-timed
    step, the dominant kernel alone, the roofline, e2e through the module
    API and (rank 0, N = 1) the CPU baseline.  Returns the result dict."""
    from qi_b200 import _lib, kernels as K

    c = CONFIGS[cfg_name]
    case = c["case"]
    M, N, Kd = case.M, case.N, case.K
    if N % (8 * world):
        raise SystemExit(f"N={N} not divisible into {world} shards of multiples of 8")
    Nl = N // world
    x_cpu, w_cpu, b_cpu = make_linear_inputs(case)
    w_shard, b_shard = w_cpu[rank * Nl:(rank + 1) * Nl], b_cpu[rank * Nl:(rank + 1) * Nl]

    g_full = None
    if c["kind"] == "nvfp4":
        from qi_b200.quantization.quantize import nvfp4_global_scale
        g_full = nvfp4_global_scale(w_cpu.float().abs().amax())
    layer = build_layer(cfg_name, w_shard, b_shard, device, nvfp4_global=g_full)
    kind = {"fp8": _lib.KIND_FP8_E4M3, "int8": _lib.KIND_INT8, "w4a16": None, "nvfp4": None}[c["kind"]]
    if c["kind"] == "fp8":
        wq, ws = layer.weight_fp8, layer.weight_scale
    elif c["kind"] == "int8":
        wq, ws = layer.qweight, layer.scales[:, 0].contiguous()
    elif c["kind"] == "nvfp4":
        wq, ws = layer.qweight_packed, layer.weight_global_scale
    else:
        wq, ws = layer.qweight_packed, None
        wq_bytes = wq.numel() * 4 + layer.scale_factors.numel() * 2 + layer.zeros.numel() * 4

    # rotate input copies so consecutive steps touch more distinct bytes than L2
    per_copy = x_cpu.numel() * 2 + wq.numel() * wq.element_size()
    ncopy = max(2, -(-3 * L2_BYTES // per_copy))
    xs = [x_cpu.to(device) for _ in range(ncopy)]
    wqs = [wq.clone() for _ in range(ncopy)]
    bias = layer.bias
    # NCCL all-gather target: rank-major [P*M, N/P] (the layout ColumnShardedLinear's "rank" gather returns)
    gathered = torch.empty((world * M, Nl), dtype=torch.bfloat16, device=device) if world > 1 else None
    stream = torch.cuda.current_stream(device)

    quant = K.quantize_fp8_rowwise if c["kind"] == "fp8" else K.quantize_int8_rowwise
    # kernels per step: w4a16 1; nvfp4 3 (amax, quantize, GEMM; plus a 4-byte memset); int8/fp8 2
    launches_per_step = {"w4a16": 1, "nvfp4": 3}.get(c["kind"], 2)
    w4_dequant = c["kind"] == "w4a16" and M >= _lib.W4A16_DEQUANT_MIN_M
    if w4_dequant:
        launches_per_step = 2  # weights dequantized once into a workspace, then the bf16 GEMM
    # N > 1, INT8/FP8: the all-gather fused into the GEMM epilogue (peer stores over NVLink)
    # auto: the fused gather where it has been validated on the GPU (2 and 4
    # ranks: 2x NCCL's all-gather after the GEMM at 4); NCCL beyond that
    gather = args.gather if args.gather != "auto" else ("peer" if world in (2, 4) else "nccl")
    peer = world > 1 and gather == "peer" and c["kind"] in ("fp8", "int8")
    peer_api = None
    if peer:
        from qi_b200.sharding import PeerGatherLinear
        peer_api = PeerGatherLinear(layer, max_tokens=M, shard=False)
        launches_per_step = 4  # quantizer, barrier, GEMM with the fused gather, barrier

    def step(i):
        if peer:
            return peer_api(xs[i % ncopy])
        x, w = xs[i % ncopy], wqs[i % ncopy]
        if c["kind"] == "w4a16":
            y = K.w4a16_linear(x, w, layer.scale_factors, layer.zeros, c["group"], bias)
        elif c["kind"] == "nvfp4":
            qa, sfa, ga = K.quantize_nvfp4(x, K.NVFP4_DYNAMIC_TENSOR)
            y = K.nvfp4_gemm(qa, sfa, w, layer.scale_factors, ga, ws, bias)
        else:
            q, s = quant(x)
            y = K.gemm(kind, q, w, s, ws, bias, gelu=c["gelu"])
        if world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(gathered, y)
        return y

    # the dominant kernel alone (activations quantized beforehand): its
    # duration is timed over a graph of back-to-back launches below
    pre = None
    if not peer and c["kind"] in ("nvfp4", "int8", "fp8"):
        pre = [K.quantize_nvfp4(x, K.NVFP4_DYNAMIC_TENSOR) if c["kind"] == "nvfp4" else quant(x) for x in xs]

    def gemm_only(i):
        if peer or pre is None:
            return step(i) if peer else K.w4a16_linear(xs[i % ncopy], wqs[i % ncopy], layer.scale_factors,
                                                       layer.zeros, c["group"], bias)
        if c["kind"] == "nvfp4":
            qa, sfa, ga = pre[i % ncopy]
            return K.nvfp4_gemm(qa, sfa, wqs[i % ncopy], layer.scale_factors, ga, ws, bias)
        q, s = pre[i % ncopy]
        return K.gemm(kind, q, wqs[i % ncopy], s, ws, bias, gelu=c["gelu"])

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(device)

    # Single GPU: the K timed steps are captured once in a CUDA graph (the
    # reference deploys its DiT under CUDA graphs too) so host launch latency
    # does not leak into the device time of small configs.  Multi-GPU: eager
    # steps (the all-gather dominates; NCCL stays outside capture), except the
    # fused peer gather, which is graph-safe.
    use_graph = (world == 1 or peer) and not args.eager
    for i in range(args.warmup):
        step(i)
        gemm_only(i)
    plan = _lib.last_launch()  # the dominant kernel (last launch of gemm_only)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph = None
    launches0 = _lib.launch_count()  # this library's kernels in the K timed steps (graph: counted at capture)
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                step(i)
        graph.replay()  # untimed: uploads the graph
        barrier()
    with ClockSampler(local) as clk:
        barrier()
        t0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                step(i)
        t1.record(stream)
        barrier()
    gpu_launches = _lib.launch_count() - launches0
    if gpu_launches != launches_per_step * args.steps:
        print(f"warning: {gpu_launches} library launches, expected {launches_per_step} x {args.steps}",
              file=sys.stderr)
    ms_total = max_over_ranks(t0.elapsed_time(t1), world, device)
    # dominant kernel: CUDA events around a graph of K back-to-back launches
    # on the same rotating inputs (no event nodes between launches, which
    # would add a launch gap to every small kernel); eager launches for the
    # multi-rank NCCL path
    barrier()
    if use_graph:
        gemm_ms = time_gemm_alone(gemm_only, args.steps, stream)
        gemm_src = f"cuda events around a graph of {args.steps} back-to-back launches (same rotating inputs)"
    else:
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(args.steps):
            gemm_only(i)
        g1.record(stream)
        torch.cuda.synchronize(device)
        gemm_ms = g0.elapsed_time(g1) / args.steps
        gemm_src = f"cuda events around {args.steps} back-to-back eager launches"
    gemm_ms = max_over_ranks(gemm_ms, world, device)
    library = None
    if world == 1 and pre is not None and c["kind"] in ("fp8", "int8"):
        library = library_comparison(kind, pre, wqs, ws, bias, ncopy, args.steps, stream)
    sustained = None
    if args.sustain > 0 and world == 1 and pre is not None:
        sustained = sustained_gemm(c, kind, pre, wqs, ws, layer, bias, ncopy, args, local, stream,
                                   2.0 * M * Nl * Kd)
    _lib.raise_on_device_error()  # a bounded device wait timed out: the numbers are void

    flops_total = 2.0 * M * N * Kd
    ms_step = ms_total / args.steps
    value = flops_total / (ms_step * 1e-3) / 1e12

    # ---- e2e through the public module API with host buffers (N > 1: the
    # column-parallel wrapper around this rank's shard, rank-major gather)
    x_host = x_cpu.pin_memory()
    x_dev = torch.empty_like(xs[0])
    out_shape = (world, M, Nl) if world > 1 else (M, N)
    y_host = torch.empty(out_shape, dtype=torch.bfloat16).pin_memory()
    api_layer = layer
    if peer:
        api_layer = peer_api  # returns the rank-major [P, M, N/P] view
    elif world > 1:
        from qi_b200.sharding import GATHER_RANK_MAJOR, ColumnShardedLinear
        api_layer = ColumnShardedLinear.from_shard(layer, N, gather=GATHER_RANK_MAJOR)

    if world == 1:
        # pinned host rows through HostLinearPipeline: the H2D copy of chunk
        # i + 1, the linear on chunk i and the D2H copy of chunk i - 1 overlap
        from qi_b200.pipeline import HostLinearPipeline, plan_chunks, rows_independent
        pipe = HostLinearPipeline(api_layer)
        from qi_b200.pipeline import M_VARIANT_MIN_CHUNK, m_invariant
        inv = m_invariant(api_layer)
        e2e_chunks = len(plan_chunks(M, None, rows_independent(api_layer), row_bytes=2 * (Kd + N),
                                     min_chunk=1 if inv else M_VARIANT_MIN_CHUNK, graph=inv))
        pipe.capture(x_host, out=y_host)  # the call recorded as a CUDA graph on these pinned buffers

        def e2e_step():
            pipe.replay()
    else:
        e2e_chunks = 1

        def e2e_step():
            x_dev.copy_(x_host, non_blocking=True)
            y_host.copy_(api_layer(x_dev), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device) / args.steps
    h2d = x_host.numel() * 2
    d2h = y_host.numel() * 2

    # ---- roofline of the dominant kernel (the GEMM)
    hbm_gbs, bf16_tf, src = peaks()
    gemm_flops_launch = 2.0 * M * Nl * Kd
    traffic = load_traffic(cfg_name, world)
    if c["kind"] == "w4a16":
        alg_bytes = wq_bytes + Nl * 2 + M * Kd * 2 + M * Nl * 2
        hbm_bound = M <= 16
    elif c["kind"] == "nvfp4":
        # GEMM operands: packed A and B, their block scales, bias, bf16 output
        alg_bytes = (M + Nl) * Kd // 2 + (M + Nl) * Kd // 16 + Nl * 2 + M * Nl * 2
        hbm_bound = False
    else:
        alg_bytes = wq.numel() + Nl * 8 + M * Kd + M * 4 + M * Nl * 2
        hbm_bound = False
    if peer:
        # fused compute + collective: the target time is the slower of the
        # tensor-core time and the NVLink time of the bytes this rank sends
        # (M x N/P bf16 to each of P-1 peers at the measured 770 GB/s per direction)
        link_bytes = M * Nl * 2 * (world - 1)
        t_tensor = gemm_flops_launch / (2 * bf16_tf * 1e12)
        t_link = link_bytes / 770e9
        target = max(t_tensor, t_link)
        roofline = {"bound": "nvlink" if t_link > t_tensor else "tensor",
                    "achieved": round(gemm_flops_launch / (gemm_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                    "peak": round(gemm_flops_launch / target / 1e12, 1), "frac": round(target / (gemm_ms * 1e-3), 4),
                    "traffic": traffic, "algorithmic_bytes": alg_bytes, "nvlink_bytes_sent": link_bytes,
                    "peak_source": f"max(flops / 2 x bf16 measured dense, NVLink bytes / 770 GB/s measured peer copy)"
                                   f" = {target * 1e6:.1f} us; {src}"}
    elif hbm_bound:
        achieved = alg_bytes / (gemm_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_gbs, "unit": "GB/s",
                    "frac": round(achieved / hbm_gbs, 4), "traffic": traffic, "algorithmic_bytes": alg_bytes,
                    "peak_source": src}
    else:
        achieved = gemm_flops_launch / (gemm_ms * 1e-3) / 1e12
        # dense tensor rate relative to bf16 on B200: 8-bit 2x, fp4 4x
        mult = {"w4a16": 1.0, "nvfp4": 4.0}.get(c["kind"], 2.0)
        peak = mult * bf16_tf
        roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "traffic": traffic, "algorithmic_bytes": alg_bytes,
                    "peak_source": f"{mult:g} x bf16 dense, " + src}
    label = kernel_label(plan)
    if w4_dequant:
        label = "k_w4a16_dequant + " + label + ", timed together"
    elif peer:
        label += (" with the all-gather fused into its epilogue (TMA stores to every rank) + 2 barriers "
                  "(activation quantizer included)")
    roofline.update({"kernel": label, "kernel_ms": round(gemm_ms, 5), "kernel_timing": gemm_src})
    if library is not None:
        roofline["library"] = library
    if sustained is not None:
        roofline["sustained"] = sustained

    result = {
        "metric": "quantized_gemm_tops", "value": round(value, 2), "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": c["dtype"], "data": "synthetic (seeded, BASELINE shapes)",
        "config": dict(linear_config(cfg_name),
                       parallelism=(f"N-shard x{world}, all-gather fused into the GEMM epilogue (TMA stores "
                                    "into IPC-mapped peer buffers over NVLink)" if peer
                                    else f"N-shard x{world} + NCCL all_gather") if world > 1 else "single GPU",
                       launch="cuda_graph" if use_graph else "eager",
                       l2=f"{ncopy} rotating input copies ({ncopy * per_copy / 2**20:.0f} MiB > L2)"),
        "e2e": {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TOPS",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "api": (f"qi_b200.pipeline.HostLinearPipeline over WeightOnlyLinear.forward ({e2e_chunks} row "
                        "chunks; H2D, linear and D2H on three streams; captured once, replayed per step)")
                       if world == 1
                       else ("qi_b200.sharding.PeerGatherLinear.forward" if peer
                             else "qi_b200.sharding.ColumnShardedLinear.forward")},
        "gpu_launches": gpu_launches,
        "roofline": roofline,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg_name, samples=3)
    graph = None
    if peer:
        peer_api.check()
        peer_api.close()
    return result


# --------------------------------------------------------------------------
# DiT step
# --------------------------------------------------------------------------


def measure_dit(args, world: int, rank: int, local: int, device, partition: str = "sequence") -> dict:
    """One MoT DiT denoising step (30 blocks, video 3120 + action 32 tokens,
    every Linear INT8 W8A8) replayed from a CUDA graph.  N > 1, partition
    "sequence": video tokens sharded, K/V all-gathered over NCCL once per
    layer; "heads": QKV / cross / ffn.0 N-sharded by heads and FFN columns,
    o / cross-o / ffn.2 row-parallel with exact int32 reductions."""
    from qi_b200 import _lib, dit as D, kernels as K

    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    cfg = D.CFG5 if not args.layers else D.DiTConfig(layers=args.layers)
    model = D.build_mot_dit(cfg, device=device, seed=0)
    tokens, rope, ctx, t_mod, _ = D.make_step_inputs(cfg, device, seed=0)
    runner = D.DiTStepRunner(model, group=group, partition=partition)
    tok_l, rope_l = runner.shard(tokens, rope)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(device)

    if args.eager:  # launch-list profiling: every kernel launched from the host
        runner.static_in = (tok_l, rope_l, ctx, t_mod)

        def run_step():
            runner.static_out = runner.step(*runner.static_in)
            return runner.static_out
        runner.replay = run_step
        run_step()
        per_step_launches = None
    else:
        c0 = _lib.launch_count()
        runner.capture(tok_l, rope_l, ctx, t_mod, warmup=2)  # 2 eager warm-up steps + the captured one
        per_step_launches = (_lib.launch_count() - c0) // 3
    for _ in range(args.warmup):
        runner.replay()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        barrier()
        t0.record(stream)
        for _ in range(args.steps):
            runner.replay()
        t1.record(stream)
        barrier()
    # this library's kernels in the timed steps (graph replays: as captured)
    gpu_launches = (_lib.launch_count() - c0 if per_step_launches is None
                    else per_step_launches * args.steps)
    ms_step = max_over_ranks(t0.elapsed_time(t1), world, device) / args.steps
    runner.check()  # raises if a bounded device wait timed out during the timed steps

    # e2e: host tokens in (pinned), graph replay, this rank's tokens back to host
    host_in = {n: x.cpu().pin_memory() for n, x in tok_l.items()}
    host_out = {n: torch.empty(x.shape, dtype=x.dtype).pin_memory() for n, x in runner.static_out.items()}

    def e2e_step():
        for n, x in host_in.items():
            runner.static_in[0][n].copy_(x, non_blocking=True)
        out = runner.replay()
        for n, x in out.items():
            host_out[n].copy_(x, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device) / args.steps
    h2d = sum(x.numel() * x.element_size() for x in host_in.values())
    d2h = sum(x.numel() * x.element_size() for x in host_out.values())

    # dominant kernel: the video FFN GEMMs (55 % of the step's INT8 ops);
    # time ffn.0 (M = this rank's video tokens, N 14336, K 3072, bias+GELU)
    w0, s0, b0 = runner.tp["video"][0].f0 if partition == "heads" else runner.plans["video"][0].f0
    xa = torch.randn(runner.video_local, cfg.experts[0].hidden, device=device).to(torch.bfloat16)
    qa, sa = K.quantize_int8_rowwise(xa)
    K.gemm(_lib.KIND_INT8, qa, w0, sa, s0, b0, gelu=True)
    plan = _lib.last_launch()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(20):
            K.gemm(_lib.KIND_INT8, qa, w0, sa, s0, b0, gelu=True)
    g.replay()
    torch.cuda.synchronize(device)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    g.replay()
    k1.record(stream)
    torch.cuda.synchronize(device)
    gemm_ms = k0.elapsed_time(k1) / 20
    del g
    m_l = runner.video_local
    # release the step's CUDA graph now: at N > 1 it holds NCCL calls, and a
    # graph still alive at destroy_process_group makes the exit wait
    runner.graph = None
    torch.cuda.synchronize(device)
    hbm_gbs, bf16_tf, src = peaks()
    gemm_ops = 2.0 * m_l * w0.shape[0] * w0.shape[1]
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(2 * bf16_tf, 1),
                "unit": "TFLOP/s", "frac": round(achieved / (2 * bf16_tf), 4),
                "traffic": load_traffic(f"dit_ffn0_m{m_l}", 1),
                "algorithmic_bytes": m_l * w0.shape[1] + w0.numel() + w0.shape[0] * 6 + m_l * 4
                                     + m_l * w0.shape[0] * 2,
                "peak_source": "2 x bf16 dense, " + src, "kernel": kernel_label(plan) + ", video ffn.0 + GELU",
                "kernel_ms": round(gemm_ms, 5), "kernel_timing": "cuda events over 20 graph-captured launches",
                "step_linear_tops": round(cfg.linear_ops() / world / (ms_step * 1e-3) / 1e12, 1)}
    result = {
        "metric": "dit_step_latency_ms", "value": round(ms_step, 4), "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": CONFIGS["dit"]["dtype"],
        "data": "synthetic (seeded random-init MoT weights and tokens)",
        "config": {"workload": "mot_dit_step_cfg5", "layers": cfg.layers, "video_tokens": cfg.experts[0].tokens,
                   "action_tokens": cfg.experts[1].tokens, "heads": f"{cfg.heads}x{cfg.head_dim}",
                   "ctx_tokens": cfg.ctx_tokens, "attention": "bf16 SDPA, first_frame_causal mask in block form",
                   "parallelism": ("single GPU" if world == 1 else
                                   f"video tokens sharded x{world} + NCCL all_gather of K/V per layer"
                                   if partition == "sequence" else
                                   f"heads / FFN columns sharded x{world}: QKV, cross, ffn.0 column-parallel; o, "
                                   "cross-o, ffn.2 row-parallel (NCCL all_reduce MAX of scales + SUM of int32); "
                                   "per-head RMS sums all-gathered"),
                   "launch": "eager" if args.eager else "cuda_graph", "linear_ops_per_step": cfg.linear_ops(),
                   "l2": "5.9 GB of INT8 weights streamed per step (> L2), no flush needed"},
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "qi_b200.dit.DiTStepRunner (graph replay) with pinned host tokens"},
        "gpu_launches": gpu_launches,
        "roofline": roofline,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = dit_cpu_baseline()
    return result


# the configs of one full run: N = 1 every BASELINE config, N > 1 the ones
# that shard (config 2 is the headline line itself)
ALL_CONFIGS_1GPU = ["int8", "w4a16_m1", "w4a16_m16", "w4a16_m256", "w4a16_m4096", "nvfp4", "fp8", "dit"]
ALL_CONFIGS_NGPU = ["fp8", "dit", "dit_tp"]


def run_ours(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def measure(name):
        torch.cuda.empty_cache()
        if CONFIGS[name]["kind"] == "dit":
            return measure_dit(args, world, rank, local, device, CONFIGS[name]["partition"])
        return measure_linear(name, args, world, rank, local, device)

    result = measure(args.config)
    if not args.only:
        result["configs"] = {}
        for name in (ALL_CONFIGS_1GPU if world == 1 else ALL_CONFIGS_NGPU):
            if name != args.config:
                result["configs"][name] = measure(name)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(result)


def _dit_cpu_layer_sample():
    """The reference's CPU path for the 20 quantized Linears of ONE layer
    (video + action, full token counts), INT8 per-token fake quant through
    the ported ``ReferenceBackend.linear``."""
    from oracle import reference_port as RP
    from qi_b200.dit import CFG5
    from qi_b200.quantization.quantize import quantize_weight_rtn

    cfg = CFG5
    g = torch.Generator().manual_seed(0)
    a = cfg.attn_dim
    calls = []
    for e in cfg.experts:
        shapes = [(e.tokens, e.hidden, a)] * 3 + [(e.tokens, a, e.hidden)] + [(e.tokens, e.hidden, a)] \
            + [(cfg.ctx_tokens, e.hidden, a)] * 2 + [(e.tokens, a, e.hidden)] \
            + [(e.tokens, e.hidden, e.ffn), (e.tokens, e.ffn, e.hidden)]
        for m, kd, n in shapes:
            x = torch.randn(m, kd, generator=g).to(torch.bfloat16)
            qw, sw, _ = quantize_weight_rtn(torch.randn(n, kd, generator=g) * 0.02, 8, -1, True)
            b = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
            calls.append((x, qw, sw, b))

    def fn():
        for x, qw, sw, b in calls:
            RP.reference_linear(x, qw, sw, None, b, 8, -1, True, activation_granularity="per_token")
    return fn, cfg


def dit_cpu_baseline():
    torch.set_num_threads(os.cpu_count() or 1)
    fn, cfg = _dit_cpu_layer_sample()
    fn()
    t = time.perf_counter()
    fn()
    dt = time.perf_counter() - t
    return {"value": round(dt * 1e3 * cfg.layers, 1), "unit": "ms", "cores": torch.get_num_threads(),
            "cpu_model": cpu_model(), "kind": "port",
            "sample": "ReferenceBackend.linear port over the 20 INT8 Linears of 1 of 30 layers (full token "
                      "counts), scaled x30; attention and norms not included",
            "ms_per_layer": round(dt * 1e3, 1)}


def library_comparison(kind, pre, wqs, ws, bias, ncopy, steps, stream) -> dict:
    """The same quantized GEMM through NVIDIA's library on the same operands,
    timed like the dominant kernel (a graph of back-to-back launches), beside
    this library's kernel with the same epilogue: FP8 through cuBLASLt
    (torch._scaled_mm: per-row x per-column scales, bias, bf16 out; it fuses
    no GELU), INT8 through cuBLAS (torch._int_mm: int32 accumulators out, so
    ours returns its raw int32 accumulators too).  Each side is timed twice,
    interleaved, best of the two."""
    from qi_b200 import _lib, kernels as K

    fp8 = kind == _lib.KIND_FP8_E4M3
    if fp8:
        f8 = torch.float8_e4m3fn
        ws_row = ws.reshape(1, -1).float().contiguous()
        sas = [s.reshape(-1, 1).contiguous() for _, s in pre]
        name = "cuBLASLt FP8 via torch._scaled_mm (per-row x per-column scales, bias, bf16 out)"

        def lib(i):
            q, _ = pre[i % ncopy]
            return torch._scaled_mm(q.view(f8), wqs[i % ncopy].view(f8).t(), scale_a=sas[i % ncopy],
                                    scale_b=ws_row, bias=bias, out_dtype=torch.bfloat16)

        def ours(i):
            q, s = pre[i % ncopy]
            return K.gemm(kind, q, wqs[i % ncopy], s, ws, bias)
    else:
        name = "cuBLAS INT8 via torch._int_mm (int32 accumulators out)"

        def lib(i):
            return torch._int_mm(pre[i % ncopy][0], wqs[i % ncopy].t())

        def ours(i):
            return K.gemm(kind, pre[i % ncopy][0], wqs[i % ncopy], None, None, raw_acc=True)
    try:
        lib(0)  # eager first call: the library sets up its handle and workspace outside graph capture
        ours(0)
        torch.cuda.synchronize()
        t_lib, t_ours = [], []
        for _ in range(2):
            t_ours.append(time_gemm_alone(ours, steps, stream))
            t_lib.append(time_gemm_alone(lib, steps, stream))
    except Exception as e:  # the library may not take this shape
        return {"name": name, "error": repr(e)[:200]}
    return {"name": name, "library_ms": round(min(t_lib), 5), "ours_same_epilogue_ms": round(min(t_ours), 5),
            "library_over_ours": round(min(t_lib) / min(t_ours), 3)}


def sustained_gemm(c, kind, pre, wqs, ws, layer, bias, ncopy, args, local, stream, flops) -> dict:
    """The dominant GEMM replayed back to back for ``args.sustain`` seconds,
    with the config's operands and again with all-zero operand codes (same
    scales), while NVML samples the SM clock, throttle reasons and board power.
    Zero codes toggle no multiplier bits: the gap between the two rows is what
    the board power cap takes from the kernel."""
    from qi_b200 import kernels as K

    def make(zero):
        if c["kind"] == "nvfp4":
            ops = [(torch.zeros_like(qa) if zero else qa, sfa, ga) for qa, sfa, ga in pre]
            ws_ = [torch.zeros_like(w) if zero else w for w in wqs]
            return lambda i: K.nvfp4_gemm(*ops[i % ncopy][:2], ws_[i % ncopy], layer.scale_factors,
                                          ops[i % ncopy][2], ws, bias)
        ops = [(torch.zeros_like(q) if zero else q, s) for q, s in pre]
        ws_ = [torch.zeros_like(w) if zero else w for w in wqs]
        return lambda i: K.gemm(kind, ops[i % ncopy][0], ws_[i % ncopy], ops[i % ncopy][1], ws, bias,
                                gelu=c["gelu"])

    out = {"seconds": args.sustain}
    for name in ("operands", "zero_operands"):
        f = make(name == "zero_operands")
        n = 20
        f(0)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                f(i)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 0
        with ClockSampler(local) as clk:
            time.sleep(0.2)
            a.record(stream)
            t0 = time.time()
            while time.time() - t0 < args.sustain:
                g.replay()
                reps += 1
                if reps % 10 == 0:
                    torch.cuda.synchronize()
            b.record(stream)
            torch.cuda.synchronize()
        us = a.elapsed_time(b) / (reps * n) * 1e3
        out[name] = {"us": round(us, 2), "tflops": round(flops / (us * 1e-6) / 1e12, 1), **clk.summary()}
        del g
    return out


def time_gemm_alone(step, steps, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            step(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def load_traffic(cfg_name: str, world: int):
    """DRAM bytes per GEMM launch from a committed ncu capture, if any."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        v = d.get(f"{cfg_name}_x{world}")
        return None if v is None else v["bytes_per_launch"]
    except Exception:
        return None


# --------------------------------------------------------------------------
# CPU baseline: the reference's own algorithm (port) on this host's cores
# --------------------------------------------------------------------------


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the baseline's record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def _cpu_sample(cfg_name: str):
    """Inputs and a callable for one CPU call of the reference path over the
    config's full input (every row)."""
    from oracle import reference_port as RP
    from qi_b200.quantization.quantize import quantize_to_fp8_e4m3_rowwise, quantize_weight_rtn

    c = CONFIGS[cfg_name]
    case = c["case"]
    x, w, b = make_linear_inputs(case)
    rows = case.M
    xs = x[:rows].contiguous()
    if c["kind"] == "nvfp4":
        from qi_b200.quantization.quantize import quantize_nvfp4
        wp, wsf, wg = quantize_nvfp4(w)
        fn = lambda: RP.nvfp4_linear_port(xs, wp, wsf, wg, b)
        desc = f"dequantise-then-F.linear NVFP4 port (per-tensor fake-quant, fp32 compute), {rows} of {case.M} rows"
    elif c["kind"] == "w4a16":
        qw, sw, zw = quantize_weight_rtn(w, 4, c["group"], False)
        fn = lambda: RP.reference_linear(xs, qw, sw, zw, b, 4, c["group"], False)
        desc = f"ReferenceBackend.linear port (bf16 input, int4 g{c['group']} dequant loop, F.linear), {rows} of {case.M} rows"
    elif c["kind"] == "int8":
        qw, sw, _ = quantize_weight_rtn(w, 8, -1, True)
        fn = lambda: RP.reference_linear(xs, qw, sw, None, b, 8, -1, True, activation_granularity="per_token")
        desc = f"ReferenceBackend.linear port (bf16 input, per-token int8 fake-quant, dequant loop, F.linear), {rows} of {case.M} rows"
    else:
        wq, ws = quantize_to_fp8_e4m3_rowwise(w)
        fn = lambda: RP.fp8_linear_port(xs, wq, ws, b, gelu=c["gelu"])
        desc = f"dequantise-then-F.linear FP8 port (per-token fake-quant, fp32 compute, GELU), {rows} of {case.M} rows"
    return fn, rows, case, desc


def cpu_baseline(cfg_name: str, samples: int = 3):
    torch.set_num_threads(os.cpu_count() or 1)
    fn, rows, case, desc = _cpu_sample(cfg_name)
    fn()
    ts = []
    for _ in range(samples):
        t = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t)
    t = statistics.median(ts)
    return {"value": round(2.0 * rows * case.N * case.K / t / 1e12, 5), "unit": "TOPS",
            "cores": torch.get_num_threads(), "cpu_model": cpu_model(), "kind": "port",
            "sample": desc + f", median of {samples}", "ms_per_call": round(t * 1e3, 2)}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    result = reference_result(args.config, args, world)
    if not args.only:
        # the other configs' reference CPU path, a few calls each (same keys as ours)
        result["configs"] = {}
        for name in (ALL_CONFIGS_1GPU if world == 1 else ALL_CONFIGS_NGPU):
            if name != args.config:
                result["configs"][name] = reference_result(name, args, world, steps=2, warmup=1)
    emit(result)


def reference_result(cfg_name: str, args, world: int, steps: int | None = None, warmup: int | None = None) -> dict:
    """The reference's CPU algorithm (port) for one config, timed on all host threads."""
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    if CONFIGS[cfg_name]["kind"] == "dit":
        fn, cfg = _dit_cpu_layer_sample()
        for _ in range(max(1, warmup)):
            fn()
        t = time.perf_counter()
        for _ in range(steps):
            fn()
        ms = (time.perf_counter() - t) / steps * 1e3 * cfg.layers
        return {
            "impl": "reference", "metric": "dit_step_latency_ms", "value": round(ms, 1), "unit": "ms",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 1),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": CONFIGS["dit"]["dtype"],
            "data": "synthetic", "config": {"workload": "mot_dit_step_cfg5"},
            "cpu_baseline": {"value": round(ms, 1), "unit": "ms", "cores": torch.get_num_threads(),
                             "cpu_model": cpu_model(), "kind": "port",
                             "sample": "20 INT8 Linears of 1 of 30 layers per step (full token counts), scaled x30"},
            "e2e": {"value": round(ms, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    fn, rows, case, desc = _cpu_sample(cfg_name)
    for _ in range(warmup):
        fn()
    t = time.perf_counter()
    for _ in range(steps):
        fn()
    dt = (time.perf_counter() - t) / steps
    value = 2.0 * rows * case.N * case.K / dt / 1e12
    c = CONFIGS[cfg_name]
    return {
        "impl": "reference", "metric": "quantized_gemm_tops", "value": round(value, 5), "unit": "TOPS",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": c["dtype"],
        "data": "synthetic (seeded, BASELINE shapes)",
        "config": linear_config(cfg_name),
        "cpu_baseline": {"value": round(value, 5), "unit": "TOPS", "cores": torch.get_num_threads(),
                         "cpu_model": cpu_model(), "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 5), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# The JSON result line goes to the process's original stdout; everything
# else that would reach fd 1 (library banners such as NCCL's version line,
# stray prints) is sent to stderr, so stdout carries exactly one line.
_RESULT_FD = None


def emit(obj) -> None:
    line = (json.dumps(obj) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, line)


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="fp8", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", action="store_true", help="measure --config alone (no configs map)")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph for the timed steps")
    ap.add_argument("--gather", default="auto", choices=["auto", "peer", "nccl"],
                    help="N > 1, INT8/FP8: all-gather fused into the GEMM epilogue (peer), a separate "
                         "NCCL call (nccl), or auto (peer at 2 ranks, NCCL beyond)")
    ap.add_argument("--sustain", type=float, default=0.0,
                    help="single-linear configs, 1 GPU: also replay the dominant GEMM for this many seconds "
                         "with the config's operands and with all-zero codes, sampling clocks and power")
    ap.add_argument("--layers", type=int, default=0,
                    help="dit only: fewer layers than config 5's 30 (profiling captures; not a bench value)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
