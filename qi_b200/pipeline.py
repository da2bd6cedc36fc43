"""Quantized linears over pinned HOST buffers, with the copies overlapped.

A ``WeightOnlyLinear`` (``qi_b200.quantization.modules``) computes on device
tensors, as the reference's module does (``src/qi/quantization/modules.py``).
A caller whose activations live in host memory otherwise pays three
serialised legs per call: host -> device of x, the linear, device -> host of
y.  ``HostLinearPipeline`` splits the rows into chunks and overlaps the host
-> device copy of chunk i + 1, the linear on chunk i and the device -> host
copy of chunk i - 1 (the two copy directions use separate copy engines and
PCIe is full duplex).  The call then costs about the larger of the two
transfers.

Rows are independent for every activation format except dynamic per-tensor
NVFP4, whose global scale is the amax of the whole input: that format runs
as one chunk.  The linear on a chunk is the module's own forward, so results
equal ``layer(x.cuda()).cpu()`` bit for bit wherever the GEMM's per-element
arithmetic does not depend on M: always for INT8; for FP8 / NVFP4 unless the
full-size launch splits its last wave along K (long K only); weight-only
formats keep chunks above their small-M kernels' 256 rows.
"""

from __future__ import annotations

import math

import torch


def rows_independent(layer) -> bool:
    """False only for dynamic per-tensor NVFP4 activations (one global scale
    from the amax of all rows)."""
    nvfp4 = (getattr(layer, "qweight_packed", None) is not None and layer.qweight_packed.dtype == torch.uint8
             and getattr(layer, "scale_factors", None) is not None
             and getattr(layer, "weight_global_scale", None) is not None)
    if not nvfp4:
        return True
    return layer.activation_scale is not None or layer.activation_granularity == "per_token"


# Weight-only formats pick their kernel by M (small-M kernels up to 256 rows,
# dequantize + bf16 GEMM above), and the kernels round differently: their
# chunks stay above that bound so every chunk runs the full-M arithmetic.
M_VARIANT_MIN_CHUNK = 384


def m_invariant(layer) -> bool:
    """True when each output element's arithmetic does not depend on the
    number of rows in the call (activation-quantized formats); False for the
    weight-only formats (W4A16 packed, or the reference's int8 code layout
    without per-token activations)."""
    qp = getattr(layer, "qweight_packed", None)
    if qp is not None and qp.dtype == torch.int32:
        return False
    if (getattr(layer, "qweight", None) is not None and getattr(layer, "weight_fp8", None) is None
            and qp is None and getattr(layer, "activation_granularity", None) != "per_token"):
        return False
    return True


def plan_chunks(rows: int, chunk_rows: int | None, independent: bool,
                row_bytes: int = 0, min_chunk: int = 1, graph: bool = False) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) of the chunks.  By default (``chunk_rows`` None)
    the transfer is split only when it is large: one chunk per 16 MiB of
    host<->device bytes (``row_bytes`` per row, in + out), at most 8 chunks
    (``graph``: one per 8 MiB, at most 16, since a CUDA-graph replay has no
    per-chunk host cost), each a multiple of 128 rows and at least 256 rows.
    Below that the copies take less time than the extra stream
    synchronisation saves.  Chunks are never shorter than ``min_chunk`` rows
    (one chunk when rows <= min_chunk)."""
    if rows <= 0:
        return []
    if not independent or rows <= min_chunk:
        return [(0, rows)]
    if chunk_rows is None:
        n = min(16, (rows * row_bytes) // (8 << 20)) if graph else min(8, (rows * row_bytes) // (16 << 20))
        if n <= 1:
            return [(0, rows)]
        chunk_rows = max(256, 128 * math.ceil(rows / n / 128))
    if chunk_rows <= 0:
        raise ValueError(f"chunk_rows must be positive, got {chunk_rows}.")
    chunk_rows = max(chunk_rows, min_chunk)
    spans = [(r0, min(rows, r0 + chunk_rows)) for r0 in range(0, rows, chunk_rows)]
    if len(spans) > 1 and spans[-1][1] - spans[-1][0] < min_chunk:  # fold a short tail into its neighbour
        spans[-2:] = [(spans[-2][0], rows)]
    return spans


class HostLinearPipeline:
    """``y_host = layer(x_host)`` for pinned host tensors, pipelined by row chunks.

    ``x_host`` is a pinned CPU tensor [..., in_features] (bf16, or any dtype the
    layer accepts); the result is written into ``out`` (a pinned CPU tensor
    [..., out_features] of the layer's output dtype, allocated pinned when not
    given).  Three streams: host -> device copies, the linear, device -> host
    copies.  The linear's output is allocated, copied into one of two
    persistent device output slots and freed on the compute stream, so the
    caching allocator never tracks a block across streams (a block freed
    while another stream still reads it is held back from reuse, and in a
    loop that starves the pool into fresh allocations).  Everything is
    asynchronous after the work already on the caller's current stream, which
    waits for the last copy: synchronise it before reading ``out`` on the
    host, as with any non-blocking copy."""

    def __init__(self, layer, chunk_rows: int | None = None, device: torch.device | str | None = None):
        self.layer = layer
        self.chunk_rows = chunk_rows
        if device is None:
            buf = next((b for b in layer.buffers()), None)
            device = buf.device if buf is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("HostLinearPipeline runs the layer on a CUDA device.")
        self.independent = rows_independent(layer)
        self.m_invariant = m_invariant(layer)
        self.s_h2d = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_d2h = torch.cuda.Stream(self.device)
        self._x = [None, None]
        self._y = [None, None]
        self._h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
        self._comp_done = [torch.cuda.Event(), torch.cuda.Event()]
        self._d2h_done = [torch.cuda.Event(), torch.cuda.Event()]

    def _buf(self, bufs, s: int, rows: int, cols: int, dtype, users) -> torch.Tensor:
        b = bufs[s]
        if b is None or b.shape[0] < rows or b.shape[1] != cols or b.dtype != dtype:
            if b is not None:
                for st in users:  # freed now: not reused before the pending copies that touch it end
                    b.record_stream(st)
            b = bufs[s] = torch.empty((rows, cols), dtype=dtype, device=self.device)
        return b[:rows]

    def capture(self, x_host: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Record one call on these pinned buffers as a CUDA graph (after one
        eager call that sets up the staging buffers); ``replay()`` then reruns
        all its copies and kernels with no per-chunk host work, so finer chunks
        pay off.  The buffers' contents may change between replays, their
        addresses may not.  Returns ``out``."""
        if out is None:
            out = torch.empty((*x_host.shape[:-1], self.layer.out_features), dtype=x_host.dtype).pin_memory()
        self._graph_chunks = True
        try:
            self(x_host, out)
            torch.cuda.current_stream(self.device).synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self(x_host, out)
        finally:
            self._graph_chunks = False
        self._graph, self._graph_out = g, out
        return out

    def replay(self) -> torch.Tensor:
        """Rerun the captured call on the caller's current stream's device
        (asynchronous, as the call itself); returns its ``out``."""
        if getattr(self, "_graph", None) is None:
            raise RuntimeError("capture() first.")
        self._graph.replay()
        return self._graph_out

    def __call__(self, x_host: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x_host.is_cuda:
            raise ValueError("HostLinearPipeline takes a host tensor; call the layer directly on device tensors.")
        kin = self.layer.in_features
        if x_host.shape[-1] != kin:
            raise ValueError(f"x_host has {x_host.shape[-1]} features, the layer takes {kin}.")
        x2 = x_host.reshape(-1, kin)
        if not x2.is_contiguous():
            raise ValueError("x_host must be contiguous.")
        rows, n_out = x2.shape[0], self.layer.out_features
        if out is None:
            out = torch.empty((*x_host.shape[:-1], n_out), dtype=x_host.dtype).pin_memory()
        if out.is_cuda or not out.is_contiguous():
            raise ValueError("out must be a contiguous pinned host tensor.")
        if out.numel() != rows * n_out:
            raise ValueError(f"out must hold {rows} x {n_out} elements.")
        if not (x_host.is_pinned() and out.is_pinned()):
            raise ValueError("x_host and out must be in pinned memory (tensor.pin_memory()).")
        y2 = out.view(rows, n_out)
        chunks = plan_chunks(rows, self.chunk_rows, self.independent,
                             row_bytes=kin * x2.element_size() + n_out * out.element_size(),
                             min_chunk=1 if self.m_invariant else M_VARIANT_MIN_CHUNK,
                             # weight-only formats dequantize the weights for every chunk: few chunks
                             graph=getattr(self, "_graph_chunks", False) and self.m_invariant)
        if not chunks:
            return out
        main = torch.cuda.current_stream(self.device)
        if len(chunks) == 1:
            # one chunk: the three legs in order on the caller's stream
            xs = self._buf(self._x, 0, rows, kin, x2.dtype, (main, self.s_h2d, self.s_comp))
            xs.copy_(x2, non_blocking=True)
            y2.copy_(self.layer(xs).view(rows, n_out), non_blocking=True)
            return out
        span = max(r1 - r0 for r0, r1 in chunks)
        for st in (self.s_h2d, self.s_comp, self.s_d2h):
            st.wait_stream(main)
        for i, (r0, r1) in enumerate(chunks):
            s, n = i % 2, r1 - r0
            xs = self._buf(self._x, s, span, kin, x2.dtype, (main, self.s_h2d, self.s_comp))[:n]
            ys = self._buf(self._y, s, span, n_out, out.dtype, (main, self.s_comp, self.s_d2h))[:n]
            with torch.cuda.stream(self.s_h2d):
                if i >= 2:
                    self.s_h2d.wait_event(self._comp_done[s])  # the linear has read this x slot
                xs.copy_(x2[r0:r1], non_blocking=True)
                self._h2d_done[s].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self._h2d_done[s])
                if i >= 2:
                    self.s_comp.wait_event(self._d2h_done[s])  # this y slot has been copied out
                ys.copy_(self.layer(xs).view(n, n_out))
                self._comp_done[s].record(self.s_comp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(self._comp_done[s])
                y2[r0:r1].copy_(ys, non_blocking=True)
                self._d2h_done[s].record(self.s_d2h)
        main.wait_stream(self.s_d2h)
        return out
