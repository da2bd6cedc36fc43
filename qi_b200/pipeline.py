"""Quantized linears over pinned HOST buffers, with the copies overlapped.

A ``WeightOnlyLinear`` (``qi_b200.quantization.modules``) computes on device
tensors, as the reference's module does (``src/qi/quantization/modules.py``).
A caller whose activations live in host memory otherwise pays three
serialised legs per call: host -> device of x, the linear, device -> host of
y.  ``HostLinearPipeline`` splits the rows into chunks and runs the legs on
three CUDA streams, so the host -> device copy of chunk i + 1, the linear on
chunk i and the device -> host copy of chunk i - 1 run at the same time (the
two copy directions use separate copy engines and PCIe is full duplex).  The
call then costs about the larger of the two transfers.

Rows are independent for every activation format except dynamic per-tensor
NVFP4, whose global scale is the amax of the whole input: that format runs
as one chunk.  The linear on a chunk is the module's own forward, so results
equal ``layer(x.cuda()).cpu()`` bit for bit wherever the GEMM's per-element
arithmetic does not depend on M (always for INT8; for the floating-point
formats unless the full-size launch splits its last wave along K).
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


def plan_chunks(rows: int, chunk_rows: int | None, independent: bool) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) of the chunks.  Default chunk: an eighth of the
    rows rounded up to a multiple of 128, at least 256 rows (fewer, longer
    GEMMs once the copies are short)."""
    if rows <= 0:
        return []
    if not independent:
        return [(0, rows)]
    if chunk_rows is None:
        chunk_rows = max(256, 128 * math.ceil(rows / 8 / 128))
    if chunk_rows <= 0:
        raise ValueError(f"chunk_rows must be positive, got {chunk_rows}.")
    return [(r0, min(rows, r0 + chunk_rows)) for r0 in range(0, rows, chunk_rows)]


class HostLinearPipeline:
    """``y_host = layer(x_host)`` for pinned host tensors, pipelined by row chunks.

    ``x_host`` is a pinned CPU tensor [..., in_features] (bf16, or any dtype the
    layer accepts); the result is written into ``out`` (a pinned CPU tensor
    [..., out_features] of the layer's output dtype, allocated pinned when not
    given).  Everything is enqueued asynchronously after the work already on
    the caller's current stream, and the current stream waits for the last
    copy: synchronise it before reading ``out`` on the host, as with any
    non-blocking copy.  Device staging buffers (two chunks of x) are kept
    between calls; the linear's own outputs and workspaces come from torch's
    caching allocator on the compute stream."""

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
        self.s_h2d = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_d2h = torch.cuda.Stream(self.device)
        self._x = [None, None]
        self._h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
        self._comp_done = [torch.cuda.Event(), torch.cuda.Event()]

    def _slot(self, s: int, rows: int, cols: int, dtype) -> torch.Tensor:
        b = self._x[s]
        if b is None or b.shape[0] < rows or b.shape[1] != cols or b.dtype != dtype:
            with torch.cuda.stream(self.s_h2d):
                b = torch.empty((rows, cols), dtype=dtype, device=self.device)
            b.record_stream(self.s_comp)
            self._x[s] = b
        return b[:rows]

    def __call__(self, x_host: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x_host.is_cuda:
            raise ValueError("HostLinearPipeline takes a host tensor; call the layer directly on device tensors.")
        if not x_host.is_pinned():
            raise ValueError("x_host must be in pinned memory (tensor.pin_memory()).")
        kin = self.layer.in_features
        if x_host.shape[-1] != kin:
            raise ValueError(f"x_host has {x_host.shape[-1]} features, the layer takes {kin}.")
        x2 = x_host.reshape(-1, kin)
        if not x2.is_contiguous():
            raise ValueError("x_host must be contiguous.")
        rows, n_out = x2.shape[0], self.layer.out_features
        if out is None:
            out = torch.empty((*x_host.shape[:-1], n_out), dtype=x_host.dtype).pin_memory()
        if out.is_cuda or not out.is_pinned() or not out.is_contiguous():
            raise ValueError("out must be a contiguous pinned host tensor.")
        if out.numel() != rows * n_out:
            raise ValueError(f"out must hold {rows} x {n_out} elements.")
        y2 = out.view(rows, n_out)
        chunks = plan_chunks(rows, self.chunk_rows, self.independent)
        if not chunks:
            return out
        span = max(r1 - r0 for r0, r1 in chunks)
        main = torch.cuda.current_stream(self.device)
        for s in (self.s_h2d, self.s_comp, self.s_d2h):
            s.wait_stream(main)
        for i, (r0, r1) in enumerate(chunks):
            s = i % 2
            xs = self._slot(s, span, kin, x2.dtype)[: r1 - r0]
            with torch.cuda.stream(self.s_h2d):
                if i >= 2:
                    self.s_h2d.wait_event(self._comp_done[s])  # the linear has read this slot
                xs.copy_(x2[r0:r1], non_blocking=True)
                self._h2d_done[s].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self._h2d_done[s])
                y = self.layer(xs)
                self._comp_done[s].record(self.s_comp)
            y.record_stream(self.s_d2h)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(self._comp_done[s])
                y2[r0:r1].copy_(y.view(r1 - r0, n_out), non_blocking=True)
        main.wait_stream(self.s_d2h)
        return out
