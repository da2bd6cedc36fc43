"""Tensor-parallel sharding of quantized linears over GPUs of one node.

One process per GPU, ``torch.distributed`` (NCCL over NVLink/NVSwitch) for the
exchange.  Two layouts:

* **Column parallel** (``ColumnShardedLinear``).  Rank ``r`` of ``P`` holds
  output channels ``[r*N/P, (r+1)*N/P)`` of the quantized weight, with its
  per-channel scales, zeros and bias.  X is replicated.  Each rank runs the
  local B200 kernel.  ``dist.all_gather_into_tensor`` then assembles Y.  Every
  output column is computed by exactly one rank with the single-GPU kernel.
  So the gathered Y equals the single-GPU Y bit for bit in every format.
  This is the BASELINE scheme for QKV (N = 3x3072) and FFN-up (N = 14336).
  The reference runs one GPU only; its linear is ``modules.py:113-133`` ->
  ``backend.linear``.
* **Row parallel, INT8 W8A8** (``RowShardedInt8Linear``).  Rank ``r`` holds
  input channels ``[r*K/P, (r+1)*K/P)`` of ``qweight``.  It receives the
  matching slice of X, for example the un-gathered output of a
  column-parallel FFN-up.  The reference's per-token scale needs the amax of
  the whole row (``quantize_int8.cu:7-59``), so the flow is:

  1. each rank computes the INT8 scales of its slice;
  2. ``all_reduce(MAX)`` on those scales (M fp32).  Division by 127 and
     ``max`` are monotone, so this is exactly the whole-row scale;
  3. each rank quantizes its slice with the shared scales and runs the raw
     int32 GEMM;
  4. ``all_reduce(SUM)`` on the int32 partials is exact and associative;
  5. one epilogue kernel applies the scales, the bias (added once) and an
     optional GELU.

  The result is bit-identical to the single-GPU ``int8_linear``.

The collectives are plain NCCL calls on torch's current stream.  No kernel
here reads peer memory; every TMA load has one destination CTA.  The local compute
goes through an ``ops`` object.  The default is the sm_100a kernels.  CPU
tests pass an oracle-backed stand-in and run the same exchange logic on
``gloo``.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn as nn

from .quantization.modules import WeightOnlyLinear

GATHER_FULL = "full"          # Y as [..., N] (rank-major blocks are re-interleaved)
GATHER_RANK_MAJOR = "rank"    # Y as [P, M, N/P] (no copy after the collective)
GATHER_NONE = "none"          # this rank's [..., N/P] only (feeds a row-parallel layer)


def _group_info(group):
    return dist.get_rank(group), dist.get_world_size(group)


def _split(n: int, world: int, what: str, multiple: int = 1) -> int:
    if n % world:
        raise ValueError(f"{what}={n} is not divisible by the world size {world}.")
    part = n // world
    if part % multiple:
        raise ValueError(f"{what}/world={part} must be a multiple of {multiple} for this format.")
    return part


# ---------------------------------------------------------------------------
# weight slicing (host side, done once at load)
# ---------------------------------------------------------------------------


def _nvfp4_sf_block_bytes(k: int) -> int:
    """Bytes of one 128-row block of the NVFP4 scale-factor atom layout."""
    s = k // 16
    return -(-s // 4) * 512


def column_shard_buffers(layer: WeightOnlyLinear, rank: int, world: int) -> WeightOnlyLinear:
    """A ``WeightOnlyLinear`` holding output channels ``[rank*N/P, (rank+1)*N/P)``.

    Per-output-channel buffers are sliced on dim 0.  Per-tensor buffers
    (``weight_global_scale``, a 1-element ``weight_scale``,
    ``activation_scale``) and the per-input-channel ``input_scale`` are
    shared.  For NVFP4, ``scale_factors`` is the flat atom layout.  Its
    outermost dimension is 128-row blocks, so N/P must be a multiple of 128
    and the slice is a contiguous byte range.
    """
    n = layer.out_features
    part = _split(n, world, "out_features")
    lo, hi = rank * part, (rank + 1) * part

    def rows(t):
        return None if t is None else t[lo:hi].contiguous()

    nvfp4 = layer.qweight_packed is not None and layer.qweight_packed.dtype == torch.uint8 \
        and layer.scale_factors is not None and layer.weight_global_scale is not None
    if nvfp4:
        _split(n, world, "out_features", 128)
        blk = _nvfp4_sf_block_bytes(layer.in_features)
        sf = layer.scale_factors.reshape(-1)[lo // 128 * blk: hi // 128 * blk].contiguous()
    else:
        sf = rows(layer.scale_factors)
    ws = layer.weight_scale
    if ws is not None and ws.numel() == n:
        ws = ws.reshape(n)[lo:hi].contiguous()
    scales = layer.scales
    if scales is not None and scales.numel() == 1:
        scales = scales.clone()
    else:
        scales = rows(scales)
    out = WeightOnlyLinear(
        qweight=rows(layer.qweight), scales=scales, zeros=rows(layer.zeros),
        bias=rows(layer.bias), in_features=layer.in_features, out_features=part, bits=layer.bits,
        group_size=layer.group_size, symmetric=layer.symmetric, backend=layer.backend,
        input_scale=layer.input_scale, qweight_packed=rows(layer.qweight_packed), scale_factors=sf,
        weight_global_scale=layer.weight_global_scale, activation_scale=layer.activation_scale,
        weight_scale=ws, weight_fp8=rows(layer.weight_fp8),
        activation_granularity=layer.activation_granularity, weight_granularity=layer.weight_granularity,
        keep_output_dtype=layer.keep_output_dtype)
    out.fuse_gelu = layer.fuse_gelu
    return out


# ---------------------------------------------------------------------------
# column parallel
# ---------------------------------------------------------------------------


class ColumnShardedLinear(nn.Module):
    """Output-channel shard of a quantized linear plus an NCCL all-gather.

    ``forward(x)`` takes the replicated activation ``[..., K]``.  The return
    value depends on ``gather``: ``"full"`` gives ``[..., N]``; ``"rank"``
    gives ``[P, M, N/P]`` with no copy after the collective; ``"none"`` gives
    this rank's ``[..., N/P]`` (the head-local QKV of tensor-parallel
    attention, or the input of a row-parallel layer).
    """

    def __init__(self, layer: WeightOnlyLinear, group=None, gather: str = GATHER_FULL):
        super().__init__()
        rank, world = _group_info(group)
        self._setup(column_shard_buffers(layer, rank, world), layer.out_features, group, gather)

    @classmethod
    def from_shard(cls, local: WeightOnlyLinear, out_features: int, group=None,
                   gather: str = GATHER_FULL) -> "ColumnShardedLinear":
        """Wrap a layer that already holds only this rank's output channels
        (weights quantized per rank at load time, never materialized whole)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self._setup(local, out_features, group, gather)
        return self

    def _setup(self, local, out_features, group, gather):
        if gather not in (GATHER_FULL, GATHER_RANK_MAJOR, GATHER_NONE):
            raise ValueError(f"gather must be 'full', 'rank' or 'none', got {gather!r}.")
        self.group = group
        self.rank, self.world = _group_info(group)
        if local.out_features * self.world != out_features:
            raise ValueError(f"shard has {local.out_features} outputs; {self.world} ranks x that != {out_features}.")
        self.in_features = local.in_features
        self.out_features = out_features
        self.local = local
        self.gather = gather

    @property
    def local_out_features(self) -> int:
        return self.local.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        if self.gather == GATHER_NONE or self.world == 1:
            if self.gather == GATHER_RANK_MAJOR:
                return y.reshape(1, -1, y.shape[-1])
            return y
        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        m, n_loc = y2.shape
        flat = torch.empty((self.world * m, n_loc), dtype=y2.dtype, device=y2.device)
        dist.all_gather_into_tensor(flat, y2, group=self.group)
        buf = flat.view(self.world, m, n_loc)
        if self.gather == GATHER_RANK_MAJOR:
            return buf
        return buf.permute(1, 0, 2).reshape(*lead, self.world * n_loc)


# ---------------------------------------------------------------------------
# peer memory: the all-gather fused into the GEMM epilogue
# ---------------------------------------------------------------------------


class _CudaArray:
    """A raw device range as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """``nbytes`` of device memory on every rank of ``group``, each rank's
    buffer mapped into every other rank over CUDA IPC, with a block of
    barrier flags in front (``QI_B200_PEER_FLAG_BYTES``).

    The allocations are plain ``cudaMalloc`` ranges.  No NVLink multicast
    object is bound to them, so a rank that leaves takes no other GPU's
    mapping with it.  Collective: every rank constructs it, with the same
    ``nbytes``, at the same point of the program."""

    FLAG_BYTES = 256

    def __init__(self, nbytes: int, group=None):
        from . import _lib

        self._lib = _lib
        self.group = group
        self.rank, self.world = _group_info(group)
        if self.world > 8:
            raise ValueError("peer buffers support at most 8 ranks (one node).")
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.call("qi_b200_peer_alloc", ctypes.c_size_t(self.FLAG_BYTES + self.nbytes), ctypes.byref(ptr), handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs, self._opened = [], []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.ptrs.append(ptr.value)
                continue
            peer = ctypes.c_void_p()
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            _lib.call("qi_b200_peer_open", hb, ctypes.byref(peer))
            self.ptrs.append(peer.value)
            self._opened.append(peer.value)
        self._own = ptr.value
        self._flags = (ctypes.c_void_p * self.world)(*self.ptrs)
        self.data = [p + self.FLAG_BYTES for p in self.ptrs]

    def local(self, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """This rank's data region as a tensor (no copy)."""
        code = {torch.bfloat16: "<i2", torch.float16: "<i2", torch.float32: "<f4", torch.int8: "|i1"}[dtype]
        n = 1
        for d in shape:
            n *= d
        if n * torch.empty((), dtype=dtype).element_size() > self.nbytes:
            raise ValueError("view exceeds the peer buffer.")
        dev = torch.device("cuda", torch.cuda.current_device())
        t = torch.as_tensor(_CudaArray(self.data[self.rank], shape, code), device=dev)
        return t.view(dtype) if dtype in (torch.bfloat16, torch.float16) else t

    def barrier(self, stream=None):
        """Bounded cross-GPU barrier on ``stream`` (default: torch's current)."""
        st = stream if stream is not None else torch.cuda.current_stream()
        self._lib.call("qi_b200_peer_barrier", self._flags, self.world, self.rank, st.cuda_stream)

    def close(self):
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            self._lib.call("qi_b200_peer_close", ctypes.c_void_p(p))
        dist.barrier(group=self.group)
        self._lib.call("qi_b200_peer_free", ctypes.c_void_p(self._own))
        self._own = None


class PeerGatherLinear(nn.Module):
    """Column-parallel INT8 / FP8 W8A8 linear whose all-gather runs inside the
    GEMM.

    Rank r writes its [M, N/P] output into block r of a rank-major
    [P, M, N/P] buffer that every rank has mapped (``PeerBuffer``).  One
    CTA-pair GEMM kernel (``qi_b200_gemm_gather``) writes every finished
    32 x 64 output box with TMA stores into block r of all P buffers: its own
    HBM and, over NVLink, the peers'.  The transfer of each tile runs while the
    tensor cores compute the next ones, so no separate collective runs and no
    SM time is set aside for one.

    Per call:

    1. a barrier (every rank has finished reading the previous output);
    2. the activation quantizer;
    3. the GEMM with the gather in its epilogue;
    4. a barrier (all blocks have landed).

    Both barriers are bounded.  Every column is computed by one rank with
    the single-GPU kernel, so the gathered result is bit-identical to one
    GPU.

    ``forward`` returns the rank-major [P, M, N/P] view of the buffer (the
    layout of ``ColumnShardedLinear(gather="rank")``).  It stays valid until
    the layer's next call."""

    def __init__(self, layer: WeightOnlyLinear, max_tokens: int, group=None, shard: bool = True):
        super().__init__()
        from . import _lib
        from . import kernels as K

        self._lib, self.K = _lib, K
        self.group = group
        self.rank, self.world = _group_info(group)
        self.local = column_shard_buffers(layer, self.rank, self.world) if shard else layer
        self.n_local = self.local.out_features
        self.out_features = self.n_local * self.world
        self.in_features = self.local.in_features
        loc = self.local
        if loc.weight_fp8 is not None:
            self.kind = _lib.KIND_FP8_E4M3
            self.w = loc.weight_fp8.contiguous()
            self.ws = loc.weight_scale.reshape(-1).float().contiguous()
        elif loc.qweight is not None and loc.qweight.dtype == torch.int8 and loc.activation_granularity == "per_token":
            self.kind = _lib.KIND_INT8
            self.w = loc.qweight.contiguous()
            self.ws = loc.scales.reshape(-1).float().contiguous()
        else:
            raise ValueError("PeerGatherLinear serves INT8 and FP8 W8A8 layers.")
        self.static_act = None if self.kind == _lib.KIND_INT8 or loc.activation_granularity == "per_token" \
            else loc.activation_scale.float().reshape(1).contiguous()
        self.bias = None if loc.bias is None else loc.bias.to(torch.bfloat16).contiguous()
        self.gelu = bool(loc.fuse_gelu)
        self.max_tokens = int(max_tokens)
        self.buf = PeerBuffer(self.world * self.max_tokens * self.n_local * 2, group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K, L = self.K, self._lib
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        m = x2.shape[0]
        if m > self.max_tokens:
            raise ValueError(f"{m} tokens exceed this layer's peer buffer ({self.max_tokens}).")
        if self.kind == L.KIND_INT8:
            q, s = K.quantize_int8_rowwise(x2)
        elif self.static_act is None:
            q, s = K.quantize_fp8_rowwise(x2)
        else:
            q, s = K.quantize_fp8_static(x2, self.static_act), self.static_act
        main = torch.cuda.current_stream()
        nl, P, r = self.n_local, self.world, self.rank
        blk = self.max_tokens * nl * 2                     # bytes of one rank block
        out = self.buf.local((P, self.max_tokens, nl))     # rank-major, this GPU's copy
        self.buf.barrier(main)  # every rank has finished reading the previous output
        # this rank's block of all P buffers, own HBM first, then the peers' over NVLink
        dst = [self.buf.data[(r + j) % P] + r * blk for j in range(P)]
        L.call("qi_b200_gemm_gather", self.kind, q.data_ptr(), self.w.data_ptr(), s.data_ptr(),
               0 if s.numel() == 1 else 1, self.ws.data_ptr(), 0 if self.ws.numel() == 1 else 1,
               None if self.bias is None else self.bias.data_ptr(), (ctypes.c_void_p * P)(*dst), P, nl, m, nl,
               self.w.shape[1], L.EPI_GELU if self.gelu else 0, main.cuda_stream)
        self.buf.barrier(main)  # every rank's tiles have landed here
        return out[:, :m]

    def check(self) -> None:
        """Raise ``QiB200DeviceError`` if a barrier or GEMM wait of this rank
        timed out since the last check (a peer that never arrived, for
        example); the outputs of those calls are incomplete.  Synchronizes
        the host with the device: call it between steps."""
        self._lib.raise_on_device_error()

    def close(self):
        self.buf.close()


# ---------------------------------------------------------------------------
# row parallel (INT8 W8A8, exact)
# ---------------------------------------------------------------------------


class KernelOps:
    """The sm_100a kernels used by ``RowShardedInt8Linear`` (C ABI
    ``qi_b200_int8_row_scales`` / ``qi_b200_quantize_int8_rowwise_given`` /
    ``qi_b200_gemm`` with raw accumulators / ``qi_b200_int8_epilogue``)."""

    def __init__(self):
        from . import _lib
        from . import kernels

        self._lib = _lib
        self._k = kernels

    def row_scales(self, x):
        return self._k.int8_row_scales(x)

    def quantize_given(self, x, scales):
        return self._k.quantize_int8_rowwise_given(x, scales)

    def gemm_acc(self, q, qweight):
        return self._k.gemm(self._lib.KIND_INT8, q, qweight, None, None, raw_acc=True)

    def epilogue(self, acc, scales, weight_scales, bias, gelu):
        return self._k.int8_epilogue(acc, scales, weight_scales, bias, gelu=gelu)


class RowShardedInt8Linear(nn.Module):
    """Input-channel (K) shard of an INT8 W8A8 linear with exact reductions.

    ``forward(x_local)`` takes this rank's activation slice ``[..., K/P]``.
    It returns the full ``[..., N]`` on every rank, bit-identical to the
    single-GPU INT8 linear.  The exchange is ``4*M`` bytes of scales
    (all-reduce MAX) plus ``4*M*N`` bytes of int32 partials (all-reduce SUM).
    """

    def __init__(self, layer: WeightOnlyLinear, group=None, ops=None):
        super().__init__()
        if layer.bits != 8 or layer.activation_granularity != "per_token" or layer.qweight is None:
            raise ValueError("RowShardedInt8Linear needs an INT8 W8A8 layer with per-token activations.")
        if layer.group_size != -1 or not layer.symmetric:
            raise ValueError("RowShardedInt8Linear needs symmetric per-channel INT8 weights.")
        self.group = group
        self.rank, self.world = _group_info(group)
        self.in_features = layer.in_features
        self.out_features = layer.out_features
        part = _split(layer.in_features, self.world, "in_features", 16)
        lo, hi = self.rank * part, (self.rank + 1) * part
        self.k_lo, self.k_hi = lo, hi
        self.register_buffer("qweight", layer.qweight[:, lo:hi].contiguous())
        ws = layer.scales.reshape(-1)
        if ws.numel() != layer.out_features:
            raise ValueError("RowShardedInt8Linear needs one weight scale per output channel.")
        self.register_buffer("weight_scales", ws.float().contiguous())
        self.register_buffer("bias", None if layer.bias is None else layer.bias.to(torch.bfloat16).contiguous())
        isc = layer.input_scale
        self.register_buffer("input_scale", None if isc is None else isc.reshape(-1)[lo:hi].contiguous())
        self.fuse_gelu = layer.fuse_gelu
        self.keep_output_dtype = layer.keep_output_dtype
        self.ops = ops if ops is not None else KernelOps()

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        if x_local.shape[-1] != self.k_hi - self.k_lo:
            raise ValueError(f"expected this rank's K slice of {self.k_hi - self.k_lo}, got {x_local.shape[-1]}.")
        out_dtype = x_local.dtype if self.keep_output_dtype == "input" else {
            "fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[self.keep_output_dtype]
        lead = x_local.shape[:-1]
        x = x_local
        if self.input_scale is not None:  # SmoothQuant division before quantization (int8_w8a8_ops.py:138-139)
            x = x / self.input_scale.to(dtype=x.dtype)
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        s = self.ops.row_scales(x2)
        if self.world > 1:
            dist.all_reduce(s, op=dist.ReduceOp.MAX, group=self.group)
        q = self.ops.quantize_given(x2, s)
        acc = self.ops.gemm_acc(q, self.qweight)
        if self.world > 1:
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        y = self.ops.epilogue(acc, s, self.weight_scales, self.bias, self.fuse_gelu)
        return y.reshape(*lead, y.shape[-1]).to(out_dtype)


def local_k_slice(x: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's K slice of a replicated activation (for a row-parallel layer
    whose input was not produced column-parallel)."""
    rank, world = _group_info(group)
    k = x.shape[-1]
    part = _split(k, world, "K")
    return x[..., rank * part:(rank + 1) * part].contiguous()
