"""GPU parity: the CUDA kernels (through the C ABI in include/qi_b200.h)
against the CPU oracle on identical seeded inputs.

Bars: bit-exact for quantized codes, scales and int32 accumulators, and for
the INT8 bf16 output (its epilogue is deterministic fp32 math); relative
Frobenius error for fp32-accumulated tensor-core outputs:
  FP8 vs oracle <= 2e-3 (accumulation order only), vs reference <= 1e-2.
"""

import numpy as np
import pytest
import torch

from oracle import qi_oracle as O
from qi_b200 import _lib, kernels as K
from qi_b200.synthetic import CFG_FP8, CFG_INT8, make_linear_inputs, make_small_case

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


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


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (numpy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


# --------------------------------------------------------------------------
# activation quantizers
# --------------------------------------------------------------------------

@pytest.mark.parametrize("M,Kd", [(1, 128), (17, 256), (512, 3072), (64, 14336), (3, 100), (5, 24), (33, 20000)])
def test_quantize_int8_rowwise_bit_exact(M, Kd):
    x, _, _ = make_small_case(M, 8, Kd, seed=M + Kd, outlier_frac=0.01)
    x = x.clone()
    if M > 2:
        x[1] = 0  # all-zero row -> scale floor 1e-10
    q, s = K.quantize_int8_rowwise(x.to(DEV))
    qo, so = O.quantize_int8_rowwise(bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


@pytest.mark.parametrize("M,Kd", [(1, 64), (17, 256), (256, 3072), (8, 14336), (3, 40)])
def test_quantize_fp8_rowwise_and_static_bit_exact(M, Kd):
    x, _, _ = make_small_case(M, 8, Kd, seed=7 * M + Kd)
    x = x.clone()
    x[0, :3] = torch.tensor([0.0, -0.0, 1e-30])
    q, s = K.quantize_fp8_rowwise(x.to(DEV))
    qo, so = O.quantize_fp8_rowwise(O.bf16_to_f32(bits(x)))
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    np.testing.assert_array_equal(u8(q), qo)
    st = torch.tensor([0.0123], dtype=torch.float32)
    qs = K.quantize_fp8_static(x.to(DEV), st.to(DEV))
    np.testing.assert_array_equal(u8(qs), O.quantize_fp8_static(O.bf16_to_f32(bits(x)), st.numpy()[0]))


def _bf16_round(v):
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(v, np.float32)))


@pytest.mark.parametrize("Kd", [256, 3072])
def test_quantize_fp8_rowwise_rounding_boundaries(Kd):
    """Quotients x / s that land exactly on (or one bf16 step beside) a
    rounding boundary of E4M3: the kernel's reciprocal-product bracket cannot
    decide them and must fall back to the correctly rounded division; ties go
    to the even code as in torch's float8 cast.  Row 0 has s = 1 exactly
    (amax 448), row 1 s = 3 (amax 1344, so x r is inexact), row 2 holds the
    boundary values nudged by one bf16 step either way, row 3 the negated
    ones (negative ties and signed zeros)."""
    vals = O.e4m3_to_f32(np.arange(0x7F, dtype=np.uint8)).astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)      # 126 boundaries, exact in bf16
    up = O.bf16_to_f32(O.f32_to_bf16(mids) + np.uint16(1))
    dn = O.bf16_to_f32(O.f32_to_bf16(mids) - np.uint16(1))

    def row(head, body):
        r = np.concatenate([[head], body]).astype(np.float32)
        r = np.resize(r, Kd)   # repeat the pattern over K
        r[0] = head
        return _bf16_round(r)

    rows = [row(448.0, np.concatenate([mids, -mids])),
            row(1344.0, np.concatenate([3 * mids, -3 * mids])),
            row(448.0, np.concatenate([up[:-1], dn[1:]])),
            row(-448.0, np.concatenate([-mids, -up[:-1], -dn[1:], [-1e-30, -0.0]]))]
    xf = np.stack(rows)
    xb = torch.from_numpy(O.f32_to_bf16(xf).view(np.int16)).view(torch.bfloat16)
    q, s = K.quantize_fp8_rowwise(xb.to(DEV))
    qo, so = O.quantize_fp8_rowwise(xf)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    np.testing.assert_array_equal(u8(q), qo)
    assert np.all(so[:2] == np.array([1.0, 3.0], np.float32))


# --------------------------------------------------------------------------
# INT8 GEMM
# --------------------------------------------------------------------------

SHAPES = [(1, 64, 128), (17, 192, 256), (128, 256, 512), (129, 136, 272), (300, 520, 1024), (512, 3072, 3072)]


@pytest.mark.parametrize("M,N,Kd", SHAPES + [(3120, 3072, 1024)])
@pytest.mark.parametrize("tile_n", [0, 64, 128, 192, 256, -128, -192, -256])
def test_int8_gemm_int32_accumulators_bit_exact(M, N, Kd, tile_n):
    """tile_n < 0: the CTA-pair kernel (cta_group::2, 256-row tiles over two SMs)."""
    g = torch.Generator().manual_seed(M * 7 + N + Kd)
    a = torch.randint(-127, 128, (M, Kd), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (N, Kd), generator=g, dtype=torch.int8)
    acc = K.gemm(_lib.KIND_INT8, a.to(DEV), b.to(DEV), None, None, raw_acc=True, tile_n=tile_n)
    ref = O.int8_gemm_acc(a.numpy(), b.numpy())
    np.testing.assert_array_equal(acc.cpu().numpy().astype(np.int64), ref)


@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("tile_n", [-256, -192, -128])
def test_pair_kernel_epilogue_matches_single_cta(tile_n, gelu):
    """The CTA-pair kernel's epilogue (per-token x per-channel scales, bias,
    GELU) gives the same bytes as the single-CTA kernel."""
    x, w, b = make_small_case(3120, 3072, 1024, seed=7, outlier_frac=0.002)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    qa, sa = K.quantize_int8_rowwise(x.to(DEV))
    args = (_lib.KIND_INT8, qa, torch.from_numpy(qw).to(DEV), sa, torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV))
    y1 = K.gemm(*args, gelu=gelu, tile_n=256)
    y2 = K.gemm(*args, gelu=gelu, tile_n=tile_n)
    assert _lib.last_launch()["kernel"] == "gemm_int8_pair"
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,N,Kd", SHAPES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_int8_linear_bf16_bit_exact(M, N, Kd, with_bias):
    x, w, b = make_small_case(M, N, Kd, seed=M + 3 * N, outlier_frac=0.002)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    bias = b if with_bias else None
    y = K.int8_linear(x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV),
                      None if bias is None else bias.to(DEV))
    yo, _, _, _ = O.int8_linear(bits(x), qw, sw[:, 0], None if bias is None else bits(bias))
    np.testing.assert_array_equal(bits(y), yo)


def test_int8_config1_full_size():
    """BASELINE config 1 at full size: bf16 output bit-exact vs the oracle,
    and within 5e-3 of the reference's fp32-input dequant-matmul path."""
    x, w, b = make_linear_inputs(CFG_INT8)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    y = K.int8_linear(x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV))
    yo, acc, qa, sa = O.int8_linear(bits(x), qw, sw[:, 0], bits(b))
    np.testing.assert_array_equal(bits(y), yo)
    yref = O.reference_linear_f32(O.bf16_to_f32(bits(x)), qw, sw, None, -1, O.bf16_to_f32(bits(b)), per_token_bits=8)
    assert O.rel_fro(O.bf16_to_f32(bits(y)), yref) <= 5e-3
    # the C-ABI _bias entry point (reference name) gives the same bytes
    # (device tensors are held in locals so their memory outlives the async launch)
    qa_d, sa_d = K.quantize_int8_rowwise(x.to(DEV))
    qw_d, sw_d, b_d = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).contiguous().to(DEV), b.to(DEV)
    out = torch.empty_like(y)
    _lib.call("qi_b200_int8_rowwise_bf16out_bias", qa_d.data_ptr(), qw_d.data_ptr(), sa_d.data_ptr(),
              sw_d.data_ptr(), b_d.data_ptr(), out.data_ptr(), CFG_INT8.M, CFG_INT8.N, CFG_INT8.K,
              torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(bits(out), yo)
    out2 = torch.empty_like(y)
    _lib.call("qi_b200_int8_rowwise_bf16out", qa_d.data_ptr(), qw_d.data_ptr(), sa_d.data_ptr(),
              sw_d.data_ptr(), out2.data_ptr(), CFG_INT8.M, CFG_INT8.N, CFG_INT8.K,
              torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(bits(out2), O.int8_epilogue(acc, sa, sw[:, 0], None))


# --------------------------------------------------------------------------
# FP8 GEMM
# --------------------------------------------------------------------------

@pytest.mark.parametrize("M,N,Kd", [(1, 64, 128), (17, 192, 256), (129, 264, 384), (256, 2048, 3072)])
@pytest.mark.parametrize("gelu", [False, True])
def test_fp8_linear_per_token_vs_oracle(M, N, Kd, gelu):
    x, w, b = make_small_case(M, N, Kd, seed=11 * M + N)
    qw, sw = O.quantize_fp8_rowwise(w.numpy())
    y = K.fp8_linear(x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw).to(DEV), None,
                     b.to(DEV), gelu=gelu)
    qa, sa = O.quantize_fp8_rowwise(O.bf16_to_f32(bits(x)))
    yo = O.fp8_linear(qa, sa, qw, sw, bits(b), gelu=gelu)
    e = O.rel_fro(O.bf16_to_f32(bits(y)), O.bf16_to_f32(yo))
    assert e <= 2e-3, e


def test_fp8_per_tensor_static_matches_reference_semantics():
    """Per-tensor weight scale + static activation scale (the reference's FP8
    granularity, flashrt_fp8_ops.py:207-229)."""
    x, w, b = make_small_case(64, 256, 512, seed=5)
    qw, sw = O.quantize_fp8_per_tensor(w.numpy())
    act_scale = np.asarray([np.abs(O.bf16_to_f32(bits(x))).max() / 448.0], np.float32)
    y = K.fp8_linear(x.to(DEV), torch.from_numpy(qw).to(DEV), torch.from_numpy(sw).to(DEV),
                     torch.from_numpy(act_scale).to(DEV), b.to(DEV))
    qa = O.quantize_fp8_static(O.bf16_to_f32(bits(x)), act_scale[0])
    yo = O.fp8_linear(qa, act_scale, qw, sw, bits(b))
    assert O.rel_fro(O.bf16_to_f32(bits(y)), O.bf16_to_f32(yo)) <= 2e-3
    yref = O.bf16_to_f32(bits(x)).astype(np.float64) @ w.numpy().astype(np.float64).T + O.bf16_to_f32(bits(b))
    assert O.rel_fro(O.bf16_to_f32(bits(y)), yref) <= 1e-1  # per-tensor fp8 vs unquantized


def test_fp8_per_token_vs_reference_fixture():
    """Per-token / per-channel FP8 against the reference's own quantizer
    applied row by row (tests/golden/fp8_per_token_M33_N256_K512.npz): the
    kernel's activation codes and scales bit-exact, the module path's weight
    codes bit-exact, and the linear (with and without the fused GELU) within
    the north-star 1e-2 of the reference-style dequantise-then-F.linear
    output (measured ~1e-3: fp32 summation order and scale order only)."""
    from pathlib import Path

    from qi_b200.quantization import WeightActivationQuantConfig, WeightOnlyLinear
    from qi_b200.quantization.backends import get_backend
    from qi_b200.quantization.quantize import quantize_linear_weight

    f = dict(np.load(Path(__file__).resolve().parent / "golden" / "fp8_per_token_M33_N256_K512.npz"))
    xb = torch.from_numpy(f["x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    bb = torch.from_numpy(f["bias"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = K.quantize_fp8_rowwise(xb)
    np.testing.assert_array_equal(u8(q), f["qx"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), f["sx"].view(np.uint32))
    qw, sw = torch.from_numpy(f["qw"]).to(DEV), torch.from_numpy(f["sw"]).to(DEV)
    for gelu, key in ((False, "y_ref"), (True, "y_ref_gelu")):
        y = K.fp8_linear(xb, qw, sw, None, bb, gelu=gelu)
        e = O.rel_fro(y.float().cpu().numpy(), O.bf16_to_f32(f[key]))
        assert e <= 1e-2, (key, e)
    cfg = WeightActivationQuantConfig(enabled=True, quant_dtype="fp8", backend="b200",
                                      activation_granularity="per_token", weight_granularity="per_channel")
    lin = torch.nn.Linear(f["w"].shape[1], f["w"].shape[0])
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(f["w"]))
        lin.bias.copy_(bb.float().cpu())
    layer = WeightOnlyLinear.from_linear(lin, quantize_linear_weight(lin.weight.detach(), cfg), cfg,
                                         get_backend("b200")).to(DEV)
    layer.bias = bb
    np.testing.assert_array_equal(u8(layer.weight_fp8), f["qw"])
    e = O.rel_fro(layer(xb).float().cpu().numpy(), O.bf16_to_f32(f["y_ref"]))
    assert e <= 1e-2, e


def _decode_e4m3(codes: torch.Tensor) -> torch.Tensor:
    """E4M3 codes (uint8, on the GPU) -> exact fp64 values."""
    return codes.view(torch.float8_e4m3fn).to(torch.float32).to(torch.float64)


def test_fp8_config2_full_size_all_rows():
    """BASELINE config 2 (M=4096, N=14336, K=3072, bias + GELU) at full size,
    every one of the 4096 x 14336 outputs checked.

    * activation codes and per-token scales: bit-exact against the oracle on
      all rows (the oracle's per-row quantizer is pinned to the reference's
      quantize_to_fp8_e4m3 applied row by row, tests/test_oracle.py);
    * raw fp32 accumulators: within 1e-5 (relative to the largest) of the
      exact sum.  The checker is a test-only fp64 GEMM on the GPU of the
      decoded codes: E4M3 x E4M3 products are exact and 3072 of them sum
      exactly in 53 bits;
    * bf16 output: rel-Frobenius <= 2e-3 against the fused epilogue applied to
      the exact sum, and <= 1e-2 against the
      reference-style dequantise-then-matmul path (both operands dequantised,
      product + bias, bf16, GELU), before and after GELU.
    """
    x, w, b = make_linear_inputs(CFG_FP8)
    qw, sw = O.quantize_fp8_rowwise(w.numpy())
    xd, bd = x.to(DEV), b.to(DEV)
    qwd, swd = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw).to(DEV)
    qa, sa = K.quantize_fp8_rowwise(xd)
    qo, so = O.quantize_fp8_rowwise(O.bf16_to_f32(bits(x)))
    np.testing.assert_array_equal(sa.cpu().numpy().view(np.uint32), so.view(np.uint32))
    np.testing.assert_array_equal(u8(qa), qo)
    del qo
    exact = _decode_e4m3(qa) @ _decode_e4m3(qwd).T                      # [4096, 14336] fp64, exact
    acc = K.gemm(_lib.KIND_FP8_E4M3, qa, qwd, None, None, raw_acc=True)
    e_acc = ((acc.double() - exact).abs().max() / exact.abs().max()).item()
    assert e_acc <= 1e-5, e_acc
    del acc
    y = K.fp8_linear(xd, qwd, swd, None, bd, gelu=True)
    lin = K.gemm(_lib.KIND_FP8_E4M3, qa, qwd, sa, swd, bd)             # the same without GELU
    # the kernel's epilogue order on the exact sum: ((acc * s_tok) * s_ch) + bias -> bf16 -> GELU -> bf16
    t = (exact.float() * sa[:, None]) * swd[None, :] + bd.float()[None, :]
    y_epi = torch.nn.functional.gelu(t.bfloat16().float(), approximate="tanh").bfloat16()
    e_epi = O.rel_fro(y.float().cpu().numpy(), y_epi.float().cpu().numpy())
    assert e_epi <= 2e-3, e_epi
    # reference-style: dequantise both operands, matmul, + bias (fp64), bf16, GELU
    ref = (_decode_e4m3(qa) * sa.double()[:, None]) @ (_decode_e4m3(qwd) * swd.double()[:, None]).T
    ref_lin = (ref + bd.double()[None, :]).bfloat16()
    ref_gelu = torch.nn.functional.gelu(ref_lin.float(), approximate="tanh").bfloat16()
    e_lin = O.rel_fro(lin.float().cpu().numpy(), ref_lin.float().cpu().numpy())
    e_gelu = O.rel_fro(y.float().cpu().numpy(), ref_gelu.float().cpu().numpy())
    print(f"cfg2 all rows: acc {e_acc:.2e}, vs epilogue(exact) {e_epi:.2e}, vs dequantise-then-matmul "
          f"{e_lin:.2e} (pre-GELU) / {e_gelu:.2e} (GELU)")
    assert e_lin <= 1e-2 and e_gelu <= 1e-2, (e_lin, e_gelu)
    assert _lib.device_status()[0] == 0


# --------------------------------------------------------------------------
# BF16 GEMM (mainloop of the W4A16 path)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("tile_n", [0, 192, -256, -192, -128])
@pytest.mark.parametrize("M,N,Kd", [(1, 64, 128), (300, 520, 512), (3120, 3072, 1024)])
def test_fp8_gemm_accumulators_vs_fp64(M, N, Kd, tile_n):
    """FP8 E4M3 raw fp32 accumulators against the exact (fp64) sum of the
    decoded operands, including the 192-column tile."""
    g = torch.Generator().manual_seed(M + N + tile_n)
    a = (torch.randn(M, Kd, generator=g) * 4).to(torch.float8_e4m3fn)
    b = (torch.randn(N, Kd, generator=g) * 4).to(torch.float8_e4m3fn)
    acc = K.gemm(_lib.KIND_FP8_E4M3, a.to(DEV), b.to(DEV), None, None, raw_acc=True, tile_n=tile_n)
    ref = a.double() @ b.double().T
    err = ((acc.cpu().double() - ref).norm() / ref.norm()).item()
    assert err < 1e-6, err


@pytest.mark.parametrize("tile_n", [0, -256, -128])
@pytest.mark.parametrize("M,N,Kd", [(1, 64, 64), (100, 192, 320), (256, 512, 1024), (700, 1024, 512)])
def test_bf16_gemm_vs_fp64(M, N, Kd, tile_n):
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(M, Kd, generator=g).bfloat16()
    b = (torch.randn(N, Kd, generator=g) * 0.02).bfloat16()
    y = K.gemm(_lib.KIND_BF16, a.to(DEV), b.to(DEV), None, None, tile_n=tile_n)
    ref = a.double() @ b.double().T
    assert O.rel_fro(y.float().cpu().numpy(), ref.numpy()) <= 5e-3


# --------------------------------------------------------------------------
# CUDA-graph capture (the reference runs its DiT under CUDA graphs by default)
# --------------------------------------------------------------------------

def test_linears_capture_in_cuda_graph_and_replay():
    x, w, b = make_small_case(64, 512, 1024, seed=21)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    fq, fs = O.quantize_fp8_rowwise(w.numpy())
    qw_d, sw_d = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).contiguous().to(DEV)
    fq_d, fs_d, b_d = torch.from_numpy(fq).to(DEV), torch.from_numpy(fs).to(DEV), b.to(DEV)
    x_static = x.to(DEV)
    # warm up outside capture (first-call host state: attributes, descriptors)
    K.int8_linear(x_static, qw_d, sw_d, b_d)
    K.fp8_linear(x_static, fq_d, fs_d, None, b_d, gelu=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y8 = K.int8_linear(x_static, qw_d, sw_d, b_d)
        yf = K.fp8_linear(x_static, fq_d, fs_d, None, b_d, gelu=True)
    x2, _, _ = make_small_case(64, 512, 1024, seed=22)
    x_static.copy_(x2.to(DEV))
    g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y8), O.int8_linear(bits(x2), qw, sw[:, 0], bits(b))[0])
    qa, sa = O.quantize_fp8_rowwise(O.bf16_to_f32(bits(x2)))
    assert O.rel_fro(O.bf16_to_f32(bits(yf)), O.bf16_to_f32(O.fp8_linear(qa, sa, fq, fs, bits(b), gelu=True))) <= 2e-3


@pytest.mark.parametrize("M,N,Kd,tile_n,splits", [(512, 3072, 3072, 0, 0), (512, 3072, 3072, 256, 2),
                                                   (100, 520, 2048, 128, 4), (32, 9216, 1024, 0, 0),
                                                   (390, 3072, 3072, 192, 2), (1, 256, 4096, 256, 3)])
@pytest.mark.parametrize("gelu", [False, True])
def test_cluster_splitk_matches_unsplit(M, N, Kd, tile_n, splits, gelu):
    """qi_b200_gemm_csk: S CTAs of a cluster split K and add their partial
    tiles through distributed shared memory.  INT8 outputs are bit-identical
    to the unsplit kernel (int32 sums); FP8 agrees to fp32 summation order."""
    x, w, b = make_small_case(M, N, Kd, seed=M + 3 * N, outlier_frac=0.002)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    qa, sa = K.quantize_int8_rowwise(x.to(DEV))
    qwd, swd, bd = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV)
    st = torch.cuda.current_stream().cuda_stream
    flags = _lib.EPI_GELU if gelu else 0

    def csk(kind, a, bw, s_a, s_b):
        y = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
        _lib.call("qi_b200_gemm_csk", kind, a.data_ptr(), bw.data_ptr(), s_a.data_ptr(), 1, s_b.data_ptr(), 1,
                  bd.data_ptr(), y.data_ptr(), N, M, N, Kd, flags, tile_n, splits, st)
        return y

    y = csk(_lib.KIND_INT8, qa, qwd, sa, swd)
    plan = _lib.last_launch()
    assert plan["kernel"] == "gemm_int8_csk" and plan["cluster"] >= 2, plan
    y_ref = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, gelu=gelu, tile_n=128)
    assert torch.equal(y, y_ref)
    if not gelu:
        yo, _, _, _ = O.int8_linear(bits(x), qw, sw[:, 0], bits(b))
        np.testing.assert_array_equal(bits(y), yo)
    qf, sf = K.quantize_fp8_rowwise(x.to(DEV))
    wf = (w * 20).to(torch.float8_e4m3fn).view(torch.uint8).to(DEV)
    wsf = torch.full((N,), 0.05, device=DEV)
    f = csk(_lib.KIND_FP8_E4M3, qf, wf, sf, wsf)
    f_ref = K.gemm(_lib.KIND_FP8_E4M3, qf, wf, sf, wsf, bd, gelu=gelu, tile_n=128)
    assert O.rel_fro(f.float().cpu().numpy(), f_ref.float().cpu().numpy()) <= 2e-3


def test_cluster_splitk_auto_for_few_tiles_long_k():
    """qi_b200_gemm picks the cluster split-K kernel on its own for very few
    tiles over a long K (the DiT action expert's FFN-down shape); INT8
    outputs stay bit-identical to the unsplit kernel."""
    M, N, Kd = 32, 1024, 4096
    x, w, b = make_small_case(M, N, Kd, seed=77)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    qa, sa = K.quantize_int8_rowwise(x.to(DEV))
    qwd, swd, bd = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV)
    y = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd)
    assert _lib.last_launch()["kernel"] == "gemm_int8_csk"
    y_ref = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, tile_n=128)
    assert _lib.last_launch()["kernel"] == "gemm_int8"
    assert torch.equal(y, y_ref)
    yo, _, _, _ = O.int8_linear(bits(x), qw, sw[:, 0], bits(b))
    np.testing.assert_array_equal(bits(K.int8_linear(x.to(DEV), qwd, swd, bd)), yo)


@pytest.mark.parametrize("M,Kd", [(33, 512), (7, 100), (256, 3072)])
def test_int8_quantizer_fused_smoothing(M, Kd):
    """SmoothQuant / AWQ input smoothing fused into the activation quantizer
    (int8_w8a8_ops.py:138-139: x / input_scale.to(x.dtype), in bf16): codes
    and scales bit-identical to dividing first with torch, and to the oracle
    on the smoothed rows.  K = 100 takes the scalar (unaligned) kernel."""
    x, _, _ = make_small_case(M, 8, Kd, seed=M + Kd, outlier_frac=0.01)
    g = torch.Generator().manual_seed(Kd)
    isc = (0.25 + 2 * torch.rand(Kd, generator=g)).float()
    xd, isd = x.to(DEV), isc.to(DEV)
    q, s = K.quantize_int8_rowwise(xd, input_scale=isd)
    xs = xd / isd.to(torch.bfloat16)
    q_ref, s_ref = K.quantize_int8_rowwise(xs.contiguous())
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
    qo, so = O.quantize_int8_rowwise(bits(xs))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_int8_module_with_input_scale_fuses_smoothing():
    """A WeightOnlyLinear with an input_scale buffer on the B200 backend gives
    the same bits as the reference order (divide, then the INT8 linear)."""
    from qi_b200.quantization import WeightActivationQuantConfig, replace_linear_with_weight_only

    M, N, Kd = 40, 256, 512
    x, w, b = make_small_case(M, N, Kd, seed=5)
    model = torch.nn.Module()
    model.ffn = torch.nn.Sequential(torch.nn.Linear(Kd, N))  # a target name of the swap
    with torch.no_grad():
        model.ffn[0].weight.copy_(w)
        model.ffn[0].bias.copy_(b.float())
    cfg = WeightActivationQuantConfig(enabled=True, algo="rtn", quant_dtype="int", backend="b200",
                                      activation_granularity="per_token", weight_granularity="per_channel")
    replace_linear_with_weight_only(model, cfg)
    model.to(DEV)
    lin = model.ffn[0]
    assert type(lin).__name__ == "WeightOnlyLinear"
    g = torch.Generator().manual_seed(3)
    isc = (0.5 + torch.rand(Kd, generator=g)).float().to(DEV)
    lin.input_scale = isc
    xd = x.to(DEV)
    y = lin(xd)
    y_ref = K.int8_linear((xd / isc.to(torch.bfloat16)).contiguous(), lin.qweight, lin.scales[:, 0].contiguous(),
                          lin.bias.to(torch.bfloat16))
    assert torch.equal(y, y_ref)


def _expected_tail_split(M, N, Kd, bn, elem, mode):
    """Splits per tail tile the library should pick (its rule, restated)."""
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    tiles = -(-M // 256) * -(-N // bn)
    kb = -(-Kd * elem // 128)
    rem = tiles % pairs
    if mode == 1 or tiles <= pairs or rem == 0:
        return 1
    s = pairs // rem
    if mode >= 2:
        s = min(s, mode)
    s = min(s, 8, kb)
    if s < 2 or (mode == 0 and kb - -(-kb // s) < 64):
        return 1
    return s


@pytest.mark.parametrize("M,N,Kd,tile_n,tail", [(1000, 4744, 1024, -256, 8), (1000, 4744, 1024, -192, 2),
                                                (1000, 4744, 1024, -128, 5), (2304, 2304, 12288, -256, 0),
                                                (3120, 3072, 14336, 0, 0)])
@pytest.mark.parametrize("gelu", [False, True])
def test_pair_tail_split_matches_unsplit(M, N, Kd, tile_n, tail, gelu):
    """The CTA-pair kernel's partial last wave (tiles % pairs tiles) split
    along K over the idle pairs: INT8 outputs bit-identical to the same
    kernel without the split (and to the oracle); FP8 and BF16 agree to fp32
    summation order.  Ragged M and N put partial tiles into the tail; the
    last two cases are the library's own choice (long K), the last one also
    of the kernel (the DiT FFN-down shape; unsplit it runs single-CTA
    tiles)."""
    x, w, b = make_small_case(M, N, Kd, seed=M + N + Kd, outlier_frac=0.002)
    qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
    qa, sa = K.quantize_int8_rowwise(x.to(DEV))
    qwd, swd, bd = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV)
    bn = -tile_n if tile_n else 256

    y = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, gelu=gelu, tile_n=tile_n, tail_split=tail)
    want = _expected_tail_split(M, N, Kd, bn, 1, tail)
    assert _lib.last_launch()["kernel"] == "gemm_int8_pair"
    assert want > 1 and _lib.last_tail_split() == want
    y_ref = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, gelu=gelu, tile_n=tile_n, tail_split=1)
    assert _lib.last_tail_split() == 1 or _lib.last_launch()["kernel"] == "gemm_int8"
    assert torch.equal(y, y_ref)
    if not gelu and tile_n == -256 and M == 1000:
        yo, _, _, _ = O.int8_linear(bits(x), qw, sw[:, 0], bits(b))
        np.testing.assert_array_equal(bits(y), yo)

    qf, sf = K.quantize_fp8_rowwise(x.to(DEV))
    wf = (w * 20).to(torch.float8_e4m3fn).view(torch.uint8).to(DEV)
    wsf = torch.full((N,), 0.05, device=DEV)
    f = K.gemm(_lib.KIND_FP8_E4M3, qf, wf, sf, wsf, bd, gelu=gelu, tile_n=tile_n, tail_split=tail)
    assert _lib.last_tail_split() == _expected_tail_split(M, N, Kd, bn, 1, tail)
    f_ref = K.gemm(_lib.KIND_FP8_E4M3, qf, wf, sf, wsf, bd, gelu=gelu, tile_n=tile_n, tail_split=1)
    assert O.rel_fro(f.float().cpu().numpy(), f_ref.float().cpu().numpy()) <= 1e-3

    xb, wb = x.to(DEV), w.to(torch.bfloat16).to(DEV)
    h = K.gemm(_lib.KIND_BF16, xb, wb, None, None, bd, gelu=gelu, tile_n=tile_n, tail_split=tail)
    assert _lib.last_tail_split() == _expected_tail_split(M, N, Kd, bn, 2, tail)
    h_ref = K.gemm(_lib.KIND_BF16, xb, wb, None, None, bd, gelu=gelu, tile_n=tile_n, tail_split=1)
    assert O.rel_fro(h.float().cpu().numpy(), h_ref.float().cpu().numpy()) <= 1e-3
    assert _lib.device_status() == (0, 0, 0, 0)


def test_pair_tail_split_repeated_and_in_cuda_graph():
    """Tail-split launches leave their counters at zero: back-to-back launches
    on new data, and replays of a CUDA graph captured on a stream that had
    not used the split before (its workspace is allocated during capture),
    all stay bit-identical to the unsplit kernel."""
    M, N, Kd = 1000, 4744, 1024
    qwd = swd = bd = None
    outs = []
    for seed in (5, 6, 7):
        x, w, b = make_small_case(M, N, Kd, seed=seed, outlier_frac=0.002)
        if qwd is None:
            qw, sw, _ = O.quantize_weight_rtn(w.numpy(), 8, -1, True)
            qwd, swd, bd = torch.from_numpy(qw).to(DEV), torch.from_numpy(sw[:, 0]).to(DEV), b.to(DEV)
        qa, sa = K.quantize_int8_rowwise(x.to(DEV))
        y = K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, tile_n=-256, tail_split=8)
        assert _lib.last_tail_split() == 8
        assert torch.equal(y, K.gemm(_lib.KIND_INT8, qa, qwd, sa, swd, bd, tile_n=-256, tail_split=1))
        outs.append((qa, sa, y))

    qa_s = outs[0][0].clone()
    sa_s = outs[0][1].clone()
    y_s = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            K.gemm(_lib.KIND_INT8, qa_s, qwd, sa_s, swd, bd, out=y_s, tile_n=-256, tail_split=8)
    assert _lib.last_tail_split() == 8
    for qa, sa, y in outs[1:] + outs[:1]:
        qa_s.copy_(qa)
        sa_s.copy_(sa)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y_s, y)
    del g
    assert _lib.device_status() == (0, 0, 0, 0)
