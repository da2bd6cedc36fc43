// Torch operators over the C ABI of libqi_b200 (include/qi_b200.h).
//
// qi_int8_w8a8::linear keeps the schema of the reference's extension
// (src/qi/quantization/csrc/int8_w8a8/bindings.cpp:159-165), so code that
// calls torch.ops.qi_int8_w8a8.linear (backends/int8_w8a8_ops.py:176) runs
// on these kernels unchanged.  The qi_b200 namespace adds the other formats
// of this library with the same conventions: inputs are CUDA tensors on one
// device, outputs and workspaces come from torch's caching allocator, work
// goes to the current stream, nothing synchronizes, and a non-zero status
// from the library becomes a c10::Error carrying its message.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <torch/library.h>

#include <optional>

#include "../../include/qi_b200.h"

namespace {

void expect_cuda(const at::Tensor& t, const char* name, const at::Device& dev) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor.");
  TORCH_CHECK(t.device() == dev, name, " must be on the same device as the activations.");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous.");
}

void ok(int rc, const char* what) {
  TORCH_CHECK(rc == QI_B200_OK, what, " failed with status ", rc, ": ", qi_b200_error_string(rc));
}

cudaStream_t stream_of(const at::Device& dev) { return at::cuda::getCurrentCUDAStream(dev.index()).stream(); }

const void* opt_ptr(const std::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}

std::optional<at::Tensor> checked_bias(const std::optional<at::Tensor>& bias, int64_t n, const at::Device& dev) {
  if (!bias.has_value() || !bias->defined()) return std::nullopt;
  expect_cuda(*bias, "bias", dev);
  TORCH_CHECK(bias->scalar_type() == at::kBFloat16, "bias must be bfloat16.");
  TORCH_CHECK(bias->numel() == n, "bias length must match the weight's N dimension.");
  return bias;
}

// The GEMM of a quantized activation with a caller-side tail-split workspace.
void gemm(int kind, const at::Tensor& a, const at::Tensor& b, const at::Tensor& a_scale, int a_stride,
          const at::Tensor& b_scale, int b_stride, const std::optional<at::Tensor>& bias, at::Tensor& out, int flags,
          cudaStream_t stream) {
  const int M = static_cast<int>(a.size(0)), K = static_cast<int>(a.size(1)), N = static_cast<int>(b.size(0));
  size_t ws_bytes = 0;
  ok(qi_b200_gemm_workspace_bytes(kind, M, N, K, flags, 0, &ws_bytes), "qi_b200_gemm_workspace_bytes");
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({static_cast<int64_t>(ws_bytes)}, a.options().dtype(at::kByte));
  ok(qi_b200_gemm_ws(kind, a.data_ptr(), b.data_ptr(), a_scale.data_ptr<float>(), a_stride,
                     b_scale.data_ptr<float>(), b_stride, opt_ptr(bias), out.data_ptr(), N, M, N, K, flags, 0,
                     ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream),
     "qi_b200_gemm_ws");
}

at::Tensor int8_linear_impl(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& weight_scales,
                            const std::optional<at::Tensor>& bias_in, bool gelu) {
  const auto dev = x.device();
  expect_cuda(x, "x_bf16_2d", dev);
  expect_cuda(qweight, "qweight", dev);
  expect_cuda(weight_scales, "weight_scales", dev);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "x_bf16_2d must be a 2-D bfloat16 tensor.");
  TORCH_CHECK(qweight.scalar_type() == at::kChar && qweight.dim() == 2, "qweight must be a 2-D int8 tensor.");
  TORCH_CHECK(weight_scales.scalar_type() == at::kFloat && weight_scales.dim() == 1,
              "weight_scales must be a 1-D float32 tensor.");
  const int64_t M = x.size(0), K = x.size(1), N = qweight.size(0);
  TORCH_CHECK(qweight.size(1) == K, "qweight K dimension must match x_bf16_2d.");
  TORCH_CHECK(weight_scales.size(0) == N, "weight_scales length must match qweight N dimension.");
  const auto bias = checked_bias(bias_in, N, dev);
  const cudaStream_t st = stream_of(dev);
  at::Tensor q = at::empty({M, K}, x.options().dtype(at::kChar));
  at::Tensor s = at::empty({M}, x.options().dtype(at::kFloat));
  at::Tensor out = at::empty({M, N}, x.options());
  if (M == 0) return out;
  ok(qi_b200_quantize_int8_rowwise(x.data_ptr(), q.data_ptr(), s.data_ptr<float>(), static_cast<int>(M),
                                   static_cast<int>(K), st),
     "qi_b200_quantize_int8_rowwise");
  gemm(QI_B200_KIND_INT8, q, qweight, s, 1, weight_scales, 1, bias, out, gelu ? QI_B200_EPI_GELU : 0, st);
  return out;
}

// qi_int8_w8a8::linear: the reference's schema and semantics (per-token
// activation quantization, INT8 GEMM, per-channel scales, optional bias).
at::Tensor qi_int8_w8a8_linear(const at::Tensor& x_bf16_2d, const at::Tensor& qweight,
                               const at::Tensor& weight_scales, const std::optional<at::Tensor>& bias) {
  return int8_linear_impl(x_bf16_2d, qweight, weight_scales, bias, false);
}

at::Tensor int8_linear(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& weight_scales,
                       const std::optional<at::Tensor>& bias, bool gelu) {
  return int8_linear_impl(x, qweight, weight_scales, bias, gelu);
}

at::Tensor fp8_linear(const at::Tensor& x, const at::Tensor& weight_fp8, const at::Tensor& weight_scale,
                      const std::optional<at::Tensor>& activation_scale, const std::optional<at::Tensor>& bias_in,
                      bool gelu) {
  const auto dev = x.device();
  expect_cuda(x, "x", dev);
  expect_cuda(weight_fp8, "weight_fp8", dev);
  expect_cuda(weight_scale, "weight_scale", dev);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "x must be a 2-D bfloat16 tensor.");
  TORCH_CHECK(weight_fp8.element_size() == 1 && weight_fp8.dim() == 2, "weight_fp8 must be 2-D E4M3 bytes.");
  TORCH_CHECK(weight_scale.scalar_type() == at::kFloat, "weight_scale must be float32.");
  const int64_t M = x.size(0), K = x.size(1), N = weight_fp8.size(0);
  TORCH_CHECK(weight_fp8.size(1) == K, "weight_fp8 K dimension must match x.");
  TORCH_CHECK(weight_scale.numel() == 1 || weight_scale.numel() == N, "weight_scale must have 1 or N values.");
  const bool stat = activation_scale.has_value() && activation_scale->defined();
  if (stat) {
    expect_cuda(*activation_scale, "activation_scale", dev);
    TORCH_CHECK(activation_scale->scalar_type() == at::kFloat && activation_scale->numel() == 1,
                "activation_scale must be one float32 value.");
  }
  const auto bias = checked_bias(bias_in, N, dev);
  const cudaStream_t st = stream_of(dev);
  at::Tensor q = at::empty({M, K}, x.options().dtype(at::kByte));
  at::Tensor out = at::empty({M, N}, x.options());
  if (M == 0) return out;
  at::Tensor s;
  if (stat) {
    s = *activation_scale;
    ok(qi_b200_quantize_fp8_static(x.data_ptr(), s.data_ptr<float>(), q.data_ptr(), static_cast<int>(M),
                                   static_cast<int>(K), st),
       "qi_b200_quantize_fp8_static");
  } else {
    s = at::empty({M}, x.options().dtype(at::kFloat));
    ok(qi_b200_quantize_fp8_rowwise(x.data_ptr(), q.data_ptr(), s.data_ptr<float>(), static_cast<int>(M),
                                    static_cast<int>(K), st),
       "qi_b200_quantize_fp8_rowwise");
  }
  gemm(QI_B200_KIND_FP8_E4M3, q, weight_fp8, s, stat ? 0 : 1, weight_scale, weight_scale.numel() == N && N > 1,
       bias, out, gelu ? QI_B200_EPI_GELU : 0, st);
  return out;
}

at::Tensor w4a16_linear(const at::Tensor& x, const at::Tensor& qweight_packed, const at::Tensor& scales_fp16,
                        const at::Tensor& zeros_packed, int64_t group_size, const std::optional<at::Tensor>& bias_in) {
  const auto dev = x.device();
  expect_cuda(x, "x", dev);
  expect_cuda(qweight_packed, "qweight_packed", dev);
  expect_cuda(scales_fp16, "scale_factors", dev);
  expect_cuda(zeros_packed, "zeros", dev);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "x must be a 2-D bfloat16 tensor.");
  TORCH_CHECK(qweight_packed.scalar_type() == at::kInt, "qweight_packed must be int32.");
  TORCH_CHECK(scales_fp16.scalar_type() == at::kHalf, "scale_factors must be float16.");
  TORCH_CHECK(zeros_packed.scalar_type() == at::kInt, "zeros must be packed int32.");
  const int64_t M = x.size(0), K = x.size(1), N = qweight_packed.size(0);
  TORCH_CHECK(qweight_packed.size(1) * 8 == K, "qweight_packed K dimension must match x.");
  const auto bias = checked_bias(bias_in, N, dev);
  const cudaStream_t st = stream_of(dev);
  at::Tensor out = at::empty({M, N}, x.options());
  if (M == 0) return out;
  if (M >= QI_B200_W4A16_DEQUANT_MIN_M) {
    at::Tensor ws = at::empty({N * K * 2}, x.options().dtype(at::kByte));
    ok(qi_b200_w4a16_linear_ws(x.data_ptr(), qweight_packed.data_ptr(), scales_fp16.data_ptr(),
                               zeros_packed.data_ptr(), static_cast<int>(group_size), opt_ptr(bias), out.data_ptr(),
                               static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), ws.data_ptr(),
                               static_cast<size_t>(ws.numel()), st),
       "qi_b200_w4a16_linear_ws");
  } else {
    ok(qi_b200_w4a16_linear(x.data_ptr(), qweight_packed.data_ptr(), scales_fp16.data_ptr(), zeros_packed.data_ptr(),
                            static_cast<int>(group_size), opt_ptr(bias), out.data_ptr(), static_cast<int>(M),
                            static_cast<int>(N), static_cast<int>(K), st),
       "qi_b200_w4a16_linear");
  }
  return out;
}

}  // namespace

TORCH_LIBRARY(qi_int8_w8a8, m) {
  m.def("linear(Tensor x_bf16_2d, Tensor qweight, Tensor weight_scales, Tensor? bias=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(qi_int8_w8a8, CUDA, m) { m.impl("linear", &qi_int8_w8a8_linear); }

TORCH_LIBRARY(qi_b200, m) {
  m.def("int8_linear(Tensor x, Tensor qweight, Tensor weight_scales, Tensor? bias=None, bool gelu=False) -> Tensor");
  m.def("fp8_linear(Tensor x, Tensor weight_fp8, Tensor weight_scale, Tensor? activation_scale=None, "
        "Tensor? bias=None, bool gelu=False) -> Tensor");
  m.def("w4a16_linear(Tensor x, Tensor qweight_packed, Tensor scale_factors, Tensor zeros, int group_size, "
        "Tensor? bias=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(qi_b200, CUDA, m) {
  m.impl("int8_linear", &int8_linear);
  m.impl("fp8_linear", &fp8_linear);
  m.impl("w4a16_linear", &w4a16_linear);
}
