// Per-token activation quantizers (bf16 rows -> int8 / fp8-e4m3 + fp32 scale).
//
// Row-parallel, HBM-bound: each row is read once with 16-byte vector loads and
// held in registers (up to 8 x uint4 per thread) across the absmax reduction
// (warp shuffles, then shared memory when a row spans several warps) and the
// quantization pass, so HBM traffic is exactly K*2 bytes in + K bytes out per
// row plus one fp32 scale.
//
// Semantics (restated from the reference):
//   int8  (csrc/int8_w8a8/quantize_int8.cu:7-59): s = max(amax/127, 1e-10),
//         q = clamp(rint(x * (1/s)), -127, 127) with an IEEE reciprocal.
//   fp8   (backends/flashrt_fp8_ops.py:38-48, one scale per row instead of one
//         per tensor): s = max(amax/448, 1e-12), q = e4m3_rn(clamp(x/s, +-448)),
//         x/s proven from a bracketed reciprocal product (see QuantFp8).
//   fp8 static (flashrt_fp8_ops.py:207-216): q = e4m3_rn(clamp(x/s_static, +-448)).
#pragma once

#include "launch_count.cuh"
#include "sm100_ptx.cuh"
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

namespace qib {

constexpr int kQuantThreads = 256;
constexpr int kQuantMaxChunks = 8;  // uint4 chunks (8 bf16 each) held per thread

struct QuantInt8 {
  static constexpr bool kNeedsAmax = true;
  static constexpr bool kStoreQ = true;
  __device__ __forceinline__ static float scale_from_amax(float amax) {
    return fmaxf(__fdiv_rn(amax, 127.0f), 1e-10f);
  }
  __device__ __forceinline__ static float aux(float s) { return __frcp_rn(s); }
  __device__ __forceinline__ static uint8_t q1(float x, float /*s*/, float inv) {
    int q = __float2int_rn(__fmul_rn(x, inv));
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    return static_cast<uint8_t>(static_cast<int8_t>(q));
  }
  // two elements -> two codes (low byte = f.x)
  __device__ __forceinline__ static uint32_t q2(float2 f, float s, float inv) {
    return q1(f.x, s, inv) | (static_cast<uint32_t>(q1(f.y, s, inv)) << 8);
  }
};

// Two fp32 values -> two E4M3 codes, round to nearest even, saturating to
// +-448 (NaN stays NaN); low byte = lo.  cvt...e4m3x2.f32 puts its first
// source operand in the upper byte.
__device__ __forceinline__ uint32_t e4m3x2_rn_sat(float lo, float hi) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// int8 with per-row scales supplied by the caller (e.g. reduced across ranks
// that each hold a K-slice of the row): q = clamp(rint(x * (1/s)), -127, 127).
struct QuantInt8Given : QuantInt8 {
  static constexpr bool kNeedsAmax = false;
};

// Only the int8 per-row scales, no codes (q may be null).  For a row split over
// ranks by K, the MAX over ranks of these local scales equals the scale of the
// whole row, because fp32 division by 127 and max() are both monotone.
struct QuantInt8ScalesOnly : QuantInt8 {
  static constexpr bool kStoreQ = false;
};

// FP8 codes are e4m3_rn(clamp(fl32(x / s), +-448)) (flashrt_fp8_ops.py:43-48;
// the saturating conversion is that clamp).  The division is avoided: with
// r = rn(1/s), t = rn(x r) is within 2^-22.4 (relative) of fl32(x / s)
// (x r carries 2^-23 + 2^-48, fl32(x / s) 2^-24), so fl32(x / s) lies between
// t (1 - 2^-20) and t (1 + 2^-20), both ends computed with one more rounding
// of 2^-24.  Rounding to E4M3 is monotone, so when both ends give the same
// code that code is proven; otherwise (the bracket straddles a rounding
// boundary, about 1 in 2^16 elements) the pair is redone with the correctly
// rounded division.  Below fp32's normal range every value involved is
// smaller than half the least E4M3 subnormal, so all three give a zero of
// the same sign.
struct QuantFp8 {
  static constexpr bool kNeedsAmax = true;
  static constexpr bool kStoreQ = true;
  __device__ __forceinline__ static float scale_from_amax(float amax) {
    return fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f);
  }
  __device__ __forceinline__ static float aux(float s) { return __frcp_rn(s); }
  __device__ __forceinline__ static uint8_t q1(float x, float s, float /*aux*/) {
    const float v = __fdiv_rn(x, s);
    return static_cast<uint8_t>(e4m3x2_rn_sat(v, 0.0f) & 0xFFu);
  }
  __device__ __forceinline__ static uint32_t q2(float2 f, float s, float r) {
    constexpr float kLo = 1.0f - 0x1p-20f, kHi = 1.0f + 0x1p-20f;
    const float2 t = __fmul2_rn(f, make_float2(r, r));
    const float2 a = __fmul2_rn(t, make_float2(kLo, kLo)), b = __fmul2_rn(t, make_float2(kHi, kHi));
    const uint32_t lo = e4m3x2_rn_sat(a.x, a.y);
    const uint32_t hi = e4m3x2_rn_sat(b.x, b.y);
    if (__builtin_expect(lo == hi, 1)) return lo;
    return e4m3x2_rn_sat(__fdiv_rn(f.x, s), __fdiv_rn(f.y, s));
  }
};

struct QuantFp8Static : QuantFp8 {
  static constexpr bool kNeedsAmax = false;
};

// max |x| of 8 bf16 values, taken on packed bf16x2 (|x| and max are exact in
// bf16, so this equals the fp32 max of the widened values).
__device__ __forceinline__ float absmax_bf16x8(const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  const __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__low2float(m), __high2float(m));
}

// SmoothQuant / AWQ input smoothing of 8 bf16 values, x / input_scale in
// bf16 as the reference does it (int8_w8a8_ops.py:138-139: the fp32 scale is
// first cast to the activation dtype): bf16(fp32(x) / fp32(bf16(d))).
__device__ __forceinline__ uint4 smooth_bf16x8(const uint4& v, const float* __restrict__ d8) {
  const float4 d0 = __ldg(reinterpret_cast<const float4*>(d8));
  const float4 d1 = __ldg(reinterpret_cast<const float4*>(d8) + 1);
  const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    const float a = __fdiv_rn(f.x, __bfloat162float(__float2bfloat16_rn(d[2 * i])));
    const float b = __fdiv_rn(f.y, __bfloat162float(__float2bfloat16_rn(d[2 * i + 1])));
    __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
    o[i] = *reinterpret_cast<uint32_t*>(&r);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <class Op>
__device__ __forceinline__ uint2 quant_bf16x8(const uint4& v, float s, float aux) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t pair = Op::q2(__bfloat1622float2(h[i]), s, aux);
    if (i < 2) lo |= pair << (16 * i);
    else hi |= pair << (16 * (i - 2));
  }
  return make_uint2(lo, hi);
}

// TPR threads per row, kQuantThreads / TPR rows per block.  cols % 8 == 0,
// row starts 16-byte aligned, ceil(cols/8 / TPR) <= kQuantMaxChunks.
template <class Op, int TPR>
__global__ void __launch_bounds__(kQuantThreads)
k_rowquant_vec(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scales,
               const float* __restrict__ static_scale, int rows, int cols, const float* __restrict__ col_div) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int RPB = kQuantThreads / TPR;
  constexpr int WPR = TPR / 32;
  __shared__ float red[RPB][WPR];
  const int r_local = threadIdx.x / TPR;
  const int t = threadIdx.x % TPR;
  const int row = blockIdx.x * RPB + r_local;
  const bool valid = row < rows;
  const int nvec = cols >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(valid ? row : 0) * cols);

  uint4 v[kQuantMaxChunks];
  float amax = 0.f;
#pragma unroll
  for (int c = 0; c < kQuantMaxChunks; ++c) {
    const int idx = c * TPR + t;
    if (valid && idx < nvec) {
      v[c] = __ldg(xr + idx);
      if (col_div != nullptr) v[c] = smooth_bf16x8(v[c], col_div + idx * 8);
      if (Op::kNeedsAmax) amax = fmaxf(amax, absmax_bf16x8(v[c]));
    }
  }
  float s;
  if (Op::kNeedsAmax) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (WPR > 1) {
      if ((threadIdx.x & 31) == 0) red[r_local][t >> 5] = amax;
      __syncthreads();
      amax = red[r_local][0];
#pragma unroll
      for (int w = 1; w < WPR; ++w) amax = fmaxf(amax, red[r_local][w]);
    }
    s = Op::scale_from_amax(amax);
    if (valid && t == 0 && scales != nullptr) scales[row] = s;
  } else {
    // given scale: one per tensor (static_scale) or one per row (scales, read)
    s = static_scale != nullptr ? __ldg(static_scale) : (valid ? __ldg(scales + row) : 1.0f);
  }
  if (!Op::kStoreQ) return;
  const float aux = Op::aux(s);
  uint2* qr = reinterpret_cast<uint2*>(q + static_cast<size_t>(valid ? row : 0) * cols);
#pragma unroll
  for (int c = 0; c < kQuantMaxChunks; ++c) {
    const int idx = c * TPR + t;
    if (valid && idx < nvec) qr[idx] = quant_bf16x8<Op>(v[c], s, aux);
  }
}

// Any cols / alignment: one warp per row, two scalar passes (second pass hits L1/L2).
template <class Op>
__global__ void __launch_bounds__(kQuantThreads)
k_rowquant_scalar(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scales,
                  const float* __restrict__ static_scale, int rows, int cols, const float* __restrict__ col_div) {
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x * (kQuantThreads / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * cols;
  // element j, smoothed as in smooth_bf16x8 when col_div is given
  auto xv = [&](int j) {
    const float f = __bfloat162float(xr[j]);
    if (col_div == nullptr) return f;
    return __bfloat162float(__float2bfloat16_rn(__fdiv_rn(f, __bfloat162float(__float2bfloat16_rn(col_div[j])))));
  };
  float s;
  if (Op::kNeedsAmax) {
    float amax = 0.f;
    for (int j = lane; j < cols; j += 32) amax = fmaxf(amax, fabsf(xv(j)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    s = Op::scale_from_amax(amax);
    if (lane == 0 && scales != nullptr) scales[row] = s;
  } else {
    s = static_scale != nullptr ? __ldg(static_scale) : __ldg(scales + row);
  }
  if (!Op::kStoreQ) return;
  const float aux = Op::aux(s);
  uint8_t* qr = q + static_cast<size_t>(row) * cols;
  for (int j = lane; j < cols; j += 32) qr[j] = Op::q1(xv(j), s, aux);
}

// ---------------------------------------------------------------------------
// Persistent row quantizer fed by bulk copies (cp.async.bulk, one destination
// CTA).  The register kernels above hold a row in registers between the amax
// and the quantization pass; at 90+ registers a thread that caps an SM at 16
// warps, and each CTA's loads are in flight only at its start, so HBM sits at
// about 20 % (ncu, 4096 x 3072 FP8).  Here a CTA of 128 threads keeps a ring
// of `stages` whole rows in shared memory: thread 0 keeps the next rows'
// copies in flight while all threads reduce and quantize the current one out
// of shared memory, so every SM always has several rows of loads outstanding
// and a thread needs few registers.  Rows r = blockIdx.x + i * gridDim.x.
// Requires cols % 8 == 0 and 16-byte aligned rows; the same per-element
// arithmetic as k_rowquant_vec (bit-identical codes and scales).
// ---------------------------------------------------------------------------
constexpr int kBulkQuantThreads = 128;
constexpr unsigned int kTagRowQuant = 0x500u;

__host__ __device__ constexpr int bulk_row_stride(int cols) { return (cols * 2 + 127) & ~127; }

template <class Op>
__global__ void __launch_bounds__(kBulkQuantThreads)
k_rowquant_bulk(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scales,
                const float* __restrict__ static_scale, int rows, int cols, const float* __restrict__ col_div,
                int stages) {
  extern __shared__ __align__(128) uint8_t qsm[];
  const int stride = bulk_row_stride(cols);
  uint64_t* full = reinterpret_cast<uint64_t*>(qsm + static_cast<size_t>(stages) * stride);
  float* red = reinterpret_cast<float*>(full + stages);   // [kBulkQuantThreads / 32]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red + kBulkQuantThreads / 32);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 2u;
  const int nvec = cols >> 3;
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  const int my_rows = rows > static_cast<int>(blockIdx.x) ? (rows - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;
  auto issue = [&](int i) {  // row i of this CTA into stage i % stages
    uint64_t* bar = &full[i % stages];
    mbar_expect_tx(bar, row_bytes);
    bulk_load(qsm + static_cast<size_t>(i % stages) * stride,
              x + (static_cast<long long>(blockIdx.x) + static_cast<long long>(i) * gridDim.x) * cols, row_bytes, bar);
  };
  if (tid == 0)
    for (int i = 0; i < stages && i < my_rows; ++i) issue(i);
  int i = 0;
  for (; i < my_rows; ++i) {
    const int st = i % stages;
    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>(i / stages) & 1u, abort_flag, kTagRowQuant, 1);
    if (!__syncthreads_and(ok)) break;
    const long long row = static_cast<long long>(blockIdx.x) + static_cast<long long>(i) * gridDim.x;
    const uint4* rb = reinterpret_cast<const uint4*>(qsm + static_cast<size_t>(st) * stride);
    float s;
    if (Op::kNeedsAmax) {
      float amax = 0.f;
      for (int j = tid; j < nvec; j += kBulkQuantThreads) {
        uint4 v = rb[j];
        if (col_div != nullptr) v = smooth_bf16x8(v, col_div + j * 8);
        amax = fmaxf(amax, absmax_bf16x8(v));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      if (lane == 0) red[warp] = amax;
      __syncthreads();
      amax = red[0];
#pragma unroll
      for (int w = 1; w < kBulkQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
      s = Op::scale_from_amax(amax);
      if (tid == 0 && scales != nullptr) scales[row] = s;
    } else {
      s = static_scale != nullptr ? __ldg(static_scale) : __ldg(scales + row);
    }
    const float aux = Op::aux(s);
    uint2* qr = reinterpret_cast<uint2*>(q + row * cols);
    for (int j = tid; j < nvec; j += kBulkQuantThreads) {
      uint4 v = rb[j];
      if (col_div != nullptr) v = smooth_bf16x8(v, col_div + j * 8);
      qr[j] = quant_bf16x8<Op>(v, s, aux);
    }
    __syncthreads();  // every thread is done with this stage (and with red[])
    if (tid == 0 && i + stages < my_rows) {
      fence_async_shared();  // the threads' reads of the stage precede the copy that overwrites it
      issue(i + stages);
    }
  }
  if (i < my_rows && tid == 0) {
    // aborted: let the copies still in flight land before the CTA exits
    for (int k = i; k < my_rows && k < i + stages; ++k)
      mbar_wait_drain(&full[k % stages], static_cast<uint32_t>(k / stages) & 1u);
  }
}

// Warp-per-row form of k_rowquant_bulk for short rows (a row of up to 8 KB):
// each warp owns a ring of `stages` row buffers and its own mbarriers, lane 0
// keeps the warp's next rows in flight, and the whole row is reduced and
// quantized by the warp with shuffles only (no block barrier per row).  Rows
// r = gwarp + i * total_warps.  Eight warps per CTA: with one 6 KB row
// buffer per warp (rows of 3072), 32 warps of an SM hold every row a
// 4096-row launch gives the SM at once (FP8 4096 x 3072: 16.6 -> 13.6 us
// against four warps with two buffers each).
constexpr int kBulkWarpRowThreads = 256;

template <class Op>
__global__ void __launch_bounds__(kBulkWarpRowThreads)
k_rowquant_bulk_warp(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scales,
                     const float* __restrict__ static_scale, int rows, int cols, const float* __restrict__ col_div,
                     int stages) {
  extern __shared__ __align__(128) uint8_t qsm[];
  constexpr int kWarps = kBulkWarpRowThreads / 32;
  const int stride = bulk_row_stride(cols);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* ring = qsm + static_cast<size_t>(warp) * stages * stride;
  uint64_t* full = reinterpret_cast<uint64_t*>(qsm + static_cast<size_t>(kWarps) * stages * stride) + warp * stages;
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(reinterpret_cast<uint64_t*>(qsm + static_cast<size_t>(kWarps) * stages * stride) +
                                      kWarps * stages) + warp;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 2u;
  const int nvec = cols >> 3;
  if (lane == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  griddep_wait();
  griddep_launch_dependents();
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kWarps + warp;
  const int my_rows = rows > gw ? static_cast<int>((rows - 1 - gw) / nw) + 1 : 0;
  auto issue = [&](int i) {
    uint64_t* bar = &full[i % stages];
    mbar_expect_tx(bar, row_bytes);
    bulk_load(ring + static_cast<size_t>(i % stages) * stride, x + (gw + static_cast<long long>(i) * nw) * cols,
              row_bytes, bar);
  };
  if (lane == 0)
    for (int i = 0; i < stages && i < my_rows; ++i) issue(i);
  int i = 0;
  for (; i < my_rows; ++i) {
    const int st = i % stages;
    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>(i / stages) & 1u, abort_flag, kTagRowQuant, 2);
    if (!__all_sync(0xffffffffu, ok)) break;
    const long long row = gw + static_cast<long long>(i) * nw;
    const uint4* rb = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(st) * stride);
    float s;
    if (Op::kNeedsAmax) {
      float amax = 0.f;
      for (int j = lane; j < nvec; j += 32) {
        uint4 v = rb[j];
        if (col_div != nullptr) v = smooth_bf16x8(v, col_div + j * 8);
        amax = fmaxf(amax, absmax_bf16x8(v));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      s = Op::scale_from_amax(amax);
      if (lane == 0 && scales != nullptr) scales[row] = s;
    } else {
      s = static_scale != nullptr ? __ldg(static_scale) : __ldg(scales + row);
    }
    const float aux = Op::aux(s);
    uint2* qr = reinterpret_cast<uint2*>(q + row * cols);
    for (int j = lane; j < nvec; j += 32) {
      uint4 v = rb[j];
      if (col_div != nullptr) v = smooth_bf16x8(v, col_div + j * 8);
      qr[j] = quant_bf16x8<Op>(v, s, aux);
    }
    __syncwarp();  // the warp is done with this stage
    if (lane == 0 && i + stages < my_rows) {
      fence_async_shared();
      issue(i + stages);
    }
  }
  if (i < my_rows && lane == 0)
    for (int k = i; k < my_rows && k < i + stages; ++k)
      mbar_wait_drain(&full[k % stages], static_cast<uint32_t>(k / stages) & 1u);
}

template <class Op>
inline cudaError_t launch_rowquant(const void* x, void* q, float* scales, const float* static_scale, int rows,
                                   int cols, cudaStream_t stream, const float* col_div = nullptr) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  const bool aligned = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(q) % 8 == 0) &&
                       (col_div == nullptr || reinterpret_cast<uintptr_t>(col_div) % 16 == 0);
  const int nvec = cols / 8;
  const dim3 blk(kQuantThreads);
  // many rows: the persistent bulk-copy kernels (whole rows in flight per
  // warp for short rows, per CTA for long ones)
  if (aligned && Op::kStoreQ && rows >= 256 && bulk_row_stride(cols) <= 48 * 1024 &&
      reinterpret_cast<uintptr_t>(x) % 16 == 0) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int stride = bulk_row_stride(cols);
    const bool per_warp = stride <= 8 * 1024;
    const int threads = per_warp ? kBulkWarpRowThreads : kBulkQuantThreads;
    const int rings = per_warp ? kBulkWarpRowThreads / 32 : 1;    // row rings per CTA
    // ring depth from a 48 KB budget per CTA; one buffer when a row (or a
    // warp's rows) fills it: more rows in flight per SM through more CTAs /
    // warps beats double buffering here (INT8 3120 x 14336: 27.8 -> 25.7 us)
    const int stages = std::max(1, std::min(8, (48 * 1024) / (rings * stride)));
    const size_t smem = static_cast<size_t>(rings) * stages * stride + rings * stages * 8 + 64;
    auto kern = per_warp ? k_rowquant_bulk_warp<Op> : k_rowquant_bulk<Op>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) ==
        cudaSuccess) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
      const int grid = std::min((rows + rings - 1) / rings, sms * per_sm);
      launch_pdl(kern, dim3(grid), dim3(threads), smem, stream, 1, xb, qb, scales, static_scale, rows, cols, col_div,
                 stages);
      count_launches(1);
      return cudaGetLastError();
    }
    cudaGetLastError();
  }
  if (aligned) {
    auto fits = [&](int tpr) { return (nvec + tpr - 1) / tpr <= kQuantMaxChunks; };
    if (fits(32)) {
      constexpr int RPB = kQuantThreads / 32;
      launch_pdl(k_rowquant_vec<Op, 32>, dim3((rows + RPB - 1) / RPB), blk, 0, stream, 1, xb, qb, scales,
                 static_scale, rows, cols, col_div);
    } else if (fits(64)) {
      constexpr int RPB = kQuantThreads / 64;
      launch_pdl(k_rowquant_vec<Op, 64>, dim3((rows + RPB - 1) / RPB), blk, 0, stream, 1, xb, qb, scales,
                 static_scale, rows, cols, col_div);
    } else if (fits(128)) {
      constexpr int RPB = kQuantThreads / 128;
      launch_pdl(k_rowquant_vec<Op, 128>, dim3((rows + RPB - 1) / RPB), blk, 0, stream, 1, xb, qb, scales,
                 static_scale, rows, cols, col_div);
    } else if (fits(256)) {
      launch_pdl(k_rowquant_vec<Op, 256>, dim3(rows), blk, 0, stream, 1, xb, qb, scales, static_scale, rows, cols,
                 col_div);
    } else {
      launch_pdl(k_rowquant_scalar<Op>, dim3((rows + 7) / 8), blk, 0, stream, 1, xb, qb, scales, static_scale, rows,
                 cols, col_div);
    }
  } else {
    launch_pdl(k_rowquant_scalar<Op>, dim3((rows + 7) / 8), blk, 0, stream, 1, xb, qb, scales, static_scale, rows,
               cols, col_div);
  }
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace qib

