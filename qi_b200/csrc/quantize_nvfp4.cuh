// NVFP4 activation quantization: bf16 [rows, cols] -> E2M1 codes (two per
// byte, element 2j in the low nibble), E4M3 block scales (one per 16
// elements along K) in the tensor-core scale-factor atom layout, and an fp32
// second-level scale g (per tensor or per row).
//
// Recipe (NVFP4 as published by NVIDIA; restated in oracle/qi_oracle.py):
//   g  = max(amax / (6 * 448), 1e-12)                   amax of the tensor or row
//   sf = e4m3_rn( min(amax_16 / (6 g), 448) )           per 16-element block
//   q  = e2m1_rn( clamp(x / (f32(sf) g), +-6) ), 0 where sf == 0
// Scale-factor atom layout: 512-byte atoms of 128 rows x 4 block scales,
// atoms ordered K-fastest then by 128-row block; row r = r0 + 32 r1 of an
// atom at byte r0*16 + r1*4 + j.  Exactly what tcgen05.cp 32x128b.warpx4
// copies into tensor memory for the block-scaled MMA.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "quantize_act.cuh"

namespace qib {

constexpr float kNvfp4GDiv = 6.0f * 448.0f;

__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u32.u8 %0, t;\n\t}\n"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

__device__ __forceinline__ float nvfp4_g_from_amax(float amax) { return fmaxf(__fdiv_rn(amax, kNvfp4GDiv), 1e-12f); }

__device__ __forceinline__ long long sf_atom_offset(int row, int blk, int ka_per_rowblock) {
  const int ra = row >> 7, r = row & 127, ka = blk >> 2, j = blk & 3;
  return (static_cast<long long>(ra) * ka_per_rowblock + ka) * 512 + (r & 31) * 16 + (r >> 5) * 4 + j;
}

// amax of a whole bf16 tensor into *amax_bits (float bits).  part == nullptr:
// blocks atomicMax into *amax_bits, which must start at 0.  Otherwise each
// block stores its maximum in part[blockIdx.x] and the last block to finish
// (ticket, zero on entry and left zero) reduces them into *amax_bits, so the
// word needs no clearing before the launch.
__global__ void __launch_bounds__(256)
k_amax_bf16(const __nv_bfloat16* __restrict__ x, long long n, unsigned int* __restrict__ amax_bits,
            unsigned int* __restrict__ part, unsigned int* __restrict__ ticket) {
  griddep_wait();
  griddep_launch_dependents();
  float m = 0.f;
  const long long nvec = n / 8;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  // kLoads 16-byte loads in flight per thread (the pass is bound by DRAM
  // latency with two); bf16 |x| max taken exactly in bf16x2
  constexpr int kLoads = 8;
  const long long stride = 256ll * gridDim.x;
  __nv_bfloat162 m2 = __float2bfloat162_rn(0.f);
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < nvec; i += kLoads * stride) {
    uint4 v[kLoads];
#pragma unroll
    for (int u = 0; u < kLoads; ++u)
      v[u] = i + u * stride < nvec ? __ldg(xv + i + u * stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[k])));
    }
  }
  m = fmaxf(__low2float(m2), __high2float(m2));
  for (long long i = nvec * 8 + blockIdx.x * 256ll + threadIdx.x; i < n; i += 256ll * gridDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  __shared__ float wm[8];
  __shared__ unsigned int last_sh;
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) m = fmaxf(m, wm[w]);
    if (part == nullptr) {
      atomicMax(amax_bits, __float_as_uint(m));  // non-negative floats order like their bits
    } else {
      part[blockIdx.x] = __float_as_uint(m);
      __threadfence();
      last_sh = atomicAdd(ticket, 1u) == gridDim.x - 1 ? 1u : 0u;
    }
  }
  if (part == nullptr) return;
  __syncthreads();
  if (last_sh == 0) return;
  __threadfence();  // every block's part is visible
  unsigned int r = 0;
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += 256) r = max(r, __ldcg(part + i));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) r = max(r, __shfl_xor_sync(0xffffffffu, r, off));
  __shared__ unsigned int wr[8];
  if ((threadIdx.x & 31) == 0) wr[threadIdx.x >> 5] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) r = max(r, wr[w]);
    *amax_bits = r;
    atomicExch(ticket, 0u);  // ready for the next launch
  }
}

__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ uint32_t e4m3_code(float v) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
// E4M3 codes of two floats in one conversion: lo in bits 0-7, hi in 8-15.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
  return out;
}
// E2M1 codes of 8 floats (pairs a..d, .x the lower nibble of each byte),
// packed into 4 bytes in element order.
__device__ __forceinline__ uint32_t e2m1x8(float2 a, float2 b, float2 c, float2 d) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}\n"
      : "=r"(out)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y), "f"(d.x), "f"(d.y));
  return out;
}

// One 16-element block -> its packed E2M1 codes (8 bytes) and E4M3 block-scale
// code, with divisions only where they decide the result, for a given g.  Each quotient the recipe rounds (bm / fl(6 g) for the block
// scale, x / fl(sf g) for the codes) is bracketed by two products with a
// reciprocal widened by +-2^-20 (8 ulp, more than the approximate
// reciprocal's and the products' rounding): the exact quotient and its fp32
// rounding both lie inside the bracket, and E4M3 / E2M1 rounding is
// monotonic, so when both ends convert to the same code that code is the
// recipe's.  Where they differ (a quotient within a few ulp of a rounding
// boundary; exact ties occur, e.g. when sf carries a factor that cancels
// against g's), that scale or the block's codes are recomputed with
// correctly rounded divisions.  Both bracket ends of the scale go through one
// E4M3x2 conversion and the codes eight at a time (E2M1x2 conversions packed
// into a word), so the common case costs one comparison per 8 codes.  A zero
// block scale gives +0 codes (the recipe's q = 0 where sf == 0, also for
// negative inputs).  rg = the bracket ends of 1 / fl(6 g).  Saturating
// conversions are the recipe's clamps (448, +-6).
__device__ __forceinline__ uint2 nvfp4_block_fast(const uint4& v0, const uint4& v1, float g, float g6, float2 rg,
                                                  uint8_t& sfc) {
  const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  __nv_bfloat162 m2 = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[0]));
#pragma unroll
  for (int k = 1; k < 8; ++k) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[k])));
  const float bm = fmaxf(__low2float(m2), __high2float(m2));  // exact: max of the same values
  const uint32_t cc = e4m3x2(__fmul_rn(bm, rg.x), __fmul_rn(bm, rg.y));  // both bracket ends at once
  uint32_t c = cc & 0xffu;
  if (c != (cc >> 8)) c = e4m3_code(fminf(__fdiv_rn(bm, g6), 448.0f));
  sfc = static_cast<uint8_t>(c);
  if (c == 0) return make_uint2(0u, 0u);  // sf == 0: every code is +0
  __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(sfc), __NV_E4M3);
  const float denom = __fmul_rn(__half2float(__half(hr)), g);
  const float inv = rcp_approx(denom);
  const float il = inv * (1.0f - 0x1p-20f), ih = inv * (1.0f + 0x1p-20f);
  const float2 il2 = make_float2(il, il), ih2 = make_float2(ih, ih);
  float2 f[8], a[8], b[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    f[k] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
    a[k] = __fmul2_rn(f[k], il2);
    b[k] = __fmul2_rn(f[k], ih2);
  }
  uint32_t lo = e2m1x8(a[0], a[1], a[2], a[3]), hi = e2m1x8(a[4], a[5], a[6], a[7]);
  // nibbles whose bracket ends convert differently: a quotient within a few
  // ulp of a rounding boundary.  Only those elements are recomputed by
  // correctly rounded division.  Exact ties are common with a per-tensor g
  // (amax / 2688 = amax / (2^7 * 3 * 7) against E4M3 block scales carrying a
  // factor 3 or 7, such as 1.5 or 1.75):
  // on N(0, 1) data about 1 % of the blocks have one, so recomputing a whole
  // block would run 16 divisions in a quarter of all 32-block warp steps;
  // per element, a division runs only where some lane needs that element.
  const uint32_t dlo = lo ^ e2m1x8(b[0], b[1], b[2], b[3]), dhi = hi ^ e2m1x8(b[4], b[5], b[6], b[7]);
  if ((dlo | dhi) != 0u) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t d = k < 4 ? dlo : dhi;
      uint32_t& word = k < 4 ? lo : hi;
      const int sh = 8 * (k & 3);  // element 2k in the low nibble of byte k & 3, element 2k + 1 in the high one
      if (d & (0xFu << sh)) word = (word & ~(0xFu << sh)) | ((e2m1x2(__fdiv_rn(f[k].x, denom), 0.f) & 0xFu) << sh);
      if (d & (0xF0u << sh))
        word = (word & ~(0xF0u << sh)) | ((e2m1x2(__fdiv_rn(f[k].y, denom), 0.f) & 0xFu) << (sh + 4));
    }
  }
  return make_uint2(lo, hi);
}

// Per-tensor g (GMODE 0: *g_in, 1: from *amax_bits, g written to g_out[0]).
// One thread per 16-element block; a warp covers 32 consecutive blocks, and
// warps walk the tensor from its END, so the part of x that the amax pass
// read last (still in L2) is read first.  Four lanes' block scales (one 4-byte
// word of an atom row) are stored together.  rows_pad * bpr % 32 == 0.
template <int GMODE>
__global__ void __launch_bounds__(256)
k_quant_nvfp4_tensor(const __nv_bfloat16* __restrict__ x, int rows, int cols, const float* __restrict__ g_in,
                     const unsigned int* __restrict__ amax_bits, float* __restrict__ g_out, uint8_t* __restrict__ q,
                     uint8_t* __restrict__ sf, int ka_per_rowblock) {
  griddep_wait();
  griddep_launch_dependents();
  const int bpr = cols >> 4;
  const int rows_pad = (rows + 127) & ~127;
  float g;
  if (GMODE == 0) {
    g = __ldg(g_in);
  } else {
    g = nvfp4_g_from_amax(__uint_as_float(*amax_bits));
    if (blockIdx.x == 0 && threadIdx.x == 0) g_out[0] = g;
  }
  const int lane = threadIdx.x & 31;
  const float g6 = __fmul_rn(6.0f, g);
  const float rg0 = rcp_approx(g6);
  const float2 rg = make_float2(rg0 * (1.0f - 0x1p-20f), rg0 * (1.0f + 0x1p-20f));
  const int chunks = rows_pad * bpr / 32;  // the host keeps rows_pad * bpr < 2^31
  const int cstride = 256 * gridDim.x / 32;
  // t / bpr for 0 <= t < 2^31 as mulhi(t, m) >> (l - 1), m = ceil(2^(31 + l) /
  // bpr), l = ceil(log2 bpr) >= 2 (bpr = cols / 16 >= 4): the product's
  // excess over t / bpr is below t / 2^(31 + l) < 1 / bpr, so the floor is exact
  const uint32_t dl = 32u - static_cast<uint32_t>(__clz(bpr - 1));
  const uint32_t dm = static_cast<uint32_t>(((1ull << (31 + dl)) + static_cast<unsigned>(bpr) - 1) / static_cast<unsigned>(bpr));
  auto div_bpr = [&](int t) { return static_cast<int>(__umulhi(static_cast<uint32_t>(t), dm) >> (dl - 1)); };
  // quantize + store one block (row < rows), then the atom word of 4 lanes
  auto finish = [&](const uint4& v0, const uint4& v1, int row, int b) {
    uint8_t sfc = 0;
    if (row < rows) {
      const uint2 packed = nvfp4_block_fast(v0, v1, g, g6, rg, sfc);
      *reinterpret_cast<uint2*>(q + static_cast<long long>(row) * (cols >> 1) + b * 8) = packed;
    }
    // blocks b .. b+3 (b % 4 == 0) of one row share a 4-byte word of the atom
    // row: lanes 4i .. 4i + 3 hold them (b & 3 == lane & 3), OR-reduced
    uint32_t wd = static_cast<uint32_t>(sfc) << (8 * (b & 3));
    wd |= __shfl_xor_sync(0xffffffffu, wd, 1);
    wd |= __shfl_xor_sync(0xffffffffu, wd, 2);
    if ((b & 3) == 0) *reinterpret_cast<uint32_t*>(sf + sf_atom_offset(row, b, ka_per_rowblock)) = wd;
  };
  // two chunks per iteration: both chunks' loads are in flight before either
  // is quantized (chunk indices are warp-uniform, so are the branches)
  for (int ch = (blockIdx.x * 256 + threadIdx.x) / 32; ch < chunks; ch += 2 * cstride) {
    const int ch2 = ch + cstride;
    const int t = (chunks - 1 - ch) * 32 + lane;
    const int row = div_bpr(t), b = t - row * bpr;
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, w0 = v0, w1 = v0;
    if (row < rows) {
      const uint4* p = reinterpret_cast<const uint4*>(x + static_cast<long long>(row) * cols + b * 16);
      v0 = __ldg(p);
      v1 = __ldg(p + 1);
    }
    int row2 = rows, b2 = 0;
    if (ch2 < chunks) {
      const int t2 = (chunks - 1 - ch2) * 32 + lane;
      row2 = div_bpr(t2);
      b2 = t2 - row2 * bpr;
      if (row2 < rows) {
        const uint4* p = reinterpret_cast<const uint4*>(x + static_cast<long long>(row2) * cols + b2 * 16);
        w0 = __ldg(p);
        w1 = __ldg(p + 1);
      }
    }
    finish(v0, v1, row, b);
    if (ch2 < chunks) finish(w0, w1, row2, b2);
  }
}

// Per-row g (GMODE 2; the per-tensor modes run k_quant_nvfp4_tensor): a CTA
// per row reduces the row's amax, writes g to g_out[row], then one thread per
// 16-element block.  cols % 16 == 0.  Scale-factor entries of the padding
// rows (up to the next multiple of 128) are written as zero so the GEMM never
// reads stale bytes.
template <int GMODE>
__global__ void __launch_bounds__(256)
k_quant_nvfp4(const __nv_bfloat16* __restrict__ x, int rows, int cols, const float* __restrict__ g_in,
              const unsigned int* __restrict__ amax_bits, float* __restrict__ g_out, uint8_t* __restrict__ q,
              uint8_t* __restrict__ sf, int ka_per_rowblock) {
  static_assert(GMODE == 2, "per-row g only");
  griddep_wait();
  griddep_launch_dependents();
  const int bpr = cols >> 4;  // blocks per row
  const int rows_pad = (rows + 127) & ~127;
  if (GMODE == 2) {
    __shared__ float wm[8];
    __shared__ float g_sh;
    for (int row = blockIdx.x; row < rows_pad; row += gridDim.x) {
      if (row >= rows) {
        for (int b = threadIdx.x; b < bpr; b += 256) sf[sf_atom_offset(row, b, ka_per_rowblock)] = 0;
        continue;
      }
      const __nv_bfloat16* xr = x + static_cast<long long>(row) * cols;
      float m = 0.f;
      for (int b = threadIdx.x; b < bpr; b += 256) {
        const uint4* p = reinterpret_cast<const uint4*>(xr + b * 16);
        const uint4 v0 = __ldg(p), v1 = __ldg(p + 1);
        m = fmaxf(m, fmaxf(absmax_bf16x8(v0), absmax_bf16x8(v1)));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) m = fmaxf(m, wm[w]);
        g_sh = nvfp4_g_from_amax(m);
        g_out[row] = g_sh;
      }
      __syncthreads();
      const float g = g_sh;
      const float g6 = __fmul_rn(6.0f, g);
      const float rg0 = rcp_approx(g6);
      const float2 rg = make_float2(rg0 * (1.0f - 0x1p-20f), rg0 * (1.0f + 0x1p-20f));
      for (int b = threadIdx.x; b < bpr; b += 256) {
        const uint4* p = reinterpret_cast<const uint4*>(xr + b * 16);
        uint8_t sfc;
        const uint2 packed = nvfp4_block_fast(__ldg(p), __ldg(p + 1), g, g6, rg, sfc);
        *reinterpret_cast<uint2*>(q + static_cast<long long>(row) * (cols >> 1) + b * 8) = packed;
        sf[sf_atom_offset(row, b, ka_per_rowblock)] = sfc;
      }
      __syncthreads();
    }
    return;
  }
}

}  // namespace qib
