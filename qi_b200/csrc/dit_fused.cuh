// Fused elementwise kernels of the MoT DiT block, around the quantized
// Linears.  Each replaces a chain of bf16 tensor ops of the reference block
// (src/qi/models/wan22/wan_video_dit.py:147-268, mot.py:100-122) with one
// pass over HBM.
//
// k_resid_ln_quant: one row per CTA, one 16-byte chunk per thread.  In order:
//   x  <- bf16(x + bf16(gate * y))  or  bf16(x + y)   (GateModule / residual)
//   n  <- bf16(LayerNorm(x) [* w + b])                 (norm1/norm2/norm3)
//   n  <- bf16(bf16(n * scale1) + shift)               (modulate; scale1 = bf16(1+scale))
//   q, s <- per-token INT8 quantization of n           (quantize_int8.cu:7-59)
// Each stage is optional.  The bf16 rounding points are those of the
// reference's tensor ops.  The row stays in registers between stages.
//
// k_rms_rope: RMSNorm over the whole attention width (all heads), times the
// norm weight, then an optional rotary embedding of (even, odd) pairs.  Up to
// two inputs (q and k) go through one launch, as blockIdx.y.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "launch_count.cuh"

namespace qib {

// One thread per 8-element chunk of a row: blockDim = D/8 rounded up to a
// whole warp (D <= 4096 -> at most 512 threads, 16 warps).
constexpr int kRowMaxThreads = 512;

__host__ __device__ inline int row_threads(int d) { return ((d / 8 + 31) / 32) * 32; }

struct ResLnParams {
  __nv_bfloat16* x;                 // [M, D] residual stream; updated in place when y != nullptr
  const __nv_bfloat16* y;           // [M, ldy] branch output, or nullptr
  long long ldy;
  const __nv_bfloat16* gate;        // [D] or nullptr (plain residual add)
  const __nv_bfloat16* ln_w;        // [D] or nullptr (no affine)
  const __nv_bfloat16* ln_b;        // [D] or nullptr
  const __nv_bfloat16* mod_scale1;  // [D] = bf16(1 + scale), or nullptr (no modulate)
  const __nv_bfloat16* mod_shift;   // [D] (with mod_scale1)
  int8_t* q;                        // [M, D] INT8 codes, or nullptr (residual update only)
  float* s;                         // [M] per-token scales (with q)
  __nv_bfloat16* xn;                // [M, D] bf16 normalized/modulated row, or nullptr
  int M, D;
  float eps;
};

// Block-wide sums / maxima of R values at once (one shared-memory round for
// all R rows of a CTA).  red holds [R][kRowMaxThreads/32] floats.
template <int R, bool MAX>
__device__ __forceinline__ void block_reduce(float (&v)[R], float* red) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v[r], o);
      v[r] = MAX ? fmaxf(v[r], u) : v[r] + u;
    }
  }
  const int nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[r * (kRowMaxThreads / 32) + (threadIdx.x >> 5)] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) {
      const float u = red[r * (kRowMaxThreads / 32) + w];
      t = MAX ? fmaxf(t, u) : t + u;
    }
    v[r] = t;
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Round 8 fp32 values to bf16 (kept as fp32), two per conversion instruction.
__device__ __forceinline__ void round8(float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(__floats2bfloat162_rn(v[2 * i], v[2 * i + 1]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Pack 8 values that are already exactly bf16 (upper halves of their fp32 bits).
__device__ __forceinline__ uint4 pack8_exact(const float (&v)[8]) {
  uint4 u;
  u.x = __byte_perm(__float_as_uint(v[0]), __float_as_uint(v[1]), 0x7632);
  u.y = __byte_perm(__float_as_uint(v[2]), __float_as_uint(v[3]), 0x7632);
  u.z = __byte_perm(__float_as_uint(v[4]), __float_as_uint(v[5]), 0x7632);
  u.w = __byte_perm(__float_as_uint(v[6]), __float_as_uint(v[7]), 0x7632);
  return u;
}

// Packed-pair forms of the helpers above.
__device__ __forceinline__ void unpack8x2(const uint4& u, float2 (&f)[4]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = __bfloat1622float2(h[i]);
}
__device__ __forceinline__ uint4 pack8x2(const float2 (&f)[4]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[i].x, f[i].y);
  return u;
}
__device__ __forceinline__ float2 round2(float2 v) { return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y)); }
__device__ __forceinline__ uint4 pack8x2_exact(const float2 (&v)[4]) {
  uint4 u;
  u.x = __byte_perm(__float_as_uint(v[0].x), __float_as_uint(v[0].y), 0x7632);
  u.y = __byte_perm(__float_as_uint(v[1].x), __float_as_uint(v[1].y), 0x7632);
  u.z = __byte_perm(__float_as_uint(v[2].x), __float_as_uint(v[2].y), 0x7632);
  u.w = __byte_perm(__float_as_uint(v[3].x), __float_as_uint(v[3].y), 0x7632);
  return u;
}

// INT8 codes clamp(rint(v * inv), -127, 127) of 8 values.  rint is done by
// adding 1.5 * 2^23 in the FP32 adder (round-to-nearest-even, exact for the
// pre-clamped |t| <= 128), which equals cvt.rni without the conversion unit.
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float inv) {
  uint32_t b[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float t = fminf(fmaxf(__fmul_rn(v[e], inv), -128.0f), 128.0f);
    int qi = static_cast<int>(__float_as_uint(__fadd_rn(t, 12582912.0f))) - 0x4B400000;
    qi = max(-127, min(127, qi));
    b[e] = static_cast<uint32_t>(qi) & 0xFFu;
  }
  return make_uint2(b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24), b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24));
}

// quant8 of 8 bf16 values whose absolute maximum over the row gave
// inv = rcp_rn(max(amax / 127, 1e-10)): then |v * inv| <= 127.00002, so of
// quant8's clamps only the lower float bound is kept, and only because it
// keeps the product and the 1.5 * 2^23 rounding add two roundings (without
// an operation between them the compiler may fuse them into one fma, which
// rounds differently at ties).  Packed fp32x2 products, bytes packed with
// byte permutes.
__device__ __forceinline__ uint2 quant8_bf16x8(const uint4& u, float inv) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 inv2 = make_float2(inv, inv), magic = make_float2(12582912.0f, 12582912.0f);
  int qi[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 t = __fmul2_rn(__bfloat1622float2(h[e]), inv2);
    t = make_float2(fmaxf(t.x, -128.0f), fmaxf(t.y, -128.0f));
    t = __fadd2_rn(t, magic);
    qi[2 * e] = max(-127, static_cast<int>(__float_as_uint(t.x)) - 0x4B400000);
    qi[2 * e + 1] = max(-127, static_cast<int>(__float_as_uint(t.y)) - 0x4B400000);
  }
  const uint32_t lo = __byte_perm(__byte_perm(qi[0], qi[1], 0x0040), __byte_perm(qi[2], qi[3], 0x0040), 0x5410);
  const uint32_t hi = __byte_perm(__byte_perm(qi[4], qi[5], 0x0040), __byte_perm(qi[6], qi[7], 0x0040), 0x5410);
  return make_uint2(lo, hi);
}

// R rows per CTA: their loads are all issued before the first reduction and
// the three block reductions (sum, sum of squares, max) serve all R rows, so
// a CTA keeps R times the bytes in flight per synchronization.
template <int R>
__global__ void __launch_bounds__(kRowMaxThreads) k_resid_ln_quant(ResLnParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[R * (kRowMaxThreads / 32)];
  const int row0 = blockIdx.x * R;
  const int j = threadIdx.x;                 // this thread's 8-element chunk of each row
  const bool act_col = j < (p.D >> 3);
  float v[R][8];
  bool act[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    act[r] = act_col && (row0 + r) < p.M;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[r][e] = 0.f;
  }

  // residual update (all R rows' loads first)
  uint4 xu[R], yu[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (!act[r]) continue;
    const long long rr = row0 + r;
    xu[r] = reinterpret_cast<const uint4*>(p.x + rr * p.D)[j];
    if (p.y != nullptr) yu[r] = reinterpret_cast<const uint4*>(p.y + rr * p.ldy)[j];
  }
  float g[8];
  if (p.gate != nullptr && act_col) unpack8(reinterpret_cast<const uint4*>(p.gate)[j], g);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (!act[r]) continue;
    unpack8(xu[r], v[r]);
    if (p.y != nullptr) {
      float yv[8];
      unpack8(yu[r], yv);
      if (p.gate != nullptr) {
#pragma unroll
        for (int e = 0; e < 8; ++e) yv[e] = __fmul_rn(g[e], yv[e]);
        round8(yv);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[r][e] = __fadd_rn(v[r][e], yv[e]);
      round8(v[r]);
      reinterpret_cast<uint4*>(p.x + static_cast<long long>(row0 + r) * p.D)[j] = pack8_exact(v[r]);
    }
  }
  if (p.q == nullptr && p.xn == nullptr) return;

  // LayerNorm statistics (two passes over registers)
  float st[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    st[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) st[r] += v[r][e];
  }
  block_reduce<R, false>(st, red);
  float mean[R], rstd[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    mean[r] = st[r] / static_cast<float>(p.D);
    st[r] = 0.f;
    if (act[r]) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[r][e] - mean[r];
        st[r] = fmaf(d, d, st[r]);
      }
    }
  }
  block_reduce<R, false>(st, red);
#pragma unroll
  for (int r = 0; r < R; ++r) rstd[r] = rsqrtf(st[r] / static_cast<float>(p.D) + p.eps);

  // normalize, affine, modulate (bf16 after each reference tensor op)
  float w[8], b[8], s1[8], sh[8];
  if (act_col) {
    if (p.ln_w != nullptr) {
      unpack8(reinterpret_cast<const uint4*>(p.ln_w)[j], w);
      unpack8(reinterpret_cast<const uint4*>(p.ln_b)[j], b);
    }
    if (p.mod_scale1 != nullptr) {
      unpack8(reinterpret_cast<const uint4*>(p.mod_scale1)[j], s1);
      unpack8(reinterpret_cast<const uint4*>(p.mod_shift)[j], sh);
    }
  }
  float amax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    amax[r] = 0.f;
    if (!act[r]) continue;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float n = (v[r][e] - mean[r]) * rstd[r];
      if (p.ln_w != nullptr) n = fmaf(n, w[e], b[e]);
      v[r][e] = n;
    }
    round8(v[r]);
    if (p.mod_scale1 != nullptr) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[r][e] = __fmul_rn(v[r][e], s1[e]);
      round8(v[r]);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[r][e] = __fadd_rn(v[r][e], sh[e]);
      round8(v[r]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) amax[r] = fmaxf(amax[r], fabsf(v[r][e]));
    if (p.xn != nullptr)
      reinterpret_cast<uint4*>(p.xn + static_cast<long long>(row0 + r) * p.D)[j] = pack8_exact(v[r]);
  }
  if (p.q == nullptr) return;

  // per-token INT8: s = max(amax/127, 1e-10), q = clamp(rint(n * (1/s)), +-127)
  block_reduce<R, true>(amax, red);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (row0 + r >= p.M) continue;
    const float s = fmaxf(__fdiv_rn(amax[r], 127.0f), 1e-10f);
    const float inv = __frcp_rn(s);
    if (j == 0) p.s[row0 + r] = s;
    if (!act[r]) continue;
    reinterpret_cast<uint2*>(p.q + static_cast<long long>(row0 + r) * p.D)[j] = quant8(v[r], inv);
  }
}

struct RmsRopeParams {
  const __nv_bfloat16* in[2];  // [M, ld_in] rows (q and k), A used columns
  long long ld_in;
  __nv_bfloat16* out[2];       // [M, ld_out]
  long long ld_out;
  const __nv_bfloat16* w[2];   // [A] RMSNorm weights
  const float* rope;           // [M, head_dim/2, 2] fp32 (cos, sin) per token and pair within a head, or nullptr
  int pairs_per_head;          // head_dim / 2
  int M, A;
  float eps;
  // per-head reduction (k_rms_rope_heads): head width, and for rows whose
  // heads are split over ranks the per-head partial sums of squares:
  // part_out [nparts][M][A / head_dim] written by this rank; part_in
  // [ranks][nparts][M][A / head_dim] from every rank (rank-major = head
  // order), normalizing over A_total = ranks * A columns
  int head_dim;
  float* part_out;
  const float* part_in;
  int ranks;
};

// One row of one part per CTA.  RMSNorm: bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)
// (wan_video_dit.py:147-158); RoPE on (even, odd) pairs within each head:
// (e c - o s, e s + o c) in fp32 (wan_video_dit.py:55-61).
template <int R>
__global__ void __launch_bounds__(kRowMaxThreads) k_rms_rope(RmsRopeParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[R * (kRowMaxThreads / 32)];
  const int row0 = blockIdx.x * R;
  const int part = blockIdx.y;
  const int j = threadIdx.x;
  const bool act_col = j < (p.A >> 3);
  const __nv_bfloat16* in = part ? p.in[1] : p.in[0];
  __nv_bfloat16* out = part ? p.out[1] : p.out[0];
  const __nv_bfloat16* wp = part ? p.w[1] : p.w[0];
  float v[R][8];
  float sq[R];
  uint4 u[R];
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (act_col && row0 + r < p.M) u[r] = reinterpret_cast<const uint4*>(in + static_cast<long long>(row0 + r) * p.ld_in)[j];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    sq[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[r][e] = 0.f;
    if (act_col && row0 + r < p.M) {
      unpack8(u[r], v[r]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sq[r] = fmaf(v[r][e], v[r][e], sq[r]);
    }
  }
  block_reduce<R, false>(sq, red);
  if (!act_col) return;
  float w[8];
  unpack8(reinterpret_cast<const uint4*>(wp)[j], w);
  const int pair0 = (j * 4) % p.pairs_per_head;  // chunk j holds pairs 4j..4j+3; index within the head
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row >= p.M) continue;
    const float rr = rsqrtf(sq[r] / static_cast<float>(p.A) + p.eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[r][e] = __fmul_rn(v[r][e], rr);
    round8(v[r]);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[r][e] = __fmul_rn(v[r][e], w[e]);
    round8(v[r]);
    if (p.rope != nullptr) {
      const float4* tab = reinterpret_cast<const float4*>(
          p.rope + (static_cast<long long>(row) * p.pairs_per_head + pair0) * 2);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float4 cs = tab[i];  // (cos, sin) of two consecutive pairs
        const float e0 = v[r][4 * i], o0 = v[r][4 * i + 1], e1 = v[r][4 * i + 2], o1 = v[r][4 * i + 3];
        v[r][4 * i] = __fsub_rn(__fmul_rn(e0, cs.x), __fmul_rn(o0, cs.y));
        v[r][4 * i + 1] = __fadd_rn(__fmul_rn(e0, cs.y), __fmul_rn(o0, cs.x));
        v[r][4 * i + 2] = __fsub_rn(__fmul_rn(e1, cs.z), __fmul_rn(o1, cs.w));
        v[r][4 * i + 3] = __fadd_rn(__fmul_rn(e1, cs.w), __fmul_rn(o1, cs.z));
      }
    }
    reinterpret_cast<uint4*>(out + static_cast<long long>(row) * p.ld_out)[j] = pack8(v[r]);
  }
}

// ---------------------------------------------------------------------------
// Warp-per-row variants for D % 256 == 0 (C = D/256 16-byte chunks per lane).
// A row lives in registers as packed bf16 (4C registers); reductions are warp
// shuffles only, so the 4 warps of a CTA work on 4 rows with no block barrier and
// many rows' loads are in flight per SM.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

constexpr int kWarpRowThreads = 128;

// The per-column vectors (gate, LayerNorm affine, modulation) are staged in
// shared memory once per CTA, so the per-chunk loops read them without an L2
// round trip each (the loops would otherwise wait on C dependent loads).
// Dynamic shared memory: 5 * D bf16.
template <int C>
__global__ void __launch_bounds__(kWarpRowThreads) k_resid_ln_quant_warp(ResLnParams p) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint4 vecs[];  // [5][C * 32]: gate, ln_w, ln_b, scale1, shift
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kWarpRowThreads / 32) + (threadIdx.x >> 5);
  {
    const __nv_bfloat16* src[5] = {p.gate, p.ln_w, p.ln_b, p.mod_scale1, p.mod_shift};
#pragma unroll
    for (int v = 0; v < 5; ++v)
      if (src[v] != nullptr)
        for (int i = threadIdx.x; i < C * 32; i += kWarpRowThreads)
          vecs[v * C * 32 + i] = __ldg(reinterpret_cast<const uint4*>(src[v]) + i);
  }
  uint4 xu[C];
  if (row < p.M) {
    const uint4* xr0 = reinterpret_cast<const uint4*>(p.x + static_cast<long long>(row) * p.D);
#pragma unroll
    for (int c = 0; c < C; ++c) xu[c] = xr0[c * 32 + lane];
  }
  __syncthreads();
  if (row >= p.M) return;
  uint4* xr = reinterpret_cast<uint4*>(p.x + static_cast<long long>(row) * p.D);
  if (p.y != nullptr) {
    const uint4* yr = reinterpret_cast<const uint4*>(p.y + static_cast<long long>(row) * p.ldy);
    uint4 yu[C];
#pragma unroll
    for (int c = 0; c < C; ++c) yu[c] = yr[c * 32 + lane];
    // bf16x2 multiply / add, each rounded once (the _rn forms are never
    // contracted into an fma): the product of two bf16 values is exact in
    // fp32 and a bf16 sum rounded directly equals the fp32 sum rounded to
    // bf16, so these are the reference's bf16(gate * y) and bf16(x + t)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      __nv_bfloat162* xh = reinterpret_cast<__nv_bfloat162*>(&xu[c]);
      const __nv_bfloat162* yh = reinterpret_cast<const __nv_bfloat162*>(&yu[c]);
      if (p.gate != nullptr) {
        const uint4 gu = vecs[c * 32 + lane];
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
#pragma unroll
        for (int e = 0; e < 4; ++e) xh[e] = __hadd2_rn(xh[e], __hmul2_rn(gh[e], yh[e]));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) xh[e] = __hadd2_rn(xh[e], yh[e]);
      }
      xr[c * 32 + lane] = xu[c];
    }
  }
  if (p.q == nullptr && p.xn == nullptr) return;

  // row statistics: per-lane pairwise sums, then the warp
  float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float2 v[4];
    unpack8x2(xu[c], v);
#pragma unroll
    for (int e = 0; e < 4; ++e) sum2 = __fadd2_rn(sum2, v[e]);
  }
  const float mean = warp_sum(sum2.x + sum2.y) / static_cast<float>(p.D);
  const float2 negmean2 = make_float2(-mean, -mean);  // v + (-mean) rounds as v - mean
  float2 sq2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float2 v[4];
    unpack8x2(xu[c], v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 d = __fadd2_rn(v[e], negmean2);
      sq2 = __ffma2_rn(d, d, sq2);
    }
  }
  const float rstd = rsqrtf(warp_sum(sq2.x + sq2.y) / static_cast<float>(p.D) + p.eps);
  const float2 rstd2 = make_float2(rstd, rstd);

  __nv_bfloat162 amax2 = __float2bfloat162_rn(0.f);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int j = c * 32 + lane;
    float2 v[4];
    unpack8x2(xu[c], v);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __fmul2_rn(__fadd2_rn(v[e], negmean2), rstd2);
    if (p.ln_w != nullptr) {
      float2 w[4], b[4];
      unpack8x2(vecs[1 * C * 32 + j], w);
      unpack8x2(vecs[2 * C * 32 + j], b);
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = __ffma2_rn(v[e], w[e], b[e]);
    }
    xu[c] = pack8x2(v);  // bf16(LayerNorm)
    if (p.mod_scale1 != nullptr) {
      // bf16(bf16(n * scale1) + shift) in bf16x2 (single roundings, as above)
      const uint4 su = vecs[3 * C * 32 + j], hu = vecs[4 * C * 32 + j];
      __nv_bfloat162* nh = reinterpret_cast<__nv_bfloat162*>(&xu[c]);
      const __nv_bfloat162* s1 = reinterpret_cast<const __nv_bfloat162*>(&su);
      const __nv_bfloat162* sh = reinterpret_cast<const __nv_bfloat162*>(&hu);
#pragma unroll
      for (int e = 0; e < 4; ++e) nh[e] = __hadd2_rn(__hmul2_rn(nh[e], s1[e]), sh[e]);
    }
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&xu[c]);
#pragma unroll
    for (int e = 0; e < 4; ++e) amax2 = __hmax2(amax2, __habs2(h[e]));  // exact: the values are bf16
    if (p.xn != nullptr) reinterpret_cast<uint4*>(p.xn + static_cast<long long>(row) * p.D)[j] = xu[c];
  }
  if (p.q == nullptr) return;
  float amax = fmaxf(__low2float(amax2), __high2float(amax2));
  amax = warp_max(amax);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-10f);
  const float inv = __frcp_rn(s);
  if (lane == 0) p.s[row] = s;
  uint2* qr = reinterpret_cast<uint2*>(p.q + static_cast<long long>(row) * p.D);
#pragma unroll
  for (int c = 0; c < C; ++c) qr[c * 32 + lane] = quant8_bf16x8(xu[c], inv);
}

// The RMSNorm weight is staged in shared memory once per CTA; when a head's
// pair count divides 128 every chunk of a lane covers the same pairs of its
// head, so the row's (cos, sin) for them are loaded once.  Dynamic shared
// memory: A bf16.
template <int C>
__global__ void __launch_bounds__(kWarpRowThreads) k_rms_rope_warp(RmsRopeParams p) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint4 wsm[];  // [C * 32] RMSNorm weight of this part
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kWarpRowThreads / 32) + (threadIdx.x >> 5);
  const int part = blockIdx.y;
  {
    const uint4* wsrc = reinterpret_cast<const uint4*>(part ? p.w[1] : p.w[0]);
    for (int i = threadIdx.x; i < C * 32; i += kWarpRowThreads) wsm[i] = __ldg(wsrc + i);
  }
  uint4 u[C];
  const bool rope_fixed = p.rope != nullptr && (128 % p.pairs_per_head) == 0;
  float4 cs_fixed[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  if (row < p.M) {
    const uint4* ir = reinterpret_cast<const uint4*>((part ? p.in[1] : p.in[0]) + static_cast<long long>(row) * p.ld_in);
#pragma unroll
    for (int c = 0; c < C; ++c) u[c] = ir[c * 32 + lane];
    if (rope_fixed) {
      const float4* tab = reinterpret_cast<const float4*>(
          p.rope + (static_cast<long long>(row) * p.pairs_per_head + (lane * 4) % p.pairs_per_head) * 2);
      cs_fixed[0] = tab[0];
      cs_fixed[1] = tab[1];
    }
  }
  __syncthreads();
  if (row >= p.M) return;
  uint4* orow = reinterpret_cast<uint4*>((part ? p.out[1] : p.out[0]) + static_cast<long long>(row) * p.ld_out);
  const uint4* wp = wsm;
  float2 sq2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float2 v2[4];
    unpack8x2(u[c], v2);
#pragma unroll
    for (int e = 0; e < 4; ++e) sq2 = __ffma2_rn(v2[e], v2[e], sq2);
  }
  const float r = rsqrtf(warp_sum(sq2.x + sq2.y) / static_cast<float>(p.A) + p.eps);
  const float2 r2 = make_float2(r, r);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int j = c * 32 + lane;
    float2 v2[4], w2[4];
    unpack8x2(u[c], v2);
    unpack8x2(wp[j], w2);
#pragma unroll
    for (int e = 0; e < 4; ++e) v2[e] = round2(__fmul2_rn(round2(__fmul2_rn(v2[e], r2)), w2[e]));
    float v[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[2 * e] = v2[e].x;
      v[2 * e + 1] = v2[e].y;
    }
    if (p.rope != nullptr) {
      const int pair0 = (j * 4) % p.pairs_per_head;
      const float4* tab = reinterpret_cast<const float4*>(
          p.rope + (static_cast<long long>(row) * p.pairs_per_head + pair0) * 2);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float4 cs = rope_fixed ? cs_fixed[i] : tab[i];
        const float e0 = v[4 * i], o0 = v[4 * i + 1], e1 = v[4 * i + 2], o1 = v[4 * i + 3];
        v[4 * i] = __fsub_rn(__fmul_rn(e0, cs.x), __fmul_rn(o0, cs.y));
        v[4 * i + 1] = __fadd_rn(__fmul_rn(e0, cs.y), __fmul_rn(o0, cs.x));
        v[4 * i + 2] = __fsub_rn(__fmul_rn(e1, cs.z), __fmul_rn(o1, cs.w));
        v[4 * i + 3] = __fadd_rn(__fmul_rn(e1, cs.w), __fmul_rn(o1, cs.z));
      }
    }
    orow[j] = pack8(v);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm (+ RoPE) with a reduction that does not depend on how the heads
// are split over ranks.  Every head's sum of squares is formed the same way
// (each lane adds the squares of its 8 consecutive elements in order, then a
// butterfly over the head_dim/8 lanes of the head), and the row total is the
// sum of the per-head sums in head order.  A rank that holds a contiguous
// range of whole heads computes those heads' sums bit for bit as one GPU
// does; with every rank's sums gathered (part_in), its total and hence its
// normalized outputs are bit-identical to the single-GPU kernel's.
//   MODE 0: whole row on this GPU: per-head sums, total, normalize, RoPE.
//   MODE 1: per-head sums only, written to part_out.
//   MODE 2: total from part_in (every rank's sums), normalize, RoPE.
// Warp per row, C = ceil(A / 256) 16-byte chunks per lane (chunk c of lane l
// = elements (32 c + l) * 8 ..+7); head_dim in {8, 16, 32, 64, 128, 256}.
// ---------------------------------------------------------------------------
template <int C, int MODE>
__global__ void __launch_bounds__(kWarpRowThreads) k_rms_rope_heads(RmsRopeParams p) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint4 wsm[];  // [A / 8] RMSNorm weight of this part (MODE != 1)
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kWarpRowThreads / 32) + (threadIdx.x >> 5);
  const int part = blockIdx.y;
  const int nvec = p.A >> 3;
  if (MODE != 1) {
    const uint4* wsrc = reinterpret_cast<const uint4*>(part ? p.w[1] : p.w[0]);
    for (int i = threadIdx.x; i < nvec; i += kWarpRowThreads) wsm[i] = __ldg(wsrc + i);
  }
  uint4 u[C];
  if (row < p.M) {
    const uint4* ir = reinterpret_cast<const uint4*>((part ? p.in[1] : p.in[0]) + static_cast<long long>(row) * p.ld_in);
#pragma unroll
    for (int c = 0; c < C; ++c)
      if (c * 32 + lane < nvec) u[c] = ir[c * 32 + lane];
  }
  if (MODE != 1) __syncthreads();
  if (row >= p.M) return;
  const int lph = p.head_dim >> 3;        // lanes per head
  const int hpc = 32 / lph;               // heads per chunk
  const int heads = p.A / p.head_dim;     // heads on this GPU
  float hs[C];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float s = 0.f;
    if (c * 32 + lane < nvec) {
      float v[8];
      unpack8(u[c], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[e], v[e], s);
    }
    for (int o = lph >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    hs[c] = s;
  }
  if (MODE == 1) {
    float* dst = p.part_out + (static_cast<long long>(part) * p.M + row) * heads;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int h = c * hpc + lane / lph;
      if (lane % lph == 0 && h < heads) dst[h] = hs[c];
    }
    return;
  }
  float tot = 0.f;
  if (MODE == 0) {
#pragma unroll
    for (int c = 0; c < C; ++c)
      for (int g = 0; g < hpc; ++g) {
        const float hv = __shfl_sync(0xffffffffu, hs[c], g * lph);
        if (c * hpc + g < heads) tot += hv;
      }
  } else {
    const int nparts = gridDim.y;
    for (int r = 0; r < p.ranks; ++r) {
      const float* src = p.part_in + ((static_cast<long long>(r) * nparts + part) * p.M + row) * heads;
      for (int h = 0; h < heads; ++h) tot += __ldg(src + h);
    }
  }
  const float rr = rsqrtf(tot / static_cast<float>(p.A * (MODE == 2 ? p.ranks : 1)) + p.eps);
  uint4* orow = reinterpret_cast<uint4*>((part ? p.out[1] : p.out[0]) + static_cast<long long>(row) * p.ld_out);
  const bool rope_fixed = p.rope != nullptr && (128 % p.pairs_per_head) == 0;
  float4 cs_fixed[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  if (rope_fixed) {
    const float4* tab = reinterpret_cast<const float4*>(
        p.rope + (static_cast<long long>(row) * p.pairs_per_head + (lane * 4) % p.pairs_per_head) * 2);
    cs_fixed[0] = tab[0];
    cs_fixed[1] = tab[1];
  }
  const float2 rr2 = make_float2(rr, rr);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int j = c * 32 + lane;
    if (j >= nvec) continue;
    // bf16(x * rr) (fp32 product, then bf16), then bf16(n * w): a product of
    // two bf16 values rounded once, in bf16x2 (never contracted)
    uint4 nb;
    {
      float2 f[4];
      unpack8x2(u[c], f);
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = __fmul2_rn(f[e], rr2);
      nb = pack8x2(f);
      const uint4 wu = wsm[j];
      __nv_bfloat162* nh = reinterpret_cast<__nv_bfloat162*>(&nb);
      const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wu);
#pragma unroll
      for (int e = 0; e < 4; ++e) nh[e] = __hmul2_rn(nh[e], wh[e]);
    }
    if (p.rope == nullptr) {
      orow[j] = nb;
      continue;
    }
    float v[8];
    unpack8(nb, v);
    {
      const float4* tab = nullptr;
      if (!rope_fixed)
        tab = reinterpret_cast<const float4*>(
            p.rope + (static_cast<long long>(row) * p.pairs_per_head + (j * 4) % p.pairs_per_head) * 2);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float4 cs = rope_fixed ? cs_fixed[i] : tab[i];
        const float e0 = v[4 * i], o0 = v[4 * i + 1], e1 = v[4 * i + 2], o1 = v[4 * i + 3];
        v[4 * i] = __fsub_rn(__fmul_rn(e0, cs.x), __fmul_rn(o0, cs.y));
        v[4 * i + 1] = __fadd_rn(__fmul_rn(e0, cs.y), __fmul_rn(o0, cs.x));
        v[4 * i + 2] = __fsub_rn(__fmul_rn(e1, cs.z), __fmul_rn(o1, cs.w));
        v[4 * i + 3] = __fadd_rn(__fmul_rn(e1, cs.w), __fmul_rn(o1, cs.z));
      }
    }
    orow[j] = pack8(v);
  }
}

}  // namespace qib
