// Attention over a short key sequence (at most 256 keys, head dim 128) on the
// tensor cores: O = softmax(Q K^T * scale) V per head, all keys of a head in
// one tile, so the softmax is exact over the row (no running rescale).
//
// The DiT step has three such attentions per layer: the cross-attention of the
// video queries over the 128 context tokens (wan_video_dit.py:122-140), the
// first-frame queries over the first-frame keys, and the 32 action queries
// over first-frame video keys plus their own (mot.py:361-463).  The long
// video self-attention (3120 keys) is not this kernel's.
//
// One work item = (head h, 128 query rows).  A persistent CTA of 4 warps runs
// items in turn:
//   thread 0: TMA loads Q [128 x 128], K [KEYS x 128] and V^T [128 x KEYS]
//             (bf16, 128-byte swizzled, out-of-range rows / keys read 0),
//             then S = Q K^T with tcgen05.mma kind::f16 into TMEM (fp32);
//   4 warps:  each thread owns one query row (its TMEM lane): row max, then
//             p = 2^((s - max) * scale * log2 e) rounded to bf16, written to
//             shared memory in the swizzled K-major layout the MMA reads (over
//             the dead Q or K tile), and the row sum of the rounded p;
//   thread 0: O = P V (V^T as the K-major B operand) into TMEM;
//   4 warps:  O / sum -> bf16 into a swizzled staging tile; thread 0 stores it
//             with TMA (asynchronous: it overlaps the next item's loads).
// Every wait is bounded; an expired wait records the error, raises the CTA's
// abort flag and the CTA drains its copies / MMAs and exits.
#pragma once

#include <cuda_bf16.h>
#include <cuda.h>
#include <cstdint>

#include "launch_count.cuh"
#include "sm100_ptx.cuh"

namespace qib {

constexpr int kAttnThreads = 128;
constexpr unsigned int kTagAttn = 0x600u;

template <int NKB>
struct AttnCfg {
  static constexpr int KEYS = 128 * NKB;              // key capacity of one tile
  static constexpr int Q_BYTES = 2 * 128 * 128;       // 2 head-dim blocks of 64 x 128 rows
  static constexpr int K_BYTES = 2 * KEYS * 128;      // 2 head-dim blocks of 64 x KEYS rows
  static constexpr int VT_BYTES = 2 * NKB * 128 * 128;  // KEYS / 64 key blocks x 128 head-dim rows
  static constexpr int P_BYTES = 2 * NKB * 128 * 128;   // KEYS / 64 key blocks x 128 query rows
  static_assert(P_BYTES == (NKB == 1 ? Q_BYTES : K_BYTES), "P reuses the Q (one key block) or K tile");
  static constexpr int SMEM_BYTES = Q_BYTES + K_BYTES + VT_BYTES + 64 + 1024;
  static constexpr int S_COL = 0, O_COL = KEYS;       // TMEM columns of S and O
  static constexpr int TMEM_COLS = NKB == 1 ? 256 : 512;
  static constexpr uint32_t IDESC_S = make_idesc(kDF32, kFmtBF16, kFmtBF16, 128, KEYS);
  static constexpr uint32_t IDESC_O = make_idesc(kDF32, kFmtBF16, kFmtBF16, 128, 128);
};

struct AttnParams {
  int sq, sk, heads;
  float scale_log2e;  // softmax scale * log2(e)
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// p = 2^(s * scale_log2e + off) of 32 scores (keys c .. c+31), masked beyond
// sk, rounded to bf16 and packed in pairs; returns their fp32 sum.
__device__ __forceinline__ float attn_p32(const uint32_t (&r)[32], int c, int sk, float sl2e, float off,
                                          uint32_t (&pk)[16]) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float e0 = (c + 2 * i < sk) ? ex2_approx(fmaf(__uint_as_float(r[2 * i]), sl2e, off)) : 0.f;
    const float e1 = (c + 2 * i + 1 < sk) ? ex2_approx(fmaf(__uint_as_float(r[2 * i + 1]), sl2e, off)) : 0.f;
    const __nv_bfloat162 b = __floats2bfloat162_rn(e0, e1);
    const float2 f = __bfloat1622float2(b);
    sum += f.x;
    sum += f.y;
    pk[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return sum;
}

// 16 packed words (32 bf16 of columns c .. c+31 of `row`) into a tile of
// 64-column, 128-row, 128-byte-swizzled regions (the layout TMA and the MMA
// descriptors use).
__device__ __forceinline__ void st_sw128_32(uint8_t* tile, int row, int c, const uint32_t (&pk)[16]) {
  uint8_t* prow = tile + (c >> 6) * (128 * 128) + row * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int chunk = ((c & 63) >> 3) + q;
    *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) << 4)) =
        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

template <int NKB>
__global__ void __launch_bounds__(kAttnThreads)
k_attn_short(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
             const __grid_constant__ CUtensorMap tmVt, const __grid_constant__ CUtensorMap tmO,
             const AttnParams p) {
  using C = AttnCfg<NKB>;
  extern __shared__ uint8_t attn_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;
  uint8_t* sVt = sK + C::K_BYTES;
  uint8_t* sP = NKB == 1 ? sQ : sK;
  uint8_t* sO = NKB == 1 ? sK : sQ;  // bf16 O staging for the TMA store: the tile P does not hold
  uint64_t* full = reinterpret_cast<uint64_t*>(sVt + C::VT_BYTES);
  uint64_t* sdone = full + 1;
  uint64_t* odone = full + 2;
  uint64_t* drain = full + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(full, 1);
    mbar_init(sdone, 1);
    mbar_init(odone, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_map(&tmQ);
    tma_prefetch_map(&tmK);
    tma_prefetch_map(&tmVt);
    tma_prefetch_map(&tmO);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  const int q_tiles = (p.sq + 127) / 128;
  const int items = q_tiles * p.heads;
  const int row = warp * 32 + lane;  // query row of the tile = TMEM lane
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
  constexpr uint32_t kTxBytes = C::Q_BYTES + C::K_BYTES + C::VT_BYTES;
  bool ok = true;
  uint32_t phase = 0;
  int issued = 0;  // items whose loads thread 0 has issued
#pragma unroll 1
  for (int item = blockIdx.x; item < items; item += gridDim.x, phase ^= 1u) {
    const int h = item / q_tiles, m0 = (item - h * q_tiles) * 128;
    if (threadIdx.x == 0) {
      bulk_wait_read_all();  // the previous item's O store has read its staging tile
      mbar_expect_tx(full, kTxBytes);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        tma_load_2d(sQ + kb * 128 * 128, &tmQ, full, h * 128 + kb * 64, m0);
        tma_load_2d(sK + kb * C::KEYS * 128, &tmK, full, h * 128 + kb * 64, 0);
      }
#pragma unroll
      for (int j = 0; j < 2 * NKB; ++j) tma_load_2d(sVt + j * 128 * 128, &tmVt, full, j * 64, h * 128);
      ++issued;
      if (!mbar_wait(full, phase, abort_flag, kTagAttn, 1)) {
        ok = false;
      } else {
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem_base + C::S_COL, sw128_kmajor_desc(smem_u32(sQ + kb * 128 * 128) + kk * 32),
                     sw128_kmajor_desc(smem_u32(sK + kb * C::KEYS * 128) + kk * 32), C::IDESC_S,
                     (kb | kk) != 0 ? 1u : 0u);
        tc_commit(sdone);
      }
    }
    if (!mbar_wait(sdone, phase, abort_flag, kTagAttn, 2)) { ok = false; break; }
    tc_fence_after();

    // ---- softmax of this thread's row: max, then 2^(..) as bf16 into P (swizzled),
    // the fp32 sum of the rounded values.  One key block: the 128 scores stay in
    // registers (one TMEM pass); two: max pass, then exp pass.
    float sum = 0.f;
    if constexpr (NKB == 1) {
      uint32_t r[4][32];
#pragma unroll
      for (int b = 0; b < 4; ++b) tmem_ld_32x32b_x32(t_row + C::S_COL + 32 * b, r[b]);
      tmem_ld_wait();
      float mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (32 * b + i < p.sk) mx = fmaxf(mx, __uint_as_float(r[b][i]));
      const float off = -mx * p.scale_log2e;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t pk[16];
        sum += attn_p32(r[b], 32 * b, p.sk, p.scale_log2e, off, pk);
        st_sw128_32(sP, row, 32 * b, pk);
      }
    } else {
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < C::KEYS; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + C::S_COL + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c + i < p.sk) mx = fmaxf(mx, __uint_as_float(r[i]));
      }
      const float off = -mx * p.scale_log2e;
#pragma unroll 1
      for (int c = 0; c < C::KEYS; c += 32) {
        uint32_t r[32], pk[16];
        tmem_ld_32x32b_x32(t_row + C::S_COL + c, r);
        tmem_ld_wait();
        sum += attn_p32(r, c, p.sk, p.scale_log2e, off, pk);
        st_sw128_32(sP, row, c, pk);
      }
    }
    fence_async_shared();  // P (generic-proxy writes) visible to the tensor core
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < 2 * NKB; ++j)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem_base + C::O_COL, sw128_kmajor_desc(smem_u32(sP + j * 128 * 128) + kk * 32),
                   sw128_kmajor_desc(smem_u32(sVt + j * 128 * 128) + kk * 32), C::IDESC_O,
                   (j | kk) != 0 ? 1u : 0u);
      tc_commit(odone);
    }
    if (!mbar_wait(odone, phase, abort_flag, kTagAttn, 3)) { ok = false; break; }
    tc_fence_after();

    // ---- O / sum -> bf16 into the staging tile (swizzled), then one TMA store
    // of the 128 x 128 tile at (row m0, column h*128); rows past sq are clipped
    const float inv = 1.0f / sum;
    {
      uint32_t r[4][32];
#pragma unroll
      for (int b = 0; b < 4; ++b) tmem_ld_32x32b_x32(t_row + C::O_COL + 32 * b, r[b]);
      tmem_ld_wait();
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(r[b][2 * i]) * inv,
                                                         __uint_as_float(r[b][2 * i + 1]) * inv);
          pk[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
        st_sw128_32(sO, row, 32 * b, pk);
      }
    }
    fence_async_shared();  // the staging tile (generic-proxy writes) visible to the TMA store
    // S / O columns and the Q, K, V^T tiles are free for the next item
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
      for (int b = 0; b < 2; ++b) tma_store_2d(&tmO, sO + b * 128 * 128, h * 128 + b * 64, m0);
      bulk_commit_group();
    }
  }
  if (threadIdx.x == 0) bulk_wait_all();  // the stores have landed before the CTA exits
  if (!ok && threadIdx.x == 0) {
    // drain: the last item's copies and any MMA still in flight
    if (issued > 0) mbar_wait_drain(full, phase);
    tc_commit(drain);
    mbar_wait_drain(drain, 0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace qib
