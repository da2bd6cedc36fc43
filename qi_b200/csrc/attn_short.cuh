// Attention over a short key sequence (at most 128 keys, head dim 128) on the
// tensor cores: O = softmax(Q K^T * scale) V per head, all keys of a head in
// one tile, so the softmax is exact over the row (no running rescale).
//
// In the DiT step this is the cross-attention of the video (and action)
// queries over the 128 context tokens (wan_video_dit.py:122-140); cuDNN's
// SDPA runs an sm80 kernel for that shape.  The video self-attention (3120
// keys), the first-frame recompute and the action queries' attention stay on
// SDPA.
//
// One work item = (head h, 128 query rows):
//   thread 0: TMA loads Q [128 x 128], K [keys x 128] and V^T [128 x keys]
//             (bf16, 128-byte swizzled, out-of-range rows / keys read 0),
//             then S = Q K^T with tcgen05.mma kind::f16 into TMEM (fp32);
//   warps:    each query row (a TMEM lane) is owned by one or two threads: row
//             max, then p = 2^((s - max) * scale * log2 e) rounded to bf16,
//             written to shared memory in the swizzled K-major layout the MMA
//             reads (over a dead operand tile), and the fp32 row sum of the
//             rounded p;
//   thread 0: O = P V (V^T as the K-major B operand) into TMEM;
//   warps:    O / sum -> bf16 into a swizzled staging tile; thread 0 stores it
//             with TMA (asynchronous: it overlaps the next item's work).
// Every wait is bounded; an expired wait records the error, raises the CTA's
// abort flag and the CTA drains its copies / MMAs and exits.
#pragma once

#include <cuda_bf16.h>
#include <cuda.h>
#include <cstdint>

#include "launch_count.cuh"
#include "sm100_ptx.cuh"

namespace qib {

constexpr unsigned int kTagAttn = 0x600u;

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

// ---------------------------------------------------------------------------
// At most 128 keys, double-buffered (the DiT's cross-attention: 3120 queries x
// 24 heads = 600 items over 128 context keys).  One CTA per SM takes a
// contiguous range of items (mostly one head), so K / V^T are loaded once per
// head; Q and K / V^T have two buffers each, and the next item's loads are
// issued right after the current item's S MMA, so they overlap its softmax,
// P V MMA and epilogue.  P and the O staging tile reuse the current item's Q
// buffer.  Shared memory: 2 x 32 KB Q + 2 x (32 + 32) KB K / V^T = 192 KB.
// ---------------------------------------------------------------------------
struct AttnDbCfg {
  static constexpr int TILE = 128 * 128 * 2;  // one 128 x 128 bf16 operand (2 swizzled 64-column blocks)
  static constexpr int THREADS = 256;         // 8 warps: two per TMEM lane quadrant, one per 64-column half
  static constexpr int SMEM_BYTES = 6 * TILE + 128 + 2 * 2 * 128 * 4 + 1024;
  static constexpr int S_COL = 0, O_COL = 128;
  static constexpr int TMEM_COLS = 256;
  static constexpr uint32_t IDESC = make_idesc(kDF32, kFmtBF16, kFmtBF16, 128, 128);
};

__global__ void __launch_bounds__(AttnDbCfg::THREADS, 1)
k_attn_short_db(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmVt, const __grid_constant__ CUtensorMap tmO,
                const AttnParams p) {
  using C = AttnDbCfg;
  extern __shared__ uint8_t attn_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  // buffers: Q b at b * TILE, K b at (2 + b) * TILE, V^T b at (4 + b) * TILE
  auto sQ = [&](int b) { return smem + b * C::TILE; };
  auto sK = [&](int b) { return smem + (2 + b) * C::TILE; };
  auto sVt = [&](int b) { return smem + (4 + b) * C::TILE; };
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + 6 * C::TILE);  // [2]
  uint64_t* kv_full = q_full + 2;                                       // [2]
  uint64_t* sdone = q_full + 4;
  uint64_t* odone = q_full + 5;
  uint64_t* drain = q_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xchg = reinterpret_cast<float*>(smem + 6 * C::TILE + 128);  // [2 halves][2 (max, sum)][128 rows]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, half = warp >> 2;  // TMEM lane quadrant (rows), 64-column half

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&kv_full[i], 1);
    }
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
  const long long items = static_cast<long long>(q_tiles) * p.heads;
  const int i0 = static_cast<int>(items * blockIdx.x / gridDim.x);
  const int i1 = static_cast<int>(items * (blockIdx.x + 1) / gridDim.x);
  const int row = quad * 32 + lane;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(half * 64);

  // loads of item j: Q into buffer qb; K / V^T of its head into buffer kvb when `kv`
  auto load_item = [&](int j, int qb, bool kv, int kvb) {
    const int h = j / q_tiles, m0 = (j - h * q_tiles) * 128;
    mbar_expect_tx(&q_full[qb], C::TILE);
    for (int kb = 0; kb < 2; ++kb) tma_load_2d(sQ(qb) + kb * (C::TILE / 2), &tmQ, &q_full[qb], h * 128 + kb * 64, m0);
    if (kv) {
      mbar_expect_tx(&kv_full[kvb], 2 * C::TILE);
      for (int kb = 0; kb < 2; ++kb) {
        tma_load_2d(sK(kvb) + kb * (C::TILE / 2), &tmK, &kv_full[kvb], h * 128 + kb * 64, 0);
        tma_load_2d(sVt(kvb) + kb * (C::TILE / 2), &tmVt, &kv_full[kvb], kb * 64, h * 128);
      }
    }
  };

  bool ok = true;
  // thread 0: loads issued and not yet consumed (buffer, phase parity), for the drain
  int q_pend = -1, kv_pend = -1;
  uint32_t q_pend_par = 0, kv_pend_par = 0;
  int seg = 0;  // head segments begun (K / V^T buffer = seg & 1)
  if (threadIdx.x == 0 && i0 < i1) {
    load_item(i0, 0, true, 0);
    q_pend = kv_pend = 0;
  }
#pragma unroll 1
  for (int j = i0; j < i1; ++j) {
    const int n = j - i0, qb = n & 1;
    const int h = j / q_tiles, m0 = (j - h * q_tiles) * 128;
    if (j != i0 && h != (j - 1) / q_tiles) ++seg;
    const int kvb = seg & 1;
    if (threadIdx.x == 0) {
      const bool new_head = (j == i0) || h != (j - 1) / q_tiles;
      if (!mbar_wait(&q_full[qb], static_cast<uint32_t>(n >> 1) & 1u, abort_flag, kTagAttn, 11) ||
          (new_head && !mbar_wait(&kv_full[kvb], static_cast<uint32_t>(seg >> 1) & 1u, abort_flag, kTagAttn, 12))) {
        ok = false;
      } else {
        q_pend = -1;
        if (new_head) kv_pend = -1;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem_base + C::S_COL, sw128_kmajor_desc(smem_u32(sQ(qb) + kb * (C::TILE / 2)) + kk * 32),
                     sw128_kmajor_desc(smem_u32(sK(kvb) + kb * (C::TILE / 2)) + kk * 32), C::IDESC,
                     (kb | kk) != 0 ? 1u : 0u);
        tc_commit(sdone);
        if (j + 1 < i1) {
          // the next item's loads: its Q buffer held item j-1's O staging tile
          // (its TMA store must have read it); a new head goes to the other
          // K / V^T buffer, whose last reader (the previous head) is done
          bulk_wait_read_all();
          const bool next_new = (j + 1) / q_tiles != h;
          load_item(j + 1, qb ^ 1, next_new, kvb ^ 1);
          q_pend = qb ^ 1;
          q_pend_par = static_cast<uint32_t>((n + 1) >> 1) & 1u;
          if (next_new) {
            kv_pend = kvb ^ 1;
            kv_pend_par = static_cast<uint32_t>((seg + 1) >> 1) & 1u;
          }
        }
      }
    }
    if (!mbar_wait(sdone, static_cast<uint32_t>(n) & 1u, abort_flag, kTagAttn, 13)) { ok = false; break; }
    tc_fence_after();

    // softmax: this thread has keys half*64 .. +63 of its row; the row max and
    // the row sum are combined with the other half's thread through shared memory
    float sum = 0.f;
    {
      uint32_t r[2][32];
#pragma unroll
      for (int b = 0; b < 2; ++b) tmem_ld_32x32b_x32(t_row + C::S_COL + 32 * b, r[b]);
      tmem_ld_wait();
      float mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (half * 64 + 32 * b + i < p.sk) mx = fmaxf(mx, __uint_as_float(r[b][i]));
      xchg[(half * 2 + 0) * 128 + row] = mx;
      __syncthreads();
      mx = fmaxf(mx, xchg[((half ^ 1) * 2 + 0) * 128 + row]);
      const float off = -mx * p.scale_log2e;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint32_t pk[16];
        sum += attn_p32(r[b], half * 64 + 32 * b, p.sk, p.scale_log2e, off, pk);
        st_sw128_32(sQ(qb), row, half * 64 + 32 * b, pk);  // P over the dead Q tile
      }
      xchg[(half * 2 + 1) * 128 + row] = sum;
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    sum = xchg[1 * 128 + row] + xchg[3 * 128 + row];  // both halves, in a fixed order
    if (threadIdx.x == 0) {
      tc_fence_after();
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem_base + C::O_COL, sw128_kmajor_desc(smem_u32(sQ(qb) + kb * (C::TILE / 2)) + kk * 32),
                   sw128_kmajor_desc(smem_u32(sVt(kvb) + kb * (C::TILE / 2)) + kk * 32), C::IDESC,
                   (kb | kk) != 0 ? 1u : 0u);
      tc_commit(odone);
    }
    if (!mbar_wait(odone, static_cast<uint32_t>(n) & 1u, abort_flag, kTagAttn, 14)) { ok = false; break; }
    tc_fence_after();

    const float inv = 1.0f / sum;
    {
      uint32_t r[2][32];
#pragma unroll
      for (int b = 0; b < 2; ++b) tmem_ld_32x32b_x32(t_row + C::O_COL + 32 * b, r[b]);
      tmem_ld_wait();
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(r[b][2 * i]) * inv,
                                                         __uint_as_float(r[b][2 * i + 1]) * inv);
          pk[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
        st_sw128_32(sQ(qb), row, half * 64 + 32 * b, pk);  // O staging over the dead P tile
      }
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
      for (int b = 0; b < 2; ++b) tma_store_2d(&tmO, sQ(qb) + b * (C::TILE / 2), h * 128 + b * 64, m0);
      bulk_commit_group();
    }
  }
  if (threadIdx.x == 0) {
    bulk_wait_all();  // the stores have landed before the CTA exits
    if (!ok) {
      // drain: loads still in flight, then any MMA
      if (q_pend >= 0) mbar_wait_drain(&q_full[q_pend], q_pend_par);
      if (kv_pend >= 0) mbar_wait_drain(&kv_full[kv_pend], kv_pend_par);
      tc_commit(drain);
      mbar_wait_drain(drain, 0);
    }
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
