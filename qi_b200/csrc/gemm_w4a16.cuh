// W4A16 GEMM: Y[M,N] = X[M,K] (bf16) . dequant(W)[N,K]^T + bias.  sm_100a
// has no int4 MMA, so the packed INT4 weight is dequantized to bf16 and fed
// to tcgen05 kind::f16 tensor cores as the A operand FROM TENSOR MEMORY:
//   D^T[n, m] = W[n, :] . X[m, :]   (M_mma = 128 weight rows = TMEM lanes,
//                                    N_mma = BT tokens from shared memory)
// Dequant warps write the bf16 weight tile with tcgen05.st straight into
// TMEM (row n in lane n, two K elements per 32-bit column), so no shared
// memory round trip and no generic->async proxy fence is needed; the
// packed words are read with plain global loads issued several stages ahead.
//
// Packed weight layout (qi_b200/quantization/quantize.py):
//   wq      int32 [N, K/8]         element k = 8w + j in bits 4j..4j+3 of word w
//   scales  fp16  [N, G]           G = ceil(K / group_size)
//   zeros   int32 [N, ceil(G/8)]   uint4 zero point of group g in word g/8, nibble g%8
// Dequantization is the reference's (src/qi/quantization/quantize.py:110-117):
//   w_bf16 = bf16_rn( fp32(q - z) * fp32(s) ), computed exactly in one FFMA:
//   f = 1 + q/16 (built from the nibble's bits), w = fma(f, 16 s, -(16 + z) s);
//   both products are exact in fp32, so the only rounding is the final bf16.
//
// CTA (768 threads): warp 0 TMA (activation tiles, 128-byte swizzled), warp 1
// TMEM allocation + MMA issue, warps 4-7 epilogue, warps 8-23 dequant (warp
// w owns TMEM lanes 32*(w%4).. and K quarter (w-8)/4 of every 64-element
// stage, i.e. 16 consecutive K elements = 2 packed words per thread).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "gemm_tc.cuh"
#include "sm100_ptx.cuh"

namespace qib {

struct W4Params {
  const int32_t* wq;      // [N, kw] packed int4
  const int32_t* zeros;   // [N, zw] packed uint4
  const __half* scales;   // [N, G]
  int kw;                 // int32 words per weight row (K / 8)
  int G;                  // groups per row
  int zw;                 // int32 words of zeros per row
  int group;              // group size in elements (multiple of 32)
  int group_shift;        // log2(group) when group is a power of two, else -1
};

namespace w4 {
constexpr int BN = 128;       // weight rows per tile (MMA M, TMEM lanes)
constexpr int BK = 64;        // K elements per stage
constexpr int A_COLS = 32;    // TMEM columns of one A stage (64 bf16 per lane)
constexpr int kPrefetch = 4;  // stages of packed weights in flight per dequant thread
constexpr int kEpiWarp0 = 4, kEpiWarpsW4 = 4;
constexpr int kDeqWarp0 = 8, kDeqWarps = 16;
constexpr int kKSplit = kDeqWarps / 4;            // dequant warps per TMEM lane quarter
constexpr int kElems = BK / kKSplit;              // K elements per dequant thread per stage (16)
constexpr int kWords = kElems / 8;                // packed int32 words per thread per stage (2)
constexpr int kThreads = (kDeqWarp0 + kDeqWarps) * 32;
constexpr int kEpiThr = kEpiWarpsW4 * 32;
constexpr int kDeqThr = kDeqWarps * 32;
constexpr int TMEM_COLS = 512;
}  // namespace w4

template <int BT>
struct W4Cfg {
  static constexpr int STAGES = BT >= 256 ? 6 : 8;
  static constexpr int X_BYTES = BT * 128;  // BT token rows x 64 bf16, 128-byte swizzled
  static constexpr int RING_BYTES = STAGES * X_BYTES;
  static constexpr int PART_BYTES = BT * w4::BN * 4;  // split-K partial tile (skinny kernel)
  static constexpr int BUF_BYTES = RING_BYTES > PART_BYTES ? RING_BYTES : PART_BYTES;
  static constexpr int SMEM_BYTES = BUF_BYTES + 256 + 1024;
  static constexpr int ACC_COL = STAGES * w4::A_COLS;  // accumulator after the A ring
  static constexpr uint32_t IDESC = make_idesc(kDF32, kFmtBF16, kFmtBF16, 128, BT);
  static_assert(ACC_COL + BT <= w4::TMEM_COLS, "TMEM");
  static_assert(SMEM_BYTES <= 232448, "smem");
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "BT");
};

// 8 nibbles of one word -> 8 bf16 (4 packed pairs, even element in the low
// half), exact reference dequant.
__device__ __forceinline__ void dequant8(uint32_t w, float s16x, float c, uint32_t* out4) {
  float f[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t nib = (w >> (4 * j)) & 0xFu;
    f[j] = fmaf(__uint_as_float(0x3F800000u | (nib << 19)), s16x, c);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) out4[j] = pack_bf16x2(f[2 * j], f[2 * j + 1]);
}

// Scale / zero of one (row, group), fetched one group ahead.
struct GroupScale {
  float s16x = 0.f, c = 0.f;  // current group: 16*s and -(16+z)*s
  float s_next = 0.f;
  uint32_t z_next = 0;
  int cur = -1, next = -1;

  __device__ __forceinline__ void fetch(const W4Params& q, long long n, int g, float& s, uint32_t& z) {
    s = __half2float(q.scales[n * q.G + g]);
    const uint32_t zw = static_cast<uint32_t>(__ldg(q.zeros + n * q.zw + (g >> 3)));
    z = (zw >> (4 * (g & 7))) & 0xFu;
  }
  __device__ __forceinline__ void set(float s, uint32_t z) {
    s16x = s * 16.0f;
    c = -(16.0f + static_cast<float>(z)) * s;
  }
  __device__ __forceinline__ void advance(const W4Params& q, long long n, int g) {
    if (g == cur) return;
    if (g == next) {
      set(s_next, z_next);
    } else {
      float s;
      uint32_t z;
      fetch(q, n, g, s, z);
      set(s, z);
    }
    cur = g;
    next = g + 1;
    if (next < q.G) fetch(q, n, next, s_next, z_next);
  }
};

// Warp-uniform bounded wait (every lane waits; all bail out if any fails),
// so the .sync.aligned tcgen05 instructions that follow see a converged warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int tag, unsigned int site) {
  const bool ok = mbar_wait(bar, parity, abort_flag, tag, site);
  return __all_sync(0xffffffffu, ok);
}

// Dequant role: stream K blocks [kb0, kb0 + nkb) of weight row n (K slice
// h of every stage: elements [h*kElems, (h+1)*kElems)) into the TMEM A ring.
// free_bar[s]: the MMA has finished reading A stage s; ready_bar[s]: this
// thread's part of stage s is in TMEM.  The packed words arrive kPrefetch
// stages ahead.  Returns false when aborting.
__device__ __forceinline__ bool dequant_rows_tmem(const W4Params& q, int n, bool row_ok, int h, int kb0, int nkb,
                                                  uint32_t tmem_a, int stages, uint64_t* free_bar,
                                                  uint64_t* ready_bar, int& stage, uint32_t& phase,
                                                  volatile int* abort_flag, unsigned int tag) {
  static_assert(w4::kWords == 2, "one 8-byte load per thread per stage");
  if (nkb <= 0) return true;
  const int32_t* src = q.wq + static_cast<long long>(n) * q.kw + w4::kWords * h;
  // this thread's word pair of K block kb exists (K % 32 == 0: a block's
  // 8 words are whole or absent past K; the activations there are zero-fill)
  auto load = [&](int kb) -> uint2 {
    return (row_ok && kb * 8 + w4::kWords * h < q.kw) ? __ldg(reinterpret_cast<const uint2*>(src + kb * 8))
                                                        : make_uint2(0, 0);
  };
  auto group_of = [&](int kb) -> int {
    const int k = kb * w4::BK + w4::kElems * h;
    return q.group_shift >= 0 ? (k >> q.group_shift) : k / q.group;
  };
  GroupScale gs;
  uint2 pf[w4::kPrefetch];
#pragma unroll
  for (int j = 0; j < w4::kPrefetch; ++j) pf[j] = (j < nkb) ? load(kb0 + j) : make_uint2(0, 0);
  for (int i0 = 0; i0 < nkb; i0 += w4::kPrefetch) {
#pragma unroll
    for (int j = 0; j < w4::kPrefetch; ++j) {
      const int i = i0 + j;
      if (i < nkb) {  // warp-uniform
        const uint2 raw = pf[j];
        if (i + w4::kPrefetch < nkb) pf[j] = load(kb0 + i + w4::kPrefetch);
        const int g = group_of(kb0 + i);
        if (row_ok && g < q.G) gs.advance(q, n, g);
        uint32_t v[8];
        dequant8(raw.x, gs.s16x, gs.c, v);
        dequant8(raw.y, gs.s16x, gs.c, v + 4);
        if (!row_ok) {
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] = 0u;
        }
        if (!warp_wait(&free_bar[stage], phase ^ 1u, abort_flag, tag, 7)) return false;
        tc_fence_after();
        tmem_st_32x32b_x8(tmem_a + stage * w4::A_COLS + (w4::kElems / 2) * h, v);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive_relaxed(&ready_bar[stage]);  // must not wait for the prefetch loads in flight
        if (++stage == stages) { stage = 0; phase ^= 1u; }
      }
    }
  }
  return true;
}

// One K block of MMAs: A stage from TMEM, activation stage from shared memory.
template <int BT>
__device__ __forceinline__ void mma_stage_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t x_smem, bool first) {
#pragma unroll
  for (int kk = 0; kk < w4::BK / 16; ++kk)
    mma_bf16_ts(d_tmem, a_tmem + kk * 8, sw128_kmajor_desc(x_smem + kk * 32), W4Cfg<BT>::IDESC,
                (!first || kk != 0) ? 1u : 0u);
}

// ---------------------------------------------------------------------------
// Large M: persistent tiles of 128 weight rows x 256 tokens.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(w4::kThreads, 1)
k_gemm_w4a16(const __grid_constant__ CUtensorMap tmX, const EpiParams p, const W4Params q) {
  constexpr int BT = 256;
  using C = W4Cfg<BT>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;  // [STAGES][256 token rows x 128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BUF_BYTES);
  uint64_t* aready = full + STAGES;
  uint64_t* empty = aready + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr unsigned int kTag = 0x200u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], w4::kDeqThr);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, w4::kEpiThr);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_map(&tmX);
  if (warp == 1) {
    tmem_alloc(tmem_slot, w4::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = (p.M + BT - 1) / BT;
  const int n_tiles = (p.N + w4::BN - 1) / w4::BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + w4::BK - 1) / w4::BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % m_tiles;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kTag, 1)) { ok = false; break; }
          mbar_expect_tx(&full[stage], C::X_BYTES);
          tma_load_2d(sX + stage * C::X_BYTES, &tmX, &full[stage], kb * w4::BK, mb * BT);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t acc = tmem_base + C::ACC_COL;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        if (!mbar_wait(tempty, (local & 1) ^ 1u, abort_flag, kTag, 2)) { ok = false; break; }
        tc_fence_after();
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kTag, 3)) { ok = false; break; }
          if (!mbar_wait(&aready[stage], phase, abort_flag, kTag, 6)) { ok = false; break; }
          tc_fence_after();
          mma_stage_ts<BT>(acc, tmem_base + stage * w4::A_COLS, smem_u32(sX + stage * C::X_BYTES), kb == 0);
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit(tfull);
      }
      if (!ok) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (warp >= w4::kDeqWarp0) {
    const int wq = warp & 3, h = (warp - w4::kDeqWarp0) >> 2;
    const uint32_t tmem_a = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int n = (tile / m_tiles) * w4::BN + wq * 32 + lane;
      if (!dequant_rows_tmem(q, n, n < p.N, h, 0, k_blocks, tmem_a, STAGES, empty, aready, stage, phase,
                             abort_flag, kTag))
        break;
    }
  } else if (warp >= w4::kEpiWarp0) {
    const int wq = warp & 3;
    const uint32_t tacc = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + C::ACC_COL;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int mb = tile % m_tiles, nb = tile / m_tiles;
      const int n = nb * w4::BN + wq * 32 + lane;
      const float bias = (p.bias != nullptr && n < p.N) ? __bfloat162float(p.bias[n]) : 0.0f;
      if (!warp_wait(tfull, local & 1, abort_flag, kTag, 4)) break;
      tc_fence_after();
      __nv_bfloat16* dcol = static_cast<__nv_bfloat16*>(p.D) + n;
#pragma unroll 1
      for (int m0 = 0; m0 < BT; m0 += 32) {
        const int mbase = mb * BT + m0;
        if (mbase >= p.M) break;  // warp-uniform
        uint32_t rr[32];
        tmem_ld_32x32b_x32(tacc + m0, rr);
        tmem_ld_wait();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (mbase + j < p.M)
              dcol[static_cast<long long>(mbase + j) * p.ldd] = __float2bfloat16_rn(__fadd_rn(__uint_as_float(rr[j]), bias));
          }
        }
      }
      tc_fence_before();
      mbar_arrive_relaxed(tempty);  // accumulator read (wait::ld); output stores need no ordering
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, w4::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Skinny W4A16 (M <= 256, BT = M rounded up to 16/32/64/128/256): one token
// tile; K split over the CTAs of a thread-block cluster (up to 8).  Each CTA
// writes its fp32 partial tile to its own shared memory and the cluster sums
// the partials through distributed shared memory in rank order (results do
// not depend on timing), adds bias and stores bf16.
// ---------------------------------------------------------------------------
template <int BT>
__global__ void __launch_bounds__(w4::kThreads, 1)
k_gemm_w4a16_skinny(const __grid_constant__ CUtensorMap tmX, const EpiParams p, const W4Params q, int kb_per_cta) {
  using C = W4Cfg<BT>;
  constexpr int STAGES = C::STAGES;
  constexpr int BN = w4::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;                            // [STAGES][BT token rows x 128 B]
  float* part = reinterpret_cast<float*>(smem);  // [BT][BN] after the main loop
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BUF_BYTES);
  uint64_t* aready = full + STAGES;
  uint64_t* empty = aready + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr unsigned int kTag = 0x300u;
  const int ks = static_cast<int>(cluster_ctarank());
  const int nks = static_cast<int>(cluster_nctarank());
  const int nb = blockIdx.x / nks;
  const int k_blocks_total = (p.K + w4::BK - 1) / w4::BK;
  const int kb0 = ks * kb_per_cta;
  const int kb1 = min(kb0 + kb_per_cta, k_blocks_total);
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], w4::kDeqThr);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_map(&tmX);
  if (warp == 1) {
    tmem_alloc(tmem_slot, w4::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool have_acc = false;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kTag, 1)) { ok = false; break; }
        mbar_expect_tx(&full[stage], C::X_BYTES);
        tma_load_2d(sX + stage * C::X_BYTES, &tmX, &full[stage], (kb0 + i) * w4::BK, 0);
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&full[stage], phase, abort_flag, kTag, 3)) { ok = false; break; }
        if (!mbar_wait(&aready[stage], phase, abort_flag, kTag, 6)) { ok = false; break; }
        tc_fence_after();
        mma_stage_ts<BT>(tmem_base + C::ACC_COL, tmem_base + stage * w4::A_COLS, smem_u32(sX + stage * C::X_BYTES),
                         i == 0);
        tc_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (ok && nkb > 0) tc_commit(tfull);
      if (!ok) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (warp >= w4::kDeqWarp0) {
    const int wq = warp & 3, h = (warp - w4::kDeqWarp0) >> 2;
    const int n = nb * BN + wq * 32 + lane;
    int stage = 0;
    uint32_t phase = 0;
    dequant_rows_tmem(q, n, n < p.N, h, kb0, nkb, tmem_base + (static_cast<uint32_t>(wq * 32) << 16), STAGES,
                      empty, aready, stage, phase, abort_flag, kTag);
  } else if (warp >= w4::kEpiWarp0) {
    // wait for the accumulator (bounded) before the ring is reused for partials
    if (nkb > 0) have_acc = warp_wait(tfull, 0, abort_flag, kTag, 4);
    if (have_acc) tc_fence_after();
  }
  // The smem ring becomes the partial buffer only after every role is done
  // with it (all MMAs completed: tfull observed by the epilogue warps).
  __syncthreads();
  if (warp >= w4::kEpiWarp0 && warp < w4::kEpiWarp0 + w4::kEpiWarpsW4) {
    const int wq = warp & 3;
    const int nl = wq * 32 + lane;  // weight row within the tile = TMEM lane
    const bool ok_acc = (nkb > 0) && !(*abort_flag);
#pragma unroll 1
    for (int m0 = 0; m0 < BT; m0 += 16) {
      uint32_t rr[16];
      if (ok_acc) {
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + C::ACC_COL + m0, rr);
        tmem_ld_wait();
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(m0 + j) * BN + nl] = ok_acc ? __uint_as_float(rr[j]) : 0.0f;
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every CTA's partial is complete and visible cluster-wide
  tc_fence_after();
  {
    const int total = BT * BN;
    const int per = (total + nks - 1) / nks;
    const int e0 = ks * per;
    const int e1 = min(e0 + per, total);
    const uint32_t part_addr = smem_u32(part);
    for (int e = e0 + static_cast<int>(threadIdx.x); e < e1; e += w4::kThreads) {
      // issue every peer's load first, then add in rank order (fixed order)
      float pv[8];
#pragma unroll
      for (int rk = 0; rk < 8; ++rk)
        pv[rk] = (rk < nks) ? ld_shared_cluster_f32(map_shared_rank(part_addr + 4u * e, rk)) : 0.0f;
      float v = pv[0];
#pragma unroll
      for (int rk = 1; rk < 8; ++rk)
        if (rk < nks) v = __fadd_rn(v, pv[rk]);
      const int m = e / BN, nl = e % BN;
      const int n = nb * BN + nl;
      if (m < p.M && n < p.N) {
        if (p.bias != nullptr) v = __fadd_rn(v, __bfloat162float(p.bias[n]));
        static_cast<__nv_bfloat16*>(p.D)[static_cast<long long>(m) * p.ldd + n] = __float2bfloat16_rn(v);
      }
    }
  }
  cluster_sync_all();  // peers' shared memory stays alive until every read is done
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, w4::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Small M (<= 8 tokens): weight-bandwidth-bound streaming kernel.
//
// At small M the GEMM reads 0.5 byte of packed weight per 2*M flops, so HBM
// bounds it.  There, the 128-row TMEM staging of the tile kernel above adds
// a serial dequant -> tcgen05.st -> MMA chain per 64-K stage.  This kernel
// instead streams the packed words with 16-byte loads issued several chunks
// ahead, dequantizes them in registers straight into the B fragments of a
// warp-level bf16 MMA (m16n8k16, the tokens as the 16-row A operand, read
// from shared memory with ldmatrix), and never stages weights in shared
// memory.
//
// CTA: 8 warps over 16 weight rows (two 8-column MMA tiles); warp w owns K
// range [w*K/8, (w+1)*K/8) in 128-element chunks.  Lane (g = lane/4,
// t = lane%4) loads words 4t..4t+3 of each chunk for rows n0+g and n0+8+g; a
// k16 step needs words 2s, 2s+1, fetched by shuffle from lane 4g + s/2.  The
// eight warps' fp32 partials are summed in shared memory in warp order, then
// bias is added and bf16 is stored.  Dequantization is the exact
// bf16((q - z) * s) of the tile kernel.
// ---------------------------------------------------------------------------

namespace w4s {
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 16;          // weight rows (output columns) per CTA
constexpr int kChunk = 128;        // K elements per chunk (16 words per row)
constexpr int kDepth = 4;          // chunks in flight per lane
constexpr int kMaxM = 8;
}  // namespace w4s

// Shared memory of k_gemm_w4a16_small: the M token rows plus one zero row
// (rows >= M of the 16-row A fragment read it), each padded by 16 bytes.
inline int w4s_smem_bytes(int M, int K) { return (M + 1) * (K + 8) * 2; }

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&a)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}

// two nibbles (elements 2t, 2t+1 of word w) -> packed bf16x2 of (q - z) * s
__device__ __forceinline__ uint32_t dequant_pair(uint32_t w, int t, float s16x, float c) {
  const uint32_t n0 = (w >> (8 * t)) & 0xFu, n1 = (w >> (8 * t + 4)) & 0xFu;
  const float f0 = fmaf(__uint_as_float(0x3F800000u | (n0 << 19)), s16x, c);
  const float f1 = fmaf(__uint_as_float(0x3F800000u | (n1 << 19)), s16x, c);
  return pack_bf16x2(f0, f1);
}

__global__ void __launch_bounds__(w4s::kThreads)
k_gemm_w4a16_small(const __nv_bfloat16* __restrict__ X, EpiParams p, W4Params q) {
  __shared__ float red[w4s::kWarps][32][8];
  extern __shared__ __align__(16) uint8_t xs_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ldx = p.K + 8;  // padded row stride of the staged tokens (elements)
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xs_raw);
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * w4s::kRows;
  const int kr = p.K / w4s::kWarps;                 // K range of this warp
  const int k_begin = warp * kr;
  const int nchunks = kr / w4s::kChunk;
  const long long row0 = n0 + g, row1 = n0 + 8 + g;
  const bool ok0 = row0 < p.N, ok1 = row1 < p.N;
  const uint4* w0p = reinterpret_cast<const uint4*>(q.wq + row0 * q.kw + k_begin / 8) + t;
  const uint4* w1p = reinterpret_cast<const uint4*>(q.wq + row1 * q.kw + k_begin / 8) + t;

  uint4 buf0[w4s::kDepth], buf1[w4s::kDepth];
#pragma unroll
  for (int i = 0; i < w4s::kDepth; ++i) {
    if (i < nchunks) {
      buf0[i] = ok0 ? __ldg(w0p + i * 4) : make_uint4(0, 0, 0, 0);
      buf1[i] = ok1 ? __ldg(w1p + i * 4) : make_uint4(0, 0, 0, 0);
    }
  }
  // stage the M token rows (and a zero row) in shared memory, 16-byte moves,
  // while this thread's first weight chunks are in flight
  {
    const int vpr = p.K / 8;  // uint4 per row
    for (int i = threadIdx.x; i < (p.M + 1) * vpr; i += w4s::kThreads) {
      const int r = i / vpr, c = i - r * vpr;
      const uint4 v = r < p.M ? __ldg(reinterpret_cast<const uint4*>(X + static_cast<long long>(r) * p.K) + c)
                              : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(xs + r * ldx + c * 8) = v;
    }
  }
  __syncthreads();
  // ldmatrix row address of this lane: matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15)
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8;
  const uint32_t a_base = smem_u32(xs + (a_row < p.M ? a_row : p.M) * ldx + (lane >> 4) * 8);

  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  int cur_group = -1;
  float s16x0 = 0.f, c0 = 0.f, s16x1 = 0.f, c1 = 0.f;
  for (int cb = 0; cb < nchunks; cb += w4s::kDepth) {
#pragma unroll
  for (int slot = 0; slot < w4s::kDepth; ++slot) {  // register slots stay compile-time
    const int ci = cb + slot;
    if (ci >= nchunks) break;
    const uint4 u0 = buf0[slot], u1 = buf1[slot];
    if (ci + w4s::kDepth < nchunks) {
      buf0[slot] = ok0 ? __ldg(w0p + (ci + w4s::kDepth) * 4) : make_uint4(0, 0, 0, 0);
      buf1[slot] = ok1 ? __ldg(w1p + (ci + w4s::kDepth) * 4) : make_uint4(0, 0, 0, 0);
    }
    const int kc = k_begin + ci * w4s::kChunk;
#pragma unroll
    for (int st = 0; st < w4s::kChunk / 16; ++st) {
      const int k0 = kc + st * 16;
      const int grp = q.group_shift >= 0 ? (k0 >> q.group_shift) : (k0 / q.group);
      if (grp != cur_group) {
        cur_group = grp;
        float sa = 0.f, sb = 0.f;
        uint32_t za = 0, zb = 0;
        if (ok0) {
          sa = __half2float(q.scales[row0 * q.G + grp]);
          za = (static_cast<uint32_t>(__ldg(q.zeros + row0 * q.zw + (grp >> 3))) >> (4 * (grp & 7))) & 0xFu;
        }
        if (ok1) {
          sb = __half2float(q.scales[row1 * q.G + grp]);
          zb = (static_cast<uint32_t>(__ldg(q.zeros + row1 * q.zw + (grp >> 3))) >> (4 * (grp & 7))) & 0xFu;
        }
        s16x0 = sa * 16.0f;
        c0 = -(16.0f + static_cast<float>(za)) * sa;
        s16x1 = sb * 16.0f;
        c1 = -(16.0f + static_cast<float>(zb)) * sb;
      }
      // words 2st, 2st+1 of this chunk live in lane 4g + st/2, at index (2st)%4
      const int src = (lane & ~3) | (st >> 1);
      const uint32_t wa0 = __shfl_sync(0xffffffffu, (st & 1) ? u0.z : u0.x, src);
      const uint32_t wa1 = __shfl_sync(0xffffffffu, (st & 1) ? u0.w : u0.y, src);
      const uint32_t wb0 = __shfl_sync(0xffffffffu, (st & 1) ? u1.z : u1.x, src);
      const uint32_t wb1 = __shfl_sync(0xffffffffu, (st & 1) ? u1.w : u1.y, src);
      uint32_t a[4];
      ldmatrix_x4(a, a_base + static_cast<uint32_t>(k0) * 2u);
      mma_bf16_16816(d0, a, dequant_pair(wa0, t, s16x0, c0), dequant_pair(wa1, t, s16x0, c0));
      mma_bf16_16816(d1, a, dequant_pair(wb0, t, s16x1, c1), dequant_pair(wb1, t, s16x1, c1));
    }
  }
  }
  // K-split reduction in warp order, then the epilogue (bias, bf16)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    red[warp][lane][i] = d0[i];
    red[warp][lane][4 + i] = d1[i];
  }
  __syncthreads();
  if (warp != 0) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = red[0][lane][i];
    for (int w = 1; w < w4s::kWarps; ++w) v += red[w][lane][i];
    acc[i] = v;
  }
  // D fragment: acc[0..1] token g, cols 2t,2t+1 of tile 0; acc[2..3] token g+8; acc[4..7] tile 1
#pragma unroll
  for (int tile = 0; tile < 2; ++tile) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = g + 8 * h;
      const int n = n0 + 8 * tile + 2 * t;
      if (m >= p.M || n >= p.N) continue;
      float y0 = acc[4 * tile + 2 * h], y1 = acc[4 * tile + 2 * h + 1];
      if (p.bias != nullptr) {
        y0 = __fadd_rn(y0, __bfloat162float(p.bias[n]));
        y1 = __fadd_rn(y1, __bfloat162float(p.bias[n + 1]));
      }
      *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(m) * p.ldd + n) =
          pack_bf16x2(y0, y1);
    }
  }
}

}  // namespace qib
