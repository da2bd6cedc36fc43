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
// half), exact reference dequant bf16(fp32((q - z) s)).  Each nibble is
// placed by a byte permute into the mantissa of 0.5 (0x3F00_0000 | q << 16 =
// 0.5 + q / 256); then fma(0.5 + q / 256, 256 s, -(128 + z) s) equals
// (q - z) s in exact arithmetic (256 s and (128 + z) s are exact in fp32), so
// its single rounding is fp32((q - z) s).  s256 = 256 s, c = -(128 + z) s.
__device__ __forceinline__ void dequant8(uint32_t w, float s256, float c, uint32_t* out4) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;  // byte b: nibble 2b / 2b + 1
  const float2 s2 = make_float2(s256, s256), c2 = make_float2(c, c);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t sel = 0x7044u | (static_cast<uint32_t>(b) << 8);  // [0, 0, byte b, 0x3F]
    const float2 v = make_float2(__uint_as_float(__byte_perm(lo, 0x3F000000u, sel)),
                                 __uint_as_float(__byte_perm(hi, 0x3F000000u, sel)));
    const float2 f = __ffma2_rn(v, s2, c2);
    out4[b] = pack_bf16x2(f.x, f.y);
  }
}

// Scale / zero of one (row, group), fetched one group ahead.
struct GroupScale {
  float s256 = 0.f, c = 0.f;  // current group: 256 s and -(128 + z) s (dequant8)
  float s_next = 0.f;
  uint32_t z_next = 0;
  int cur = -1, next = -1;

  __device__ __forceinline__ void fetch(const W4Params& q, long long n, int g, float& s, uint32_t& z) {
    s = __half2float(q.scales[n * q.G + g]);
    const uint32_t zw = static_cast<uint32_t>(__ldg(q.zeros + n * q.zw + (g >> 3)));
    z = (zw >> (4 * (g & 7))) & 0xFu;
  }
  __device__ __forceinline__ void set(float s, uint32_t z) {
    s256 = s * 256.0f;
    c = -(128.0f + static_cast<float>(z)) * s;
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
        dequant8(raw.x, gs.s256, gs.c, v);
        dequant8(raw.y, gs.s256, gs.c, v + 4);
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


// Weight-only quantized weights in the reference's own layout
// (quantize.py:32-78: one int8 code per value, fp32 scales [N, G], int16
// zero points [N, G] or none) -> bf16 [N, K], computed as the reference's
// dequantize_weight (quantize.py:81-119) does: w = fp32(q - z) * s rounded
// to fp32, then to bf16.  Serves weight-only INT8 (W8A16) and INT4 stored
// one value per byte.  16 elements per thread (one 16-byte load); K % 16 == 0.
__global__ void __launch_bounds__(256)
k_wo_dequant(const int8_t* __restrict__ q, const float* __restrict__ scales, const int16_t* __restrict__ zeros,
             int G, int group, __nv_bfloat16* __restrict__ out, int N, int K) {
  griddep_wait();
  griddep_launch_dependents();
  const int per_row = K >> 4;
  const long long total = static_cast<long long>(N) * per_row;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += 256ll * gridDim.x) {
    const int n = static_cast<int>(i / per_row);
    const int k0 = static_cast<int>(i - static_cast<long long>(n) * per_row) << 4;
    const int4 raw = __ldg(reinterpret_cast<const int4*>(q + static_cast<long long>(n) * K + k0));
    const int8_t* c = reinterpret_cast<const int8_t*>(&raw);
    uint32_t packed[8];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      float w2[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int g = (k0 + e + t) / group;
        const float sc = __ldg(scales + static_cast<long long>(n) * G + g);
        const float zc = zeros != nullptr ? static_cast<float>(__ldg(zeros + static_cast<long long>(n) * G + g)) : 0.f;
        w2[t] = __fmul_rn(__fsub_rn(static_cast<float>(c[e + t]), zc), sc);
      }
      packed[e >> 1] = pack_bf16x2(w2[0], w2[1]);
    }
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<long long>(n) * K + k0);
    o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
}

// Dequantize packed INT4 weights to bf16 [N, K] (the reference's
// bf16((q - z) s), exact), four packed words (32 elements) per thread.
// HBM-bound: K/2 + 2K bytes per row (+ scales).  group % 32 == 0, K % 32 == 0.
__global__ void __launch_bounds__(256)
k_w4a16_dequant(W4Params q, __nv_bfloat16* __restrict__ out, int N, int K) {
  griddep_wait();
  griddep_launch_dependents();
  const int qpr = q.kw / 4;  // word quads per row
  const int quads = N * qpr;  // the host keeps N * K / 32 < 2^31
  for (int i = blockIdx.x * 256 + threadIdx.x; i < quads; i += 256 * gridDim.x) {
    const int n = i / qpr;
    const int w0 = (i - n * qpr) * 4;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(q.wq + static_cast<long long>(n) * q.kw + w0));
    const int k0 = w0 * 8;
    const int grp = q.group_shift >= 0 ? (k0 >> q.group_shift) : (k0 / q.group);  // 32 elements: one group
    const float sc = __half2float(__ldg(q.scales + static_cast<long long>(n) * q.G + grp));
    const uint32_t z = (static_cast<uint32_t>(__ldg(q.zeros + static_cast<long long>(n) * q.zw + (grp >> 3))) >>
                        (4 * (grp & 7))) & 0xFu;
    const float s256 = sc * 256.0f, c = -(128.0f + static_cast<float>(z)) * sc;
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(n) * K + k0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t o[4];
      dequant8(wd[j], s256, c, o);
      dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

namespace w4s {
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowPad = 16;  // bytes after each staged weight row (spreads the rows over banks)
constexpr int kMaxM = 16;    // one m16 MMA row block
}  // namespace w4s

// Shared-memory layout of k_gemm_w4a16_small<NT, KS> (byte offsets, all
// 16-aligned): 2 mbarriers (weights, tokens) | RB = 8 NT weight rows of this
// CTA's K range (KC/2 bytes + pad) | RB x G fp16 scales | RB x zw zero words |
// M token rows of the K range (KC bf16 + pad, natural order) | warp partials |
// CTA partials (read by the cluster's rank 0).
struct W4sLayout {
  int w_off, w_stride, s_off, z_off, x_off, x_stride, red_off, part_off, total;
};
__host__ __device__ inline W4sLayout w4s_layout(int NT, int KS, int M, int K, int G, int zw, int group) {
  const int RB = 8 * NT, KC = K / KS;
  (void)group;
  W4sLayout L;
  L.w_off = 16;
  L.w_stride = KC / 2 + w4s::kRowPad;
  L.s_off = L.w_off + RB * L.w_stride;
  L.z_off = L.s_off + ((RB * G * 2 + 15) & ~15);
  L.x_off = L.z_off + ((RB * zw * 4 + 15) & ~15);
  L.x_stride = KC * 2 + w4s::kRowPad;  // bytes; the pad spreads ldmatrix rows over banks
  L.red_off = L.x_off + M * L.x_stride;
  L.part_off = L.red_off + w4s::kWarps * 32 * 4 * 4;
  L.total = L.part_off + NT * 32 * 4 * 4;
  return L;
}

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

// Elements 2t and 2t+1 of a packed word (byte t) minus the zero point, as
// bf16x2 (q_2t - z, q_2t+1 - z): each nibble goes into the low mantissa bits
// of bf16 128.0 (giving 128 + q exactly), then 128 + z is subtracted (zb =
// bf16x2 of 128 + z); every value is a small integer, so all of it is exact.
__device__ __forceinline__ uint32_t nibble_pair_minus_z(uint32_t w, int t8, uint32_t zb) {
  const uint32_t x = w >> t8;
  const uint32_t v = (x & 0x0000000Fu) | ((x << 12) & 0x000F0000u) | 0x43004300u;
  const __nv_bfloat162 r = __hsub2_rn(*reinterpret_cast<const __nv_bfloat162*>(&v),
                                      *reinterpret_cast<const __nv_bfloat162*>(&zb));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// W4A16 for M <= 16 tokens.  A CTA covers RB = 8 NT weight rows and 1/KS of K
// (KS CTAs of a cluster split K).  Thread 0 brings the CTA's weight row
// slices, scales and zeros into shared memory with bulk copies before waiting
// for the previous kernel (programmatic dependent launch: the weights are
// layer constants), then the token rows of its K range.  The MMAs
// (m16n8k16, bf16, fp32 accumulate) multiply the tokens by (q - z), exact in
// bf16; per quantization group the fp32 result D (two accumulator chains
// added) becomes s D, the group's contribution sum_k x_k (q_k - z) s.  With
// one-hot token rows this is bf16((q - z) s), the reference's dequantized
// weight, bit for bit; in general it skips the reference's bf16 rounding of
// each weight (relative difference ~1e-3).  Warps: n-tile warp % NT, K part
// warp / NT.  Partials are added in K order: warps in the CTA, then the
// cluster's CTAs by rank (distributed shared memory).
template <int NT, int KS>
__global__ void __launch_bounds__(w4s::kThreads)
k_gemm_w4a16_small(const __nv_bfloat16* __restrict__ X, EpiParams p, W4Params q) {
  static_assert(NT == KS, "each warp's K range must hold whole quantization groups: K / 8 per warp");
  constexpr int RB = 8 * NT, KP = w4s::kWarps / NT;
  extern __shared__ __align__(128) uint8_t sm[];
  const W4sLayout L = w4s_layout(NT, KS, p.M, p.K, q.G, q.zw, q.group);
  uint64_t* bar_w = reinterpret_cast<uint64_t*>(sm);
  uint64_t* bar_x = bar_w + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cr = KS > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int n0 = (blockIdx.x / KS) * RB;
  const int rows = min(RB, p.N - n0);
  const int KC = p.K / KS, kc0 = cr * KC;
  if (threadIdx.x == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_x, 1);
    fence_mbar_init();
    mbar_expect_tx(bar_w, static_cast<uint32_t>(rows * (KC / 2 + q.G * 2 + q.zw * 4)));
#pragma unroll 1
    for (int r = 0; r < rows; ++r)
      bulk_load(sm + L.w_off + r * L.w_stride, q.wq + static_cast<long long>(n0 + r) * q.kw + kc0 / 8, KC / 2, bar_w);
    bulk_load(sm + L.s_off, q.scales + static_cast<long long>(n0) * q.G, rows * q.G * 2, bar_w);
    bulk_load(sm + L.z_off, q.zeros + static_cast<long long>(n0) * q.zw, rows * q.zw * 4, bar_w);
  }
  __syncthreads();  // both mbarriers are initialized before any thread waits on them
  // The packed weights, scales and zeros are layer constants: their copies
  // above are issued before waiting for the previous kernel in the stream
  // (programmatic dependent launch), so the fetch overlaps its tail.  X is
  // read and D written only after the wait.
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_expect_tx(bar_x, static_cast<uint32_t>(p.M * KC * 2));
#pragma unroll 1
    for (int r = 0; r < p.M; ++r)
      bulk_load(sm + L.x_off + r * L.x_stride, X + static_cast<long long>(r) * p.K + kc0, KC * 2, bar_x);
  }
  bool ok = mbar_wait_drain(bar_w, 0) && mbar_wait_drain(bar_x, 0);  // bounded; copies of valid memory complete
  if (!ok && threadIdx.x == 0) record_error(kDevWaitTimeout, 0x300u, 1);

  const int g = lane >> 2, t = lane & 3;
  const int nt = warp % NT, kp = warp / NT;
  const int KW = KC / KP;  // this warp's K range (whole groups)
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (ok) {
    const uint8_t* wrow = sm + L.w_off + (nt * 8 + g) * L.w_stride + kp * KW / 2;
    // zero point of this lane's B column (weight row nt*8 + g); scales of its D columns (rows r0, r0 + 1)
    const uint32_t* zgp = reinterpret_cast<const uint32_t*>(sm + L.z_off) + (nt * 8 + g) * q.zw;
    const int r0 = nt * 8 + 2 * t;
    const __half* s0p = reinterpret_cast<const __half*>(sm + L.s_off) + r0 * q.G;
    const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8;
    const uint32_t a_base = smem_u32(sm + L.x_off + (a_row < p.M ? a_row : 0) * L.x_stride) +
                            static_cast<uint32_t>(kp * KW + (lane >> 4) * 8) * 2u;
    const int t8 = 8 * t;
#pragma unroll 1
    for (int gl = 0; gl < KW / q.group; ++gl) {
      const int grp = (kc0 + kp * KW) / q.group + gl;
      const uint32_t z = (zgp[grp >> 3] >> (4 * (grp & 7))) & 0xFu;
      const uint32_t zb = (0x4300u | z) * 0x00010001u;
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      const int kg = gl * q.group;
#pragma unroll 4
      for (int k = kg; k < kg + q.group; k += 32) {
        const uint4 w = *reinterpret_cast<const uint4*>(wrow + k / 2);  // elements k .. k + 31 of row g
        uint32_t a[4];
        ldmatrix_x4(a, a_base + static_cast<uint32_t>(k) * 2u);
        mma_bf16_16816(d0, a, nibble_pair_minus_z(w.x, t8, zb), nibble_pair_minus_z(w.y, t8, zb));
        ldmatrix_x4(a, a_base + static_cast<uint32_t>(k + 16) * 2u);
        mma_bf16_16816(d1, a, nibble_pair_minus_z(w.z, t8, zb), nibble_pair_minus_z(w.w, t8, zb));
      }
      // the group's contribution: s D, columns r0, r0 + 1
      const float sa = __half2float(s0p[grp]), sb = __half2float(s0p[q.G + grp]);
      acc[0] = fmaf(sa, d0[0] + d1[0], acc[0]);
      acc[1] = fmaf(sb, d0[1] + d1[1], acc[1]);
      acc[2] = fmaf(sa, d0[2] + d1[2], acc[2]);
      acc[3] = fmaf(sb, d0[3] + d1[3], acc[3]);
    }
  }
  // warps of one n-tile add their K parts in order
  float* red = reinterpret_cast<float*>(sm + L.red_off);
  float* part = reinterpret_cast<float*>(sm + L.part_off);
#pragma unroll
  for (int i = 0; i < 4; ++i) red[(warp * 32 + lane) * 4 + i] = acc[i];
  __syncthreads();
  if (warp < NT) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = red[(warp * 32 + lane) * 4 + i];
      for (int k = 1; k < KP; ++k) v += red[((k * NT + warp) * 32 + lane) * 4 + i];
      part[(warp * 32 + lane) * 4 + i] = v;
    }
  }
  if constexpr (KS > 1) cluster_sync_all();  // every CTA's partials are in its shared memory
  if (cr == 0 && warp < NT) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = part[(warp * 32 + lane) * 4 + i];
    if constexpr (KS > 1) {
      for (int r = 1; r < KS; ++r) {
        const uint32_t base = map_shared_rank(smem_u32(part + (warp * 32 + lane) * 4), static_cast<uint32_t>(r));
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] += ld_shared_cluster_f32(base + 4 * i);
      }
    }
    // D fragment: v[0..1] token g, weight rows n0 + 8 warp + 2t, +1; v[2..3] token g + 8
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = g + 8 * h;
      const int n = n0 + warp * 8 + 2 * t;
      if (m >= p.M || n >= p.N) continue;
      float y0 = v[2 * h], y1 = v[2 * h + 1];
      if (p.bias != nullptr) {
        y0 = __fadd_rn(y0, __bfloat162float(p.bias[n]));
        y1 = __fadd_rn(y1, __bfloat162float(p.bias[n + 1]));
      }
      *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(m) * p.ldd + n) =
          pack_bf16x2(y0, y1);
    }
  }
  if constexpr (KS > 1) cluster_sync_all();  // rank 0 has read the peers' partials
}

}  // namespace qib
