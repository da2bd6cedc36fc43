// Persistent, warp-specialized tcgen05 GEMM with a fused dequantization
// epilogue:  D[M,N] = epilogue( A[M,K] . B[N,K]^T ).
//
//   A: activations, K-major (row-major [M,K]);  B: nn.Linear weight, K-major
//   ([N,K] row-major, i.e. the column-major B operand of the GEMM).
//
// Roles (256 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0      TMA producer: 128-byte-swizzled A and B tiles into a ring of
//               STAGES shared-memory stages (cp.async.bulk.tensor, one destination CTA)
//   warp 1      TMEM allocator + single-thread MMA issuer (tcgen05.mma, M=128,
//               N=BN, accumulators in tensor memory, double buffered so the
//               epilogue of tile i overlaps the main loop of tile i+1)
//   warps 4..7  epilogue: tcgen05.ld 32 columns at a time, apply per-token /
//               per-channel scales, bias and optional GELU in fp32, store bf16
//
// Kinds: kind::i8 (int8 x int8 -> s32), kind::f8f6f4 (e4m3 x e4m3 -> f32),
// kind::f16 (bf16 x bf16 -> f32).
//
// INT8 epilogue reproduces the reference EVT (cutlass_int8_rowwise.cu:43-71):
//   y = bf16_rn( fp32( fp32( float(acc) * s_tok[m] ) * s_ch[n] ) + bias[n] ).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace qib {

enum class MmaKind : int { I8 = 0, F8 = 1, BF16 = 2, NVF4 = 3 };

// epilogue flags
constexpr int kEpiGelu = 1;     // GELU(tanh) of the bf16-rounded linear output
constexpr int kEpiRawAcc = 2;   // debug: store raw 32-bit accumulators (int32 / fp32), ld = ldd

// CTA shape: warp 0 TMA, warp 1 MMA + TMEM, warps 2-3 idle, warps 4-11 epilogue
constexpr int kFirstEpiWarp = 4;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kGemmThreads = (kFirstEpiWarp + kEpiWarps) * 32;

struct EpiParams {
  const float* sa;  // per-row (token) scale, or nullptr (= 1)
  int sa_stride;    // 0 = one scale for all rows
  const float* sb;  // per-column (channel) scale, or nullptr (= 1)
  int sb_stride;    // 0 = one scale for all columns
  const __nv_bfloat16* bias;  // [N] or nullptr
  void* D;                    // bf16 [M, ldd] (or 32-bit [M, ldd] with kEpiRawAcc)
  long long ldd;
  int M, N, K;
  int flags;
  // NVFP4 only: block-scale atoms of A and B (see quantize_nvfp4.cuh) and
  // the number of 4-scale atoms per 128-row block (= K / 64)
  const uint8_t* sfa;
  const uint8_t* sfb;
  int sf_ka;
  // CTA-pair kernel: each of the last (tiles % pairs) tiles, the partial last
  // wave, is split along K over tail_split pairs (1 = no split).  Partial
  // accumulators go to tail_ws, the caller's workspace (tail tiles x
  // tail_split x 256 x BN words; tail_ws_bytes is read on the host only);
  // tail_cnt holds 2 x kMaxTailTiles counters that are zero between launches.
  int tail_split = 1;
  uint32_t* tail_ws = nullptr;
  size_t tail_ws_bytes = 0;
  unsigned int* tail_cnt = nullptr;
};
constexpr int kMaxTailTiles = 128;
constexpr int kMaxPeers = 8;

template <MmaKind KIND, int BN_, int STAGES_, bool EPI_TMA_ = false>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr bool NVF4 = (KIND == MmaKind::NVF4);
  static constexpr int ELEM = (KIND == MmaKind::BF16) ? 2 : 1;    // bytes per TMA element (fp4: packed bytes)
  static constexpr int BK = 128 / ELEM;                          // one 128-B swizzle row per operand row
  static constexpr int UMMA_K = (KIND == MmaKind::BF16) ? 16 : 32;  // 32 bytes of K per MMA (64 fp4)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  // NVFP4: per stage (256 K elements) 4 scale atoms for A, 4 x BN/128 for B
  static constexpr int SFA_BYTES = NVF4 ? 4 * 512 : 0;
  static constexpr int SFB_BYTES = NVF4 ? 4 * 512 * (BN / 128) : 0;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr int ACC_COLS = BN;  // fp32/s32 accumulator: one TMEM column per output column
  static constexpr int SF_COLS = NVF4 ? 4 * 4 + 4 * (BN / 32) : 0;  // scale factors in TMEM
  static constexpr int TMEM_NEED = 2 * ACC_COLS + SF_COLS;
  static constexpr int TMEM_COLS = (TMEM_NEED <= 32) ? 32 : (TMEM_NEED <= 64) ? 64 : (TMEM_NEED <= 128) ? 128 : (TMEM_NEED <= 256) ? 256 : 512;
  static constexpr int COLPARAM_BYTES = 2 * BN * (4 + 2);  // double-buffered column scales + bias
  static constexpr int BAR_BYTES = 256;
  // k_gemm_tc's 128- and 192-wide 8-bit / bf16 tiles store their bf16
  // results through one swizzled 32 x 64 (or 32 x 32) shared-memory box per
  // epilogue warp and a TMA store (row-per-lane global stores write 32 rows
  // per warp instruction)
  static constexpr bool TMA_OUT = EPI_TMA_ && !NVF4 && (BN == 128 || BN == 192);
  static constexpr int STAGING_BYTES = TMA_OUT ? 8 * 32 * 64 * 2 : 0;
  static constexpr int SMEM_BYTES =
      STAGES * STAGE_BYTES + STAGING_BYTES + COLPARAM_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static constexpr uint32_t IDESC =
      (KIND == MmaKind::I8)   ? make_idesc(kDS32, kFmtS8, kFmtS8, BM, BN)
      : (KIND == MmaKind::F8) ? make_idesc(kDF32, kFmtE4M3, kFmtE4M3, BM, BN)
      : (KIND == MmaKind::NVF4) ? make_idesc_nvf4(BM, BN)
                              : make_idesc(kDF32, kFmtBF16, kFmtBF16, BM, BN);
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(TMEM_NEED <= 512, "TMEM");
  static_assert(!NVF4 || BN == 128, "NVFP4 tiles are 128 x 128");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// GELU, tanh form: 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))), with the
// hardware tanh approximation (tanh.approx.f32, relative error ~2^-11, below
// the bf16 rounding that follows).
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_tanh_fast(float v) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float inner = k0 * fmaf(k1 * v * v, v, v);
  return 0.5f * v * (1.0f + tanh_hw(inner));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// gelu_tanh_fast on two values with packed fp32x2 arithmetic: the same
// operations in the same order (each rounds the same way), half the
// instructions.
__device__ __forceinline__ float2 gelu_tanh_fast2(float2 v) {
  const float2 k0 = make_float2(0.7978845608028654f, 0.7978845608028654f);
  const float2 k1 = make_float2(0.044715f, 0.044715f);
  const float2 t = __fmul2_rn(__fmul2_rn(k1, v), v);
  const float2 inner = __fmul2_rn(k0, __ffma2_rn(t, v, v));
  const float2 one_th = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(tanh_hw(inner.x), tanh_hw(inner.y)));
  return __fmul2_rn(__fmul2_rn(make_float2(0.5f, 0.5f), v), one_th);
}

// Standalone INT8 epilogue over raw int32 accumulators, used after a
// cross-rank sum of K-sharded partial accumulators.  Same operation order as
// the fused epilogue: bf16(((float)acc * sa[m]) * sb[n] + bias[n]), then GELU
// on the bf16 value.  Elementwise and HBM-bound (4 B in, 2 B out).
__global__ void __launch_bounds__(256)
k_int8_epilogue(const int32_t* __restrict__ acc, const float* __restrict__ sa, const float* __restrict__ sb,
                const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out, int M, int N, int gelu) {
  const long long total = static_cast<long long>(M) * N;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += 256ll * gridDim.x) {
    const int m = static_cast<int>(i / N), n = static_cast<int>(i - static_cast<long long>(m) * N);
    float y = __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), __ldg(sa + m)), __ldg(sb + n));
    if (bias != nullptr) y = __fadd_rn(y, __bfloat162float(bias[n]));
    __nv_bfloat16 h = __float2bfloat16_rn(y);
    if (gelu) h = __float2bfloat16_rn(gelu_tanh_fast(__bfloat162float(h)));
    out[i] = h;
  }
}

template <MmaKind KIND>
__device__ __forceinline__ void mma_issue(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (KIND == MmaKind::I8) mma_i8(d, a, b, idesc, acc);
  else if constexpr (KIND == MmaKind::F8) mma_f8(d, a, b, idesc, acc);
  else if constexpr (KIND == MmaKind::BF16) mma_bf16(d, a, b, idesc, acc);
}

// Epilogue for one 32-column chunk of one row (this thread's row).  Column
// scales and bias come from the per-tile shared-memory copy (sb_s, bias_s,
// indexed from the chunk's first column); the row scale is in a register.
// W columns (8, 16 or 32) from the chunk's first column n0.
template <MmaKind KIND, int W = 32>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[W], const EpiParams& p, int m, int n0,
                                               float sa, const float* sb_s, const __nv_bfloat16* bias_s,
                                               uint32_t* packed_out = nullptr) {
  static_assert(W == 8 || W == 16 || W == 32, "chunk width");
  const int n_valid = p.N - n0;  // >= 1; a multiple of 8 when < W (N % 8 == 0)
  if (p.flags & kEpiRawAcc) {
    uint32_t* drow = static_cast<uint32_t*>(p.D) + static_cast<long long>(m) * p.ldd;
#pragma unroll
    for (int j = 0; j < W; j += 4) {
      if (j < n_valid) *reinterpret_cast<uint4*>(drow + n0 + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    }
    return;
  }
  // ((acc * sa) * sb + bias) -> bf16 -> GELU, on pairs of columns with packed
  // fp32x2 operations (each element rounds exactly as with scalar ones)
  float2 y[W / 2];
#pragma unroll
  for (int j = 0; j < W / 2; ++j) {
    if constexpr (KIND == MmaKind::I8)
      y[j] = make_float2(__int2float_rn(static_cast<int>(r[2 * j])), __int2float_rn(static_cast<int>(r[2 * j + 1])));
    else
      y[j] = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
  }
  if (KIND != MmaKind::BF16 || p.sa != nullptr) {
    const float2 sa2 = make_float2(sa, sa);
#pragma unroll
    for (int j = 0; j < W / 2; ++j) y[j] = __fmul2_rn(y[j], sa2);
  }
  if (p.sb != nullptr) {
#pragma unroll
    for (int j = 0; j < W / 2; j += 2) {
      const float4 s4 = *reinterpret_cast<const float4*>(sb_s + 2 * j);
      y[j] = __fmul2_rn(y[j], make_float2(s4.x, s4.y));
      y[j + 1] = __fmul2_rn(y[j + 1], make_float2(s4.z, s4.w));
    }
  }
  if (p.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < W / 2; j += 4) {
      const uint4 b4 = *reinterpret_cast<const uint4*>(bias_s + 2 * j);
      const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&b4);
#pragma unroll
      for (int i = 0; i < 4; ++i) y[j + i] = __fadd2_rn(y[j + i], __bfloat1622float2(bh[i]));
    }
  }
  uint32_t packed[W / 2];
#pragma unroll
  for (int j = 0; j < W / 2; ++j) packed[j] = pack_bf16x2(y[j].x, y[j].y);
  if (p.flags & kEpiGelu) {
#pragma unroll
    for (int j = 0; j < W / 2; ++j) {
      const float2 g = gelu_tanh_fast2(__bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&packed[j])));
      packed[j] = pack_bf16x2(g.x, g.y);
    }
  }
  if (packed_out != nullptr) {  // the caller stores the bf16 row chunk itself
#pragma unroll
    for (int j = 0; j < W / 2; ++j) packed_out[j] = packed[j];
    return;
  }
  __nv_bfloat16* drow = static_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(m) * p.ldd;
#pragma unroll
  for (int j = 0; j < W / 8; ++j) {
    if (8 * j < n_valid)
      *reinterpret_cast<uint4*>(drow + n0 + 8 * j) =
          make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  }
}

template <MmaKind KIND, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const EpiParams p,
          const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD32) {
  using C = GemmCfg<KIND, BN, STAGES, true>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sSFA = sB + STAGES * C::B_BYTES;      // NVFP4 only
  uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;  // NVFP4 only
  uint8_t* staging = sSFB + STAGES * C::SFB_BYTES;  // 1024-byte aligned: 8 output boxes (TMA_OUT)
  // per-tile column parameters, double buffered: [2][BN] fp32 scales, [2][BN] bf16 bias
  float* col_scale = reinterpret_cast<float*>(staging + C::STAGING_BYTES);
  __nv_bfloat16* col_bias = reinterpret_cast<__nv_bfloat16*>(col_scale + 2 * BN);
  uint64_t* full = reinterpret_cast<uint64_t*>(col_bias + 2 * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* epi_sync = drain + 1;  // [2]: epilogue threads' column parameters are staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_sync + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr unsigned int kTag = 0x100u + static_cast<unsigned int>(KIND) * 16u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiThreads);
      mbar_init(&epi_sync[b], kEpiThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  const int m_tiles = (p.M + C::BM - 1) / C::BM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int k_units = C::NVF4 ? p.K / 2 : p.K;  // K in TMA elements
  const int k_blocks = (k_units + C::BK - 1) / C::BK;
  // work items: (m tile, n tile), m fastest
  const int num_tiles = m_tiles * n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % m_tiles, nb = tile / m_tiles;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kTag, 1)) { ok = false; break; }
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * C::BK, mb * C::BM);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * C::BK, nb * BN);
          if constexpr (C::NVF4) {
            // the stage's 4 scale atoms are contiguous per 128-row block
            bulk_load(sSFA + stage * C::SFA_BYTES, p.sfa + (static_cast<long long>(mb) * p.sf_ka + kb * 4) * 512,
                      C::SFA_BYTES, &full[stage]);
            bulk_load(sSFB + stage * C::SFB_BYTES, p.sfb + (static_cast<long long>(nb) * p.sf_ka + kb * 4) * 512,
                      C::SFB_BYTES, &full[stage]);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) until every issued copy has landed so no TMA
        // write targets this CTA's shared memory after it exits.
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
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, kTag, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * C::ACC_COLS);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kTag, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
          if constexpr (C::NVF4) {
            // scale factors -> TMEM (in issue order with the MMAs that read them)
            const uint32_t tsfa = tmem_base + 2 * C::ACC_COLS;
            const uint32_t tsfb = tsfa + 16;
            const uint32_t sfa0 = smem_u32(sSFA + stage * C::SFA_BYTES);
            const uint32_t sfb0 = smem_u32(sSFB + stage * C::SFB_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              tc_cp_32x128b_warpx4(tsfa + 4 * kk, sf_atom_desc(sfa0 + kk * 512));
              tc_cp_32x128b_warpx4(tsfb + 4 * kk, sf_atom_desc(sfb0 + kk * 512));
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_nvf4(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), C::IDESC,
                       tsfa + 4 * kk, tsfb + 4 * kk, (kb != 0 || kk != 0) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk) {
              const uint64_t ad = sw128_kmajor_desc(a0 + kk * 32);
              const uint64_t bd = sw128_kmajor_desc(b0 + kk * 32);
              mma_issue<KIND>(d_tmem, ad, bd, C::IDESC, (kb != 0 || kk != 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit(&tfull[buf]);
      }
      if (!ok) {
        // make sure no MMA is still reading shared memory / writing TMEM
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (warp >= kFirstEpiWarp) {
    // ---------------- epilogue (8 warps) ----------------
    // Warp w may only touch TMEM lanes 32*(w%4)..+31; the two warps sharing
    // a lane quarter split the tile's columns in halves.
    const int et = threadIdx.x - kFirstEpiWarp * 32;  // 0..kEpiThreads-1
    const int wq = warp & 3;
    const int half = (warp - kFirstEpiWarp) >> 2;
    constexpr int COLS = BN / 2;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int mb = tile % m_tiles, nb = tile / m_tiles;
      const int buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      // stage this tile's column scales / bias in shared memory
      float* sb_t = col_scale + buf * BN;
      __nv_bfloat16* bias_t = col_bias + buf * BN;
      for (int j = et; j < BN; j += kEpiThreads) {
        const int n = nb * BN + j;
        float sv = 1.0f;
        if (p.sb != nullptr) sv = (n < p.N) ? __ldg(p.sb + static_cast<long long>(n) * p.sb_stride) : 0.0f;
        sb_t[j] = sv;
        bias_t[j] = (p.bias != nullptr && n < p.N) ? p.bias[n] : __float2bfloat16_rn(0.0f);
      }
      const int row = wq * 32 + lane;
      const int m = mb * C::BM + row;
      float sa = 1.0f;
      if (p.sa != nullptr && m < p.M) sa = __ldg(p.sa + static_cast<long long>(m) * p.sa_stride);
      // all epilogue threads have staged the parameters (bounded mbarrier wait
      // rather than a named barrier, so an aborting CTA cannot block here)
      mbar_arrive(&epi_sync[buf]);
      if (!mbar_wait(&epi_sync[buf], tph, abort_flag, kTag, 5)) break;
      if (!mbar_wait(&tfull[buf], tph, abort_flag, kTag, 4)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) +
                             static_cast<uint32_t>(buf * C::ACC_COLS + half * COLS);
#pragma unroll 1
      for (int c = 0; c < COLS; c += 64) {
        const int n0 = nb * BN + half * COLS + c;
        if (n0 >= p.N) break;  // warp-uniform
        if constexpr (C::TMA_OUT) {
          if (!(p.flags & kEpiRawAcc)) {
            // this warp's 32 x 64 box (a 32 x 32 box for the last 32 columns
            // of a 192-wide tile's half), one 32-column chunk at a time; rows
            // swizzled (64-column box: 16-byte chunk q of row r at q ^ (r & 7),
            // 128-byte rows; 32-column box: q ^ ((r >> 1) & 3), 64-byte rows);
            // one TMA store into D, clipped to [M, N]
            const int j0 = half * COLS + c;
            const bool wide = (COLS - c) >= 64;  // warp-uniform
            uint8_t* box = staging + (warp - kFirstEpiWarp) * (32 * 64 * 2);
            if (lane == 0) bulk_wait_read_all();  // the previous box has left shared memory
            __syncwarp();
            uint4* dst = reinterpret_cast<uint4*>(box + lane * (wide ? 128 : 64));
            const int sw = wide ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              if (hh == 1 && !wide) break;
              uint32_t r[32], pk[16];
              tmem_ld_32x32b_x32(taddr + c + 32 * hh, r);
              tmem_ld_wait();
              epilogue_chunk<KIND>(r, p, m, n0 + 32 * hh, sa, sb_t + j0 + 32 * hh, bias_t + j0 + 32 * hh, pk);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
                dst[(4 * hh + q4) ^ sw] = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(wide ? &tmD : &tmD32, box, n0, mb * C::BM + wq * 32);
              bulk_commit_group();
            }
            continue;
          }
        }
        uint32_t r0[32], r1[32];
        const bool two = (COLS - c) >= 64;
        tmem_ld_32x32b_x32(taddr + c, r0);
        if (two) tmem_ld_32x32b_x32(taddr + c + 32, r1);
        tmem_ld_wait();
        if (m < p.M) {
          const int j0 = half * COLS + c;
          epilogue_chunk<KIND>(r0, p, m, n0, sa, sb_t + j0, bias_t + j0);
          if (two && n0 + 32 < p.N)
            epilogue_chunk<KIND>(r1, p, m, n0 + 32, sa, sb_t + j0 + 32, bias_t + j0 + 32);
        }
      }
      tc_fence_before();
      mbar_arrive_relaxed(&tempty[buf]);  // accumulator read (wait::ld); output stores need no ordering
    }
    if (C::TMA_OUT && lane == 0) {
      bulk_wait_all();  // the TMA stores have completed before the kernel retires
      fence_proxy_async_global();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Split-K over a thread-block cluster, for problems whose output tiles cannot
// fill the SMs (48 tiles of 128 x 256 for 148 SMs).  The S
// CTAs of a cluster share one output tile and split its K blocks.  Each
// CTA's MMAs accumulate its K range in TMEM; the epilogue warps copy the raw
// accumulator into shared memory (the pipeline stages are free by then);
// after a cluster barrier each CTA finishes the 32-column chunks j with
// j % S == its rank: it adds the S partial chunks in rank order (its own
// from shared memory, the others over distributed shared memory; int32
// exactly for INT8) and runs the fused epilogue on the sum.  A second cluster
// barrier keeps every CTA's buffer alive until all ranks have read it.
// One tile per cluster: grid = tiles x S.
// ---------------------------------------------------------------------------
template <MmaKind KIND, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_csk(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const EpiParams p) {
  using C = GemmCfg<KIND, BN, STAGES>;
  static_assert(!C::NVF4, "block-scaled split-K is not built");
  constexpr int RED_LD = BN + 4;  // 32-bit words per staged row (16-byte pad: conflict-free row accesses)
  static_assert(128 * RED_LD * 4 <= STAGES * C::STAGE_BYTES, "reduction buffer fits in the pipeline stages");
  constexpr int TMEM_COLS = BN <= 128 ? 128 : 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint32_t* red = reinterpret_cast<uint32_t*>(smem);  // after the tile's MMAs: [128][RED_LD] raw accumulators
  float* col_scale = reinterpret_cast<float*>(sB + STAGES * C::B_BYTES);
  __nv_bfloat16* col_bias = reinterpret_cast<__nv_bfloat16*>(col_scale + BN);
  uint64_t* full = reinterpret_cast<uint64_t*>(col_bias + BN);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr unsigned int kTag = 0x400u + static_cast<unsigned int>(KIND) * 16u;
  const int S = static_cast<int>(cluster_nctarank());
  const int sk = static_cast<int>(cluster_ctarank());
  const int m_tiles = (p.M + C::BM - 1) / C::BM;
  const int tile = blockIdx.x / S;
  const int mb = tile % m_tiles, nb = tile / m_tiles;
  const int k_blocks = (p.K + C::BK - 1) / C::BK;
  const int kb_per = (k_blocks + S - 1) / S;
  const int kb0 = sk * kb_per, kb1 = min(k_blocks, kb0 + kb_per);  // the host makes every range non-empty

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: this CTA's K blocks ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kTag, 1)) { ok = false; break; }
        mbar_expect_tx(&full[stage], C::STAGE_BYTES);
        tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * C::BK, mb * C::BM);
        tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * C::BK, nb * BN);
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
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, kTag, 3)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
        const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk)
          mma_issue<KIND>(tmem_base, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), C::IDESC,
                          (kb != kb0 || kk != 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (ok) tc_commit(tfull);
      else {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  }
  const int et = threadIdx.x - kFirstEpiWarp * 32;
  const int wq = warp & 3;
  const int half = (warp - kFirstEpiWarp) >> 2;
  constexpr int COLS = BN / 2;
  const int row = wq * 32 + lane;
  const int m = mb * C::BM + row;
  float sa = 1.0f;
  if (warp >= kFirstEpiWarp) {
    // column scales / bias of the tile; raw accumulators -> shared memory
    for (int j = et; j < BN; j += kEpiThreads) {
      const int n = nb * BN + j;
      float sv = 1.0f;
      if (p.sb != nullptr) sv = (n < p.N) ? __ldg(p.sb + static_cast<long long>(n) * p.sb_stride) : 0.0f;
      col_scale[j] = sv;
      col_bias[j] = (p.bias != nullptr && n < p.N) ? p.bias[n] : __float2bfloat16_rn(0.0f);
    }
    if (p.sa != nullptr && m < p.M) sa = __ldg(p.sa + static_cast<long long>(m) * p.sa_stride);
    ok = mbar_wait(tfull, 0, abort_flag, kTag, 4);
    tc_fence_after();
    if (ok) {
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + static_cast<uint32_t>(half * COLS);
#pragma unroll 1
      for (int c = 0; c < COLS; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c, r);
        tmem_ld_wait();
        uint4* dst = reinterpret_cast<uint4*>(red + row * RED_LD + half * COLS + c);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every CTA's partial tile is in its shared memory; column parameters staged
  if (warp >= kFirstEpiWarp) {
#pragma unroll 1
    for (int c = 0; c < COLS; c += 32) {
      const int j0 = half * COLS + c;  // column of the tile
      if (((j0 >> 5) % S) != sk) continue;
      const int n0 = nb * BN + j0;
      if (n0 >= p.N || m >= p.M) continue;
      uint32_t acc[32];
      const uint32_t loc = smem_u32(red + row * RED_LD + j0);
#pragma unroll 1
      for (int r = 0; r < S; ++r) {
        const uint32_t base = map_shared_rank(loc, static_cast<uint32_t>(r));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 v = ld_shared_cluster_v4(base + 16u * q);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (r == 0) acc[4 * q + e] = w[e];
            else if constexpr (KIND == MmaKind::I8)
              acc[4 * q + e] = static_cast<uint32_t>(static_cast<int>(acc[4 * q + e]) + static_cast<int>(w[e]));
            else
              acc[4 * q + e] = __float_as_uint(__fadd_rn(__uint_as_float(acc[4 * q + e]), __uint_as_float(w[e])));
          }
        }
      }
      epilogue_chunk<KIND>(acc, p, m, n0, sa, col_scale + j0, col_bias + j0);
    }
  }
  cluster_sync_all();  // no CTA frees its buffer while another rank may still read it
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace qib
