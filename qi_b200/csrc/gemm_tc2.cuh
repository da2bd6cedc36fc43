// CTA-pair tcgen05 GEMM (cta_group::2): D[M,N] = epilogue(A[M,K] . B[N,K]^T)
// with one 256 x BN MMA tile spread over the tensor cores of two SMs.
//
// Why: with one CTA per 128 x 256 tile, every SM streams 16 KB of A plus
// 32 KB of B from L2 per 128-byte K slice, about 96 B per clock at the
// 8-bit MMA rate.  That is more than an SM's share of L2 bandwidth, so the
// single-CTA kernel plateaus near 70 % of the tensor peak.  A CTA pair
// computes a 256 x BN tile.  Each CTA loads its own 128 rows of A and half
// of B, and the even CTA's MMA reads B's halves from both shared memories.
// The L2 -> SMEM traffic per MMA drops by a third (BN = 256: 32 KB per SM
// per K slice).
//
// Roles per CTA (384 threads, one CTA per SM, clusters of 2):
//   warp 0      TMA producer: this CTA's A rows (128) and B rows (BN/2) of
//               every K slice; completion is counted on the EVEN CTA's
//               `full` barrier (the even CTA's producer posts the expected
//               bytes of both CTAs)
//   warp 1      both CTAs allocate TMEM together (cta_group::2); the even
//               CTA's lane 0 issues tcgen05.mma.cta_group::2 (M = 256) and
//               commits to `empty` / `tfull` of both CTAs (multicast commit)
//   warps 4-11  epilogue of this CTA's 128 accumulator rows, as in the
//               single-CTA kernel; each warp arrives on the even CTA's
//               `tempty` when its TMEM columns have been read
// Loads have one destination CTA each (no TMA multicast), so the kernel is
// safe in processes whose peers map this GPU's memory.
//
// NVFP4 (kind::mxf4nvf4, block16 UE4M3 scales): each CTA also loads (plain
// TMA, its own barrier) the scale-factor atoms of its own 128 A rows and of
// ALL BN columns of B, since the pair's MMA reads each CTA's scales from that
// CTA's TMEM.  Four more warps (one per TMEM lane quadrant) move the atoms
// from shared memory into a ring of TMEM scale slots with tcgen05.st, then
// arrive on the even CTA's `sf_ready`.  Measured on B200: tcgen05.cp of the
// 12 atoms of a K slice from the MMA thread costs 82 clocks per 128-clock MMA
// (serialised with the MMAs, even from another warp), while tcgen05.st from
// other warps runs concurrently with them.  Roles: warp 0 TMA, warp 1 MMA,
// warps 4-7 scale slots, warps 8-15 epilogue (512 threads).  At BN = 256 the
// accumulator is single-buffered (256 + 4 slots x 48 columns of 512).
#pragma once

#include "gemm_tc.cuh"

namespace qib {

// Output tensor maps for the column-parallel all-gather fused into the
// epilogue: map[i] describes the [M, N] bf16 block this rank owns in
// destination i (this GPU's output buffer or a peer's, mapped over NVLink).
// Every 32 x 64 output box is written with one TMA store per destination.
struct OutMaps {
  CUtensorMap map[kMaxPeers];
  int n;  // 0: plain stores to EpiParams::D
};

template <MmaKind KIND, int BN_, int STAGES_, bool GATHER_ = false>
struct Gemm2Cfg {
  static constexpr bool NVF4 = (KIND == MmaKind::NVF4);
  static constexpr int BM = 128;  // rows per CTA; a pair covers 256
  static constexpr int BN = BN_;  // output columns of a pair tile
  static constexpr int STAGES = STAGES_;
  static constexpr int ELEM = (KIND == MmaKind::BF16) ? 2 : 1;
  static constexpr int BK = 128 / ELEM;  // TMA elements per 128-byte K slice (NVF4: packed bytes, 256 values)
  static constexpr int UMMA_K = (KIND == MmaKind::BF16) ? 16 : 32;  // TMA elements per MMA
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = (BN / 2) * 128;
  static constexpr int SFA_BYTES = NVF4 ? 4 * 512 : 0;               // this CTA's 128 rows, 4 K atoms
  static constexpr int SFB_BYTES = NVF4 ? 4 * 512 * (BN / 128) : 0;  // every column of the pair tile
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr int ACC_BUFS = (NVF4 && BN == 256) ? 1 : 2;
  static constexpr int ACC_COLS = BN;
  static constexpr int SF_COLS = NVF4 ? 4 * 4 + 4 * (BN / 32) : 0;  // per K slice: A 4 x 4, B 4 x BN/32 columns
  static constexpr int SF_SLOTS = NVF4 ? (BN == 256 ? 5 : 8) : 0;  // TMEM scale slots in flight
  static constexpr int SF_COL0 = ACC_BUFS * BN;                     // first scale column
  static constexpr int TMEM_COLS = (SF_COL0 + SF_SLOTS * SF_COLS <= 256) ? 256 : 512;
  // warp roles: 0 TMA, 1 MMA, [4, 4 + 4) scale slots (NVFP4), then 8 epilogue warps
  static constexpr int SF_WARP0 = 4;
  static constexpr int EPI_WARP0 = NVF4 ? 8 : kFirstEpiWarp;
  static constexpr int THREADS = (EPI_WARP0 + kEpiWarps) * 32;
  static constexpr int COLPARAM_BYTES = 2 * BN * (4 + 2);
  static constexpr int BAR_BYTES = 512;
  // bf16 results of 256-wide tiles leave through one 32-row x 64-column box
  // (128-byte rows) of shared memory per epilogue warp and TMA stores: for
  // the fused gather to every rank (measured on 2 GPUs: 64-column boxes with
  // 5 stages beat 32-column boxes by 25 % and 128-column boxes with 4 stages
  // by 10 %), and into this GPU's output, where row-per-lane global stores
  // (32 rows per warp instruction) cost about 5 us per tile: the NVFP4 tile's
  // single accumulator buffer makes the MMAs wait for all of it (config 4
  // 92 -> 84 us), and with two buffers the stores still compete with the
  // next tile's operand loads (FP8 config 2 157 -> 147 us, INT8 3120 x 14336
  // x 3072 112 -> 105 us).  Local boxes are 128-byte swizzled (conflict-free
  // row writes); the gather's are not.  The staging costs the 8-bit and bf16
  // tiles their sixth pipeline stage (measured: no loss).
  static constexpr bool TMA_OUT = GATHER_ || BN == 256;
  static constexpr int STAGING_BYTES = TMA_OUT ? kEpiWarps * 32 * 64 * 2 : 0;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + COLPARAM_BYTES + BAR_BYTES + STAGING_BYTES + 1024;
  static constexpr uint32_t IDESC = (KIND == MmaKind::I8)     ? make_idesc(kDS32, kFmtS8, kFmtS8, 256, BN)
                                    : (KIND == MmaKind::F8)   ? make_idesc(kDF32, kFmtE4M3, kFmtE4M3, 256, BN)
                                    : (KIND == MmaKind::NVF4) ? make_idesc_nvf4(256, BN)
                                                              : make_idesc(kDF32, kFmtBF16, kFmtBF16, 256, BN);
  static_assert(!NVF4 || BN == 128 || BN == 256, "NVFP4 pair tiles: whole 128-column scale atoms");
  static_assert(!NVF4 || !GATHER_, "NVFP4 with the fused gather is not built");
  static_assert(BN % 64 == 0 && BN >= 128 && BN <= 256, "BN");
  static_assert(SF_COL0 + SF_SLOTS * SF_COLS <= 512, "TMEM");
  static_assert(SF_COLS % 16 == 0, "scale slots are written 16 columns at a time");
  static_assert(BAR_BYTES >= 8 * (3 * STAGES + 2 * SF_SLOTS + 7) + 8, "barrier region");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static_assert(!TMA_OUT || BN % 128 == 0, "output boxes are 64 columns per epilogue warp");
};

// One work item of a pair: a whole tile, or (tail split) a K range of one of
// the tiles of the partial last wave.  With S > 1 the first tiles - tail
// tiles (tail = tiles % pairs, a whole number of waves) go round-robin to the
// pairs; then pair u < tail * S takes K blocks [s kb / S, (s + 1) kb / S) of
// tail tile u / S, s = u % S.  unit = u, or -1 for a whole tile.
struct PairWork {
  int tile, kb0, kb1, unit;
};
__device__ __forceinline__ bool pair_work(int w, int pair, int npairs, int num_tiles, int S, int k_blocks,
                                          PairWork& o) {
  const int tail = S > 1 ? num_tiles % npairs : 0;
  const int whole = num_tiles - tail;
  const int tile = pair + w * npairs;
  if (tile < whole) {
    o = {tile, 0, k_blocks, -1};
    return true;
  }
  if (S > 1 && w == whole / npairs && pair < tail * S) {
    const int s = pair % S;
    o = {whole + pair / S, s * k_blocks / S, (s + 1) * k_blocks / S, pair};
    return true;
  }
  return false;
}

// Tail split, run by the 256 epilogue threads of each CTA of a tail unit once
// its partial accumulators are in the workspace: wait (bounded) until all 2S
// CTAs of the tile have stored theirs, then sum this CTA's share of the tile
// (1/2S of its 8-column row pieces, splits added in a fixed order, so the
// result is deterministic and exact for INT8) and run the usual epilogue on
// it.  The last CTA to finish resets the tile's counters for the next launch.
// Returns false when the CTA is aborting.
constexpr int kMaxTailSplit = 8;
template <MmaKind KIND, int BN>
__device__ __forceinline__ bool tail_reduce(const EpiParams& p, const PairWork& wk, int S, int rank, int mb, int nb,
                                              int et, const float* sb_t, const __nv_bfloat16* bias_t,
                                              uint64_t* tail_sync, uint32_t& ph, volatile int* abort_flag,
                                              unsigned int tag) {
  auto epi_bar = [&](unsigned int site) {
    mbar_arrive(tail_sync);
    const bool ok = mbar_wait(tail_sync, ph, abort_flag, tag, site);
    ph ^= 1u;
    return ok;
  };
  const int tt = wk.unit / S;
  unsigned int* cnt = p.tail_cnt + tt;
  unsigned int* done = p.tail_cnt + kMaxTailTiles + tt;
  const unsigned int need = 2u * static_cast<unsigned int>(S);
  if (!epi_bar(10)) return false;  // every partial store of this CTA is issued
  if (et == 0) {
    __threadfence();
    atomicAdd(cnt, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu(cnt) < need) {
      if (*abort_flag) break;
      if (globaltimer_ns() - t0 > QI_WAIT_TIMEOUT_NS) {
        record_error(kDevWaitTimeout, tag, 11);
        *abort_flag = 1;
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
  }
  if (!epi_bar(12) || *abort_flag) return false;

  constexpr int PPR = BN / 8;   // 8-column pieces per row
  constexpr int P = 256 * PPR;  // pieces per tile
  const int R = 2 * S, c = 2 * (wk.unit % S) + rank;
  const int q1 = (c + 1) * P / R;
  const uint32_t* base = p.tail_ws + static_cast<size_t>(tt) * S * 256 * BN;
  for (int q = c * P / R + et; q < q1; q += kEpiThreads) {
    const int rt = q / PPR, j0 = (q - rt * PPR) * 8;
    const int m = mb * 256 + rt, n0 = nb * BN + j0;
    if (m >= p.M || n0 >= p.N) continue;
    const uint4* src = reinterpret_cast<const uint4*>(base + static_cast<size_t>(rt) * BN + j0);
    constexpr int kSplitWords = 256 * BN / 4;  // uint4 per split
    constexpr int kBatch = 4;                  // splits loaded together (registers: 8 per split)
    uint32_t r[8];
#pragma unroll
    for (int s0 = 0; s0 < kMaxTailSplit; s0 += kBatch) {
      if (s0 < S) {
        uint4 part[kBatch][2];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (s0 + i < S) {
            part[i][0] = __ldcg(src + (s0 + i) * kSplitWords);
            part[i][1] = __ldcg(src + (s0 + i) * kSplitWords + 1);
          }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (s0 + i < S) {
            const uint32_t v[8] = {part[i][0].x, part[i][0].y, part[i][0].z, part[i][0].w,
                                   part[i][1].x, part[i][1].y, part[i][1].z, part[i][1].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if (s0 + i == 0) r[e] = v[e];
              else if constexpr (KIND == MmaKind::I8) r[e] += v[e];  // two's-complement int32 sum
              else r[e] = __float_as_uint(__fadd_rn(__uint_as_float(r[e]), __uint_as_float(v[e])));
            }
          }
        }
      }
    }
    float sa = 1.0f;
    if (p.sa != nullptr) sa = __ldg(p.sa + static_cast<long long>(m) * p.sa_stride);
    epilogue_chunk<KIND, 8>(r, p, m, n0, sa, sb_t + j0, bias_t + j0);
  }

  if (!epi_bar(13)) return false;  // this CTA has read its share
  if (et == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == need - 1u) {  // every CTA of the tile is past its wait and its reads
      atomicExch(cnt, 0u);
      atomicExch(done, 0u);
    }
  }
  return true;
}

template <MmaKind KIND, int BN, int STAGES, bool GATHER = false>
__global__ void __launch_bounds__(Gemm2Cfg<KIND, BN, STAGES, GATHER>::THREADS, 1)
k_gemm_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmSFA, const __grid_constant__ CUtensorMap tmSFB, const EpiParams p,
           const __grid_constant__ OutMaps om) {
  using C = Gemm2Cfg<KIND, BN, STAGES, GATHER>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sSFA = sB + STAGES * C::B_BYTES;      // NVFP4 only
  uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;  // NVFP4 only
  uint8_t* staging = sSFB + STAGES * C::SFB_BYTES;  // 1024-byte aligned: 8 boxes of 32 x 64 bf16 (TMA_OUT)
  float* col_scale = reinterpret_cast<float*>(staging + C::STAGING_BYTES);
  __nv_bfloat16* col_bias = reinterpret_cast<__nv_bfloat16*>(col_scale + 2 * BN);
  uint64_t* full = reinterpret_cast<uint64_t*>(col_bias + 2 * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* epi_sync = drain + 1;
  uint64_t* sf_full = epi_sync + 2;          // [STAGES] this CTA's scale atoms landed (NVFP4)
  uint64_t* sf_ready = sf_full + STAGES;     // [SF_SLOTS] even CTA: both CTAs' slot written
  uint64_t* sf_free = sf_ready + C::SF_SLOTS;  // [SF_SLOTS] the MMAs reading the slot are done
  uint64_t* tail_sync = sf_free + C::SF_SLOTS;  // epilogue threads of a tail-split unit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tail_sync + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr int kFirstEpi = C::EPI_WARP0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = the CTA that issues the MMAs
  const bool leader = rank == 0;
  constexpr unsigned int kTag = 0x200u + static_cast<unsigned int>(KIND) * 16u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);  // one arrive per epilogue warp of both CTAs
      mbar_init(&epi_sync[b], kEpiThreads);
    }
    if constexpr (C::NVF4) {
      for (int s = 0; s < STAGES; ++s) mbar_init(&sf_full[s], 1);
      for (int s = 0; s < C::SF_SLOTS; ++s) {
        mbar_init(&sf_ready[s], 2 * 4);  // one arrive per scale warp of both CTAs
        mbar_init(&sf_free[s], 1);
      }
    }
    mbar_init(drain, 1);
    mbar_init(tail_sync, kEpiThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    if constexpr (C::NVF4) {
      tma_prefetch_map(&tmSFA);
      tma_prefetch_map(&tmSFB);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive / complete_tx
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int m_tiles = (p.M + 255) / 256;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_units = C::NVF4 ? p.K / 2 : p.K;  // K in TMA elements
  const int k_blocks = (k_units + C::BK - 1) / C::BK;
  // tail split (host: tail * S <= pairs, S <= k_blocks).  Not for NVFP4: its
  // 512-thread CTA has 128 registers a thread, and the split's reduction
  // made the kernel spill (measured 92 -> 98 us at config 4)
  const int S = (C::NVF4 || GATHER) ? 1 : p.tail_split;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      PairWork wk;
      for (int w = 0; ok && pair_work(w, pair, npairs, num_tiles, S, k_blocks, wk); ++w) {
        const int mb = wk.tile % m_tiles, nb = wk.tile / m_tiles;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kTag, 1)) { ok = false; break; }
          const uint32_t lfull = map_shared_rank(smem_u32(&full[stage]), 0);
          if (leader) mbar_expect_tx(&full[stage], 2 * (C::A_BYTES + C::B_BYTES));
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, lfull, kb * C::BK, mb * 256 + rank * C::BM);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, lfull, kb * C::BK, nb * BN + rank * (BN / 2));
          if constexpr (C::NVF4) {
            // scale atoms (this CTA's barrier): rows are [128-row block][K atom of 64
            // values]; 4 atoms per K slice
            mbar_expect_tx(&sf_full[stage], C::SFA_BYTES + C::SFB_BYTES);
            tma_load_2d(sSFA + stage * C::SFA_BYTES, &tmSFA, &sf_full[stage], 0,
                        (2 * mb + static_cast<int>(rank)) * p.sf_ka + kb * 4);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d(sSFB + stage * C::SFB_BYTES + j * 2048, &tmSFB, &sf_full[stage], 0,
                          (nb * (BN / 128) + j) * p.sf_ka + kb * 4);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok && leader) {
        // the pair's copies complete on the even CTA's barriers: wait (bounded)
        // until the stages in flight have landed before the pair exits
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&full[s], ph);
        }
      }
      if (!ok && C::NVF4) {
        // this CTA's scale loads complete on its own barriers
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&sf_full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (even CTA) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      int g = 0;  // K slices issued so far (scale slot ring)
      bool ok = true;
      PairWork wk;
      for (int w = 0; ok && pair_work(w, pair, npairs, num_tiles, S, k_blocks, wk); ++w, ++local) {
        const int buf = local % C::ACC_BUFS;
        const uint32_t tph = (local / C::ACC_BUFS) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, kTag, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * C::ACC_COLS);
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kTag, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
          if constexpr (C::NVF4) {
            // both CTAs' scale slot for this K slice is in TMEM
            const int slot = g % C::SF_SLOTS;
            if (!mbar_wait(&sf_ready[slot], (g / C::SF_SLOTS) & 1, abort_flag, kTag, 6)) { ok = false; break; }
            tc_fence_after();
            const uint32_t tsfa = tmem_base + static_cast<uint32_t>(C::SF_COL0 + slot * C::SF_COLS);
            const uint32_t tsfb = tsfa + 16;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_nvf4_pair(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), C::IDESC,
                            tsfa + 4 * kk, tsfb + (BN / 32) * kk, (kb != wk.kb0 || kk != 0) ? 1u : 0u);
            tc_commit_pair_mc(&sf_free[slot], 0x3);
            ++g;
          } else {
#pragma unroll
            for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk)
              mma_pair<static_cast<int>(KIND)>(d_tmem, sw128_kmajor_desc(a0 + kk * 32),
                                               sw128_kmajor_desc(b0 + kk * 32), C::IDESC,
                                               (kb != wk.kb0 || kk != 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit_pair_mc(&tfull[buf], 0x3);
      }
      if (!ok) {
        tc_commit_pair_mc(drain, 0x1);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (C::NVF4 && warp >= C::SF_WARP0 && warp < C::SF_WARP0 + 4) {
    // ---------------- scale slots (NVFP4): shared-memory atoms -> TMEM ----------------
    // Atom layout: row r (0..31) holds 16 bytes, the 4 K scales of rows r, r+32,
    // r+64, r+96; each lane quadrant of TMEM gets the same 32 rows (the layout
    // a 32x128b.warpx4 copy produces): lane l, column 4a + c of atom a = bytes
    // [4c, 4c + 4) of row l % 32.  Slot columns: A atoms kk at 4kk, B atoms
    // (kk, j) at 16 + (BN/32) kk + 4j.
    if constexpr (C::NVF4) {
    const uint32_t tq = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    int stage = 0;
    uint32_t phase = 0;
    int g = 0;
    bool ok = true;
    PairWork wk;
    for (int w = 0; ok && pair_work(w, pair, npairs, num_tiles, S, k_blocks, wk); ++w) {
      for (int kb = wk.kb0; kb < wk.kb1; ++kb, ++g) {
        const int slot = g % C::SF_SLOTS;
        if (!mbar_wait(&sf_free[slot], ((g / C::SF_SLOTS) & 1) ^ 1u, abort_flag, kTag, 7)) { ok = false; break; }
        if (!mbar_wait(&sf_full[stage], phase, abort_flag, kTag, 8)) { ok = false; break; }
        const uint4* fa = reinterpret_cast<const uint4*>(sSFA + stage * C::SFA_BYTES) + lane;
        const uint4* fb = reinterpret_cast<const uint4*>(sSFB + stage * C::SFB_BYTES) + lane;
        uint32_t r[C::SF_COLS];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint4 v = fa[kk * 32];
          r[4 * kk] = v.x; r[4 * kk + 1] = v.y; r[4 * kk + 2] = v.z; r[4 * kk + 3] = v.w;
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) {
            const uint4 u = fb[j * 128 + kk * 32];
            const int c = 16 + (BN / 32) * kk + 4 * j;
            r[c] = u.x; r[c + 1] = u.y; r[c + 2] = u.z; r[c + 3] = u.w;
          }
        }
        const uint32_t taddr = tq + static_cast<uint32_t>(C::SF_COL0 + slot * C::SF_COLS);
#pragma unroll
        for (int c = 0; c < C::SF_COLS; c += 16)
          tmem_st_32x32b_x16(taddr + c, *reinterpret_cast<const uint32_t(*)[16]>(&r[c]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(map_shared_rank(smem_u32(&sf_ready[slot]), 0));
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    }
  } else if (warp >= kFirstEpi) {
    // ---------------- epilogue (8 warps, this CTA's 128 rows) ----------------
    const int et = threadIdx.x - kFirstEpi * 32;
    const int wq = warp & 3;
    const int half = (warp - kFirstEpi) >> 2;
    constexpr int COLS = BN / 2;
    int local = 0;
    uint32_t tail_ph = 0;
    PairWork wk;
    for (int w = 0; pair_work(w, pair, npairs, num_tiles, S, k_blocks, wk); ++w, ++local) {
      const int mb = wk.tile % m_tiles, nb = wk.tile / m_tiles;
      const int buf = local % C::ACC_BUFS;
      const uint32_t tph = (local / C::ACC_BUFS) & 1;
      // column parameters alternate between two buffers whatever ACC_BUFS is:
      // a warp that is done with work item w stages those of w + 1 while other
      // warps may still read w's; epi_sync of w + 1 proves all are done with
      // w - 1, whose buffer w + 1 reuses
      const int pb = local & 1;
      const uint32_t pph = (local >> 1) & 1;
      float* sb_t = col_scale + pb * BN;
      __nv_bfloat16* bias_t = col_bias + pb * BN;
      for (int j = et; j < BN; j += kEpiThreads) {
        const int n = nb * BN + j;
        float sv = 1.0f;
        if (p.sb != nullptr) sv = (n < p.N) ? __ldg(p.sb + static_cast<long long>(n) * p.sb_stride) : 0.0f;
        sb_t[j] = sv;
        bias_t[j] = (p.bias != nullptr && n < p.N) ? p.bias[n] : __float2bfloat16_rn(0.0f);
      }
      const int row = wq * 32 + lane;
      const int m = mb * 256 + static_cast<int>(rank) * C::BM + row;
      float sa = 1.0f;
      if (p.sa != nullptr && m < p.M) sa = __ldg(p.sa + static_cast<long long>(m) * p.sa_stride);
      mbar_arrive(&epi_sync[pb]);
      if (!mbar_wait(&epi_sync[pb], pph, abort_flag, kTag, 5)) break;
      if (!mbar_wait(&tfull[buf], tph, abort_flag, kTag, 4)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) +
                             static_cast<uint32_t>(buf * C::ACC_COLS + half * COLS);
#pragma unroll 1
      for (int c = 0; c < COLS; c += 64) {
        const int n0 = nb * BN + half * COLS + c;
        if (n0 >= p.N) break;  // warp-uniform
        if constexpr (C::TMA_OUT && !GATHER) {
          if (!(p.flags & kEpiRawAcc) && wk.unit < 0) {  // tail-split units store raw partials below
            // this warp's 32 x 64 box, one 32-column chunk at a time (fewer
            // live registers), rows 128-byte swizzled (16-byte chunk q of row
            // r at q ^ (r & 7)); one TMA store into D, clipped to [M, N]
            const int j0 = half * COLS + c;
            uint8_t* box = staging + (warp - kFirstEpi) * (32 * 64 * 2);
            const int row_base = mb * 256 + static_cast<int>(rank) * C::BM + wq * 32;
            if (lane == 0) bulk_wait_read_all();  // the previous box has left shared memory
            __syncwarp();
            uint4* dst = reinterpret_cast<uint4*>(box + lane * 128);
            const int sw = lane & 7;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
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
              tma_store_2d(&om.map[0], box, n0, row_base);
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
        const int j0 = half * COLS + c;
        if constexpr (!GATHER) {
          if (wk.unit >= 0) {
            // K range of a tail tile: raw partial accumulators to the workspace
            uint4* wrow = reinterpret_cast<uint4*>(
                p.tail_ws + (static_cast<size_t>(wk.unit) * 256 + static_cast<int>(rank) * C::BM + row) * BN + j0);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcg(wrow + q, make_uint4(r0[4 * q], r0[4 * q + 1], r0[4 * q + 2], r0[4 * q + 3]));
            if (two) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                __stcg(wrow + 8 + q, make_uint4(r1[4 * q], r1[4 * q + 1], r1[4 * q + 2], r1[4 * q + 3]));
            }
          } else if (m < p.M) {
            epilogue_chunk<KIND>(r0, p, m, n0, sa, sb_t + j0, bias_t + j0);
            if (two && n0 + 32 < p.N) epilogue_chunk<KIND>(r1, p, m, n0 + 32, sa, sb_t + j0 + 32, bias_t + j0 + 32);
          }
        } else {
          // fused all-gather: stage this warp's 32 x 64 box (one 128-byte row
          // per lane), then one TMA store per destination (clipped to [M, N]
          // by the tensor maps)
          uint8_t* box = staging + (warp - kFirstEpi) * (32 * 64 * 2);
          const int row_base = mb * 256 + static_cast<int>(rank) * C::BM + wq * 32;
          uint32_t pk[32];
          epilogue_chunk<KIND>(r0, p, m, n0, sa, sb_t + j0, bias_t + j0, pk);
          if (two) epilogue_chunk<KIND>(r1, p, m, n0 + 32, sa, sb_t + j0 + 32, bias_t + j0 + 32, pk + 16);
          if (lane == 0) bulk_wait_read_all();  // the previous box has left shared memory
          __syncwarp();
          uint4* dst = reinterpret_cast<uint4*>(box + lane * 128);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) dst[q4] = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int d = 0; d < om.n; ++d) tma_store_2d(&om.map[d], box, n0, row_base);
            bulk_commit_group();
          }
        }
      }
      // this warp's TMEM columns are read: tell the MMA issuer (even CTA)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_shared_rank(smem_u32(&tempty[buf]), 0));
      if constexpr (!GATHER && !C::NVF4) {
        if (wk.unit >= 0 &&
            !tail_reduce<KIND, BN>(p, wk, S, static_cast<int>(rank), mb, nb, et, sb_t, bias_t, tail_sync, tail_ph,
                                   abort_flag, kTag))
          break;
      }
    }
  }

  if (C::TMA_OUT && warp >= kFirstEpi && lane == 0) {
    // the TMA stores have completed before the kernel retires (the fused
    // gather's have reached every destination; the cross-GPU barrier that
    // follows publishes them)
    bulk_wait_all();
    fence_proxy_async_global();
    if (GATHER) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no MMA of the pair still targets either CTA's TMEM or smem
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace qib
