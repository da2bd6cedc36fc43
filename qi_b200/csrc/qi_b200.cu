// libqi_b200: the C-ABI of the B200-native quantized-linear kernels.
//
// One translation unit (the device status word and the kernels live in the
// same module).  Every entry point:
//   * takes plain device pointers, sizes and a cudaStream_t,
//   * launches asynchronously on that stream, never synchronizes, never
//     allocates device memory (callers own all memory; the only allocating
//     entry points are the explicit qi_b200_peer_alloc / _free), so calls can
//     be captured in CUDA graphs,
//   * returns an int status (0 = ok), see include/qi_b200.h.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "attn_short.cuh"
#include "dit_fused.cuh"
#include "launch_count.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_w4a16.cuh"
#include "quantize_act.cuh"
#include "quantize_nvfp4.cuh"
#include "sm100_ptx.cuh"
#include "../../include/qi_b200.h"

namespace qib {

// ---------------------------------------------------------------------------
// per-device host state
// ---------------------------------------------------------------------------
// Per-stream slots (up to kTailSlots streams per device; further streams run
// without what a slot provides).  A slot holds the arrival / done counters of
// the CTA-pair GEMM's tail split in g_tail_cnt (zero at load; each launch
// leaves them zero unless it aborted, and qi_b200_device_status(clear)
// re-zeroes them after an error); the partial accumulators themselves go to
// a workspace the caller passes (qi_b200_gemm_ws).
constexpr int kTailSlots = 8;
__device__ unsigned int g_tail_cnt[kTailSlots][2 * kMaxTailTiles];
// Per-stream slots also hold the NVFP4 tensor amax pass's per-block maxima
// and its ticket (zero at load and after every launch), so that pass needs
// no memset before it.
constexpr int kAmaxParts = 2048;
__device__ unsigned int g_amax_part[kTailSlots][kAmaxParts];
__device__ unsigned int g_amax_ticket[kTailSlots];

struct DeviceInfo {
  int checked = 0;  // 0 unknown, 1 ok, -1 wrong arch
  int num_sms = 0;
  int n_tail = 0;
  cudaStream_t tail[kTailSlots] = {};
  unsigned int* tail_cnt = nullptr;
  unsigned int* amax_part = nullptr;
  unsigned int* amax_ticket = nullptr;
};
constexpr int kMaxDevices = 64;
static DeviceInfo g_dev[kMaxDevices];
static std::mutex g_dev_mu;

// Slot of `stream` (registered on first use, up to kTailSlots per device),
// -1 when the table is full or the slot arrays cannot be located.  Call with
// g_dev_mu held.
static int stream_slot(DeviceInfo* di, cudaStream_t stream) {
  if (di->tail_cnt == nullptr) {
    void *a = nullptr, *b = nullptr, *c = nullptr;
    if (cudaGetSymbolAddress(&a, g_tail_cnt) != cudaSuccess || cudaGetSymbolAddress(&b, g_amax_part) != cudaSuccess ||
        cudaGetSymbolAddress(&c, g_amax_ticket) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    di->amax_part = static_cast<unsigned int*>(b);
    di->amax_ticket = static_cast<unsigned int*>(c);
    di->tail_cnt = static_cast<unsigned int*>(a);
  }
  int i = 0;
  while (i < di->n_tail && di->tail[i] != stream) ++i;
  if (i == di->n_tail) {
    if (i == kTailSlots) return -1;
    di->tail[i] = stream;
    di->n_tail = i + 1;
  }
  return i;
}

// Tail-split counters of `stream`'s slot; false when the slot table is full
// (the launch then runs without the split).  Nothing is allocated.
static bool tail_counters(DeviceInfo* di, cudaStream_t stream, unsigned int** cnt) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  const int i = stream_slot(di, stream);
  if (i < 0) return false;
  *cnt = di->tail_cnt + static_cast<size_t>(i) * 2 * kMaxTailTiles;
  return true;
}

// Splits per tail tile for `tiles` pair tiles on `pairs` pairs: the partial
// last wave (tiles % pairs tiles) spreads its K over the idle pairs.  mode 0
// is automatic: only when it takes at least 64 K blocks (about 16 us at the
// 8-bit MMA rate) off the critical path.  A split unit costs a pipeline fill,
// a workspace round trip and a wait for the slowest pair of its group
// (pairs finish their whole tiles up to a tile apart), which measured on
// B200 ate the gain at K = 3072: FP8 4096 x 14336 x 3072 139 -> 150 us,
// INT8 3120 x 9216 x 3072 74 -> 86 us, while INT8 3120 x 3072 x 14336 went
// 125 -> 107 us.  1 = none; S >= 2 = at most S.
static int tail_plan(int tiles, int pairs, int k_blocks, int mode) {
  if (mode == 1 || tiles <= pairs) return 1;
  const int tail = tiles % pairs;
  if (tail == 0 || tail > kMaxTailTiles) return 1;
  int S = pairs / tail;
  if (mode >= 2) S = std::min(S, mode);
  S = std::min(S, std::min(kMaxTailSplit, k_blocks));
  if (S < 2) return 1;
  if (mode == 0 && k_blocks - (k_blocks + S - 1) / S < 64) return 1;
  return S;
}

static int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QI_B200_ECUDA;
  DeviceInfo& d = g_dev[dev];
  if (d.checked == 0) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (d.checked == 0) {
      int major = 0, minor = 0, sms = 0;
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      d.num_sms = sms;
      d.checked = (major == 10 && minor == 0) ? 1 : -1;
    }
  }
  *out = &d;
  return d.checked == 1 ? QI_B200_OK : QI_B200_EARCH;
}

// ---------------------------------------------------------------------------
// TMA descriptors (cuTensorMapEncodeTiled through the runtime's driver
// entry-point lookup, so the library does not link libcuda directly)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor [rows, inner] with a byte row stride, 128-byte
// swizzled boxes of [box_rows, box_inner].  Out-of-range box elements read 0.
static int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return QI_B200_ETMAP;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QI_B200_OK : QI_B200_ETMAP;
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch plan of the calling thread's most recent GEMM launch (diagnostics:
// kernel id, grid, cluster size, tile N, stages, dynamic shared memory).
struct LaunchPlan {
  int kernel, grid, cluster, tile_n, stages, smem;
};
static thread_local LaunchPlan g_last_plan = {0, 0, 0, 0, 0, 0};
static thread_local int g_last_tail = 1;  // splits per tail tile of the last CTA-pair launch
enum PlanKernel { kPlanGemmI8 = 1, kPlanGemmF8 = 2, kPlanGemmBF16 = 3, kPlanGemmNVF4 = 4,
                  kPlanW4Skinny = 6, kPlanW4Small = 7,
                  kPlanGemmPair = 8 /* + kind: 8 int8, 9 fp8, 10 bf16, 11 nvfp4 */,
                  kPlanGemmCsk = 12 /* + kind: 12 int8, 13 fp8, 14 bf16 */ };

// ---------------------------------------------------------------------------
// GEMM launch
// ---------------------------------------------------------------------------
template <MmaKind KIND, int BN, int STAGES>
static int launch_gemm_cfg(const void* A, const void* B, const EpiParams& p, int num_sms, cudaStream_t stream) {
  using C = GemmCfg<KIND, BN, STAGES, true>;
  const CUtensorMapDataType dt =
      (KIND == MmaKind::BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint64_t ku = C::NVF4 ? (uint64_t)p.K / 2 : (uint64_t)p.K;  // K in TMA elements (fp4: packed bytes)
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, dt, ku, (uint64_t)p.M, ku * C::ELEM, C::BK, C::BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, dt, ku, (uint64_t)p.N, ku * C::ELEM, C::BK, BN);
  if (rc) return rc;
  CUtensorMap td = {}, td32 = {};  // bf16 output boxes of 32 rows x 64 (32) columns (TMA-store epilogue)
  if (C::TMA_OUT && !(p.flags & kEpiRawAcc)) {
    rc = make_tmap_2d(&td, p.D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.ldd * 2,
                      64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (BN == 192) {
      rc = make_tmap_2d(&td32, p.D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)p.N, (uint64_t)p.M,
                        (uint64_t)p.ldd * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc) return rc;
    }
  }
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(k_gemm_tc<KIND, BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[dev] = true;
  }
  const int tiles = ((p.M + C::BM - 1) / C::BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  g_last_plan = {1 + static_cast<int>(KIND), grid, 1, BN, STAGES, C::SMEM_BYTES};
  const cudaError_t e =
      launch_pdl(k_gemm_tc<KIND, BN, STAGES>, dim3(grid), dim3(kGemmThreads), C::SMEM_BYTES, stream, 1, ta, tb, p, td, td32);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

// CTA-pair kernel (cta_group::2): 256 x BN tiles over clusters of 2 CTAs.
template <MmaKind KIND, int BN, int STAGES, bool GATHER = false>
static int launch_gemm2_cfg(const void* A, const void* B, const EpiParams& p, int num_sms, cudaStream_t stream,
                            const OutMaps* om_in = nullptr) {
  using C = Gemm2Cfg<KIND, BN, STAGES, GATHER>;
  static OutMaps kNoMaps = {};  // n = 0: plain epilogue stores
  OutMaps local = {};           // TMA-store epilogue into this GPU's output (bf16 results)
  if constexpr (C::TMA_OUT && !GATHER) {
    if (!(p.flags & kEpiRawAcc)) {
      const int rc = make_tmap_2d(&local.map[0], p.D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)p.N,
                                  (uint64_t)p.M, (uint64_t)p.ldd * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      local.n = 1;
    }
  }
  const OutMaps& om = om_in != nullptr ? *om_in : (C::TMA_OUT && !GATHER ? local : kNoMaps);
  const CUtensorMapDataType dt =
      (KIND == MmaKind::BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint64_t ku = C::NVF4 ? (uint64_t)p.K / 2 : (uint64_t)p.K;  // K in TMA elements (fp4: packed bytes)
  CUtensorMap ta, tb, tsa = {}, tsb = {};
  int rc = make_tmap_2d(&ta, A, dt, ku, (uint64_t)p.M, ku * C::ELEM, C::BK, C::BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, dt, ku, (uint64_t)p.N, ku * C::ELEM, C::BK, BN / 2);
  if (rc) return rc;
  if constexpr (C::NVF4) {
    // scale atoms as rows of 512 bytes (128 x u32): [128-row block][K atom]; 4 atoms per box
    const uint64_t rows_a = (uint64_t)((p.M + 127) / 128) * p.sf_ka;
    const uint64_t rows_b = (uint64_t)((p.N + 127) / 128) * p.sf_ka;
    rc = make_tmap_2d(&tsa, p.sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128, rows_a, 512, 128, 4,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = make_tmap_2d(&tsb, p.sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128, rows_b, 512, 128, 4,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(k_gemm_tc2<KIND, BN, STAGES, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[dev] = true;
  }
  const int tiles = ((p.M + 255) / 256) * ((p.N + BN - 1) / BN);
  const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
  EpiParams q = p;
  q.tail_split = 1;
  q.tail_cnt = nullptr;
  if (!C::NVF4 && !GATHER && p.tail_split != 1 && p.tail_ws != nullptr) {
    // the split needs the caller's workspace to hold every tail tile's S
    // partial accumulators (256 x BN words each)
    const int S = tail_plan(tiles, pairs, static_cast<int>((ku + C::BK - 1) / C::BK), p.tail_split);
    const size_t need = static_cast<size_t>(tiles % pairs) * S * 256 * BN * 4;
    DeviceInfo* di = nullptr;
    if (S > 1 && need <= p.tail_ws_bytes && device_info(&di) == QI_B200_OK && tail_counters(di, stream, &q.tail_cnt))
      q.tail_split = S;
  }
  g_last_plan = {kPlanGemmPair + static_cast<int>(KIND), 2 * pairs, 2, BN, STAGES, C::SMEM_BYTES};
  g_last_tail = q.tail_split;
  const cudaError_t e = launch_pdl(k_gemm_tc2<KIND, BN, STAGES, GATHER>, dim3(2 * pairs), dim3(C::THREADS),
                                   C::SMEM_BYTES, stream, 2, ta, tb, tsa, tsb, q, om);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

// Cluster split-K (k_gemm_csk): S CTAs of a cluster share one 128 x BN tile.
template <MmaKind KIND, int BN, int STAGES>
static int launch_gemm_csk_cfg(const void* A, const void* B, const EpiParams& p, int S, cudaStream_t stream) {
  using C = GemmCfg<KIND, BN, STAGES>;
  const CUtensorMapDataType dt =
      (KIND == MmaKind::BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint64_t ku = (uint64_t)p.K;
  const int k_blocks = (p.K + C::BK - 1) / C::BK;
  const int kbp = (k_blocks + S - 1) / S;
  if (S < 2 || S > 8 || (long long)kbp * (S - 1) >= k_blocks) return QI_B200_ESHAPE;  // a rank without K blocks
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, dt, ku, (uint64_t)p.M, ku * C::ELEM, C::BK, C::BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, dt, ku, (uint64_t)p.N, ku * C::ELEM, C::BK, BN);
  if (rc) return rc;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(k_gemm_csk<KIND, BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[dev] = true;
  }
  const int tiles = ((p.M + C::BM - 1) / C::BM) * ((p.N + BN - 1) / BN);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(tiles * S, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  g_last_plan = {kPlanGemmCsk + static_cast<int>(KIND), tiles * S, S, BN, STAGES, C::SMEM_BYTES};
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_csk<KIND, BN, STAGES>, ta, tb, p);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

template <MmaKind KIND>
static int launch_gemm_csk(const void* A, const void* B, const EpiParams& p, int bn, int S, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_gemm_csk_cfg<KIND, 256, 4>(A, B, p, S, stream);
    case 192: return launch_gemm_csk_cfg<KIND, 192, 5>(A, B, p, S, stream);
    case 128: return launch_gemm_csk_cfg<KIND, 128, 6>(A, B, p, S, stream);
    default: return QI_B200_EINVAL;
  }
}

// The cluster split-K plan for a problem whose tiles leave most SMs idle:
// the tile width and cluster size (2..4, >= 4 K blocks per rank) that put the
// most CTAs to work; {0, 1} when the tiles already fill half the SMs.
static void csk_plan(int kind, int M, int N, int K, int num_sms, int* bn_out, int* s_out) {
  *bn_out = 0;
  *s_out = 1;
  if (kind < 0 || kind > 2) return;
  const int bk = kind == QI_B200_KIND_BF16 ? 64 : 128;
  const int k_blocks = (K + bk - 1) / bk;
  int best = 0;
  for (int bn : {256, 192, 128}) {
    const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
    if (tiles * 2 > num_sms) continue;
    int S = std::min(4, std::min(num_sms / tiles, k_blocks / 4));
    if (S < 2) continue;
    const int kbp = (k_blocks + S - 1) / S;
    S = (k_blocks + kbp - 1) / kbp;  // every rank gets >= 1 K block
    if (S < 2) continue;
    if (tiles * S > best) {
      best = tiles * S;
      *bn_out = bn;
      *s_out = S;
    }
  }
}

// Column-tile width: minimise (tiles per CTA) x (BN + fixed per-tile cost).
static int pick_bn(int M, int N, int num_sms) {
  const int mt = (M + 127) / 128;
  int best_bn = 256;
  long best = -1;
  for (int bn : {256, 192, 128, 64}) {
    const long tiles = (long)mt * ((N + bn - 1) / bn);
    const long waves = (tiles + num_sms - 1) / num_sms;
    const long cost = waves * (bn + 64);
    if (best < 0 || cost < best) {
      best = cost;
      best_bn = bn;
    }
  }
  return best_bn;
}

template <MmaKind KIND>
static int launch_gemm(const void* A, const void* B, const EpiParams& p, cudaStream_t stream, int force_bn) {
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  if constexpr (KIND == MmaKind::NVF4) {
    // 128 x 128 single-CTA tiles, or CTA pairs: 256 x 128 (double-buffered
    // accumulator) or 256 x 256 (single-buffered: the scale factors take TMEM
    // columns too)
    if (force_bn == -256) return launch_gemm2_cfg<KIND, 256, 5>(A, B, p, di->num_sms, stream);
    if (force_bn == -128) return launch_gemm2_cfg<KIND, 128, 7>(A, B, p, di->num_sms, stream);
    if (force_bn == 0 && p.M >= 1024 &&
        (long long)((p.M + 255) / 256) * ((p.N + 255) / 256) >= di->num_sms / 2)
      return launch_gemm2_cfg<KIND, 256, 5>(A, B, p, di->num_sms, stream);
    return launch_gemm_cfg<KIND, 128, 6>(A, B, p, di->num_sms, stream);
  } else {
    if (force_bn < 0) {  // the CTA-pair kernel with tile width -force_bn
      switch (-force_bn) {
        case 256: return launch_gemm2_cfg<KIND, 256, 5>(A, B, p, di->num_sms, stream);
        case 192: return launch_gemm2_cfg<KIND, 192, 7>(A, B, p, di->num_sms, stream);
        case 128: return launch_gemm2_cfg<KIND, 128, 8>(A, B, p, di->num_sms, stream);
        default: return QI_B200_EINVAL;
      }
    }
    if (force_bn == 0) {
      // very few tiles over a long K (e.g. the DiT action expert's FFN-down,
      // M = 32, N = 1024, K = 4096: 12.5 -> 8.8 us): split K inside clusters
      const int bk = KIND == MmaKind::BF16 ? 64 : 128;
      const int k_blocks = (p.K + bk - 1) / bk;
      const int tiles128 = ((p.M + 127) / 128) * ((p.N + 127) / 128);
      if (tiles128 <= 16 && k_blocks >= 32) {
        int cbn, cs;
        csk_plan(static_cast<int>(KIND), p.M, p.N, p.K, di->num_sms, &cbn, &cs);
        if (cbn != 0) return launch_gemm_csk<KIND>(A, B, p, cbn, cs, stream);
      }
    }
    if (force_bn == 0 && p.M >= 1024 && p.tail_split != 1) {
      // long K with a partial last wave: CTA pairs with that wave split along
      // K (INT8 3120 x 3072 x 14336: 124 us on single-CTA 192-wide tiles,
      // 107 us as pairs with the split)
      const int bk = KIND == MmaKind::BF16 ? 64 : 128;
      const int ptiles = ((p.M + 255) / 256) * ((p.N + 255) / 256);
      if (ptiles >= di->num_sms / 2 && tail_plan(ptiles, di->num_sms / 2, (p.K + bk - 1) / bk, p.tail_split) > 1)
        return launch_gemm2_cfg<KIND, 256, 5>(A, B, p, di->num_sms, stream);
    }
    const int bn = force_bn > 0 ? force_bn : pick_bn(p.M, p.N, di->num_sms);
    // Large problems on 256-wide tiles run as CTA pairs (256 x 256 tiles on two
    // SMs): a third less L2 -> SMEM traffic per MMA.  Measured on B200: FP8
    // 4096x14336x3072 72 -> 78 %, INT8 3120x14336x3072 74 -> 81 %, BF16
    // 4096^3 77 -> 85 % of peak; small M stays on single-CTA tiles.
    if (force_bn == 0 && bn == 256 && p.M >= 1024 &&
        (long long)((p.M + 255) / 256) * ((p.N + 255) / 256) >= di->num_sms / 2)
      return launch_gemm2_cfg<KIND, 256, 5>(A, B, p, di->num_sms, stream);
    switch (bn) {
      case 256: return launch_gemm_cfg<KIND, 256, 4>(A, B, p, di->num_sms, stream);
      case 192: return launch_gemm_cfg<KIND, 192, 4>(A, B, p, di->num_sms, stream);
      case 128: return launch_gemm_cfg<KIND, 128, 6>(A, B, p, di->num_sms, stream);
      case 64: return launch_gemm_cfg<KIND, 64, 8>(A, B, p, di->num_sms, stream);
      default: return QI_B200_EINVAL;
    }
  }
}

static int check_gemm_args(int kind, const void* A, const void* B, const float* sa, int sa_stride, const float* sb,
                           int sb_stride, const void* bias, const void* D, long long ldd, int M, int N, int K,
                           int flags) {
  if (A == nullptr || B == nullptr || D == nullptr) return QI_B200_EINVAL;
  if (kind < 0 || kind > 2) return QI_B200_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0) return QI_B200_ESHAPE;
  const int elem = (kind == 2) ? 2 : 1;
  if (N % 8 != 0 || (K * elem) % 16 != 0) return QI_B200_ESHAPE;
  if (ldd < N || ldd % 8 != 0) return QI_B200_ESHAPE;
  if (!aligned16(A) || !aligned16(B) || !aligned16(D)) return QI_B200_EALIGN;
  if (bias != nullptr && !aligned16(bias)) return QI_B200_EALIGN;
  if (sb != nullptr && sb_stride != 0 && (sb_stride != 1 || !aligned16(sb))) return QI_B200_EALIGN;
  if (sa != nullptr && sa_stride < 0) return QI_B200_EINVAL;
  if (flags & ~(kEpiGelu | kEpiRawAcc)) return QI_B200_EINVAL;
  return QI_B200_OK;
}

// Workspace bytes the tail split of the GEMM that launch_gemm would run for
// this problem needs (0 when that launch does not split): the same kernel
// and tile choice as launch_gemm, then tail tiles x splits x 256 x BN words.
static size_t tail_ws_plan(int kind, int M, int N, int K, int mode, int force_bn, int num_sms) {
  if (mode == 1 || kind < 0 || kind > 2 || M <= 0 || N <= 0 || K <= 0 || force_bn > 0) return 0;
  const int bk = kind == QI_B200_KIND_BF16 ? 64 : 128;
  const int k_blocks = (K + bk - 1) / bk;
  const int pairs_max = num_sms / 2;
  int bn = 0;
  if (force_bn < 0) {
    bn = -force_bn;
  } else {
    const int tiles128 = ((M + 127) / 128) * ((N + 127) / 128);
    if (tiles128 <= 16 && k_blocks >= 32) {
      int cbn, cs;
      csk_plan(kind, M, N, K, num_sms, &cbn, &cs);
      if (cbn != 0) return 0;  // cluster split-K: no workspace
    }
    const long long ptiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    if (M >= 1024 && ptiles >= pairs_max) {
      if (tail_plan(static_cast<int>(ptiles), pairs_max, k_blocks, mode) > 1 || pick_bn(M, N, num_sms) == 256)
        bn = 256;
    }
  }
  if (bn == 0) return 0;
  const int tiles = ((M + 255) / 256) * ((N + bn - 1) / bn);
  const int pairs = tiles < pairs_max ? tiles : pairs_max;
  const int S = tail_plan(tiles, pairs, k_blocks, mode);
  return S > 1 ? static_cast<size_t>(tiles % pairs) * S * 256 * bn * 4 : 0;
}

// workspace == nullptr runs without the tail split (as tail mode 1).
static int gemm_dispatch(int kind, const void* A, const void* B, const float* sa, int sa_stride, const float* sb,
                         int sb_stride, const void* bias, void* D, long long ldd, int M, int N, int K, int flags,
                         int force_bn, cudaStream_t stream, void* workspace = nullptr, size_t workspace_bytes = 0) {
  int tail_mode = (flags >> QI_B200_TAIL_SPLIT_SHIFT) & 15;
  flags &= ~(15 << QI_B200_TAIL_SPLIT_SHIFT);
  int rc = check_gemm_args(kind, A, B, sa, sa_stride, sb, sb_stride, bias, D, ldd, M, N, K, flags);
  if (rc) return rc;
  if (workspace != nullptr && !aligned16(workspace)) return QI_B200_EALIGN;
  if (workspace == nullptr || workspace_bytes == 0) tail_mode = 1;
  EpiParams p{};
  p.tail_split = tail_mode;  // 0 automatic, 1 none, S >= 2 at most S (resolved by the pair launcher)
  p.tail_ws = static_cast<uint32_t*>(workspace);
  p.tail_ws_bytes = workspace_bytes;
  p.sa = sa;
  p.sa_stride = sa_stride;
  p.sb = sb;
  p.sb_stride = sb_stride;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.D = D;
  p.ldd = ldd;
  p.M = M;
  p.N = N;
  p.K = K;
  p.flags = flags;
  switch (kind) {
    case QI_B200_KIND_INT8: return launch_gemm<MmaKind::I8>(A, B, p, stream, force_bn);
    case QI_B200_KIND_FP8_E4M3: return launch_gemm<MmaKind::F8>(A, B, p, stream, force_bn);
    default: return launch_gemm<MmaKind::BF16>(A, B, p, stream, force_bn);
  }
}

static int quant_status(cudaError_t e) { return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA; }

// ---------------------------------------------------------------------------
// Peer memory for the column-parallel all-gather overlapped with the GEMM:
// buffers shared over CUDA IPC (plain device allocations, no multicast
// object), a bounded cross-GPU barrier on per-rank flag words, and an
// asynchronous copy (copy engine over NVLink) into a peer's buffer.
// ---------------------------------------------------------------------------

struct PeerFlags {
  unsigned int* flag[kMaxPeers];  // rank i's flag block: word j written by rank j; word kMaxPeers = i's counter
  int P, rank;
  unsigned long long timeout_ns;  // wait limit per lane
};

// One warp.  This rank's barrier counter (in its own flag block, so a CUDA
// graph replay advances it too) gives the epoch.  Lane i < P publishes the
// epoch in rank i's block (release, system scope), then waits (acquire,
// bounded by f.timeout_ns) until rank i has published the same epoch in
// this rank's block.  Every rank runs the same sequence of barriers.
__global__ void k_peer_barrier(PeerFlags f) {
  const int lane = threadIdx.x;
  unsigned int epoch = 0;
  if (lane == 0) {
    unsigned int* ctr = f.flag[f.rank] + kMaxPeers;
    epoch = *ctr + 1u;
    *ctr = epoch;
  }
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  if (lane < f.P) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.flag[lane] + f.rank), "r"(epoch) : "memory");
    const unsigned int* mine = f.flag[f.rank] + lane;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (static_cast<int>(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > f.timeout_ns) {
        record_error(kDevWaitTimeout, 0x300u, static_cast<unsigned int>(lane));
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
}

static_assert(sizeof(cudaIpcMemHandle_t) <= QI_B200_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int qi_b200_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes == 0) return QI_B200_EINVAL;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return QI_B200_ECUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return QI_B200_ECUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return QI_B200_ECUDA;
  }
  std::memset(ipc_handle, 0, QI_B200_IPC_HANDLE_BYTES);
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return QI_B200_OK;
}

extern "C" int qi_b200_peer_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return QI_B200_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

extern "C" int qi_b200_peer_close(void* ptr) {
  if (ptr == nullptr) return QI_B200_EINVAL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

extern "C" int qi_b200_peer_free(void* ptr) {
  if (ptr == nullptr) return QI_B200_EINVAL;
  return cudaFree(ptr) == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

extern "C" int qi_b200_peer_barrier_timed(void* const* flags, int P, int rank, unsigned long long timeout_ns,
                                          cudaStream_t stream) {
  if (flags == nullptr || P < 1 || P > kMaxPeers || rank < 0 || rank >= P) return QI_B200_EINVAL;
  if (timeout_ns == 0 || timeout_ns > QI_WAIT_TIMEOUT_NS) return QI_B200_EINVAL;
  PeerFlags f{};
  for (int i = 0; i < P; ++i) {
    if (flags[i] == nullptr || (reinterpret_cast<uintptr_t>(flags[i]) & 3u) != 0) return QI_B200_EALIGN;
    f.flag[i] = static_cast<unsigned int*>(flags[i]);
  }
  f.P = P;
  f.rank = rank;
  f.timeout_ns = timeout_ns;
  k_peer_barrier<<<1, 32, 0, stream>>>(f);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

extern "C" int qi_b200_peer_barrier(void* const* flags, int P, int rank, cudaStream_t stream) {
  return qi_b200_peer_barrier_timed(flags, P, rank, QI_WAIT_TIMEOUT_NS, stream);
}

extern "C" int qi_b200_gemm_gather(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                                   const float* b_scale, int b_scale_stride, const void* bias, void* const* dst,
                                   int ndst, long long ldd, int M, int N, int K, int flags, cudaStream_t stream) {
  if (dst == nullptr || ndst < 1 || ndst > kMaxPeers) return QI_B200_EINVAL;
  if (kind != QI_B200_KIND_INT8 && kind != QI_B200_KIND_FP8_E4M3 && kind != QI_B200_KIND_BF16) return QI_B200_EINVAL;
  if (flags & ~kEpiGelu) return QI_B200_EINVAL;  // bf16 outputs only
  for (int i = 0; i < ndst; ++i)
    if (dst[i] == nullptr || !aligned16(dst[i])) return QI_B200_EALIGN;
  int rc = check_gemm_args(kind, A, B, a_scale, a_scale_stride, b_scale, b_scale_stride, bias, dst[0], ldd, M, N, K,
                           flags);
  if (rc) return rc;
  DeviceInfo* di = nullptr;
  rc = device_info(&di);
  if (rc) return rc;
  OutMaps om = {};
  om.n = ndst;
  for (int i = 0; i < ndst; ++i) {
    rc = make_tmap_2d(&om.map[i], dst[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)N, (uint64_t)M,
                      (uint64_t)ldd * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  EpiParams p{};
  p.sa = a_scale;
  p.sa_stride = a_scale_stride;
  p.sb = b_scale;
  p.sb_stride = b_scale_stride;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.D = dst[0];
  p.ldd = ldd;
  p.M = M;
  p.N = N;
  p.K = K;
  p.flags = flags;
  switch (kind) {
    case QI_B200_KIND_INT8: return launch_gemm2_cfg<MmaKind::I8, 256, 5, true>(A, B, p, di->num_sms, stream, &om);
    case QI_B200_KIND_FP8_E4M3:
      return launch_gemm2_cfg<MmaKind::F8, 256, 5, true>(A, B, p, di->num_sms, stream, &om);
    default: return launch_gemm2_cfg<MmaKind::BF16, 256, 5, true>(A, B, p, di->num_sms, stream, &om);
  }
}

extern "C" int qi_b200_gemm_csk(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                                const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd,
                                int M, int N, int K, int flags, int tile_n, int splits, cudaStream_t stream) {
  int rc = check_gemm_args(kind, A, B, a_scale, a_scale_stride, b_scale, b_scale_stride, bias, D, ldd, M, N, K,
                           flags);
  if (rc) return rc;
  DeviceInfo* di = nullptr;
  rc = device_info(&di);
  if (rc) return rc;
  if (tile_n == 0 || splits == 0) {
    int bn, S;
    csk_plan(kind, M, N, K, di->num_sms, &bn, &S);
    if (bn == 0) return QI_B200_ESHAPE;
    if (tile_n == 0) tile_n = bn;
    if (splits == 0) splits = S;
  }
  EpiParams p{};
  p.sa = a_scale;
  p.sa_stride = a_scale_stride;
  p.sb = b_scale;
  p.sb_stride = b_scale_stride;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.D = D;
  p.ldd = ldd;
  p.M = M;
  p.N = N;
  p.K = K;
  p.flags = flags;
  switch (kind) {
    case QI_B200_KIND_INT8: return launch_gemm_csk<MmaKind::I8>(A, B, p, tile_n, splits, stream);
    case QI_B200_KIND_FP8_E4M3: return launch_gemm_csk<MmaKind::F8>(A, B, p, tile_n, splits, stream);
    default: return launch_gemm_csk<MmaKind::BF16>(A, B, p, tile_n, splits, stream);
  }
}

// ---------------------------------------------------------------------------
// NVFP4
// ---------------------------------------------------------------------------
static int nvfp4_quantize(const void* x, int rows, int cols, int g_mode, const float* g_in, unsigned int* ws_amax,
                          float* g_out, void* q, void* sf, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return QI_B200_ESHAPE;
  if (cols % 64 != 0) return QI_B200_ESHAPE;
  if (x == nullptr || q == nullptr || sf == nullptr) return QI_B200_EINVAL;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) || !aligned16(sf)) return QI_B200_EALIGN;
  if (g_mode == 0 && g_in == nullptr) return QI_B200_EINVAL;
  if (g_mode == 1 && (ws_amax == nullptr || g_out == nullptr)) return QI_B200_EINVAL;
  if (g_mode == 2 && g_out == nullptr) return QI_B200_EINVAL;
  if (g_mode < 0 || g_mode > 2) return QI_B200_EINVAL;
  if ((long long)((rows + 127) & ~127) * (cols / 16) >= (1ll << 31)) return QI_B200_ESHAPE;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  const int ka = cols / 64;
  const int rows_pad = (rows + 127) & ~127;
  const long long blocks = (long long)rows_pad * (cols / 16);
  // the tensor-scale kernels walk x from its end in grid-stride order: a grid
  // of exactly the resident blocks keeps that order (all blocks run together)
  static int occ[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (occ[dev] == 0) {
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_quant_nvfp4_tensor<1>, 256, 0) != cudaSuccess || o < 1)
      o = 4;
    occ[dev] = o;
  }
  const int grid_flat = (int)std::min<long long>((blocks + 255) / 256, (long long)di->num_sms * occ[dev]);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  auto* sb = static_cast<uint8_t*>(sf);
  if (g_mode == 1) {
    const long long n = (long long)rows * cols;
    const int g2 = (int)std::min<long long>(
        std::min<long long>((n / 8 + 255) / 256 + 1, (long long)di->num_sms * 8), kAmaxParts);
    // per-block maxima in this stream's slot, reduced by the last block: no
    // memset of ws_amax (and no graph node that breaks the launch chain)
    unsigned int *part = nullptr, *ticket = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_dev_mu);
      const int slot = stream_slot(di, stream);
      if (slot >= 0) {
        part = di->amax_part + static_cast<size_t>(slot) * kAmaxParts;
        ticket = di->amax_ticket + slot;
      }
    }
    if (part == nullptr && cudaMemsetAsync(ws_amax, 0, sizeof(unsigned int), stream) != cudaSuccess)
      return QI_B200_ECUDA;
    launch_pdl(k_amax_bf16, dim3(g2), dim3(256), 0, stream, 1, xb, n, ws_amax, part, ticket);
    launch_pdl(k_quant_nvfp4_tensor<1>, dim3(grid_flat), dim3(256), 0, stream, 1, xb, rows, cols,
               static_cast<const float*>(nullptr), static_cast<const unsigned int*>(ws_amax), g_out, qb, sb, ka);
    count_launches(2);
  } else if (g_mode == 0) {
    launch_pdl(k_quant_nvfp4_tensor<0>, dim3(grid_flat), dim3(256), 0, stream, 1, xb, rows, cols, g_in,
               static_cast<const unsigned int*>(nullptr), static_cast<float*>(nullptr), qb, sb, ka);
    count_launches(1);
  } else {
    const int g3 = std::min(rows_pad, di->num_sms * 8);
    launch_pdl(k_quant_nvfp4<2>, dim3(g3), dim3(256), 0, stream, 1, xb, rows, cols,
               static_cast<const float*>(nullptr), static_cast<const unsigned int*>(nullptr), g_out, qb, sb, ka);
    count_launches(1);
  }
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

static int nvfp4_gemm(const void* A, const void* SFA, const void* B, const void* SFB, const float* a_g,
                      int a_g_stride, const float* b_g, const void* bias, void* D, long long ldd, int M, int N, int K,
                      int flags, cudaStream_t stream) {
  if (A == nullptr || B == nullptr || SFA == nullptr || SFB == nullptr || D == nullptr) return QI_B200_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0) return QI_B200_ESHAPE;
  if (K % 256 != 0 || N % 8 != 0 || ldd < N || ldd % 8 != 0) return QI_B200_ESHAPE;
  if (!aligned16(A) || !aligned16(B) || !aligned16(D) || !aligned16(SFA) || !aligned16(SFB)) return QI_B200_EALIGN;
  const int tile = (flags >> QI_B200_NVFP4_TILE_SHIFT) & 3;
  flags &= ~(3 << QI_B200_NVFP4_TILE_SHIFT);
  if (flags & ~(kEpiGelu | kEpiRawAcc)) return QI_B200_EINVAL;
  EpiParams p = {};
  p.sa = a_g;
  p.sa_stride = a_g_stride;
  p.sb = b_g;
  p.sb_stride = 0;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.D = D;
  p.ldd = ldd;
  p.M = M;
  p.N = N;
  p.K = K;
  p.flags = flags;
  p.sfa = static_cast<const uint8_t*>(SFA);
  p.sfb = static_cast<const uint8_t*>(SFB);
  p.sf_ka = K / 64;
  static const int kTileForce[4] = {0, 128, -128, -256};
  return launch_gemm<MmaKind::NVF4>(A, B, p, stream, kTileForce[tile]);
}

// ---------------------------------------------------------------------------
// W4A16 launch: skinny split-K kernel for M <= 256, 256x128 tiles above.
// ---------------------------------------------------------------------------
template <int MP>
static int launch_w4_skinny(const void* X, const EpiParams& p, const W4Params& q,
                            int num_sms, cudaStream_t stream) {
  using C = W4Cfg<MP>;
  CUtensorMap tx;
  int rc = make_tmap_2d(&tx, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.K * 2,
                        w4::BK, MP);
  if (rc) return rc;
  static bool attr_done[kMaxDevices] = {};
  int adev = 0;
  cudaGetDevice(&adev);
  if (!attr_done[adev]) {
    if (cudaFuncSetAttribute(k_gemm_w4a16_skinny<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM_BYTES) != cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[adev] = true;
  }
  const int n_tiles = (p.N + w4::BN - 1) / w4::BN;
  const int k_blocks = (p.K + w4::BK - 1) / w4::BK;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(w4::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // K split = cluster size: the largest (<= 8) for which every cluster of
  // the grid is resident at once (cluster placement is per GPC, so this is
  // asked of the occupancy API rather than derived from the SM count).
  static int ks_cache[kMaxDevices][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int key = n_tiles < 64 ? n_tiles : 63;
  int ks = ks_cache[dev][key];
  if (ks == 0) {
    ks = 1;
    for (int cand = 8; cand >= 2; --cand) {
      if (cand > k_blocks || n_tiles * cand > num_sms) continue;
      int nclusters = 0;
      attr[0].val.clusterDim.x = cand;
      cfg.gridDim = dim3(n_tiles * cand, 1, 1);
      if (cudaOccupancyMaxActiveClusters(&nclusters, k_gemm_w4a16_skinny<MP>, &cfg) == cudaSuccess &&
          nclusters >= n_tiles) {
        ks = cand;
        break;
      }
    }
    cudaGetLastError();  // clear a failed occupancy query
    ks_cache[dev][key] = ks;
  }
  if (ks > k_blocks) ks = k_blocks;
  const int kbc = (k_blocks + ks - 1) / ks;
  ks = (k_blocks + kbc - 1) / kbc;  // every CTA of the cluster gets >= 1 K block
  cfg.gridDim = dim3(n_tiles * ks, 1, 1);
  attr[0].val.clusterDim.x = ks;
  g_last_plan = {kPlanW4Skinny, n_tiles * ks, ks, MP, C::STAGES, C::SMEM_BYTES};
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_w4a16_skinny<MP>, tx, p, q, kbc);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

template <int NT, int KS>
static int launch_w4_small(const void* X, const EpiParams& p, const W4Params& q, cudaStream_t stream) {
  const W4sLayout L = w4s_layout(NT, KS, p.M, p.K, q.G, q.zw, q.group);
  if (L.total > 200 * 1024) return QI_B200_ESHAPE;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(k_gemm_w4a16_small<NT, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024) != cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[dev] = true;
  }
  const int blocks = (p.N + 8 * NT - 1) / (8 * NT);
  g_last_plan = {kPlanW4Small, blocks * KS, KS, p.M, 0, L.total};
  const cudaError_t e = launch_pdl(k_gemm_w4a16_small<NT, KS>, dim3(blocks * KS), dim3(w4s::kThreads), L.total,
                                   stream, KS, static_cast<const __nv_bfloat16*>(X), p, q);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

static int launch_w4a16(const void* X, const void* wq, const void* scales, const void* zeros, int group,
                        const void* bias, void* D, long long ldd, int M, int N, int K, cudaStream_t stream) {
  if (X == nullptr || wq == nullptr || scales == nullptr || zeros == nullptr || D == nullptr) return QI_B200_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0) return QI_B200_ESHAPE;
  if (group <= 0 || group > K) group = K;
  if (K % 32 != 0 || N % 8 != 0 || group % 32 != 0) return QI_B200_ESHAPE;
  if (ldd < N || ldd % 8 != 0) return QI_B200_ESHAPE;
  if (!aligned16(X) || !aligned16(wq) || !aligned16(D)) return QI_B200_EALIGN;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  EpiParams p = {};
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.D = D;
  p.ldd = ldd;
  p.M = M;
  p.N = N;
  p.K = K;
  W4Params q;
  q.G = (K + group - 1) / group;
  q.zw = (q.G + 7) / 8;
  q.group = group;
  q.group_shift = ((group & (group - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(group)) : -1;
  q.scales = static_cast<const __half*>(scales);
  q.zeros = static_cast<const int32_t*>(zeros);
  q.wq = static_cast<const int32_t*>(wq);
  q.kw = K / 8;
  if (M <= w4s::kMaxM && group >= 32 && group <= 256 && (group & (group - 1)) == 0 && K % (8 * group) == 0 &&
      aligned16(scales) && aligned16(zeros)) {
    // small M (3072 x 3072, g128, compared in one process): one token, one
    // column of CTAs (5.2 us against 7.0 as CTA pairs); more, CTA pairs
    // splitting K (M = 4 / 16: 6.7 / 8.4 us against 13.0 on one column / 9.8
    // on clusters of 4)
    if (M <= 1) rc = launch_w4_small<1, 1>(X, p, q, stream);
    else rc = launch_w4_small<2, 2>(X, p, q, stream);
    if (rc != QI_B200_ESHAPE) return rc;  // ESHAPE: shared memory too small, use the split-K kernel
  }
  if (M <= 16) return launch_w4_skinny<16>(X, p, q, di->num_sms, stream);
  if (M <= 32) return launch_w4_skinny<32>(X, p, q, di->num_sms, stream);
  if (M <= 64) return launch_w4_skinny<64>(X, p, q, di->num_sms, stream);
  if (M <= 128) return launch_w4_skinny<128>(X, p, q, di->num_sms, stream);
  if (M <= 256) return launch_w4_skinny<256>(X, p, q, di->num_sms, stream);
  // M > 256 without a workspace (qi_b200_w4a16_linear): the skinny kernel
  // over 256-row blocks of x.  With a workspace, qi_b200_w4a16_linear_ws
  // dequantizes the weights once instead, which is faster at these M.
  const auto* xb = static_cast<const __nv_bfloat16*>(X);
  auto* db = static_cast<__nv_bfloat16*>(D);
  for (int m0 = 0; m0 < M; m0 += 256) {
    EpiParams pc = p;
    pc.M = std::min(256, M - m0);
    pc.D = db + static_cast<long long>(m0) * ldd;
    const void* xc = xb + static_cast<long long>(m0) * K;
    rc = pc.M <= 128 ? launch_w4_skinny<128>(xc, pc, q, di->num_sms, stream)
                     : launch_w4_skinny<256>(xc, pc, q, di->num_sms, stream);
    if (rc) return rc;
  }
  return QI_B200_OK;
}

}  // namespace qib

using namespace qib;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int qi_b200_abi_version(void) { return QI_B200_ABI_VERSION; }

const char* qi_b200_error_string(int code) {
  switch (code) {
    case QI_B200_OK: return "ok";
    case QI_B200_EINVAL: return "invalid argument";
    case QI_B200_ESHAPE: return "unsupported shape (need M,N,K > 0, N % 8 == 0, K*elem % 16 == 0)";
    case QI_B200_EALIGN: return "pointer not 16-byte aligned";
    case QI_B200_ECUDA: return "CUDA launch error";
    case QI_B200_ETMAP: return "TMA descriptor encoding failed";
    case QI_B200_EARCH: return "current device is not sm_100 (B200)";
    case QI_B200_ETOOBIG: return "size exceeds the entry point's fixed maximum";
    default: return "unknown status";
  }
}

int qi_b200_launch_count(unsigned long long* out) {
  if (out == nullptr) return QI_B200_EINVAL;
  *out = launch_counter().load(std::memory_order_relaxed);
  return QI_B200_OK;
}

int qi_b200_last_launch(int* out6) {
  if (out6 == nullptr) return QI_B200_EINVAL;
  const LaunchPlan& p = g_last_plan;
  const int v[6] = {p.kernel, p.grid, p.cluster, p.tile_n, p.stages, p.smem};
  for (int i = 0; i < 6; ++i) out6[i] = v[i];
  return QI_B200_OK;
}

int qi_b200_last_tail_split(void) { return g_last_tail; }

int qi_b200_device_status(unsigned int* out4, int clear) {
  unsigned int h[4] = {0, 0, 0, 0};
  if (cudaMemcpyFromSymbol(h, g_status, sizeof(h)) != cudaSuccess) return QI_B200_ECUDA;
  if (out4 != nullptr)
    for (int i = 0; i < 4; ++i) out4[i] = h[i];
  if (clear) {
    unsigned int z[4] = {0, 0, 0, 0};
    if (cudaMemcpyToSymbol(g_status, z, sizeof(z)) != cudaSuccess) return QI_B200_ECUDA;
    if (h[0] != 0) {  // an aborted launch may have left its slot counters raised
      static const unsigned int zc[kTailSlots][2 * kMaxTailTiles] = {};
      static const unsigned int zt[kTailSlots] = {};
      if (cudaMemcpyToSymbol(g_tail_cnt, zc, sizeof(zc)) != cudaSuccess) return QI_B200_ECUDA;
      if (cudaMemcpyToSymbol(g_amax_ticket, zt, sizeof(zt)) != cudaSuccess) return QI_B200_ECUDA;
    }
  }
  return QI_B200_OK;
}

int qi_b200_quantize_int8_rowwise(const void* x_bf16, void* q_int8, float* scales, int rows, int cols,
                                  cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (rows == 0 || cols == 0) return QI_B200_OK;
  if (x_bf16 == nullptr || q_int8 == nullptr || scales == nullptr) return QI_B200_EINVAL;
  return quant_status(launch_rowquant<QuantInt8>(x_bf16, q_int8, scales, nullptr, rows, cols, stream));
}

int qi_b200_quantize_int8_rowwise_smooth(const void* x_bf16, const float* input_scale, void* q_int8, float* scales,
                                         int rows, int cols, cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (x_bf16 == nullptr || input_scale == nullptr || q_int8 == nullptr || scales == nullptr) return QI_B200_EINVAL;
  return quant_status(launch_rowquant<QuantInt8>(x_bf16, q_int8, scales, nullptr, rows, cols, stream, input_scale));
}

int qi_b200_quantize_int8_rowwise_given(const void* x_bf16, const float* scales, void* q_int8, int rows, int cols,
                                        cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (rows == 0 || cols == 0) return QI_B200_OK;
  if (x_bf16 == nullptr || q_int8 == nullptr || scales == nullptr) return QI_B200_EINVAL;
  return quant_status(
      launch_rowquant<QuantInt8Given>(x_bf16, q_int8, const_cast<float*>(scales), nullptr, rows, cols, stream));
}

int qi_b200_resid_ln_quant(void* x_bf16, const void* y_bf16, long long ldy, const void* gate, const void* ln_w,
                           const void* ln_b, const void* mod_scale1, const void* mod_shift, void* q_int8,
                           float* scales, void* xn_bf16, int M, int D, float eps, cudaStream_t stream) {
  if (M < 0 || D <= 0) return QI_B200_ESHAPE;
  if (M == 0) return QI_B200_OK;
  if (x_bf16 == nullptr) return QI_B200_EINVAL;
  if (D % 8 != 0 || D > kRowMaxThreads * 8) return QI_B200_ESHAPE;
  if ((ln_w == nullptr) != (ln_b == nullptr) || (mod_scale1 == nullptr) != (mod_shift == nullptr) ||
      (q_int8 != nullptr && scales == nullptr) || (y_bf16 == nullptr && gate != nullptr))
    return QI_B200_EINVAL;
  if (y_bf16 != nullptr && (ldy < D || ldy % 8 != 0)) return QI_B200_ESHAPE;
  const void* ptrs[] = {x_bf16, y_bf16, gate, ln_w, ln_b, mod_scale1, mod_shift, xn_bf16};
  for (const void* ptr : ptrs)
    if (ptr != nullptr && !aligned16(ptr)) return QI_B200_EALIGN;
  if (q_int8 != nullptr && (reinterpret_cast<uintptr_t>(q_int8) & 7u) != 0) return QI_B200_EALIGN;
  ResLnParams p;
  p.x = static_cast<__nv_bfloat16*>(x_bf16);
  p.y = static_cast<const __nv_bfloat16*>(y_bf16);
  p.ldy = ldy;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.ln_w = static_cast<const __nv_bfloat16*>(ln_w);
  p.ln_b = static_cast<const __nv_bfloat16*>(ln_b);
  p.mod_scale1 = static_cast<const __nv_bfloat16*>(mod_scale1);
  p.mod_shift = static_cast<const __nv_bfloat16*>(mod_shift);
  p.q = static_cast<int8_t*>(q_int8);
  p.s = scales;
  p.xn = static_cast<__nv_bfloat16*>(xn_bf16);
  p.M = M;
  p.D = D;
  p.eps = eps;
  const int wgrid = (M + kWarpRowThreads / 32 - 1) / (kWarpRowThreads / 32);
  switch (D) {  // warp per row where the row splits into whole 256-element slices
    case 1024: launch_pdl(k_resid_ln_quant_warp<4>, dim3(wgrid), dim3(kWarpRowThreads), 5 * 1024 * 2, stream, 1, p); break;
    case 2048: launch_pdl(k_resid_ln_quant_warp<8>, dim3(wgrid), dim3(kWarpRowThreads), 5 * 2048 * 2, stream, 1, p); break;
    case 3072: launch_pdl(k_resid_ln_quant_warp<12>, dim3(wgrid), dim3(kWarpRowThreads), 5 * 3072 * 2, stream, 1, p); break;
    case 4096: launch_pdl(k_resid_ln_quant_warp<16>, dim3(wgrid), dim3(kWarpRowThreads), 5 * 4096 * 2, stream, 1, p); break;
    default: launch_pdl(k_resid_ln_quant<1>, dim3(M), dim3(row_threads(D)), 0, stream, 1, p);
  }
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

}  // extern "C"

namespace qib {

// k_rms_rope_heads<C, MODE> for C = ceil(A / 256) chunks per lane (A <= 4096).
template <int MODE>
static cudaError_t launch_rms_heads(const RmsRopeParams& p, int nparts, cudaStream_t stream) {
  const dim3 grid((p.M + kWarpRowThreads / 32 - 1) / (kWarpRowThreads / 32), nparts);
  const size_t smem = MODE == 1 ? 0 : static_cast<size_t>(p.A) * 2;
  switch ((p.A + 255) / 256) {
#define QI_RMS_HEADS_CASE(c) \
  case c: return launch_pdl(k_rms_rope_heads<c, MODE>, grid, dim3(kWarpRowThreads), smem, stream, 1, p);
    QI_RMS_HEADS_CASE(1) QI_RMS_HEADS_CASE(2) QI_RMS_HEADS_CASE(3) QI_RMS_HEADS_CASE(4)
    QI_RMS_HEADS_CASE(5) QI_RMS_HEADS_CASE(6) QI_RMS_HEADS_CASE(7) QI_RMS_HEADS_CASE(8)
    QI_RMS_HEADS_CASE(9) QI_RMS_HEADS_CASE(10) QI_RMS_HEADS_CASE(11) QI_RMS_HEADS_CASE(12)
    QI_RMS_HEADS_CASE(13) QI_RMS_HEADS_CASE(14) QI_RMS_HEADS_CASE(15) QI_RMS_HEADS_CASE(16)
#undef QI_RMS_HEADS_CASE
    default: return cudaErrorInvalidValue;
  }
}

static bool rms_heads_ok(int A, int head_dim) {
  return head_dim >= 8 && head_dim <= 256 && (head_dim & (head_dim - 1)) == 0 && A % head_dim == 0 && A <= 4096;
}

// Shared argument checks and parameter block of the RMSNorm entry points.
static int rms_params(RmsRopeParams* p, const void* in0, const void* in1, long long ld_in, void* out0, void* out1,
                      long long ld_out, const void* w0, const void* w1, const float* rope, int head_dim, int nparts,
                      int M, int A, float eps, bool need_out) {
  if (M < 0 || A <= 0 || nparts < 1 || nparts > 2) return QI_B200_ESHAPE;
  if (A % 8 != 0 || A > kRowMaxThreads * 8 || ld_in < A || ld_in % 8) return QI_B200_ESHAPE;
  if (need_out && (ld_out < A || ld_out % 8)) return QI_B200_ESHAPE;
  if (rope != nullptr && (head_dim <= 0 || head_dim % 8 != 0 || A % head_dim != 0)) return QI_B200_ESHAPE;
  const void* ins[2] = {in0, in1};
  void* outs[2] = {out0, out1};
  const void* ws[2] = {w0, w1};
  for (int i = 0; i < nparts; ++i) {
    if (ins[i] == nullptr || (need_out && (outs[i] == nullptr || ws[i] == nullptr))) return QI_B200_EINVAL;
    if (!aligned16(ins[i]) || (need_out && (!aligned16(outs[i]) || !aligned16(ws[i])))) return QI_B200_EALIGN;
  }
  if (rope != nullptr && !aligned16(rope)) return QI_B200_EALIGN;
  for (int i = 0; i < 2; ++i) {
    const int k = i < nparts ? i : 0;
    p->in[i] = static_cast<const __nv_bfloat16*>(ins[k]);
    p->out[i] = static_cast<__nv_bfloat16*>(outs[k]);
    p->w[i] = static_cast<const __nv_bfloat16*>(ws[k]);
  }
  p->ld_in = ld_in;
  p->ld_out = ld_out;
  p->rope = rope;
  p->pairs_per_head = rope != nullptr ? head_dim / 2 : 1;
  p->M = M;
  p->A = A;
  p->eps = eps;
  p->head_dim = head_dim;
  p->part_out = nullptr;
  p->part_in = nullptr;
  p->ranks = 1;
  return QI_B200_OK;
}

}  // namespace qib

extern "C" {

int qi_b200_rms_head_partials(const void* in0, const void* in1, long long ld_in, float* partials, int head_dim,
                              int nparts, int M, int A, cudaStream_t stream) {
  RmsRopeParams p;
  int rc = rms_params(&p, in0, in1, ld_in, nullptr, nullptr, 0, nullptr, nullptr, nullptr, head_dim, nparts, M, A,
                      0.f, false);
  if (rc) return rc;
  if (!rms_heads_ok(A, head_dim)) return QI_B200_ESHAPE;
  if (partials == nullptr) return QI_B200_EINVAL;
  if (M == 0) return QI_B200_OK;
  p.part_out = partials;
  const cudaError_t e = launch_rms_heads<1>(p, nparts, stream);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_rms_rope_partials(const void* in0, const void* in1, long long ld_in, void* out0, void* out1,
                              long long ld_out, const void* w0, const void* w1, const float* rope, int head_dim,
                              int nparts, int M, int A, const float* partials, int ranks, float eps,
                              cudaStream_t stream) {
  RmsRopeParams p;
  int rc = rms_params(&p, in0, in1, ld_in, out0, out1, ld_out, w0, w1, rope, head_dim, nparts, M, A, eps, true);
  if (rc) return rc;
  if (!rms_heads_ok(A, head_dim)) return QI_B200_ESHAPE;
  if (partials == nullptr || ranks < 1 || ranks > kMaxPeers) return QI_B200_EINVAL;
  if (M == 0) return QI_B200_OK;
  p.part_in = partials;
  p.ranks = ranks;
  const cudaError_t e = launch_rms_heads<2>(p, nparts, stream);
  count_launches(1);
  return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_rms_rope(const void* in0, const void* in1, long long ld_in, void* out0, void* out1, long long ld_out,
                     const void* w0, const void* w1, const float* rope, int head_dim, int nparts, int M, int A,
                     float eps, cudaStream_t stream) {
  if (rms_heads_ok(A, head_dim)) {  // the head-order reduction (same bits however the heads are split)
    RmsRopeParams p;
    int rc = rms_params(&p, in0, in1, ld_in, out0, out1, ld_out, w0, w1, rope, head_dim, nparts, M, A, eps, true);
    if (rc) return rc;
    if (M == 0) return QI_B200_OK;
    const cudaError_t e = launch_rms_heads<0>(p, nparts, stream);
    count_launches(1);
    return e == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
  }
  if (M < 0 || A <= 0 || nparts < 1 || nparts > 2) return QI_B200_ESHAPE;
  if (M == 0) return QI_B200_OK;
  if (A % 8 != 0 || A > kRowMaxThreads * 8 || ld_in < A || ld_out < A || ld_in % 8 || ld_out % 8)
    return QI_B200_ESHAPE;
  if (rope != nullptr && (head_dim <= 0 || head_dim % 8 != 0 || A % head_dim != 0)) return QI_B200_ESHAPE;
  const void* ins[2] = {in0, in1};
  void* outs[2] = {out0, out1};
  const void* ws[2] = {w0, w1};
  RmsRopeParams p;
  for (int i = 0; i < nparts; ++i) {
    if (ins[i] == nullptr || outs[i] == nullptr || ws[i] == nullptr) return QI_B200_EINVAL;
    if (!aligned16(ins[i]) || !aligned16(outs[i]) || !aligned16(ws[i])) return QI_B200_EALIGN;
  }
  if (rope != nullptr && !aligned16(rope)) return QI_B200_EALIGN;
  for (int i = 0; i < 2; ++i) {
    p.in[i] = static_cast<const __nv_bfloat16*>(ins[i < nparts ? i : 0]);
    p.out[i] = static_cast<__nv_bfloat16*>(outs[i < nparts ? i : 0]);
    p.w[i] = static_cast<const __nv_bfloat16*>(ws[i < nparts ? i : 0]);
  }
  p.ld_in = ld_in;
  p.ld_out = ld_out;
  p.rope = rope;
  p.pairs_per_head = rope != nullptr ? head_dim / 2 : 1;
  p.M = M;
  p.A = A;
  p.eps = eps;
  const dim3 wgrid((M + kWarpRowThreads / 32 - 1) / (kWarpRowThreads / 32), nparts);
  switch (A) {
    case 1024: launch_pdl(k_rms_rope_warp<4>, wgrid, dim3(kWarpRowThreads), 1024 * 2, stream, 1, p); break;
    case 2048: launch_pdl(k_rms_rope_warp<8>, wgrid, dim3(kWarpRowThreads), 2048 * 2, stream, 1, p); break;
    case 3072: launch_pdl(k_rms_rope_warp<12>, wgrid, dim3(kWarpRowThreads), 3072 * 2, stream, 1, p); break;
    case 4096: launch_pdl(k_rms_rope_warp<16>, wgrid, dim3(kWarpRowThreads), 4096 * 2, stream, 1, p); break;
    default: launch_pdl(k_rms_rope<1>, dim3(M, nparts), dim3(row_threads(A)), 0, stream, 1, p);
  }
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_int8_row_scales(const void* x_bf16, float* scales, int rows, int cols, cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (rows == 0 || cols == 0) return QI_B200_OK;
  if (x_bf16 == nullptr || scales == nullptr) return QI_B200_EINVAL;
  return quant_status(launch_rowquant<QuantInt8ScalesOnly>(x_bf16, nullptr, scales, nullptr, rows, cols, stream));
}

int qi_b200_int8_epilogue(const void* acc_int32, const float* act_scale, const float* weight_scale,
                          const void* bias, void* out_bf16, int M, int N, int flags, cudaStream_t stream) {
  if (M < 0 || N < 0) return QI_B200_ESHAPE;
  if (M == 0 || N == 0) return QI_B200_OK;
  if (acc_int32 == nullptr || act_scale == nullptr || weight_scale == nullptr || out_bf16 == nullptr)
    return QI_B200_EINVAL;
  if (flags & ~kEpiGelu) return QI_B200_EINVAL;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  const long long total = (long long)M * N;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)di->num_sms * 8);
  k_int8_epilogue<<<grid, 256, 0, stream>>>(static_cast<const int32_t*>(acc_int32), act_scale, weight_scale,
                                             static_cast<const __nv_bfloat16*>(bias),
                                             static_cast<__nv_bfloat16*>(out_bf16), M, N, flags & kEpiGelu);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_quantize_fp8_rowwise(const void* x_bf16, void* q_fp8, float* scales, int rows, int cols,
                                 cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (rows == 0 || cols == 0) return QI_B200_OK;
  if (x_bf16 == nullptr || q_fp8 == nullptr || scales == nullptr) return QI_B200_EINVAL;
  return quant_status(launch_rowquant<QuantFp8>(x_bf16, q_fp8, scales, nullptr, rows, cols, stream));
}

int qi_b200_quantize_fp8_static(const void* x_bf16, const float* scale, void* q_fp8, int rows, int cols,
                                cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QI_B200_ESHAPE;
  if (rows == 0 || cols == 0) return QI_B200_OK;
  if (x_bf16 == nullptr || q_fp8 == nullptr || scale == nullptr) return QI_B200_EINVAL;
  return quant_status(launch_rowquant<QuantFp8Static>(x_bf16, q_fp8, nullptr, scale, rows, cols, stream));
}

int qi_b200_gemm(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                 const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd, int M, int N,
                 int K, int flags, int tile_n, cudaStream_t stream) {
  return gemm_dispatch(kind, A, B, a_scale, a_scale_stride, b_scale, b_scale_stride, bias, D, ldd, M, N, K, flags,
                       tile_n, stream);
}

int qi_b200_gemm_ws(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                    const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd, int M, int N,
                    int K, int flags, int tile_n, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return gemm_dispatch(kind, A, B, a_scale, a_scale_stride, b_scale, b_scale_stride, bias, D, ldd, M, N, K, flags,
                       tile_n, stream, workspace, workspace_bytes);
}

int qi_b200_gemm_workspace_bytes(int kind, int M, int N, int K, int flags, int tile_n, size_t* bytes) {
  if (bytes == nullptr) return QI_B200_EINVAL;
  *bytes = 0;
  if (kind < 0 || kind > 2) return QI_B200_EINVAL;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  *bytes = tail_ws_plan(kind, M, N, K, (flags >> QI_B200_TAIL_SPLIT_SHIFT) & 15, tile_n, di->num_sms);
  return QI_B200_OK;
}

int qi_b200_int8_rowwise_bf16out(const void* A, const void* B, const void* act_scale, const void* weight_scale,
                                 void* D, int M, int N, int K, cudaStream_t stream) {
  return gemm_dispatch(QI_B200_KIND_INT8, A, B, static_cast<const float*>(act_scale), 1,
                       static_cast<const float*>(weight_scale), 1, nullptr, D, N, M, N, K, 0, 0, stream);
}

int qi_b200_int8_rowwise_bf16out_bias(const void* A, const void* B, const void* act_scale, const void* weight_scale,
                                      const void* bias, void* D, int M, int N, int K, cudaStream_t stream) {
  return gemm_dispatch(QI_B200_KIND_INT8, A, B, static_cast<const float*>(act_scale), 1,
                       static_cast<const float*>(weight_scale), 1, bias, D, N, M, N, K, 0, 0, stream);
}

int qi_b200_w4a16_linear(const void* x_bf16, const void* qweight_packed, const void* scales_fp16,
                         const void* zeros_packed, int group_size, const void* bias, void* out_bf16, int M, int N,
                         int K, cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  return launch_w4a16(x_bf16, qweight_packed, scales_fp16, zeros_packed, group_size, bias, out_bf16, N, M, N, K,
                      stream);
}

int qi_b200_w4a16_dequant(const void* qweight_packed, const void* scales_fp16, const void* zeros_packed,
                          int group_size, void* out_bf16, int N, int K, cudaStream_t stream) {
  if (qweight_packed == nullptr || scales_fp16 == nullptr || zeros_packed == nullptr || out_bf16 == nullptr)
    return QI_B200_EINVAL;
  if (N <= 0 || K <= 0) return QI_B200_ESHAPE;
  int group = group_size;
  if (group <= 0 || group > K) group = K;
  if (K % 32 != 0 || group % 32 != 0 || (long long)N * (K / 32) >= (1ll << 31)) return QI_B200_ESHAPE;
  if (!aligned16(out_bf16) || !aligned16(qweight_packed)) return QI_B200_EALIGN;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  W4Params q;
  q.G = (K + group - 1) / group;
  q.zw = (q.G + 7) / 8;
  q.group = group;
  q.group_shift = ((group & (group - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(group)) : -1;
  q.scales = static_cast<const __half*>(scales_fp16);
  q.zeros = static_cast<const int32_t*>(zeros_packed);
  q.wq = static_cast<const int32_t*>(qweight_packed);
  q.kw = K / 8;
  const long long quads = (long long)N * (K / 32);
  const int grid = (int)std::min<long long>((quads + 255) / 256, (long long)di->num_sms * 16);
  launch_pdl(k_w4a16_dequant, dim3(grid), dim3(256), 0, stream, 1, q, static_cast<__nv_bfloat16*>(out_bf16), N, K);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_w4a16_linear_ws(const void* x_bf16, const void* qweight_packed, const void* scales_fp16,
                            const void* zeros_packed, int group_size, const void* bias, void* out_bf16, int M, int N,
                            int K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (M < QI_B200_W4A16_DEQUANT_MIN_M || workspace == nullptr || workspace_bytes < (size_t)N * K * 2)
    return launch_w4a16(x_bf16, qweight_packed, scales_fp16, zeros_packed, group_size, bias, out_bf16, N, M, N, K,
                        stream);
  // large M: the weights are dequantized once into the workspace, then a bf16
  // tcgen05 GEMM (the dequantized tile would otherwise be rebuilt for every
  // M tile)
  int rc = qi_b200_w4a16_dequant(qweight_packed, scales_fp16, zeros_packed, group_size, workspace, N, K, stream);
  if (rc) return rc;
  return gemm_dispatch(QI_B200_KIND_BF16, x_bf16, workspace, nullptr, 0, nullptr, 0, bias, out_bf16, N, M, N, K, 0,
                       0, stream);
}

int qi_b200_wo_dequant(const void* qweight_int8, const float* scales, const void* zeros_int16, int group_size,
                       void* out_bf16, int N, int K, cudaStream_t stream) {
  if (qweight_int8 == nullptr || scales == nullptr || out_bf16 == nullptr) return QI_B200_EINVAL;
  if (N <= 0 || K <= 0 || K % 16 != 0) return QI_B200_ESHAPE;
  int group = group_size;
  if (group <= 0 || group > K) group = K;
  if (!aligned16(qweight_int8) || !aligned16(out_bf16)) return QI_B200_EALIGN;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  const int G = (K + group - 1) / group;
  const long long chunks = (long long)N * (K / 16);
  const int grid = (int)std::min<long long>((chunks + 255) / 256, (long long)di->num_sms * 16);
  launch_pdl(k_wo_dequant, dim3(grid), dim3(256), 0, stream, 1, static_cast<const int8_t*>(qweight_int8), scales,
             static_cast<const int16_t*>(zeros_int16), G, group, static_cast<__nv_bfloat16*>(out_bf16), N, K);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}

int qi_b200_wo_linear_ws(const void* x_bf16, const void* qweight_int8, const float* scales, const void* zeros_int16,
                         int group_size, const void* bias, void* out_bf16, int M, int N, int K, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (workspace == nullptr || workspace_bytes < (size_t)N * K * 2) return QI_B200_EINVAL;
  int rc = check_gemm_args(QI_B200_KIND_BF16, x_bf16, workspace, nullptr, 0, nullptr, 0, bias, out_bf16, N, M, N, K,
                           0);
  if (rc) return rc;
  rc = qi_b200_wo_dequant(qweight_int8, scales, zeros_int16, group_size, workspace, N, K, stream);
  if (rc) return rc;
  return gemm_dispatch(QI_B200_KIND_BF16, x_bf16, workspace, nullptr, 0, nullptr, 0, bias, out_bf16, N, M, N, K, 0,
                       0, stream);
}

int qi_b200_quantize_nvfp4(const void* x_bf16, int rows, int cols, int g_mode, const float* g_in,
                           unsigned int* ws_amax, float* g_out, void* q_packed, void* sf_atoms, cudaStream_t stream) {
  if (rows == 0) return QI_B200_OK;
  return nvfp4_quantize(x_bf16, rows, cols, g_mode, g_in, ws_amax, g_out, q_packed, sf_atoms, stream);
}

int qi_b200_nvfp4_gemm(const void* A_packed, const void* A_sf, const void* B_packed, const void* B_sf,
                       const float* a_global_scale, int a_scale_per_row, const float* b_global_scale,
                       const void* bias, void* D, long long ldd, int M, int N, int K, int flags, cudaStream_t stream) {
  return nvfp4_gemm(A_packed, A_sf, B_packed, B_sf, a_global_scale, a_scale_per_row ? 1 : 0, b_global_scale, bias, D,
                    ldd, M, N, K, flags, stream);
}

int qi_b200_nvfp4_linear(const void* x_bf16, const void* weight_packed, const void* weight_sf,
                         const float* weight_global_scale, int act_scale_mode, const float* act_global_scale,
                         const void* bias, void* out_bf16, void* ws_q, void* ws_sf, float* ws_g,
                         unsigned int* ws_amax, int M, int N, int K, int flags, cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (weight_global_scale == nullptr) return QI_B200_EINVAL;
  const float* ag = act_scale_mode == 0 ? act_global_scale : ws_g;
  if (ag == nullptr) return QI_B200_EINVAL;
  int rc = nvfp4_quantize(x_bf16, M, K, act_scale_mode, act_global_scale, ws_amax, ws_g, ws_q, ws_sf, stream);
  if (rc) return rc;
  return nvfp4_gemm(ws_q, ws_sf, weight_packed, weight_sf, ag, act_scale_mode == 2 ? 1 : 0, weight_global_scale, bias,
                    out_bf16, N, M, N, K, flags, stream);
}

// gemm_flags: epilogue flags only; these entry points take no GEMM
// workspace, so the CTA-pair kernel's tail split does not run
static int int8_linear_impl(const void* x_bf16, const void* qweight, const float* weight_scale, const void* bias,
                            void* out_bf16, void* ws_q, float* ws_scales, int M, int N, int K, int gemm_flags,
                            cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (ws_q == nullptr || ws_scales == nullptr || weight_scale == nullptr) return QI_B200_EINVAL;
  int rc = check_gemm_args(QI_B200_KIND_INT8, ws_q, qweight, ws_scales, 1, weight_scale, 1, bias, out_bf16, N, M, N,
                           K, 0);
  if (rc) return rc;
  rc = qi_b200_quantize_int8_rowwise(x_bf16, ws_q, ws_scales, M, K, stream);
  if (rc) return rc;
  return gemm_dispatch(QI_B200_KIND_INT8, ws_q, qweight, ws_scales, 1, weight_scale, 1, bias, out_bf16, N, M, N, K,
                       gemm_flags, 0, stream);
}

int qi_b200_int8_linear(const void* x_bf16, const void* qweight, const float* weight_scale, const void* bias,
                        void* out_bf16, void* ws_q, float* ws_scales, int M, int N, int K, cudaStream_t stream) {
  return int8_linear_impl(x_bf16, qweight, weight_scale, bias, out_bf16, ws_q, ws_scales, M, N, K, 0, stream);
}

int qi_b200_fp8_linear(const void* x_bf16, const void* weight_fp8, const float* weight_scale,
                       int weight_scale_per_channel, const float* static_act_scale, const void* bias,
                       void* out_bf16, void* ws_q, float* ws_scales, int M, int N, int K, int flags,
                       cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (ws_q == nullptr || weight_scale == nullptr) return QI_B200_EINVAL;
  if (static_act_scale == nullptr && ws_scales == nullptr) return QI_B200_EINVAL;
  const float* sa = static_act_scale != nullptr ? static_act_scale : ws_scales;
  const int sa_stride = static_act_scale != nullptr ? 0 : 1;
  const int sb_stride = weight_scale_per_channel ? 1 : 0;
  int rc = check_gemm_args(QI_B200_KIND_FP8_E4M3, ws_q, weight_fp8, sa, sa_stride, weight_scale, sb_stride, bias,
                           out_bf16, N, M, N, K, flags);
  if (rc) return rc;
  rc = static_act_scale != nullptr ? qi_b200_quantize_fp8_static(x_bf16, static_act_scale, ws_q, M, K, stream)
                                   : qi_b200_quantize_fp8_rowwise(x_bf16, ws_q, ws_scales, M, K, stream);
  if (rc) return rc;
  return gemm_dispatch(QI_B200_KIND_FP8_E4M3, ws_q, weight_fp8, sa, sa_stride, weight_scale, sb_stride, bias,
                       out_bf16, N, M, N, K, flags, 0, stream);
}

}  // extern "C"

// ===========================================================================
// INT8 linear without caller-provided workspace.
//
// qi_b200_int8_linear needs scratch for the quantized activations (int8
// [M,K] + fp32 [M]).  Some callers cannot obtain it: a host that hands this
// library only the layer's input and output buffers (an FFI plugin inside a
// runtime that owns all device memory, or a real-time control loop where
// cudaMalloc's implicit device-wide synchronization would stall the control
// thread).  For them the scratch lives in fixed arrays in this library's
// device image, so a call allocates nothing.
//
// The arrays exist once per device that loads the library and stay resident
// until the process exits.  All calls on a device share them: two calls whose
// kernels overlap on the GPU (different streams without ordering between
// them) race on the scratch and may produce wrong results; serialize them on
// one stream.  The quantize kernel overwrites every scratch byte a call reads
// before it is read, so nothing needs clearing between calls.
// ===========================================================================
namespace qib {

static __device__ __align__(256) int8_t g_noalloc_q[QI_B200_NOALLOC_MAX_ACT_BYTES];
static __device__ __align__(256) float g_noalloc_scales[QI_B200_NOALLOC_MAX_ROWS];

struct NoAllocScratch {
  std::atomic<int> ready{0};  // release-stored after q / scales are set
  void* q = nullptr;
  float* scales = nullptr;
};
static NoAllocScratch g_noalloc[kMaxDevices];
static std::mutex g_noalloc_mu;

// Device addresses of the scratch arrays for the current device.  In host
// code the array names are host-side shadows, not device addresses, so the
// addresses are looked up once per device (with that device current) and
// cached.  The first lookup may make the CUDA runtime load this library's
// device code onto the device.
static int noalloc_scratch(void** q, float** scales) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QI_B200_ECUDA;
  NoAllocScratch& e = g_noalloc[dev];
  if (!e.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!e.ready.load(std::memory_order_relaxed)) {
      void* pq = nullptr;
      void* ps = nullptr;
      if (cudaGetSymbolAddress(&pq, g_noalloc_q) != cudaSuccess ||
          cudaGetSymbolAddress(&ps, g_noalloc_scales) != cudaSuccess) {
        cudaGetLastError();  // leave no sticky error for the caller's next cudaGetLastError
        return QI_B200_ECUDA;
      }
      e.q = pq;
      e.scales = static_cast<float*>(ps);
      e.ready.store(1, std::memory_order_release);
    }
  }
  *q = e.q;
  *scales = e.scales;
  return QI_B200_OK;
}

}  // namespace qib

extern "C" int qi_b200_int8_linear_noalloc(const void* x_bf16, const void* qweight, const float* weight_scale,
                                           const void* bias, void* out_bf16, int M, int N, int K,
                                           cudaStream_t stream) {
  if (M == 0) return QI_B200_OK;
  if (M < 0 || K <= 0) return QI_B200_ESHAPE;
  if (M > QI_B200_NOALLOC_MAX_ROWS || static_cast<long long>(M) * K > QI_B200_NOALLOC_MAX_ACT_BYTES)
    return QI_B200_ETOOBIG;
  void* q = nullptr;
  float* scales = nullptr;
  int rc = noalloc_scratch(&q, &scales);
  if (rc) return rc;
  return int8_linear_impl(x_bf16, qweight, weight_scale, bias, out_bf16, q, scales, M, N, K, 0, stream);
}

// ---------------------------------------------------------------------------
// Attention over at most 128 keys (head dim 128): k_attn_short_db
// ---------------------------------------------------------------------------
namespace qib {
// At most 128 keys: the double-buffered kernel, one CTA per SM.
static int launch_attn_short_db(const void* q, long long ldq, const void* k, long long ldk, const void* vt,
                                long long ldvt, void* o, long long ldo, int sq, int sk, int heads, float scale,
                                cudaStream_t stream) {
  using C = AttnDbCfg;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  CUtensorMap tq, tk, tv, to;
  const uint64_t width = static_cast<uint64_t>(heads) * 128;
  if ((rc = make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, width, sq, ldq * 2, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, width, sk, ldk * 2, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, sk, width, ldvt * 2, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&to, o, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, width, sq, ldo * 2, 64, 128))) return rc;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(k_attn_short_db, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
        cudaSuccess)
      return QI_B200_ECUDA;
    attr_done[dev] = true;
  }
  AttnParams p;
  p.sq = sq;
  p.sk = sk;
  p.heads = heads;
  p.scale_log2e = scale * 1.4426950408889634f;
  const int items = heads * ((sq + 127) / 128);
  const int grid = std::min(items, di->num_sms);
  launch_pdl(k_attn_short_db, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, 1, tq, tk, tv, to, p);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? QI_B200_OK : QI_B200_ECUDA;
}
}  // namespace qib

extern "C" int qi_b200_attention_short(const void* q, long long ldq, const void* k, long long ldk, const void* vt,
                                       long long ldvt, void* o, long long ldo, int sq, int sk, int heads,
                                       int head_dim, float scale, cudaStream_t stream) {
  using namespace qib;
  if (q == nullptr || k == nullptr || vt == nullptr || o == nullptr) return QI_B200_EINVAL;
  if (head_dim != 128 || heads <= 0 || sq < 0 || sk < 1 || sk > 128) return QI_B200_ESHAPE;
  if (sq == 0) return QI_B200_OK;
  const long long width = static_cast<long long>(heads) * 128;
  if (ldq < width || ldk < width || ldo < width || ldvt < sk) return QI_B200_ESHAPE;
  if (ldq % 8 || ldk % 8 || ldo % 8 || ldvt % 8) return QI_B200_EALIGN;
  if (!aligned16(q) || !aligned16(k) || !aligned16(vt) || !aligned16(o)) return QI_B200_EALIGN;
  if (!(scale > 0.0f)) return QI_B200_EINVAL;
  return launch_attn_short_db(q, ldq, k, ldk, vt, ldvt, o, ldo, sq, sk, heads, scale, stream);
}
