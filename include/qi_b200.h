/*
 * qi_b200 — C ABI of the B200-native (sm_100a) quantized-linear kernels.
 *
 * Drop-in boundary for hongzicong/qi's quantized nn.Linear hot path.  Each
 * entry point below names the reference interface it replaces (paths inside
 * the reference project, src/qi/quantization/...).
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers on the current CUDA device; tensors
 *     are dense row-major; bf16 = IEEE bfloat16 bits, fp8 = E4M3 ("fn")
 *     codes, int8 = two's complement;
 *   - work is enqueued on `stream`; nothing synchronizes and nothing
 *     allocates device memory (callers own every buffer, workspaces
 *     included; only qi_b200_peer_alloc / qi_b200_peer_free allocate, and
 *     they are explicit set-up calls), so calls can be captured in CUDA
 *     graphs;
 *   - the return value is a status code (QI_B200_OK = 0); a non-zero code
 *     means nothing was enqueued, except QI_B200_ECUDA which reports a launch
 *     error from the CUDA runtime;
 *   - device-side pipeline waits are bounded; a wait that runs out of time
 *     records its site in the device status word (qi_b200_device_status) and
 *     the kernel returns instead of hanging;
 *   - kernels are launched with programmatic dependent launch: activations
 *     and outputs are touched only after the previous kernel in the stream
 *     has finished, but the small-M W4A16 kernel (qi_b200_w4a16_linear,
 *     M <= 16) starts fetching its packed weights, scales and zeros before
 *     that point (M = 1: 7.0 -> 6.7 us; the same for the large GEMMs' B
 *     tiles measured slower, so they do not).  Weight buffers are layer
 *     constants: do not write one with a kernel of this library immediately
 *     before a W4A16 call on the same stream reads it (a torch or other
 *     kernel in between, or a synchronized stream, is enough).
 */
#ifndef QI_B200_H_
#define QI_B200_H_

#include <cuda_runtime_api.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QI_B200_ABI_VERSION 1

/* status codes */
#define QI_B200_OK 0
#define QI_B200_EINVAL 1  /* null pointer, bad enum or flag */
#define QI_B200_ESHAPE 2  /* unsupported dimensions */
#define QI_B200_EALIGN 3  /* pointer not 16-byte aligned */
#define QI_B200_ECUDA 4   /* CUDA runtime reported a launch error */
#define QI_B200_ETMAP 5   /* TMA descriptor could not be encoded */
#define QI_B200_EARCH 6   /* current device is not sm_100 */
#define QI_B200_ETOOBIG 7 /* size above an entry point's fixed maximum */

/* GEMM operand kinds for qi_b200_gemm */
#define QI_B200_KIND_INT8 0     /* int8 x int8 -> int32 (tcgen05 kind::i8) */
#define QI_B200_KIND_FP8_E4M3 1 /* e4m3 x e4m3 -> fp32 (kind::f8f6f4)      */
#define QI_B200_KIND_BF16 2     /* bf16 x bf16 -> fp32 (kind::f16)         */

/* epilogue flags for qi_b200_gemm / qi_b200_fp8_linear */
#define QI_B200_EPI_GELU 1    /* GELU(tanh) of the bf16-rounded linear output */
#define QI_B200_EPI_RAW_ACC 2 /* store raw 32-bit accumulators instead of bf16 (debug) */
/* NVFP4 GEMM tile choice in flags bits 8-9: 0 = the library's choice (CTA
 * pairs with 256 x 256 tiles for M >= 1024 when they fill half the SMs, else
 * single-CTA 128 x 128), 1 = single-CTA 128 x 128, 2 = CTA pair 256 x 128,
 * 3 = CTA pair 256 x 256. */
#define QI_B200_NVFP4_TILE_SHIFT 8
/* qi_b200_gemm_ws flags bits 12-15: the CTA-pair kernel's partial last wave.
 * When tiles % pairs tiles are left for a last wave, each of them can have
 * its K range split over S pairs that would otherwise sit idle; the partial
 * accumulators meet in the caller's workspace (qi_b200_gemm_workspace_bytes
 * gives its size) and are summed in a fixed order, so INT8 results stay
 * bit-exact.  0 = the library's choice, 1 = no split, 2..15 = at most that
 * many splits per tile (further capped at 8 and at the idle pairs).  Without
 * a workspace (qi_b200_gemm) there is no split.  Replaces nothing in the
 * reference (its CUTLASS kernels run one tile per CTA with no split); a
 * scheduling choice of this library. */
#define QI_B200_TAIL_SPLIT_SHIFT 12

int qi_b200_abi_version(void);
const char* qi_b200_error_string(int code);

/* Device status word of the current device: out4[0] = error (0 none, 1 a
 * bounded wait timed out), out4[1] = kernel tag, out4[2] = wait site,
 * out4[3] = block index.  Synchronous (reads device memory); not for use
 * inside stream capture.  clear != 0 resets it. */
int qi_b200_device_status(unsigned int* out4, int clear);

/* Launch plan of the calling thread's most recent GEMM launch, for
 * diagnostics: out6 = {kernel (1 int8, 2 fp8, 3 bf16, 4 nvfp4, 6 w4a16
 * split-K clusters, 7 w4a16 small-M, 8/9/10/11 int8 / fp8 / bf16 / nvfp4
 * CTA-pair tiles, 12/13/14 int8 / fp8 / bf16 cluster split-K), grid, cluster
 * size, tile N (or padded M for kernel 6, M for kernel 7), pipeline stages,
 * dynamic shared memory bytes}. */
int qi_b200_last_launch(int* out6);
/* Splits per tail tile (see QI_B200_TAIL_SPLIT_SHIFT) of the calling thread's
 * most recent CTA-pair GEMM launch; 1 = its last wave ran unsplit. */
int qi_b200_last_tail_split(void);

/* Number of kernels this library has launched in this process, counting
 * launches recorded into a CUDA graph under capture once (at capture). */
int qi_b200_launch_count(unsigned long long* out);

/* ---- activation quantizers --------------------------------------------
 * Replaces qi_quantize_int8_rowwise (csrc/int8_w8a8/quantize_int8.cuh:7-13,
 * kernel quantize_int8.cu:7-59): per row s = max(amax/127, 1e-10),
 * q = clamp(rint(x * (1/s)), -127, 127) (IEEE reciprocal). */
int qi_b200_quantize_int8_rowwise(const void* x_bf16, void* q_int8, float* scales, int rows, int cols,
                                  cudaStream_t stream);

/* qi_b200_quantize_int8_rowwise of x / input_scale, fused: the SmoothQuant /
 * AWQ smoothing of Int8W8A8Backend.linear (int8_w8a8_ops.py:138-139), done
 * in bf16 as there: x' = bf16(fp32(x) / fp32(bf16(input_scale[k]))).
 * input_scale fp32 [cols]. */
int qi_b200_quantize_int8_rowwise_smooth(const void* x_bf16, const float* input_scale, void* q_int8, float* scales,
                                         int rows, int cols, cudaStream_t stream);

/* INT8 quantization with caller-provided per-row scales (no counterpart in
 * the reference): q = clamp(rint(x * (1/s[row])), -127, 127).  Used when a
 * row's K extent is split over ranks: the per-row scales are first reduced
 * with MAX across ranks, so every rank quantizes with the single-GPU scale. */
int qi_b200_quantize_int8_rowwise_given(const void* x_bf16, const float* scales, void* q_int8, int rows, int cols,
                                        cudaStream_t stream);

/* Only the INT8 per-row scales s = max(amax/127, 1e-10) of a bf16 [rows, cols]
 * block (no counterpart in the reference; K1's scale half,
 * quantize_int8.cu:7-59).  For rows split over ranks by K, the MAX over ranks
 * of these scales is exactly the scale of the whole row (division and max are
 * monotone), which qi_b200_quantize_int8_rowwise_given then applies. */
int qi_b200_int8_row_scales(const void* x_bf16, float* scales, int rows, int cols, cudaStream_t stream);

/* The INT8 GEMM epilogue on its own (same operation order as the fused one,
 * cutlass_int8_rowwise.cu:43-71): out = bf16(((float)acc * act_scale[m]) *
 * weight_scale[n] + bias[n]) (+ GELU with QI_B200_EPI_GELU).  Used after a
 * cross-rank int32 sum of K-sharded partial accumulators. */
int qi_b200_int8_epilogue(const void* acc_int32, const float* act_scale, const float* weight_scale,
                          const void* bias, void* out_bf16, int M, int N, int flags, cudaStream_t stream);

/* qi_b200_gemm split over K inside a thread-block cluster: `splits` (2..8)
 * CTAs share one 128 x tile_n output tile (tile_n 128, 192 or 256), each
 * over a contiguous range of K; the partial tiles are added in rank order
 * through distributed shared memory (int32 exactly for INT8, so INT8 outputs
 * are bit-identical to qi_b200_gemm) and each rank runs the fused epilogue on
 * a share of the tile's columns.  No workspace.  tile_n = 0 / splits = 0 pick
 * the plan that puts the most CTAs to work (QI_B200_ESHAPE when the tiles
 * already fill half the SMs). */
int qi_b200_gemm_csk(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                     const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd, int M, int N,
                     int K, int flags, int tile_n, int splits, cudaStream_t stream);

/* ---- Peer memory for the column-parallel linear with an overlapped all-gather
 * (no counterpart in the reference, which runs on one GPU).  One process per
 * GPU; buffers are plain device allocations shared over CUDA IPC (no NVLink
 * multicast object).  The host exchanges the IPC handles (e.g. with
 * torch.distributed.all_gather_object) and opens the peers' handles. ---- */
#define QI_B200_IPC_HANDLE_BYTES 64
#define QI_B200_MAX_PEERS 8

/* cudaMalloc(bytes), zero it, and export its IPC handle (64 bytes). */
int qi_b200_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map a peer's buffer (cudaIpcOpenMemHandle, lazy peer access). */
int qi_b200_peer_open(const void* ipc_handle, void** ptr);
int qi_b200_peer_close(void* ptr);
int qi_b200_peer_free(void* ptr);

/* Cross-GPU barrier on the stream.  flags[i] is rank i's flag block
 * (QI_B200_PEER_FLAG_BYTES, zero-initialized): word j is written by rank j,
 * word QI_B200_MAX_PEERS is rank i's own barrier counter.  The kernel
 * advances this rank's counter (so CUDA-graph replays advance it too),
 * writes it into word `rank` of every block (release, system scope) and
 * waits until every rank has written the same value into its own block
 * (acquire).  All ranks must run the same sequence of barriers.  The wait is
 * bounded (2 s): on timeout the device status word records kernel tag 0x300
 * with the rank that did not arrive as the wait site, and the kernel
 * returns. */
#define QI_B200_PEER_FLAG_BYTES 256
int qi_b200_peer_barrier(void* const* flags, int P, int rank, cudaStream_t stream);
/* qi_b200_peer_barrier with the wait limited to timeout_ns (0 < timeout_ns
 * <= 2 s): a caller that wants a failed peer reported sooner, e.g. a health
 * check between steps. */
int qi_b200_peer_barrier_timed(void* const* flags, int P, int rank, unsigned long long timeout_ns,
                               cudaStream_t stream);

/* qi_b200_gemm (INT8 / FP8 / BF16, bf16 out, optional GELU) on the CTA-pair
 * kernel with the column-parallel all-gather fused into its epilogue: every
 * finished 32 x 64 output box is written by TMA into each of the ndst [M, N]
 * blocks dst[i] (row pitch ldd elements): this rank's block of its own
 * output buffer and of its peers' buffers, mapped with qi_b200_peer_open.
 * The NVLink transfer of a tile overlaps the MMAs of the next tiles.  When
 * the kernel retires, its stores have completed; follow with
 * qi_b200_peer_barrier before any rank reads.  ndst <= 8; N % 8 == 0. */
int qi_b200_gemm_gather(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                        const float* b_scale, int b_scale_stride, const void* bias, void* const* dst, int ndst,
                        long long ldd, int M, int N, int K, int flags, cudaStream_t stream);

/* ---- Fused elementwise stages of the MoT DiT block (no counterpart in the
 * reference's quantization package: they fuse the bf16 tensor ops of
 * src/qi/models/wan22/wan_video_dit.py:147-268 and mot.py:100-122 that sit
 * between the quantized Linears into one pass each). ----
 *
 * qi_b200_resid_ln_quant, one row of x [M, D] per CTA, every stage optional:
 *   x  <- bf16(x + bf16(gate * y))  (y and gate given) or bf16(x + y) (y only)
 *   n  <- bf16(LayerNorm(x, eps) [* ln_w + ln_b])
 *   n  <- bf16(bf16(n * mod_scale1) + mod_shift)     mod_scale1 = bf16(1 + scale)
 *   q_int8, scales <- per-token INT8 of n (quantize_int8.cu:7-59); xn_bf16 <- n
 * With q_int8 and xn_bf16 both null only the residual update runs.
 * D % 8 == 0, D <= 4096; bf16 pointers 16-byte aligned; y row stride ldy. */
int qi_b200_resid_ln_quant(void* x_bf16, const void* y_bf16, long long ldy, const void* gate, const void* ln_w,
                           const void* ln_b, const void* mod_scale1, const void* mod_shift, void* q_int8,
                           float* scales, void* xn_bf16, int M, int D, float eps, cudaStream_t stream);

/* qi_b200_rms_rope: for nparts (1 or 2) inputs of [M, A] (row stride ld_in):
 *   out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)            (RMSNorm over all A)
 *   then, with rope ([M, head_dim/2, 2] fp32 cos/sin per token), rotate each
 *   (even, odd) pair of every head: (e c - o s, e s + o c) in fp32.
 * A % 8 == 0, A <= 4096, head_dim % 8 == 0.  With head_dim a power of two
 * in [8, 256] dividing A, mean(x^2) is the sum of per-head sums of squares
 * taken in head order, the same bits however the heads are split over GPUs
 * (qi_b200_rms_head_partials / qi_b200_rms_rope_partials). */
int qi_b200_rms_rope(const void* in0, const void* in1, long long ld_in, void* out0, void* out1, long long ld_out,
                     const void* w0, const void* w1, const float* rope, int head_dim, int nparts, int M, int A,
                     float eps, cudaStream_t stream);

/* Head-parallel RMSNorm (no counterpart in the reference, which runs the
 * q/k RMSNorm of wan_video_dit.py:147-158 over all heads on one GPU).  A rank
 * holding a contiguous range of whole heads (A = its columns) writes its
 * per-head sums of squares, partials[nparts][M][A / head_dim] fp32; the ranks
 * all-gather them (rank-major: [ranks][nparts][M][A / head_dim], i.e. head
 * order); qi_b200_rms_rope_partials then normalizes this rank's columns over
 * all ranks * A columns.  The outputs are bit-identical to qi_b200_rms_rope
 * on the unsplit row.  head_dim a power of two in [8, 256] dividing A. */
int qi_b200_rms_head_partials(const void* in0, const void* in1, long long ld_in, float* partials, int head_dim,
                              int nparts, int M, int A, cudaStream_t stream);
int qi_b200_rms_rope_partials(const void* in0, const void* in1, long long ld_in, void* out0, void* out1,
                              long long ld_out, const void* w0, const void* w1, const float* rope, int head_dim,
                              int nparts, int M, int A, const float* partials, int ranks, float eps,
                              cudaStream_t stream);

/* Attention over a short key sequence (no counterpart in the reference's
 * own code: the DiT blocks call torch's scaled_dot_product_attention,
 * wan_video_dit.py:14-23).  Per head h of `heads` (head_dim must be 128):
 *   O[:, h] = softmax(Q[:, h] K[:, h]^T * scale) V[:, h]
 * for sq query rows and 1 <= sk <= 128 keys, no mask (the DiT's
 * cross-attention over its context tokens).  q [sq, ldq], k [sk, ldk]
 * and o [sq, ldo] hold head h in columns h*128 .. h*128+127; V is passed
 * transposed, vt [heads*128, ldvt] with row h*128 + d holding V[:, h, d] over
 * the keys (ldvt >= sk).  bf16 in and out, fp32 scores and accumulation,
 * probabilities rounded to bf16 before the P V product.  All leading
 * dimensions multiples of 8, pointers 16-byte aligned. */
int qi_b200_attention_short(const void* q, long long ldq, const void* k, long long ldk, const void* vt,
                            long long ldvt, void* o, long long ldo, int sq, int sk, int heads, int head_dim,
                            float scale, cudaStream_t stream);

/* Per-token FP8: s = max(amax/448, 1e-12), q = e4m3_rn(clamp(x/s, +-448)).
 * Generalises backends/flashrt_fp8_ops.py:38-48 (per tensor) to per row. */
int qi_b200_quantize_fp8_rowwise(const void* x_bf16, void* q_fp8, float* scales, int rows, int cols,
                                 cudaStream_t stream);

/* Static per-tensor FP8 with a calibrated device scale; replaces FlashRT's
 * quantize_fp8_static as called at backends/flashrt_fp8_ops.py:210-216. */
int qi_b200_quantize_fp8_static(const void* x_bf16, const float* scale, void* q_fp8, int rows, int cols,
                                cudaStream_t stream);

/* ---- GEMMs -------------------------------------------------------------
 * Replaces qi_cutlass_int8_rowwise_bf16out / _bias (csrc/int8_w8a8/
 * bindings.cpp:20-85, kernels cutlass_int8_rowwise*.cu):
 *   D[M,N] = bf16( (float(sum_k A[m,k] B[n,k]) * act_scale[m]) * weight_scale[n] (+ bias[n]) )
 * A int8 [M,K], B int8 [N,K] (nn.Linear weight), scales fp32, bias/D bf16.
 * Needs N % 8 == 0, K % 16 == 0 (the reference needs N, K % 64 == 0). */
int qi_b200_int8_rowwise_bf16out(const void* A, const void* B, const void* act_scale, const void* weight_scale,
                                 void* D, int M, int N, int K, cudaStream_t stream);
int qi_b200_int8_rowwise_bf16out_bias(const void* A, const void* B, const void* act_scale, const void* weight_scale,
                                      const void* bias, void* D, int M, int N, int K, cudaStream_t stream);

/* General form of the GEMM above for every operand kind (replaces the
 * tile-specific variants _t64x128/_t64x256/_t32x128/_t128x64 of
 * bindings.cpp:31-85 and FlashRT's GemmRunner.fp8_run_dev called at
 * backends/flashrt_fp8_ops.py:68-89):
 *   D[m, n] (row stride ldd) = epi( acc[m,n] * a_scale[m*a_scale_stride] * b_scale[n*b_scale_stride] + bias[n] )
 * a_scale / b_scale / bias may be NULL; a stride of 0 broadcasts one scale.
 * tile_n = 0 picks the kernel and tile width; 64, 128, 192 or 256 forces a
 * single-CTA tile of that width; -128, -192 or -256 forces the CTA-pair
 * kernel (tcgen05 cta_group::2, 256-row tiles over two SMs) of that width. */
int qi_b200_gemm(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                 const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd, int M, int N,
                 int K, int flags, int tile_n, cudaStream_t stream);

/* qi_b200_gemm with a caller-owned workspace for the CTA-pair kernel's split
 * of its partial last wave (QI_B200_TAIL_SPLIT_SHIFT): at least
 * qi_b200_gemm_workspace_bytes bytes, 16-byte aligned, used by one launch at
 * a time (calls that overlap on the GPU need separate workspaces).  A null
 * or too small workspace runs the launch without the split.  Same result
 * either way (bit-identical for INT8). */
int qi_b200_gemm_ws(int kind, const void* A, const void* B, const float* a_scale, int a_scale_stride,
                    const float* b_scale, int b_scale_stride, const void* bias, void* D, long long ldd, int M, int N,
                    int K, int flags, int tile_n, void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* Workspace bytes qi_b200_gemm_ws needs for this problem, flags and tile_n on
 * the current device (0: that launch does not split).  Host only. */
int qi_b200_gemm_workspace_bytes(int kind, int M, int N, int K, int flags, int tile_n, size_t* bytes);

/* ---- W4A16 (INT4 weight-only) ----------------------------------------
 * Replaces the weight-only INT4 path of ReferenceBackend.linear
 * (backends/reference.py:48-91, dequantize_weight at quantize.py:81-119) and
 * the reserved CudaExtBackend (backends/reference.py:94-96):
 *   out[M,N] = bf16( x_bf16 . W^T + bias ),  W[n,k] = bf16( (q[n,k] - z[n,g]) * s[n,g] )
 * qweight_packed int32 [N, K/8] (element 8w+j in bits 4j..4j+3 of word w),
 * scales_fp16 [N, G], zeros_packed int32 [N, ceil(G/8)] (uint4, group g in
 * word g/8 nibble g%8), G = ceil(K / group_size); group_size <= 0 means one
 * group per row.  Needs K % 32 == 0, N % 8 == 0, group_size % 32 == 0.
 * M <= 16: a streaming kernel over bulk-copied weight rows; M <= 256: a
 * split-K kernel over a thread-block cluster; larger M: that kernel per
 * 256-row block (qi_b200_w4a16_linear_ws is faster there). */
int qi_b200_w4a16_linear(const void* x_bf16, const void* qweight_packed, const void* scales_fp16,
                         const void* zeros_packed, int group_size, const void* bias, void* out_bf16, int M, int N,
                         int K, cudaStream_t stream);

/* Packed INT4 weights -> bf16 [N, K] (qweight and out_bf16 16-byte aligned),
 * exactly the reference's dequantization.  group_size % 32 == 0, K % 32 == 0. */
int qi_b200_w4a16_dequant(const void* qweight_packed, const void* scales_fp16, const void* zeros_packed,
                          int group_size, void* out_bf16, int N, int K, cudaStream_t stream);

/* qi_b200_w4a16_linear with a caller-owned workspace of at least N * K * 2
 * bytes (16-byte aligned): for M >= QI_B200_W4A16_DEQUANT_MIN_M the weights
 * are dequantized once into it and multiplied with the bf16 tcgen05 GEMM (the
 * fused kernels would rebuild each dequantized tile for every M tile); below
 * that, or without a workspace, it is qi_b200_w4a16_linear. */
#define QI_B200_W4A16_DEQUANT_MIN_M 257
int qi_b200_w4a16_linear_ws(const void* x_bf16, const void* qweight_packed, const void* scales_fp16,
                            const void* zeros_packed, int group_size, const void* bias, void* out_bf16, int M, int N,
                            int K, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- Weight-only linears on the reference's own buffers ----------------
 * Replaces the reserved CudaExtBackend (backends/reference.py:94-96) for the
 * weight-only configs the reference's ReferenceBackend.linear serves
 * (reference.py:48-91): WeightOnlyQuantConfig's default bits=8, group 128,
 * symmetric (W8A16), and INT4 kept one value per int8.  qweight int8 [N, K]
 * (codes; symmetric: -qmax..qmax, asymmetric: 0..2^bits-1), scales fp32
 * [N, G], zeros int16 [N, G] or NULL (symmetric), G = ceil(K / group_size),
 * group_size <= 0 = one group per row.  The dequantization is the
 * reference's, bit for bit: W = bf16(fp32(q - z) * s).  K % 16 == 0. */
int qi_b200_wo_dequant(const void* qweight_int8, const float* scales, const void* zeros_int16, int group_size,
                       void* out_bf16, int N, int K, cudaStream_t stream);
/* out[M, N] = bf16(x . W^T + bias): W dequantized into the caller's
 * workspace (>= N * K * 2 bytes, 16-byte aligned), then the bf16 tcgen05
 * GEMM. */
int qi_b200_wo_linear_ws(const void* x_bf16, const void* qweight_int8, const float* scales, const void* zeros_int16,
                         int group_size, const void* bias, void* out_bf16, int M, int N, int K, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream);

/* ---- NVFP4 W4A4 (no counterpart in the reference, which only names the
 * buffers qweight_packed / scale_factors / weight_global_scale at
 * src/qi/quantization/modules.py:21-23) ------------------------------------
 * Values E2M1 (two per byte, element 2j in the low nibble); E4M3 scale per 16
 * elements along K in the scale-factor atom layout (512-byte atoms of 128 rows
 * x 4 scales, atoms K-fastest, row r0 + 32 r1 at byte r0*16 + r1*4 + j; rows
 * padded to a multiple of 128); fp32 second-level scale g.
 *   g = max(amax / 2688, 1e-12); sf = e4m3(min(amax16 / (6 g), 448));
 *   q = e2m1(clamp(x / (sf g), +-6)).
 * Activation quantization, g_mode: 0 = static per-tensor g (g_in), 1 =
 * dynamic per-tensor (two passes; ws_amax is one uint32 of scratch, needing
 * no clearing; the amax pass keeps per-block maxima in a library slot of the
 * calling stream; g_out[0]),
 * 2 = dynamic per-row (g_out[rows]).  cols % 64 == 0; x and sf_atoms
 * 16-byte aligned, q_packed 8-byte aligned. */
int qi_b200_quantize_nvfp4(const void* x_bf16, int rows, int cols, int g_mode, const float* g_in,
                           unsigned int* ws_amax, float* g_out, void* q_packed, void* sf_atoms, cudaStream_t stream);
/* D = bf16( (acc * a_g[m or 0]) * b_g[0] + bias ), acc = sum over 16-blocks of
 * (q_a q_b) sf_a sf_b on tcgen05 kind::mxf4nvf4 (block16).  K % 256 == 0.
 * flags: QI_B200_EPI_GELU, QI_B200_EPI_RAW_ACC, tile choice (see
 * QI_B200_NVFP4_TILE_SHIFT). */
int qi_b200_nvfp4_gemm(const void* A_packed, const void* A_sf, const void* B_packed, const void* B_sf,
                       const float* a_global_scale, int a_scale_per_row, const float* b_global_scale,
                       const void* bias, void* D, long long ldd, int M, int N, int K, int flags, cudaStream_t stream);
/* Quantize x (act_scale_mode as g_mode above) into the caller's workspace
 * (ws_q [M, K/2], ws_sf atoms, ws_g [1 or M], ws_amax [1]) then the GEMM. */
int qi_b200_nvfp4_linear(const void* x_bf16, const void* weight_packed, const void* weight_sf,
                         const float* weight_global_scale, int act_scale_mode, const float* act_global_scale,
                         const void* bias, void* out_bf16, void* ws_q, void* ws_sf, float* ws_g,
                         unsigned int* ws_amax, int M, int N, int K, int flags, cudaStream_t stream);

/* ---- whole quantized linears -----------------------------------------
 * Replaces the torch op qi_int8_w8a8::linear (csrc/int8_w8a8/bindings.cpp:
 * 87-157, schema :159-165): quantize x per token into the caller's
 * workspace (ws_q int8 [M,K], ws_scales fp32 [M]) then run the INT8 GEMM. */
int qi_b200_int8_linear(const void* x_bf16, const void* qweight, const float* weight_scale, const void* bias,
                        void* out_bf16, void* ws_q, float* ws_scales, int M, int N, int K, cudaStream_t stream);

/* Replaces FlashRTFP8Backend.linear's device work (backends/flashrt_fp8_ops.py:
 * 207-229): static per-tensor (static_act_scale != NULL) or dynamic per-token
 * (static_act_scale == NULL, scales into ws_scales) activation quantization,
 * then the FP8 GEMM with per-tensor or per-channel weight scales, bias and
 * optional GELU fused into the epilogue. */
int qi_b200_fp8_linear(const void* x_bf16, const void* weight_fp8, const float* weight_scale,
                       int weight_scale_per_channel, const float* static_act_scale, const void* bias,
                       void* out_bf16, void* ws_q, float* ws_scales, int M, int N, int K, int flags,
                       cudaStream_t stream);

/* ---- INT8 linear that allocates nothing --------------------------------
 * No counterpart in the reference.  Same result as qi_b200_int8_linear (same
 * kernels, bit-identical output), for callers that cannot provide or
 * allocate scratch memory: hosts that pass the library only the layer's
 * input and output (an FFI plugin inside a runtime that owns all device
 * memory), or real-time loops where cudaMalloc's implicit device-wide
 * synchronization is not allowed.
 *
 * The quantized activations go to fixed scratch arrays inside the library's
 * device image (one copy per device that loads the library, resident until
 * the process exits): at most QI_B200_NOALLOC_MAX_ROWS rows and
 * QI_B200_NOALLOC_MAX_ACT_BYTES activation elements (M*K); larger calls
 * return QI_B200_ETOOBIG and enqueue nothing.
 *
 * The first call on a device looks up the scratch arrays' device addresses
 * (and may make the CUDA runtime load the library's device code); make that
 * first call before any stream capture.  All calls on a device share the
 * scratch: calls whose kernels can overlap on the GPU race and may return
 * wrong results, so issue them on one stream (or otherwise order them).
 * Nothing needs clearing between calls: every scratch byte a call reads is
 * first written by that call. */
#define QI_B200_NOALLOC_MAX_ROWS 16384
#define QI_B200_NOALLOC_MAX_ACT_BYTES (8 * 1024 * 1024)
int qi_b200_int8_linear_noalloc(const void* x_bf16, const void* qweight, const float* weight_scale,
                                const void* bias, void* out_bf16, int M, int N, int K, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QI_B200_H_ */
