// Host side of the tcgen05 GEMM: tensor maps, instantiation table, launches.
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm.cuh"
#include "launch.cuh"

namespace oasis {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  return OASIS_OK;
}

// 2-D row-major tensor [rows][ld] of `esize`-byte elements, box = box_cols x box_rows
// with 128-byte swizzle (box_cols * esize == 128).
int encode_2d(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
              int box_cols, int box_rows, int esize) {
  if (int s = get_encoder()) return s;
  if (!aligned16(base)) return fail(OASIS_ERR_ALIGNMENT, "GEMM operand base not 16-byte aligned");
  if ((ld * esize) % 16 != 0) return fail(OASIS_ERR_ALIGNMENT, "GEMM leading dim not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return OASIS_OK;
}

// Most CTA pairs of this kernel that can be resident at once (clusters are placed
// within a GPC, so this can be below num_sms() / 2).
}  // namespace

// bf16 tensor of rank 2 or 3 (dims innermost first, byte strides of dims 1..rank-1),
// 128-byte swizzled boxes (box[0] * 2 == 128).
int encode_bf16_sw128(CUtensorMap* map, const void* base, int rank, const long long* dims,
                      const long long* strides_bytes, const int* box) {
  if (int s = get_encoder()) return s;
  if (!aligned16(base)) return fail(OASIS_ERR_ALIGNMENT, "tensor map base not 16-byte aligned");
  cuuint64_t d[3], st[2];
  cuuint32_t b[3], e[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    b[i] = static_cast<cuuint32_t>(box[i]);
    if (i > 0) {
      if (strides_bytes[i - 1] % 16) return fail(OASIS_ERR_ALIGNMENT, "tensor map stride not 16-byte aligned");
      st[i - 1] = static_cast<cuuint64_t>(strides_bytes[i - 1]);
    }
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, st, b,
                        e, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return OASIS_OK;
}

namespace {

template <int BN, int EPI>
int max_pairs() {
  using S = GemmShape<BN, 2>;
  static int pairs = 0;
  if (pairs == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = S::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tcgen05_kernel<BN, EPI, 2>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    pairs = n;
  }
  return pairs;
}

// Which operand the kernel may fetch before the previous kernel ends (bit 0: B, bit 1: A).
inline int prefetch_flags(const GemmOperands& g) {
  return g.b_is_weight ? 1 : (g.a_is_weight ? 2 : 0);
}

template <int BN, int EPI, int CTAS>
int launch_one(const GemmOperands& g, const EpiParams& ep, cudaStream_t stream, int max_ctas) {
  using S = GemmShape<BN, CTAS>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tcgen05_kernel<BN, EPI, CTAS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm)");
    configured = true;
  }
  const int tiles = ((g.M + kGemmBM * CTAS - 1) / (kGemmBM * CTAS)) * ((g.N + BN - 1) / BN) *
                    (g.splits > 1 ? g.splits : 1);
  int units = num_sms();
  if constexpr (CTAS == 2) units = max_pairs<BN, EPI>();
  if (max_ctas > 0 && max_ctas / CTAS < units) units = max_ctas / CTAS > 0 ? max_ctas / CTAS : 1;
  if (tiles < units) units = tiles;
  if (epi_uses_tma(EPI) && !g.has_d)
    return fail(OASIS_ERR_INVALID_ARG, "GEMM epilogue needs an output tensor map");
  EpiParams epk = ep;
  epk.k_splits = 1;
  if (g.splits > 1) {
    if (EPI != kEpiGateResid || CTAS != 1 || !ep.split_flags || (g.K / kGemmBK) % g.splits)
      return fail(OASIS_ERR_INVALID_ARG, "GEMM K split needs the residual epilogue, single CTAs, "
                                         "split counters and whole k-blocks per split");
    epk.k_splits = g.splits;
  }
  cudaError_t e;
  if constexpr (CTAS == 2)
    e = launch_pdl_cluster(gemm_tcgen05_kernel<BN, EPI, CTAS>, dim3(units * CTAS), dim3(kGemmThreads),
                           S::kSmemBytes, stream, CTAS, g.a, g.b, g.d, g.M, g.N, g.K,
                           prefetch_flags(g), epk);
  else
    e = launch_pdl(gemm_tcgen05_kernel<BN, EPI, CTAS>, dim3(units), dim3(kGemmThreads), S::kSmemBytes,
                   stream, g.a, g.b, g.d, g.M, g.N, g.K, prefetch_flags(g), epk);
  if (e != cudaSuccess) return cuda_status(e, "gemm_tcgen05_kernel");
  return OASIS_OK;
}

template <int BN, int CTAS>
int dispatch_epi(const GemmOperands& g, int epi, const EpiParams& ep, cudaStream_t s, int mc) {
  switch (epi) {
    case kEpiStoreBF16: return launch_one<BN, kEpiStoreBF16, CTAS>(g, ep, s, mc);
    case kEpiStoreF32Bias: return launch_one<BN, kEpiStoreF32Bias, CTAS>(g, ep, s, mc);
    case kEpiQkvRope: return launch_one<BN, kEpiQkvRope, CTAS>(g, ep, s, mc);
    case kEpiBiasGelu: return launch_one<BN, kEpiBiasGelu, CTAS>(g, ep, s, mc);
    case kEpiGateResid: return launch_one<BN, kEpiGateResid, CTAS>(g, ep, s, mc);
  }
  if (CTAS == 1) {  // swap-AB and row epilogues: small shapes, single CTAs only
    switch (epi) {
      case kEpiAdaT: return launch_one<BN, kEpiAdaT, 1>(g, ep, s, mc);
      case kEpiFinal: return launch_one<BN, kEpiFinal, 1>(g, ep, s, mc);
      case kEpiAdaTSilu: return launch_one<BN, kEpiAdaTSilu, 1>(g, ep, s, mc);
    }
  }
  return fail(OASIS_ERR_INVALID_ARG, "unknown GEMM epilogue (or not available on CTA pairs)");
}

}  // namespace

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int make_gemm_operands(GemmOperands* g, const void* A, long long lda, const void* B, long long ldb,
                       int M, int N, int K, int bn, int ctas) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(OASIS_ERR_INVALID_ARG, "GEMM sizes must be positive");
  if (K % kGemmBK) return fail(OASIS_ERR_UNSUPPORTED, "GEMM K must be a multiple of 64");
  if (bn != 32 && bn != 64 && bn != 128 && bn != 192 && bn != 256)
    return fail(OASIS_ERR_UNSUPPORTED, "GEMM tile N must be 32, 64, 128, 192 or 256");
  if (ctas != 1 && !(ctas == 2 && bn == 256))
    return fail(OASIS_ERR_UNSUPPORTED, "GEMM CTA pairs need tile N 256");
  *g = GemmOperands{};
  if (int s = encode_2d(&g->a, A, M, K, lda, kGemmBK, kGemmBM, 2)) return s;
  // each CTA of a pair loads half of the tile's B rows
  if (int s = encode_2d(&g->b, B, N, K, ldb, kGemmBK, bn / ctas, 2)) return s;
  g->M = M;
  g->N = N;
  g->K = K;
  g->bn = bn;
  g->ctas = ctas;
  g->splits = 1;
  g->has_d = false;
  g->b_is_weight = false;
  return OASIS_OK;
}

int set_gemm_output(GemmOperands* g, void* D, long long ldd, bool f32) {
  const int esize = f32 ? 4 : 2;
  if (g->N % (f32 ? 32 : 64))
    return fail(OASIS_ERR_UNSUPPORTED, "TMA-store GEMM epilogue needs N % 64 == 0 (bf16) / 32 (fp32)");
  if (int s = encode_2d(&g->d, D, g->M, g->N, ldd, 128 / esize, 32, esize)) return s;
  g->has_d = true;
  return OASIS_OK;
}

int launch_gemm(const GemmOperands& g, int epi, const EpiParams& ep, cudaStream_t stream,
                int max_ctas) {
  if (g.ctas == 2) {
    if (g.bn == 256) return dispatch_epi<256, 2>(g, epi, ep, stream, max_ctas);
    return fail(OASIS_ERR_UNSUPPORTED, "GEMM CTA-pair tile N");
  }
  switch (g.bn) {
    case 32: return dispatch_epi<32, 1>(g, epi, ep, stream, max_ctas);
    case 64: return dispatch_epi<64, 1>(g, epi, ep, stream, max_ctas);
    case 128: return dispatch_epi<128, 1>(g, epi, ep, stream, max_ctas);
    case 192: return dispatch_epi<192, 1>(g, epi, ep, stream, max_ctas);
    case 256: return dispatch_epi<256, 1>(g, epi, ep, stream, max_ctas);
  }
  return fail(OASIS_ERR_UNSUPPORTED, "GEMM tile N");
}

int launch_chain(const ChainStep* steps, int n, cudaStream_t stream) {
  using S = GemmShape<256, 2>;
  if (n < 1 || n > kMaxChainOps) return fail(OASIS_ERR_INVALID_ARG, "chain: 1..4 steps");
  static bool configured = false;
  static int pairs = 0;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm_chain)");
    pairs = max_pairs<256, kEpiGateResid>();
    configured = true;
  }
  ChainParams P{};
  P.n_ops = n;
  P.prefetch_b = steps[0].g->b_is_weight ? 1 : 0;
  int max_tiles = 0;
  for (int i = 0; i < n; ++i) {
    const GemmOperands& g = *steps[i].g;
    if (g.ctas != 2 || g.bn != 256 || !g.has_d || g.N % 256)
      return fail(OASIS_ERR_UNSUPPORTED, "chain: every step needs CTA-pair 256-wide tiles");
    if (steps[i].epi != kEpiGateResid && steps[i].epi != kEpiBiasGelu && steps[i].epi != kEpiQkvRope)
      return fail(OASIS_ERR_UNSUPPORTED, "chain: epilogue kind");
    if (steps[i].ep.ln_out && (steps[i].epi != kEpiGateResid || !steps[i].tiles_done))
      return fail(OASIS_ERR_INVALID_ARG, "chain: LayerNorm phase needs a residual step with counters");
    ChainOp& op = P.op[i];
    op.a = g.a;
    op.b = g.b;
    op.d = g.d;
    op.ep = steps[i].ep;
    op.ep.ln_count = steps[i].tiles_done;
    op.M = g.M;
    op.N = g.N;
    op.K = g.K;
    op.epi = steps[i].epi;
    op.wait = steps[i].wait;
    op.wait_tiles = steps[i].wait_tiles;
    op.tiles_done = steps[i].tiles_done;
    op.rows_done = steps[i].rows_done;
    if (steps[i].publish_bits && (g.N / 256 > 32 || steps[i].ep.ln_out || !steps[i].tiles_done))
      return fail(OASIS_ERR_INVALID_ARG, "chain: tile bitmasks need at most 32 N tiles, counters and no LayerNorm");
    if (steps[i].wait_bits && (g.K / 256 > 32 || !steps[i].wait))
      return fail(OASIS_ERR_INVALID_ARG, "chain: bitmask waits need at most 32 producer tiles along K");
    op.publish_bits = steps[i].publish_bits ? 1 : 0;
    op.wait_bits = steps[i].wait_bits ? 1 : 0;
    const int tiles = ((g.M + 255) / 256) * (g.N / 256);
    if (tiles > max_tiles) max_tiles = tiles;
  }
  int units = pairs;
  if (max_tiles < units) units = max_tiles;
  cudaError_t e = launch_pdl_cluster(gemm_chain_kernel, dim3(units * 2), dim3(kGemmThreads),
                                     S::kSmemBytes, stream, 2, P);
  if (e != cudaSuccess) return cuda_status(e, "gemm_chain_kernel");
  return OASIS_OK;
}

namespace {

// Estimated microseconds of an M x N x K bf16 GEMM on 128*ctas x bn tiles with K split
// `splits` ways, `slots` units resident at once (SMs, or SM pairs).  Each unit streams
// its A rows (16 KB per k-block) and its share of the B rows (bn/ctas x 128 B) through
// one SM (~150 GB/s) and issues 2*bn tensor cycles per k-block; the whole launch moves A
// once per N tile and B once per M tile out of L2 (~20 TB/s); ~1.5 us of pipeline fill
// and epilogue per unit; split k issues its reduce-adds after split k-1's completed
// (~2.5 us each).  The constants reproduce the tile choices measured best on B200 for
// the incremental forward's shapes (M = 1152 and 2304).
double gemm_time_us(long long M, long long N, long long K, int bn, int ctas, int splits, int slots) {
  const double clk_ghz = 1.8, sm_gbps = 150.0, l2_gbps = 20000.0, fixed_us = 1.5;
  const long long m_tiles = (M + 128LL * ctas - 1) / (128LL * ctas);
  const long long n_tiles = N / bn;
  const long long units = m_tiles * n_tiles * splits;
  const long long waves = (units + slots - 1) / slots;
  const double kb = static_cast<double>(K / 64 / splits);
  const double t_load = (16384.0 + (bn / ctas) * 128.0) / (sm_gbps * 1e3);
  const double t_mma = 2.0 * bn / (clk_ghz * 1e3);
  const double t_unit = kb * (t_load > t_mma ? t_load : t_mma) + fixed_us;
  const double l2_bytes = 2.0 * M * K * n_tiles + 2.0 * N * K * m_tiles;
  const double t_l2 = l2_bytes / (l2_gbps * 1e3) + fixed_us;
  const double t = waves * t_unit > t_l2 ? waves * t_unit : t_l2;
  return t + (splits - 1) * 2.5;
}

}  // namespace

void choose_tiles(int M, int N, int K, bool allow_split, int* bn, int* ctas, int* splits) {
  const long long sms = num_sms();
  const int pairs = max_pairs<256, kEpiGateResid>();
  *splits = 1;
  if (N % 256 == 0 && M >= 32 * kGemmBM) {
    // CTA pairs on 256 x 256 tiles (the chained launch's tiles) from 4,096 rows on, unless
    // they run in fewer than four waves, the last of them under 45 % full: each SM stages
    // half the B rows, so a pair tile costs the SM less operand traffic than any
    // single-CTA tile, and from four waves on a partly filled last wave costs less than
    // leaving the pairs.  Below 4,096 rows (the incremental forward of 8-16 sessions:
    // 1,152 and 2,304 rows) single CTAs measured faster in the whole forward (2.59 vs
    // 2.64 ms at 8 sessions, 4.67 vs 4.83 ms at 16): there each projection is about one
    // wave, and a 128-row tile keeps every SM busy where 256-row pair tiles leave half
    const long long pair_m = (M + 2 * kGemmBM - 1) / (2 * kGemmBM);
    const long long units = pair_m * (N / 256);
    const long long waves = (units + pairs - 1) / pairs;
    const long long last = units - (waves - 1) * pairs;
    if (waves >= 4 || 100 * last >= 45LL * pairs) {
      *bn = 256;
      *ctas = 2;
      return;
    }
  }
  double best = 1e30;
  *bn = 64;
  *ctas = 1;
  for (int b : {64, 128, 192, 256}) {
    if (N % b) continue;
    for (int s : {1, 2, 4}) {
      if (s > 1 && (!allow_split || b < 128 || (K / kGemmBK) % s)) continue;
      const double t = gemm_time_us(M, N, K, b, 1, s, static_cast<int>(sms));
      if (t < best) {
        best = t;
        *bn = b;
        *ctas = 1;
        *splits = s;
      }
    }
  }
  if (N % *bn) {  // no candidate divides N: the widest power of two that does
    int b = 256;
    while (b > 32 && N % b) b >>= 1;
    *bn = b;
    *ctas = 1;
    *splits = 1;
  }
}

size_t split_flag_count(const GemmOperands& g) {
  if (g.splits <= 1) return 0;
  return static_cast<size_t>((g.M + kGemmBM - 1) / kGemmBM) * (g.N / g.bn) * kEpiWarps;
}

}  // namespace oasis

// ------------------------------------------------------------------ bounded-wait self-test
namespace oasis {
namespace {
__device__ unsigned int g_never_set = 0;  // no kernel ever writes it

__global__ void bounded_wait_selftest_kernel() {
  if (threadIdx.x == 0) wait_count_geq(&g_never_set, 1u);  // gives up, records the timeout
}
}  // namespace
}  // namespace oasis

// ------------------------------------------------------------------ C ABI
extern "C" int oasis_gemm_bf16(const void* A, const void* B, void* D, const float* bias, int M,
                               int N, int K, int lda, int ldb, int ldd, int epilogue,
                               cudaStream_t stream) {
  using namespace oasis;
  if (!A || !B || !D) return fail(OASIS_ERR_INVALID_ARG, "oasis_gemm_bf16: null pointer");
  if (epilogue != 0 && epilogue != 1)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_gemm_bf16: epilogue must be 0 or 1");
  if (N % (epilogue == 0 ? 64 : 32))
    return fail(OASIS_ERR_UNSUPPORTED, "oasis_gemm_bf16: N must be a multiple of 64 (bf16) / 32 (fp32)");
  if (!aligned16(D) || (epilogue == 0 ? (ldd % 8) : (ldd % 4)))
    return fail(OASIS_ERR_ALIGNMENT, "oasis_gemm_bf16: D must be 16-byte aligned rows");
  int bn = 256, ctas = 1, splits = 1;
  choose_tiles(M, N, K, false, &bn, &ctas, &splits);
  if (epilogue == 0 && bn < 64) bn = 64;  // the bf16 TMA-store box is 64 columns wide
  GemmOperands g;
  if (int s = make_gemm_operands(&g, A, lda, B, ldb, M, N, K, bn, ctas)) return s;
  if (int s = set_gemm_output(&g, D, ldd, epilogue == 1)) return s;
  EpiParams ep{};
  ep.out = D;
  ep.ldd = ldd;
  ep.bias = bias;
  return launch_gemm(g, epilogue == 0 ? kEpiStoreBF16 : kEpiStoreF32Bias, ep, stream);
}

extern "C" int oasis_selftest_bounded_wait(cudaStream_t stream) {
  using namespace oasis;
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "bounded_wait_selftest_kernel");
  return OASIS_OK;
}
