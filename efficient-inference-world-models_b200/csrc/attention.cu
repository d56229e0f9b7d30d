// Spatial (144-token, non-causal) and temporal (<=32-frame, causal) attention.
//
// Both are small, HBM/L2-bound attention problems (head dim 64): a whole
// sequence fits one tile, so softmax is exact (no online rescaling).  QK^T and PV
// run on mma.sync m16n8k16 bf16 tensor-core tiles with fp32 accumulation; q and k
// arrive post-RoPE from the QKV GEMM epilogue.  Temporal K/V may come from the
// quantised cache: FP8/INT4 codes are dequantised while they are staged into
// shared memory, so the cache is never materialised in bf16 in HBM.
#include <algorithm>

#include "launch.cuh"

namespace oasis {

constexpr int kQkvLd = 3 * OASIS_HIDDEN;  // 3072
constexpr int kSmemStride = 72;           // bf16 per staged row (64 + 8 pad: conflict-free ldmatrix)

// Address of 16-byte chunk `chunk` (0..7) of row `row` in a tile of 128-byte rows
// written by TMA with 128-byte swizzle (tile base 1024-byte aligned): the chunk index
// is XORed with row mod 8, which also makes 8-row ldmatrix reads bank-conflict free.
__device__ __forceinline__ uint32_t sw128(uint32_t tile, int row, int chunk) {
  return tile + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// ----------------------------------------------------------------------------------
// spatial attention (144 tokens of one frame, non-causal)
// ----------------------------------------------------------------------------------
constexpr int kSpTile = OASIS_TOKENS * 128;  // 18,432 B: 144 rows x 64 bf16, 128B-swizzled

// 16 query rows r0..r0+15 of one (frame, head) on the legacy tensor path (mma.sync
// m16n8k16) by one warp, from swizzled Q/K/V tiles: online softmax over 3 key blocks
// of 48; writes the 16 output rows into the swizzled tile sO (the same rows of Q, read
// into registers first).
__device__ __forceinline__ void spatial_rows16(uint32_t sQ, uint32_t sK, uint32_t sV, int r0, int lane,
                                               float scale_log2, uint8_t* sO) {
  uint32_t qa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    ldsm_x4(sw128(sQ, r0 + (lane & 15), kk * 2 + (lane >> 4)), qa[kk][0], qa[kk][1], qa[kk][2],
            qa[kk][3]);
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
#pragma unroll 1
  for (int kb = 0; kb < 3; ++kb) {
    float s[6][4];
#pragma unroll
    for (int j = 0; j < 6; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int jp = 0; jp < 3; ++jp) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1, b2, b3;
        const int key = kb * 48 + jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(sw128(sK, key, kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * jp], qa[kk], b0, b1);
        mma_bf16_16816(s[2 * jp + 1], qa[kk], b2, b3);
      }
    }
    float bm0 = m0, bm1 = m1;
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      bm0 = fmaxf(bm0, fmaxf(s[j][0], s[j][1]));
      bm1 = fmaxf(bm1, fmaxf(s[j][2], s[j][3]));
    }
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
    const float alpha0 = exp2f((m0 - bm0) * scale_log2), alpha1 = exp2f((m1 - bm1) * scale_log2);
    m0 = bm0;
    m1 = bm1;
    const float o0 = m0 * scale_log2, o1 = m1 * scale_log2;
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      s[j][0] = exp2f(s[j][0] * scale_log2 - o0);
      s[j][1] = exp2f(s[j][1] * scale_log2 - o0);
      s[j][2] = exp2f(s[j][2] * scale_log2 - o1);
      s[j][3] = exp2f(s[j][3] * scale_log2 - o1);
      sum0 += s[j][0] + s[j][1];
      sum1 += s[j][2] + s[j][3];
    }
    l0 = l0 * alpha0 + sum0;
    l1 = l1 * alpha1 + sum1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= alpha0;
      o[j][1] *= alpha0;
      o[j][2] *= alpha1;
      o[j][3] *= alpha1;
    }
#pragma unroll
    for (int kk = 0; kk < 3; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jd = 0; jd < 8; jd += 2) {
        uint32_t b0, b1, b2, b3;
        const int key = kb * 48 + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(sw128(sV, key, jd + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16_16816(o[jd], pa, b0, b1);
        mma_bf16_16816(o[jd + 1], pa, b2, b3);
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  const int g = lane >> 2, c = lane & 3;
  const int ra = r0 + g, rb = ra + 8;
#pragma unroll
  for (int jd = 0; jd < 8; ++jd) {
    *reinterpret_cast<uint32_t*>(sO + ra * 128 + ((jd ^ (ra & 7)) << 4) + 4 * c) =
        pack_bf16x2(o[jd][0] * inv0, o[jd][1] * inv0);
    *reinterpret_cast<uint32_t*>(sO + rb * 128 + ((jd ^ (rb & 7)) << 4) + 4 * c) =
        pack_bf16x2(o[jd][2] * inv1, o[jd][3] * inv1);
  }
}

// One CTA per (frame, head), 6 warps.  Q, K, V (144 x 64 each) arrive by TMA into
// 128B-swizzled tiles.  Query rows 0..127 run on tcgen05: warp 0 issues S = Q K^T
// (M=128, N=144, K=64) into TMEM; warps 2..5 (one query row per TMEM lane) read their
// row of S, take the exact softmax in registers and write P (bf16) as a K-major
// swizzled tile; warp 0 issues O = P V (M=128, N=64, K=144, V as an MN-major operand)
// into TMEM; warps 2..5 normalise O into the Q tile (free once S is computed).  Rows
// 128..143 run concurrently on warp 1 with mma.sync (spatial_rows16).  The finished
// 144 x 64 tile leaves by one TMA store.
constexpr int kSpThreads = 192;
constexpr int kSpPAtom = 128 * 128;                          // 16 KB: 128 rows x 64 keys bf16
constexpr int kSpSmem = 3 * kSpTile + 3 * kSpPAtom + 1024 + 64;  // 104,448 + slack + barriers
constexpr int kSpTmemCols = 256;                             // S: columns 0..143, O: 192..255
constexpr int kSpOCol = 192;

__global__ void __launch_bounds__(kSpThreads, 2)
    attn_spatial_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                        const __grid_constant__ CUtensorMap tm_out, float scale_log2) {
  pdl_trigger();
  extern __shared__ uint8_t sm_sp[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_sp) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t* sP = tiles + 3 * kSpTile;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 3 * kSpPAtom);  // qk, v, s, p, o
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 5);
  const int f = blockIdx.x;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    mbar_init(&bar[3], 4);  // one arrival per softmax warp
    mbar_init(&bar[4], 1);
    mbar_fence_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) tmem_alloc<kSpTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // qkv comes from the previous kernel; out is read by earlier ones
  const uint32_t sQ = smem_u32(tiles), sK = sQ + kSpTile, sV = sK + kSpTile;
  const uint32_t sPa = smem_u32(sP);

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar[0], 2 * kSpTile);
      tma_load_2d(tiles, &tm_qkv, &bar[0], h * 64, f * OASIS_TOKENS);
      tma_load_2d(tiles + kSpTile, &tm_qkv, &bar[0], OASIS_HIDDEN + h * 64, f * OASIS_TOKENS);
      mbar_arrive_expect_tx(&bar[1], kSpTile);
      tma_load_2d(tiles + 2 * kSpTile, &tm_qkv, &bar[1], 2 * OASIS_HIDDEN + h * 64, f * OASIS_TOKENS);
      if (mbar_wait(&bar[0], 0)) {
        tc_fence_after();
        constexpr uint32_t idesc_s = umma_idesc_bf16(128, OASIS_TOKENS);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tmem, umma_desc_sw128(sQ + k * 32), umma_desc_sw128(sK + k * 32), idesc_s, k > 0);
        umma_commit(&bar[2]);
        if (mbar_wait(&bar[1], 0) && mbar_wait(&bar[3], 0)) {
          tc_fence_after();
          constexpr uint32_t idesc_o = umma_idesc_bf16(128, 64, true);
#pragma unroll
          for (int k = 0; k < OASIS_TOKENS / 16; ++k)  // 9 steps of 16 keys
            umma_bf16(tmem + kSpOCol,
                      umma_desc_sw128(sPa + (k >> 2) * kSpPAtom + (k & 3) * 32),
                      umma_desc_sw128_mn(sV + k * 2048), idesc_o, k > 0);
          umma_commit(&bar[4]);
        }
      }
    }
  } else if (warp == 1) {
    if (mbar_wait(&bar[0], 0) && mbar_wait(&bar[1], 0))
      spatial_rows16(sQ, sK, sV, 128, lane, scale_log2, tiles);
  } else {
    const int quarter = warp & 3;       // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;  // this thread's query row
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = mbar_wait(&bar[2], 0);
    float inv = 0.0f;
    if (ok) {
      tc_fence_after();
      float v[64], v16[16];
      float m = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        tmem_ld64(trow + c * 64, v);
#pragma unroll
        for (int i = 0; i < 64; ++i) m = fmaxf(m, v[i]);
      }
      tmem_ld16(trow + 128, v16);
#pragma unroll
      for (int i = 0; i < 16; ++i) m = fmaxf(m, v16[i]);
      const float mo = m * scale_log2;
      float sum = 0.0f;
      // P row r, keys k: atom k / 64, 16-byte chunk (k % 64) / 8, swizzled by r mod 8
      uint8_t* prow = sP + r * 128;
      auto put8 = [&](int key0, const float* e) {
        const uint4 q = make_uint4(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]),
                                   pack_bf16x2(e[4], e[5]), pack_bf16x2(e[6], e[7]));
        *reinterpret_cast<uint4*>(prow + (key0 >> 6) * kSpPAtom + ((((key0 & 63) >> 3) ^ (r & 7)) << 4)) = q;
      };
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        tmem_ld64(trow + c * 64, v);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          v[i] = exp2f(v[i] * scale_log2 - mo);
          sum += v[i];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) put8(c * 64 + j * 8, v + j * 8);
      }
      tmem_ld16(trow + 128, v16);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v16[i] = exp2f(v16[i] * scale_log2 - mo);
        sum += v16[i];
      }
      put8(128, v16);
      put8(136, v16 + 8);
      inv = 1.0f / sum;
      fence_async_smem_cta();  // P (generic writes) is read by the tensor core next
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar[3]);
    if (ok && mbar_wait(&bar[4], 0)) {
      tc_fence_after();
      // row r of O into row r of the Q tile (the S MMA that read it has completed)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float o[32];
        tmem_ld32(trow + kSpOCol + half * 32, o);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(tiles + r * 128 + (((half * 4 + q) ^ (r & 7)) << 4)) =
              make_uint4(pack_bf16x2(o[8 * q + 0] * inv, o[8 * q + 1] * inv),
                         pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                         pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv),
                         pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
      }
    }
  }
  fence_async_smem_cta();  // the O rows (generic writes) are read by the TMA store below
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<kSpTmemCols>(tmem);
  if (threadIdx.x == 0) {
    tma_store_2d(&tm_out, tiles, h * 64, f * OASIS_TOKENS);
    bulk_commit();
    bulk_wait_read<0>();  // shared memory is read before the CTA exits
  }
}

// ----------------------------------------------------------------------------------
// temporal attention, several query frames: one warp per (session, token, head);
// CTA = 4 heads of one token
// ----------------------------------------------------------------------------------

constexpr int kTpWarps = 4;
constexpr int kTpRowsPerMat = 32;
constexpr int kTpWarpSmem = 3 * kTpRowsPerMat * kSmemStride;  // bf16 elements
constexpr int kTpTileBytes = kTpWarps * kTpWarpSmem * 2;        // 55,296 B
// raw staging of quantised cached rows, per tensor: 32 rows x 256 B of codes (4 heads of
// FP8; INT4 uses the first 128 B) + 32 x 16 B of per-row scale (8 B) and zero (8 B)
constexpr int kTpRawCodes = kTpRowsPerMat * 256;
constexpr int kTpRawTensor = kTpRawCodes + kTpRowsPerMat * 16;
constexpr int kTpSmem = kTpTileBytes + 2 * kTpRawTensor;        // 72,704 B
constexpr int kTpTmaTile = kTpRowsPerMat * 128;                   // 4 KB: 32 frames x 64 bf16
constexpr int kTpTmaTiles = kTpWarps * 3 * kTpTmaTile;            // 48 KB
constexpr int kTpSmemTma = kTpTmaTiles + 1024 + 64;               // + alignment slack, barrier

// two e4m3fn codes -> floats (hardware conversion to f16 is exact, NaN codes stay NaN)
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_codes) {
  uint32_t h;
  const uint16_t v = static_cast<uint16_t>(two_codes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Dequantised values, rounded to bf16 once as the reference's bf16 dequantisation does:
// FP8 code x scale (exact in fp32: 4 x 8 significant bits); INT4 code x scale + zero
// (code x fp16 scale is exact in fp32, so fused and unfused forms agree).
__device__ __forceinline__ float dq_fp8(float code_value, float scale) {
  return bf16_round(code_value * scale);
}
__device__ __forceinline__ float dq_int4(uint32_t code, float scale, float zero) {
  return bf16_round(__fmaf_rn(static_cast<float>(code), scale, zero));
}

// 8 codes -> 8 bf16, dequantised exactly as q.to(bf16) * scale in bf16 (one rounding)
__device__ __forceinline__ uint4 dequant_fp8x8(uint32_t lo, uint32_t hi, float scale) {
  const float2 a = e4m3x2_to_float2(lo), b = e4m3x2_to_float2(lo >> 16);
  const float2 c = e4m3x2_to_float2(hi), d = e4m3x2_to_float2(hi >> 16);
  return make_uint4(pack_bf16x2(a.x * scale, a.y * scale), pack_bf16x2(b.x * scale, b.y * scale),
                    pack_bf16x2(c.x * scale, c.y * scale), pack_bf16x2(d.x * scale, d.y * scale));
}

__device__ __forceinline__ uint4 dequant_int4x8(uint32_t w, float scale, float zero) {
  // 4 bytes = 8 codes; element 2i in the high nibble
  uint32_t r[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t byte = (w >> (8 * b)) & 0xFFu;
    r[b] = pack_bf16x2(__fmaf_rn(static_cast<float>(byte >> 4), scale, zero),
                       __fmaf_rn(static_cast<float>(byte & 0xFu), scale, zero));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// TMA = true: full-window call (no cached past): Q, K, V of the 4 heads arrive by 12
// TMA tensor loads (box = 32 frames x 64 columns of one token) into 128B-swizzled
// 4 KB tiles.  TMA = false: cached past frames.  All rows are first copied
// asynchronously (cp.async): bf16 rows straight into the tiles, FP8/INT4 codes and their
// scales into a raw area, so every load of the CTA is in flight at once; the codes are
// then dequantised from shared memory into the tiles.  Keys and values follow their own
// slot maps.
template <bool TMA>
__global__ void __launch_bounds__(kTpWarps * 32)
    attn_temporal_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                         const __grid_constant__ CUtensorMap tm_out,
                         const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                         const __grid_constant__ KvView kv, int layer, int q_frames, int q_pos0,
                         int n_past, int n_kv, float scale_log2) {
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm_tp_raw[];
  uint8_t* sm_tp = TMA ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_tp_raw) + 1023) &
                                                    ~static_cast<uintptr_t>(1023))
                       : sm_tp_raw;
  uint64_t* tbar = reinterpret_cast<uint64_t*>(sm_tp + kTpTmaTiles);
  if (TMA && threadIdx.x == 0) {
    mbar_init(tbar, 1);
    mbar_fence_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_out);
  }
  if (TMA) __syncthreads();
  pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x;                 // token within frame
  const int hg = blockIdx.y;                // group of 4 heads
  const int h = hg * kTpWarps + warp;
  const int b = blockIdx.z;                 // session
  __nv_bfloat16* smem_all = reinterpret_cast<__nv_bfloat16*>(sm_tp);
  // per head hh: Q, K, V blocks of 32 rows x kSmemStride
  auto mat = [&](int hh, int which) { return smem_all + hh * kTpWarpSmem + which * kTpRowsPerMat * kSmemStride; };

  const int m_tiles = (q_frames + 15) >> 4;  // 1 or 2
  const int n_pairs = (n_kv + 15) >> 4;      // key tiles of 16 (1 or 2)
  const int tid = threadIdx.x;
  const int n_live = n_kv - n_past;

  if constexpr (TMA) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(tbar, kTpTmaTiles);
      for (int hh = 0; hh < kTpWarps; ++hh)
        for (int which = 0; which < 3; ++which)
          tma_load_3d(sm_tp + (hh * 3 + which) * kTpTmaTile, &tm_qkv, tbar,
                      which * OASIS_HIDDEN + (hg * kTpWarps + hh) * 64, p, b * q_frames);
    }
    if (!mbar_wait(tbar, 0)) return;  // timeout recorded in the device error word
  } else {
    uint8_t* raw = sm_tp + kTpTileBytes;  // [K | V] raw areas
    // ---- phase 1: every copy in flight (the 4 heads of one (session, token) are contiguous) ----
    // Q rows and live K/V rows: 3 x 512 B per frame, 16-byte chunks
    for (int i = tid; i < q_frames * 32; i += kTpWarps * 32) {
      const int t = i >> 5, c = i & 31;
      const __nv_bfloat16* src = qkv + (static_cast<long long>(b * q_frames + t) * OASIS_TOKENS + p) * kQkvLd + hg * 256 + c * 8;
      cp_async16(mat(c >> 3, 0) + t * kSmemStride + (c & 7) * 8, src);
    }
    for (int i = tid; i < n_live * 64; i += kTpWarps * 32) {
      const int j = i >> 6, which = 1 + ((i >> 5) & 1), c = i & 31;
      const __nv_bfloat16* src = qkv + (static_cast<long long>(b * q_frames + j) * OASIS_TOKENS + p) * kQkvLd +
                                 which * OASIS_HIDDEN + hg * 256 + c * 8;
      cp_async16(mat(c >> 3, which) + (n_past + j) * kSmemStride + (c & 7) * 8, src);
    }
    // cached rows, unit u (0..31) of the (slot, tensor) row: bf16 32 x 16 B; FP8 16 x 16 B
    // of codes + the 4 heads' scales; INT4 8 x 16 B + the token's 4 scales and 4 zeros
    for (int i = tid; i < n_past * 64; i += kTpWarps * 32) {
      const int s = i >> 6, which = 1 + ((i >> 5) & 1), u = i & 31;
      const KvTensor& t = kv.t[which - 1];
      const int kind = t.kind[s];
      uint8_t* rt = raw + (which - 1) * kTpRawTensor;
      if (kind == OASIS_KV_BF16) {
        const long long page = kv_page(b, kv.layers, layer, t.n_bf16, t.index[s]);
        cp_async16(mat(u >> 3, which) + s * kSmemStride + (u & 7) * 8,
                   t.bf16 + (page * OASIS_TOKENS + p) * OASIS_HIDDEN + hg * 256 + u * 8);
      } else if (kind == OASIS_KV_FP8) {
        const long long page = kv_page(b, kv.layers, layer, t.n_fp8, t.index[s]);
        if (u < 16)
          cp_async16(rt + s * 256 + u * 16, t.fp8 + (page * OASIS_TOKENS + p) * OASIS_HIDDEN + hg * 256 + u * 16);
        else if (u == 16)
          cp_async8(rt + kTpRawCodes + s * 16, t.fp8_scale + page * OASIS_HEADS + hg * 4);
      } else {
        const long long page = kv_page(b, kv.layers, layer, t.n_int4, t.index[s]);
        const long long grp = (page * OASIS_TOKENS + p) * OASIS_HEADS + hg * 4;
        if (u < 8)
          cp_async16(rt + s * 256 + u * 16, t.int4 + grp * 32 + u * 16);
        else if (u == 8)
          cp_async8(rt + kTpRawCodes + s * 16, t.i4_scale + grp);
        else if (u == 9)
          cp_async8(rt + kTpRawCodes + s * 16 + 8, t.i4_zero + grp);
      }
    }
    cp_async_wait_all();
    __syncthreads();
    // ---- phase 2: dequantise the raw rows into the tiles (8 elements per item) ----
    for (int i = tid; i < n_past * 64; i += kTpWarps * 32) {
      const int s = i >> 6, which = 1 + ((i >> 5) & 1), u = i & 31;
      const int kind = kv.t[which - 1].kind[s];
      if (kind == OASIS_KV_BF16) continue;
      const uint8_t* rt = raw + (which - 1) * kTpRawTensor;
      const int hh = u >> 3, c = u & 7;  // head, 8-element chunk
      uint4 v;
      if (kind == OASIS_KV_FP8) {
        const uint2 w = *reinterpret_cast<const uint2*>(rt + s * 256 + hh * 64 + c * 8);
        const float scale =
            __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(rt + kTpRawCodes + s * 16)[hh]);
        v = dequant_fp8x8(w.x, w.y, scale);
      } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(rt + s * 256 + hh * 32 + c * 4);
        const __half* aux = reinterpret_cast<const __half*>(rt + kTpRawCodes + s * 16);
        v = dequant_int4x8(w, __half2float(aux[hh]), __half2float(aux[4 + hh]));
      }
      *reinterpret_cast<uint4*>(mat(hh, which) + s * kSmemStride + c * 8) = v;
    }
    // zero the padding rows the MMAs read (keeps masked products finite)
    for (int i = tid; i < kTpWarps * 3 * 32 * 8; i += kTpWarps * 32) {
      const int hh = i / (3 * 32 * 8), which = (i / (32 * 8)) % 3, r = (i >> 3) & 31, c = i & 7;
      const bool pad = which == 0 ? (r >= q_frames && r < m_tiles * 16) : (r >= n_kv && r < n_pairs * 16);
      if (pad) *reinterpret_cast<uint4*>(mat(hh, which) + r * kSmemStride + c * 8) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
  }
  // 16-byte chunk `chunk` of row `row` of this warp's Q (0), K (1) or V (2) tile
  auto at = [&](int which, int row, int chunk) -> uint32_t {
    if constexpr (TMA)
      return sw128(smem_u32(sm_tp + (warp * 3 + which) * kTpTmaTile), row, chunk);
    else
      return smem_u32(mat(warp, which) + row * kSmemStride + chunk * 8);
  };
  const int g = lane >> 2, c = lane & 3;

  for (int mt = 0; mt < m_tiles; ++mt) {
    uint32_t qa[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      ldsm_x4(at(0, mt * 16 + (lane & 15), kk * 2 + (lane >> 4)), qa[kk][0], qa[kk][1], qa[kk][2],
              qa[kk][3]);
    float s[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
    // key tiles this query tile can see: a tile whose first key lies past the tile's last
    // query position is fully masked (its products would be zeroed), so it is skipped
    const int live_pairs = min(n_pairs, (q_pos0 + mt * 16 + 15) / 16 + 1);
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
      if (jp < live_pairs) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t b0, b1, b2, b3;
          const int key = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
          ldsm_x4(at(1, key, kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
          mma_bf16_16816(s[2 * jp], qa[kk], b0, b1);
          mma_bf16_16816(s[2 * jp + 1], qa[kk], b2, b3);
        }
      }
    }
    // causal mask: query row t at window position q_pos0 + t sees keys 0..q_pos0+t
    const int qp0 = q_pos0 + mt * 16 + g;
    const int qp1 = qp0 + 8;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = j * 8 + 2 * c + e;
        const bool ok = key < n_kv;
        if (!(ok && key <= qp0)) s[j][e] = -INFINITY;
        if (!(ok && key <= qp1)) s[j][2 + e] = -INFINITY;
        mx0 = fmaxf(mx0, s[j][e]);
        mx1 = fmaxf(mx1, s[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float o0 = mx0 * scale_log2, o1 = mx1 * scale_log2;
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j][0] = exp2f(s[j][0] * scale_log2 - o0);
      s[j][1] = exp2f(s[j][1] * scale_log2 - o0);
      s[j][2] = exp2f(s[j][2] * scale_log2 - o1);
      s[j][3] = exp2f(s[j][3] * scale_log2 - o1);
      sum0 += s[j][0] + s[j][1];
      sum1 += s[j][2] + s[j][3];
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);

    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      if (kk < live_pairs) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int jd = 0; jd < 8; jd += 2) {
          uint32_t b0, b1, b2, b3;
          const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldsm_x4_t(at(2, key, jd + (lane >> 4)), b0, b1, b2, b3);
          mma_bf16_16816(o[jd], pa, b0, b1);
          mma_bf16_16816(o[jd + 1], pa, b2, b3);
        }
      }
    }
    const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
    const int t0 = mt * 16 + g, t1 = t0 + 8;
    if constexpr (TMA) {
      // O rows t0, t1 into this warp's Q tile (rows mt*16.. were read into registers
      // above and are not read again), same 128B swizzle; one TMA store per warp below
      uint8_t* otile = sm_tp + (warp * 3) * kTpTmaTile;
#pragma unroll
      for (int jd = 0; jd < 8; ++jd) {
        *reinterpret_cast<uint32_t*>(otile + t0 * 128 + ((jd ^ (t0 & 7)) << 4) + 4 * c) =
            pack_bf16x2(o[jd][0] * inv0, o[jd][1] * inv0);
        *reinterpret_cast<uint32_t*>(otile + t1 * 128 + ((jd ^ (t1 & 7)) << 4) + 4 * c) =
            pack_bf16x2(o[jd][2] * inv1, o[jd][3] * inv1);
      }
      continue;
    }
    if (t0 < q_frames) {
      __nv_bfloat16* orow = out + (static_cast<long long>(b * q_frames + t0) * OASIS_TOKENS + p) * OASIS_HIDDEN + h * 64;
#pragma unroll
      for (int jd = 0; jd < 8; ++jd)
        *reinterpret_cast<uint32_t*>(orow + jd * 8 + 2 * c) = pack_bf16x2(o[jd][0] * inv0, o[jd][1] * inv0);
    }
    if (t1 < q_frames) {
      __nv_bfloat16* orow = out + (static_cast<long long>(b * q_frames + t1) * OASIS_TOKENS + p) * OASIS_HIDDEN + h * 64;
#pragma unroll
      for (int jd = 0; jd < 8; ++jd)
        *reinterpret_cast<uint32_t*>(orow + jd * 8 + 2 * c) = pack_bf16x2(o[jd][2] * inv1, o[jd][3] * inv1);
    }
  }
  if constexpr (TMA) {
    // the warp's head: q_frames rows x 128 B, strided by a frame in the output
    fence_async_smem_cta();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(&tm_out, sm_tp + (warp * 3) * kTpTmaTile, h * 64, p, b * q_frames);
      bulk_commit();
      bulk_wait_read<0>();  // shared memory is read before the CTA exits
    }
  }
}


// ----------------------------------------------------------------------------------
// temporal attention of ONE query frame over cached frames (the incremental forward):
// a persistent grid; each CTA walks work items (session, token, 8 heads), one warp per
// head, with the next item's rows in flight while it computes the current one.
// ----------------------------------------------------------------------------------
// Per item, warp 0 brings the cached key and value rows (8 heads: 1024 B bf16, 512 B FP8
// codes, 256 B INT4 codes per slot) into one of two shared-memory stages by bulk copies
// and the per-slot scales/zeros by plain loads, and the query frame's own q, k, v rows,
// on two mbarriers (q + keys, values).  Scores and probability-weighted values of the
// cached slots run on tensor cores (mma.sync m16n8k16, f16 operands, fp32 accumulation,
// the query in row 0): FP8 codes become f16 by one cvt per pair (exact), INT4 codes by the
// 1024-offset f16 trick (exact), bf16 rows by f32 -> f16; the FP8 scale and the INT4
// scale and zero are applied to the fp32 scores (s_j = scale_j * q.c_j [+ zero_j sum(q)])
// and to the probabilities (p'_j = p_j * scale_j / max scale, plus sum_j p_j zero_j).
// The query frame's own key and value (bf16) are one more key on the CUDA cores.  Head
// dims are permuted inside each k-step so a thread's 16 dims of a key row are one load,
// and the output dims so its 8 dims of a value row are one load; each kind's rows sit in
// their own region with a stride that keeps those loads free of bank conflicts.  Slots
// past the cached frames map to rows zero-filled once, so the tiles need no branch.
constexpr int kDecHeads = 8;
constexpr int kDecThreads = kDecHeads * 32;
constexpr int kDecMaxStage = 112 * 1024;  // two stages must fit the 227 KB of a CTA
// Kinds of the decode kernel's template: one storage kind for every cached slot of a
// tensor, or kDecMixed (per-slot kinds and row offsets from the layout).
constexpr int kDecMixed = 3;

struct DecodeLayout {
  uint32_t k_row[OASIS_MAX_FRAMES], v_row[OASIS_MAX_FRAMES];  // row of slot j in a stage
  uint32_t k_base, v_base, k_stride, v_stride;  // uniform kinds: row j at base + j * stride
  uint32_t aux;          // K scales of slot j at aux + 32 j, V scales at aux + 1024 + 32 j
  uint32_t live;         // q | k | v rows of the query frame, 1 KB each
  uint32_t stage_bytes;  // one pipeline stage (a multiple of 128)
  uint32_t k_bytes, v_bytes;  // bulk-copy bytes of one item on the two barriers
  unsigned long long k_kinds, v_kinds;  // 2 bits per slot 0..31 (slots past n_past: kind of their zero row)
  int live_kv;           // the query frame's own K/V is a key (at window position n_past)
  int items;             // batch * 144 tokens * 2 head groups
};

__device__ __forceinline__ int decode_kind(unsigned long long kinds, int j) {
  return static_cast<int>((kinds >> (2 * j)) & 3ull);
}
__device__ __forceinline__ uint32_t f16x2_e4m3x2(uint32_t two_codes) {
  uint32_t h;
  const uint16_t v = static_cast<uint16_t>(two_codes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  return h;
}
__device__ __forceinline__ uint32_t f16x2_bf16x2(uint32_t w) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(bf16_hi(w)), "f"(bf16_lo(w)));
  return h;
}
// one packed byte of two INT4 codes (element 2i high) -> f16x2 (high nibble in the low half)
__device__ __forceinline__ uint32_t f16x2_nibbles(uint32_t byte) {
  const uint32_t biased = ((byte >> 4) & 0xFu) | ((byte & 0xFu) << 16) | 0x64006400u;  // 1024 + code
  uint32_t h;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h) : "r"(biased), "r"(0x64006400u));
  return h;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  return h;
}
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// f16 fragments of 16 dims (4 k-steps x 2 registers) of one key row of head hh: dims
// 16c + 4ks + {0,1} in [ks][0], + {2,3} in [ks][1].
__device__ __forceinline__ void decode_key_frag(const uint8_t* row, int kind, int hh, int c,
                                                uint32_t (&kb)[4][2]) {
  if (kind == OASIS_KV_FP8) {
    const uint4 x = *reinterpret_cast<const uint4*>(row + hh * 64 + 16 * c);
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      kb[ks][0] = f16x2_e4m3x2(w[ks] & 0xFFFFu);
      kb[ks][1] = f16x2_e4m3x2(w[ks] >> 16);
    }
  } else if (kind == OASIS_KV_INT4) {
    const uint2 x = *reinterpret_cast<const uint2*>(row + hh * 32 + 8 * c);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t h = ((ks < 2) ? x.x : x.y) >> (16 * (ks & 1));
      kb[ks][0] = f16x2_nibbles(h & 0xFFu);
      kb[ks][1] = f16x2_nibbles((h >> 8) & 0xFFu);
    }
  } else {
    const uint4* kp = reinterpret_cast<const uint4*>(row + hh * 128 + 32 * c);
    const uint4 x0 = kp[0], x1 = kp[1];
    const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      kb[ks][0] = f16x2_bf16x2(w[2 * ks]);
      kb[ks][1] = f16x2_bf16x2(w[2 * ks + 1]);
    }
  }
}

// f16 pairs of dims 8g..8g+7 of one value row of head hh (dims 8g + 2q, + 1 in F[q]).
__device__ __forceinline__ void decode_value_row(const uint8_t* row, int kind, int hh, int g,
                                                 uint32_t (&F)[4]) {
  if (kind == OASIS_KV_FP8) {
    const uint2 x = *reinterpret_cast<const uint2*>(row + hh * 64 + 8 * g);
    F[0] = f16x2_e4m3x2(x.x & 0xFFFFu);
    F[1] = f16x2_e4m3x2(x.x >> 16);
    F[2] = f16x2_e4m3x2(x.y & 0xFFFFu);
    F[3] = f16x2_e4m3x2(x.y >> 16);
  } else if (kind == OASIS_KV_INT4) {
    const uint32_t x = *reinterpret_cast<const uint32_t*>(row + hh * 32 + 4 * g);
#pragma unroll
    for (int q = 0; q < 4; ++q) F[q] = f16x2_nibbles((x >> (8 * q)) & 0xFFu);
  } else {
    const uint4 x = *reinterpret_cast<const uint4*>(row + hh * 128 + 16 * g);
    F[0] = f16x2_bf16x2(x.x);
    F[1] = f16x2_bf16x2(x.y);
    F[2] = f16x2_bf16x2(x.z);
    F[3] = f16x2_bf16x2(x.w);
  }
}

// Multiplier and offset of a cached slot's key (s_j = acc * mul + off * sum(q)) or value
// (O += p_j * mul * codes, + p_j * off) for head hh: FP8 (scale, 0), INT4 (scale, zero),
// bf16 (1, 0).
__device__ __forceinline__ float2 decode_slot_scale(const uint8_t* aux, int kind, int hh) {
  if (kind == OASIS_KV_FP8) return make_float2(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(aux)[hh]), 0.0f);
  if (kind == OASIS_KV_INT4)
    return make_float2(__half2float(reinterpret_cast<const __half*>(aux)[hh]),
                       __half2float(reinterpret_cast<const __half*>(aux + 16)[hh]));
  return make_float2(1.0f, 0.0f);
}

template <int KK, int VK>
__global__ void __launch_bounds__(kDecThreads, 2)
    attn_decode_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                       const __grid_constant__ KvView kv, const __grid_constant__ DecodeLayout lay,
                       int layer, int q_pos, int n_past, float scale_log2) {
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t sm_dec[];
  __shared__ __align__(8) uint64_t bars[2][2];  // [stage][keys, values]
  __shared__ int abort_flag;                    // a bounded wait gave up: every warp stops
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hh = warp;                   // head within the group
  const int g = lane >> 2, c = lane & 3;  // mma fragment coordinates
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int st = 0; st < 2; ++st) {
      mbar_init(&bars[st][0], 1);
      mbar_init(&bars[st][1], 1);
    }
    mbar_fence_init();
  }
  // both stages zero-filled once: rows of slots past the cached frames stay zero
  for (uint32_t i = threadIdx.x * 16; i < 2 * lay.stage_bytes; i += kDecThreads * 16)
    *reinterpret_cast<uint4*>(sm_dec + i) = make_uint4(0, 0, 0, 0);
  fence_async_smem_cta();  // the zeros land before any bulk copy writes the same bytes
  __syncthreads();
  pdl_wait();

  // warp 0: one item's rows into stage st
  auto issue = [&](int item, int st) {
    const int hg = item & 1, tok = item >> 1;
    const int p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;
    uint8_t* stage = sm_dec + st * lay.stage_bytes;
    if (lane == 0) {
      mbar_expect_tx(&bars[st][0], lay.k_bytes);
      mbar_expect_tx(&bars[st][1], lay.v_bytes);
    }
    __syncwarp();
    if (lane < n_past) {  // lane s: the keys and values of cached slot s
      const int s = lane;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const KvTensor& t = kv.t[which];
        uint64_t* bar = &bars[st][which];
        uint8_t* row = stage + (which ? lay.v_row[s] : lay.k_row[s]);
        uint8_t* aux = stage + lay.aux + which * 1024 + s * 32;
        const int tk = which ? VK : KK;
        const int kind = tk == kDecMixed ? static_cast<int>(t.kind[s]) : tk;
        const int idx = t.index[s];
        if (kind == OASIS_KV_BF16) {
          const long long page = kv_page(b, kv.layers, layer, t.n_bf16, idx);
          bulk_load(row, t.bf16 + (page * OASIS_TOKENS + p) * OASIS_HIDDEN + hg * kDecHeads * 64,
                    kDecHeads * 128, bar);
        } else if (kind == OASIS_KV_FP8) {
          const long long page = kv_page(b, kv.layers, layer, t.n_fp8, idx);
          bulk_load(row, t.fp8 + (page * OASIS_TOKENS + p) * OASIS_HIDDEN + hg * kDecHeads * 64,
                    kDecHeads * 64, bar);
          *reinterpret_cast<uint4*>(aux) =
              *reinterpret_cast<const uint4*>(t.fp8_scale + page * OASIS_HEADS + hg * kDecHeads);
        } else {
          const long long page = kv_page(b, kv.layers, layer, t.n_int4, idx);
          const long long grp = (page * OASIS_TOKENS + p) * OASIS_HEADS + hg * kDecHeads;
          bulk_load(row, t.int4 + grp * 32, kDecHeads * 32, bar);
          *reinterpret_cast<uint4*>(aux) = *reinterpret_cast<const uint4*>(t.i4_scale + grp);
          *reinterpret_cast<uint4*>(aux + 16) = *reinterpret_cast<const uint4*>(t.i4_zero + grp);
        }
      }
    } else if (lane == 31) {  // the query frame's own q, k, v (bf16 rows of the QKV output)
      const __nv_bfloat16* row = qkv + (static_cast<long long>(b) * OASIS_TOKENS + p) * kQkvLd + hg * kDecHeads * 64;
      bulk_load(stage + lay.live, row, kDecHeads * 128, &bars[st][0]);
      if (lay.live_kv) {
        bulk_load(stage + lay.live + 1024, row + OASIS_HIDDEN, kDecHeads * 128, &bars[st][0]);
        bulk_load(stage + lay.live + 2048, row + 2 * OASIS_HIDDEN, kDecHeads * 128, &bars[st][1]);
      }
    }
    __syncwarp();  // the scale stores of every lane before the arrivals release them
    if (lane == 0) {
      mbar_arrive(&bars[st][0]);
      mbar_arrive(&bars[st][1]);
    }
  };
  auto k_kind = [&](int j) { return KK == kDecMixed ? decode_kind(lay.k_kinds, j) : KK; };
  auto v_kind = [&](int j) { return VK == kDecMixed ? decode_kind(lay.v_kinds, j) : VK; };
  auto k_row = [&](int j) { return KK == kDecMixed ? lay.k_row[j] : lay.k_base + j * lay.k_stride; };
  auto v_row = [&](int j) { return VK == kDecMixed ? lay.v_row[j] : lay.v_base + j * lay.v_stride; };
  const bool live_key = lay.live_kv && n_past <= q_pos;

  int it = blockIdx.x;
  if (warp == 0 && it < lay.items) issue(it, 0);
  for (int k = 0; it < lay.items; ++k, it += gridDim.x) {
    const int st = k & 1;
    const uint32_t ph = (k >> 1) & 1;
    const bool next = it + static_cast<int>(gridDim.x) < lay.items;
    if (warp == 0 && next) issue(it + gridDim.x, st ^ 1);
    const uint8_t* stage = sm_dec + st * lay.stage_bytes;
    const int hg = it & 1, tok = it >> 1;
    // a wait that gives up records a timeout in the device error word; the CTA then
    // stops after this item (below), every warp at the same point
    bool ok = mbar_wait(&bars[st][0], ph);
    if (ok) {

    // ---- the query: lane l holds dims 2l, 2l+1 (the live key's score); lanes 0..3 also
    // hold the A operand (row 0), lane c dims 16c..16c+15 in k-step order
    const uint32_t qw = *reinterpret_cast<const uint32_t*>(stage + lay.live + hh * 128 + 4 * lane);
    float s_live = -INFINITY;
    if (live_key) {
      const uint32_t kw = *reinterpret_cast<const uint32_t*>(stage + lay.live + 1024 + hh * 128 + 4 * lane);
      float d = __fmaf_rn(bf16_hi(qw), bf16_hi(kw), bf16_lo(qw) * bf16_lo(kw));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      s_live = d;
    }
    uint32_t qa[4][2];
    float qsum = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) qa[ks][0] = qa[ks][1] = 0u;
    if (g == 0) {
      const uint4* qp = reinterpret_cast<const uint4*>(stage + lay.live + hh * 128 + 32 * c);
      const uint4 x0 = qp[0], x1 = qp[1];
      const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = f16x2_bf16x2(w[2 * ks]);
        qa[ks][1] = f16x2_bf16x2(w[2 * ks + 1]);
        if (KK == OASIS_KV_INT4 || KK == kDecMixed) {
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][0]));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][1]));
          qsum += (f0.x + f0.y) + (f1.x + f1.y);
        }
      }
    }
    if (KK == OASIS_KV_INT4 || KK == kDecMixed) {
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
    }
    // lane j: multiplier / offset of cached key j
    float2 kscale = make_float2(1.0f, 0.0f);
    if (KK != OASIS_KV_BF16 && lane < n_past) kscale = decode_slot_scale(stage + lay.aux + lane * 32, k_kind(lane), hh);

    // ---- cached scores: n-tile nt holds keys 8nt..8nt+7; this thread supplies key 8nt + g
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
      const int j = 8 * nt + g;
      uint32_t kb[4][2];
      decode_key_frag(stage + k_row(j), k_kind(j), hh, c, kb);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) mma_f16_16816(sacc[nt], qa[ks][0], qa[ks][1], kb[ks][0], kb[ks][1]);
    }

    // ---- softmax over the cached keys (row 0: lanes 0..3 hold keys 8nt + 2c + e) and the live key
    float sc[8];
    float mx = s_live;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = 8 * (i >> 1) + 2 * c + (i & 1);
      float s = sacc[i >> 1][i & 1];
      if (KK != OASIS_KV_BF16) {
        const float mul = __shfl_sync(0xffffffffu, kscale.x, j);
        if (KK == OASIS_KV_INT4 || KK == kDecMixed)
          s = __fmaf_rn(s, mul, __shfl_sync(0xffffffffu, kscale.y, j) * qsum);
        else
          s *= mul;
      }
      sc[i] = (j < n_past && j <= q_pos) ? s : -INFINITY;
      mx = fmaxf(mx, sc[i]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mxs = mx * scale_log2;
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pr = sc[i] == -INFINITY ? 0.0f : exp2f(__fmaf_rn(sc[i], scale_log2, -mxs));
      sum += pr;
      sc[i] = bf16_round(pr);  // the probability as the tensor-core path rounds it
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float p_live = live_key ? exp2f(__fmaf_rn(s_live, scale_log2, -mxs)) : 0.0f;
    sum += p_live;
    const float pb_live = bf16_round(p_live);
    ok = mbar_wait(&bars[st][1], ph);
    if (ok) {
    // value multipliers: lane j holds slot j's; their max normalises P'
    float2 vscale = make_float2(lane < n_past ? 1.0f : 0.0f, 0.0f);
    if (VK != OASIS_KV_BF16 && lane < n_past)
      vscale = decode_slot_scale(stage + lay.aux + 1024 + lane * 32, v_kind(lane), hh);
    float vmax = 1.0f, corr = 0.0f;
    if (VK != OASIS_KV_BF16) {
      vmax = vscale.x;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    const float inv_vmax = 1.0f / vmax;
    float pv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = 8 * (i >> 1) + 2 * c + (i & 1);
      pv[i] = sc[i];
      if (VK != OASIS_KV_BF16) {
        pv[i] = sc[i] * __shfl_sync(0xffffffffu, vscale.x, j) * inv_vmax;
        if (VK == OASIS_KV_INT4 || VK == kDecMixed) corr = __fmaf_rn(sc[i], __shfl_sync(0xffffffffu, vscale.y, j), corr);
      }
    }
    if (VK == OASIS_KV_INT4 || VK == kDecMixed) {
      corr += __shfl_xor_sync(0xffffffffu, corr, 1);
      corr += __shfl_xor_sync(0xffffffffu, corr, 2);
    }
    uint32_t pa[2][2];
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
      pa[k2][0] = pa[k2][1] = 0u;
      if (g == 0) {
        pa[k2][0] = pack_f16x2(pv[4 * k2], pv[4 * k2 + 1]);
        pa[k2][1] = pack_f16x2(pv[4 * k2 + 2], pv[4 * k2 + 3]);
      }
    }

    // ---- O = P' V: n-tile n2 column g is output dim 8g + n2; this thread supplies keys
    // 16 k2 + 2c + {0, 1, 8, 9}, dims 8g..8g+7 of each
    float oacc[8][4];
#pragma unroll
    for (int n2 = 0; n2 < 8; ++n2) oacc[n2][0] = oacc[n2][1] = oacc[n2][2] = oacc[n2][3] = 0.0f;
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
      uint32_t F[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int j = 16 * k2 + 2 * c + (r & 1) + 8 * (r >> 1);
        decode_value_row(stage + v_row(j), v_kind(j), hh, g, F[r]);
      }
#pragma unroll
      for (int n2 = 0; n2 < 8; ++n2) {
        const uint32_t sel = (n2 & 1) ? 0x7632u : 0x5410u;
        const uint32_t b0 = __byte_perm(F[0][n2 >> 1], F[1][n2 >> 1], sel);
        const uint32_t b1 = __byte_perm(F[2][n2 >> 1], F[3][n2 >> 1], sel);
        mma_f16_16816(oacc[n2], pa[k2][0], pa[k2][1], b0, b1);
      }
    }
    if (g == 0) {
      // lane c holds dims 16c + n2 (column 2c) and 16c + 8 + n2 (column 2c + 1)
      const float inv = 1.0f / sum;
      const uint4* vl = reinterpret_cast<const uint4*>(stage + lay.live + 2048 + hh * 128 + 32 * c);
      const uint4 v0 = vl[0], v1 = vl[1];
      const uint32_t vw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        // dims 16c + 2k, 16c + 2k + 1: accumulators of columns 2c (k < 4) / 2c + 1
        const int n2 = (2 * k) & 7, col = k >> 2;
        const float a0 = __fmaf_rn(vmax, oacc[n2][col], corr), a1 = __fmaf_rn(vmax, oacc[n2 + 1][col], corr);
        o[k] = pack_bf16x2(__fmaf_rn(pb_live, bf16_lo(vw[k]), a0) * inv, __fmaf_rn(pb_live, bf16_hi(vw[k]), a1) * inv);
      }
      uint4* orow = reinterpret_cast<uint4*>(out + (static_cast<long long>(tok) * OASIS_HIDDEN) +
                                             (hg * kDecHeads + hh) * 64 + 16 * c);
      orow[0] = make_uint4(o[0], o[1], o[2], o[3]);
      orow[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    }  // values arrived
    }  // keys arrived
    if (!ok) abort_flag = 1;
    __syncthreads();  // every warp is done with this stage before it is refilled
    if (abort_flag) {
      // the prefetched item's copies land (bounded) before the CTA exits
      if (threadIdx.x == 0 && next) {
        const uint32_t ph_next = ((k + 1) >> 1) & 1;
        mbar_wait(&bars[st ^ 1][0], ph_next);
        mbar_wait(&bars[st ^ 1][1], ph_next);
      }
      return;
    }
  }
}

// decode kernel for (key kind, value kind), each a storage kind or kDecMixed
using DecodeKernel = void (*)(const __nv_bfloat16*, __nv_bfloat16*, const KvView, const DecodeLayout, int,
                              int, int, float);
template <int KK>
DecodeKernel decode_kernel_v(int vk) {
  switch (vk) {
    case OASIS_KV_BF16: return attn_decode_kernel<KK, OASIS_KV_BF16>;
    case OASIS_KV_FP8: return attn_decode_kernel<KK, OASIS_KV_FP8>;
    case OASIS_KV_INT4: return attn_decode_kernel<KK, OASIS_KV_INT4>;
  }
  return attn_decode_kernel<KK, kDecMixed>;
}
DecodeKernel decode_kernel(int kk, int vk) {
  switch (kk) {
    case OASIS_KV_BF16: return decode_kernel_v<OASIS_KV_BF16>(vk);
    case OASIS_KV_FP8: return decode_kernel_v<OASIS_KV_FP8>(vk);
    case OASIS_KV_INT4: return decode_kernel_v<OASIS_KV_INT4>(vk);
  }
  return decode_kernel_v<kDecMixed>(vk);
}

// ----------------------------------------------------------------------------------
// host launchers
// ----------------------------------------------------------------------------------
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)

int launch_attn_spatial(const void* qkv, void* out, int frames, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_spatial_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSpSmem);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attn_spatial)");
    configured = true;
  }
  // qkv [frames * 144][3072] bf16; box = one head's 64 columns of one frame's 144 rows
  CUtensorMap tm;
  const long long dims[2] = {3 * OASIS_HIDDEN, static_cast<long long>(frames) * OASIS_TOKENS};
  const long long strides[1] = {3 * OASIS_HIDDEN * 2};
  const int box[2] = {64, OASIS_TOKENS};
  if (int st = encode_bf16_sw128(&tm, qkv, 2, dims, strides, box)) return st;
  // out [frames * 144][1024] bf16; box = one head's 64 columns of one frame's 144 rows
  CUtensorMap tm_out;
  const long long odims[2] = {OASIS_HIDDEN, static_cast<long long>(frames) * OASIS_TOKENS};
  const long long ostrides[1] = {OASIS_HIDDEN * 2};
  if (int st = encode_bf16_sw128(&tm_out, out, 2, odims, ostrides, box)) return st;
  dim3 grid(frames, OASIS_HEADS);
  cudaError_t e = launch_pdl(attn_spatial_kernel, grid, dim3(kSpThreads), kSpSmem, stream, tm,
                             tm_out, kScaleLog2);
  if (e != cudaSuccess) return cuda_status(e, "attn_spatial_kernel");
  return OASIS_OK;
}

int launch_attn_temporal(const void* qkv, const KvView& kv, int layer, void* out, int batch,
                         int q_frames, int q_pos0, int n_past, int n_kv, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_temporal_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kTpSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_temporal_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kTpSmemTma);
    for (int kk = 0; kk < 4 && e == cudaSuccess; ++kk)
      for (int vk = 0; vk < 4 && e == cudaSuccess; ++vk)
        e = cudaFuncSetAttribute(decode_kernel(kk, vk), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 2 * kDecMaxStage);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attn_temporal)");
    configured = true;
  }
  if (q_frames == 1 && n_past > 0 && n_past < OASIS_MAX_FRAMES) {
    // one query frame over cached slots: the persistent decode kernel.  A stage holds the
    // key rows and the value rows of the 32 slots, each kind in its own region with a
    // stride that keeps the fragment loads conflict-free (key rows: bf16 1040, FP8 576,
    // INT4 288 B; value rows: 1040, 528, 272 B), 2 x 32 x 32 B of scales, the live rows.
    // Slots past n_past take rows of the narrowest kind present, which stay zero.
    DecodeLayout lay{};
    lay.live_kv = n_kv > n_past ? 1 : 0;
    lay.items = batch * OASIS_TOKENS * 2;
    auto codes = [](int kind) -> uint32_t {
      return kind == OASIS_KV_BF16 ? kDecHeads * 128 : (kind == OASIS_KV_FP8 ? kDecHeads * 64 : kDecHeads * 32);
    };
    const uint32_t k_strides[3] = {1040, 576, 288}, v_strides[3] = {1040, 528, 272};
    uint32_t off = 0;
    int uniform[2];
    for (int which = 0; which < 2; ++which) {
      const KvTensor& t = kv.t[which];
      const uint32_t* stride = which ? v_strides : k_strides;
      int kinds[OASIS_MAX_FRAMES];
      bool present[3] = {false, false, false};
      for (int s = 0; s < n_past; ++s) {
        kinds[s] = t.kind[s];
        present[kinds[s]] = true;
      }
      int narrow = OASIS_KV_BF16;  // the kind with the smallest rows present
      for (int k : {OASIS_KV_FP8, OASIS_KV_INT4})
        if (present[k]) narrow = k;
      for (int s = n_past; s < OASIS_MAX_FRAMES; ++s) kinds[s] = narrow;
      uniform[which] = (present[0] + present[1] + present[2] == 1) ? narrow : kDecMixed;
      uint32_t* rows = which ? lay.v_row : lay.k_row;
      unsigned long long mask = 0;
      for (int k : {OASIS_KV_BF16, OASIS_KV_FP8, OASIS_KV_INT4}) {  // one region per kind
        for (int s = 0; s < OASIS_MAX_FRAMES; ++s)
          if (kinds[s] == k) {
            rows[s] = off;
            off += stride[k];
          }
      }
      for (int s = 0; s < OASIS_MAX_FRAMES; ++s) mask |= static_cast<unsigned long long>(kinds[s]) << (2 * s);
      uint32_t bytes = 0;
      for (int s = 0; s < n_past; ++s) bytes += codes(kinds[s]);
      if (which) {
        lay.v_kinds = mask;
        lay.v_bytes = bytes + lay.live_kv * kDecHeads * 128;
        lay.v_base = rows[0];
        lay.v_stride = stride[narrow];
      } else {
        lay.k_kinds = mask;
        lay.k_bytes = bytes + (1 + lay.live_kv) * kDecHeads * 128;
        lay.k_base = rows[0];
        lay.k_stride = stride[narrow];
      }
    }
    lay.aux = off;
    off += 2 * 1024;
    lay.live = off;
    off += 3 * kDecHeads * 128;
    lay.stage_bytes = (off + 127) & ~127u;
    if (lay.stage_bytes > static_cast<uint32_t>(kDecMaxStage))
      return fail(OASIS_ERR_UNSUPPORTED, "attn_decode_kernel: stage layout too large");
    DecodeKernel kern = decode_kernel(uniform[0], uniform[1]);
    const size_t smem = 2 * static_cast<size_t>(lay.stage_bytes);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecThreads, smem) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    const int ctas = std::min(lay.items, per_sm * num_sms());
    cudaError_t e = launch_pdl(kern, dim3(ctas), dim3(kDecThreads), smem, stream,
                               static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out),
                               kv, lay, layer, q_pos0, n_past, kScaleLog2);
    if (e != cudaSuccess) return cuda_status(e, "attn_decode_kernel");
    return OASIS_OK;
  }
  dim3 grid(OASIS_TOKENS, OASIS_HEADS / kTpWarps, batch);
  CUtensorMap tm{}, tm_out{};
  const bool tma = n_past == 0;
  if (tma) {
    // qkv viewed as [frames][144 tokens][3072]: box = 64 columns x 1 token x 32 frames
    const long long dims[3] = {3 * OASIS_HIDDEN, OASIS_TOKENS, static_cast<long long>(batch) * q_frames};
    const long long strides[2] = {3 * OASIS_HIDDEN * 2, static_cast<long long>(OASIS_TOKENS) * 3 * OASIS_HIDDEN * 2};
    const int box[3] = {64, 1, kTpRowsPerMat};
    if (int st = encode_bf16_sw128(&tm, qkv, 3, dims, strides, box)) return st;
    // out viewed as [frames][144 tokens][1024]: box = 64 columns x 1 token x q_frames frames
    // (one session's window, so a store never reaches the next session's rows)
    const long long odims[3] = {OASIS_HIDDEN, OASIS_TOKENS, static_cast<long long>(batch) * q_frames};
    const long long ostrides[2] = {OASIS_HIDDEN * 2, static_cast<long long>(OASIS_TOKENS) * OASIS_HIDDEN * 2};
    const int obox[3] = {64, 1, q_frames};
    if (int st = encode_bf16_sw128(&tm_out, out, 3, odims, ostrides, obox)) return st;
  }
  cudaError_t e = tma ? launch_pdl(attn_temporal_kernel<true>, grid, dim3(kTpWarps * 32), kTpSmemTma,
                                   stream, tm, tm_out, static_cast<const __nv_bfloat16*>(qkv),
                                   static_cast<__nv_bfloat16*>(out), kv, layer, q_frames, q_pos0,
                                   n_past, n_kv, kScaleLog2)
                      : launch_pdl(attn_temporal_kernel<false>, grid, dim3(kTpWarps * 32), kTpSmem,
                                   stream, tm, tm_out, static_cast<const __nv_bfloat16*>(qkv),
                                   static_cast<__nv_bfloat16*>(out), kv, layer, q_frames, q_pos0,
                                   n_past, n_kv, kScaleLog2);
  if (e != cudaSuccess) return cuda_status(e, "attn_temporal_kernel");
  return OASIS_OK;
}

}  // namespace oasis

extern "C" int oasis_attn_spatial(const void* qkv, void* out, int frames, cudaStream_t stream) {
  using namespace oasis;
  if (!qkv || !out || frames <= 0) return fail(OASIS_ERR_INVALID_ARG, "oasis_attn_spatial: bad args");
  if (!aligned16(qkv) || !aligned16(out)) return fail(OASIS_ERR_ALIGNMENT, "oasis_attn_spatial: alignment");
  if (frames > 65535 * 16) return fail(OASIS_ERR_UNSUPPORTED, "oasis_attn_spatial: too many frames");
  return launch_attn_spatial(qkv, out, frames, stream);
}

extern "C" int oasis_attn_temporal(const void* qkv, const oasis_kv_cache_t* cache, int layer,
                                   void* out, int batch, int q_frames, int q_pos0, int n_past,
                                   int n_kv, cudaStream_t stream) {
  using namespace oasis;
  if (!qkv || !out || batch <= 0 || q_frames <= 0)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_attn_temporal: bad args");
  if (n_kv < 1 || n_kv > OASIS_MAX_FRAMES || q_frames > OASIS_MAX_FRAMES || n_past < 0 ||
      n_past > n_kv || n_kv - n_past > q_frames || q_pos0 < 0)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_attn_temporal: inconsistent frame counts");
  if (n_past > 0 && (!cache || n_past > cache->n_slots || layer < 0 || layer >= cache->layers ||
                     batch > cache->batch))
    return fail(OASIS_ERR_INVALID_ARG, "oasis_attn_temporal: cache does not cover n_past/layer/batch");
  if (!aligned16(qkv) || !aligned16(out)) return fail(OASIS_ERR_ALIGNMENT, "oasis_attn_temporal: alignment");
  KvView v;
  if (int s = make_kv_view(n_past > 0 ? cache : nullptr, &v)) return s;
  return launch_attn_temporal(qkv, v, layer, out, batch, q_frames, q_pos0, n_past, n_kv, stream);
}
