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
  uint64_t* tbar = reinterpret_cast<uint64_t*>(sm_tp + kTpTmaTiles);  // per head: Q+K, V
  if (TMA && threadIdx.x == 0) {
    for (int i = 0; i < 2 * kTpWarps; ++i) mbar_init(&tbar[i], 1);
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
      // each head's Q and K on one barrier, its V on a second, V last: a warp starts its
      // scores once its own head's Q and K are in, while later heads and the values load
      for (int hh = 0; hh < kTpWarps; ++hh) {
        mbar_arrive_expect_tx(&tbar[2 * hh], 2 * kTpTmaTile);
        for (int which = 0; which < 2; ++which)
          tma_load_3d(sm_tp + (hh * 3 + which) * kTpTmaTile, &tm_qkv, &tbar[2 * hh],
                      which * OASIS_HIDDEN + (hg * kTpWarps + hh) * 64, p, b * q_frames);
      }
      for (int hh = 0; hh < kTpWarps; ++hh) {
        mbar_arrive_expect_tx(&tbar[2 * hh + 1], kTpTmaTile);
        tma_load_3d(sm_tp + (hh * 3 + 2) * kTpTmaTile, &tm_qkv, &tbar[2 * hh + 1],
                    2 * OASIS_HIDDEN + (hg * kTpWarps + hh) * 64, p, b * q_frames);
      }
    }
    if (!mbar_wait(&tbar[2 * warp], 0)) return;  // timeout recorded in the device error word
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
    // zero the padding rows the MMAs read (keeps masked products finite), if there are any
    if (q_frames < m_tiles * 16 || n_kv < n_pairs * 16) {
      for (int i = tid; i < kTpWarps * 3 * 32 * 8; i += kTpWarps * 32) {
        const int hh = i / (3 * 32 * 8), which = (i / (32 * 8)) % 3, r = (i >> 3) & 31, c = i & 7;
        const bool pad = which == 0 ? (r >= q_frames && r < m_tiles * 16) : (r >= n_kv && r < n_pairs * 16);
        if (pad) *reinterpret_cast<uint4*>(mat(hh, which) + r * kSmemStride + c * 8) = make_uint4(0, 0, 0, 0);
      }
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

    if constexpr (TMA) {
      if (mt == 0 && !mbar_wait(&tbar[2 * warp + 1], 0)) return;  // this head's V
    }
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
// temporal attention of ONE query frame over cached frames (the incremental forward)
// ----------------------------------------------------------------------------------
// One warp per (session, token, head): the head's 64-dim query row against up to 31
// cached key rows plus the frame's own key.  Warps are independent (no shared memory, no
// block barrier); a persistent grid walks the items, and each warp issues the next
// item's loads straight into registers as soon as the current item's copies are used
// (keys, query and key scales after the scores; values and value scales after P V), so
// one item's rows are in flight while the warp computes the other.
// Both products run on tensor cores (mma.sync m16n8k16, fp32 accumulation):
//   scores  S[1 x 32] = q K^T: the query is row 0 of A, the keys are the B columns
//           (n-tile nt = keys 8nt..8nt+7; thread (g, c) supplies key 8nt + g);
//   output  O^T[64 x 1] = V^T P^T: V^T is A (m-tile mo = 16 dims; thread (g, c) supplies
//           keys 16kv + 2c + {0, 1, 8, 9}, dims 8g..8g+7) and P^T is column 0 of B, which
//           is where the score accumulators of lanes 0..3 already hold it.
// Rows keep their storage format until the fragment is built: a tensor whose cached
// slots are all bf16 feeds bf16 mma directly; FP8 codes become f16 by one cvt per pair
// (exact); INT4 codes by the 1024-offset f16 trick on nibble pairs (exact).  Inside each
// k-step the head dims are permuted so a thread's dims of a key row are one contiguous
// load, and the query takes the same permutation.  FP8 scales and INT4 scale/zero apply
// to the fp32 scores (s_j = scale_j q.c_j + zero_j sum(q)) and to the probabilities
// (p'_j = p_j scale_j / max scale, plus sum_j p_j zero_j).  The frame's own key and value
// (bf16 rows of the QKV output) are one more key on the CUDA cores.
constexpr int kDecWarps = 4;
constexpr int kDecThreads = kDecWarps * 32;
// Kinds of the decode kernel's template: one storage kind for every cached slot of a
// tensor, or kDecMixed (per-slot kinds from the layout).
constexpr int kDecMixed = 3;
// ... or 4 + 3a + b (a != b): kind a at the key positions below the layout's split, kind b
// from it on (two kind-uniform runs of tiles: the kind branches fold at compile time)
constexpr int kDecSplit = 4;
__host__ __device__ constexpr int dec_split_code(int a, int b) { return kDecSplit + 3 * a + b; }
__host__ __device__ constexpr int dec_split_a(int code) { return (code - kDecSplit) / 3; }
__host__ __device__ constexpr int dec_split_b(int code) { return (code - kDecSplit) % 3; }
// whether a template kind code can hold rows of storage kind `kind`
__host__ __device__ constexpr bool dec_has(int code, int kind) {
  return code == kind || code == kDecMixed ||
         (code >= kDecSplit && (dec_split_a(code) == kind || dec_split_b(code) == kind));
}

struct DecodeTensor {
  uint32_t slot_page[OASIS_MAX_FRAMES];  // layer * n_kind + pool index of slot j
  unsigned long long kinds;              // 2 bits per slot (slots past n_past: any kind)
  uint32_t session_pages[3];             // per kind: layers * n_kind, the pages of one session
};
// Key positions 0..31 of the tiles hold the cached slots in an order the host picks:
// slot order when every slot of a tensor has one kind, else grouped so that each 8-key
// n-tile holds one (key kind, value kind) pair, which keeps the kind branches uniform
// across the warp.  Softmax and P V do not depend on the order.
struct DecodeLayout {
  DecodeTensor t[2];  // keys, values, indexed by key position
  uint32_t valid;     // positions holding a cached slot at or before the query's window position
  int split;          // split kind codes: first position of the second kind (a multiple of 8)
  int items;          // batch * 144 tokens * 16 heads
  int live_kv;        // the query frame's own K/V is a key (at window position n_past)
};

// bytes of one token's 1024 elements / one head's 64 elements in a pool of `kind`
__host__ __device__ constexpr uint32_t dec_row_bytes(int kind) {
  return kind == OASIS_KV_BF16 ? 2048u : (kind == OASIS_KV_FP8 ? 1024u : 512u);
}
__host__ __device__ constexpr uint32_t dec_head_bytes(int kind) { return dec_row_bytes(kind) / 16; }

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldg_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}
// rows of the QKV output (written by the preceding kernel): coherent loads
__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
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
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  return h;
}
// 2^x by the SFU (ex2.approx; 2^-inf = +0, results below the normal range flush to 0: the
// probabilities they would give are far below a bf16 ulp of the row sum)
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t sub_1024(uint32_t biased) {
  uint32_t h;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h) : "r"(biased), "r"(0x64006400u));
  return h;
}
// nibbles at bits s..s+3 and 16+s..19+s of u -> f16x2 (exact codes 0..15)
__device__ __forceinline__ uint32_t nibble_pair(uint32_t u, int s) {
  return sub_1024(((u >> s) & 0x000F000Fu) | 0x64006400u);
}
// one packed byte of two INT4 codes (element 2i high) -> f16x2 (element 2i in the low half)
__device__ __forceinline__ uint32_t f16x2_nibbles(uint32_t byte) {
  return sub_1024(((byte >> 4) & 0xFu) | ((byte & 0xFu) << 16) | 0x64006400u);
}
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Key fragments of one key row (this thread's 16 dims, one contiguous chunk) for the 4
// k-steps: kb[ks][0] pairs with the query's A register of columns 2c, 2c+1, kb[ks][1]
// with columns 2c+8, 2c+9.  Dim order: bf16 and FP8 tensors take dims 16c + 4ks + {0,1}
// and + {2,3} ("consecutive"); INT4 and mixed tensors take, for k = 0, 1, dims
// 16c + 8k + {0,4}, {1,5} (k-step 2k) and {2,6}, {3,7} (k-step 2k+1) ("nibble" order,
// the order in which a masked shift takes nibble pairs out of one 32-bit word).
__device__ __forceinline__ void key_fragments_int4(uint32_t w0, uint32_t w1, uint32_t (&kb)[4][2]) {
  const uint32_t w[2] = {w0, w1};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    kb[2 * k][0] = nibble_pair(w[k], 4);       // elements 0, 4
    kb[2 * k][1] = nibble_pair(w[k], 0);       // 1, 5
    kb[2 * k + 1][0] = nibble_pair(w[k], 12);  // 2, 6
    kb[2 * k + 1][1] = nibble_pair(w[k], 8);   // 3, 7
  }
}
template <int KK, int KW>
__device__ __forceinline__ void key_fragments(const uint32_t (&w)[KW], int kind, uint32_t (&kb)[4][2]) {
  if constexpr (KK == OASIS_KV_BF16) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      kb[ks][0] = w[2 * ks];
      kb[ks][1] = w[2 * ks + 1];
    }
  } else if constexpr (KK == OASIS_KV_FP8) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      kb[ks][0] = f16x2_e4m3x2(w[ks]);
      kb[ks][1] = f16x2_e4m3x2(w[ks] >> 16);
    }
  } else if constexpr (KK == OASIS_KV_INT4) {
    key_fragments_int4(w[0], w[1], kb);
  } else if (kind == OASIS_KV_INT4) {  // mixed tensor (8 words a row)
    key_fragments_int4(w[0], w[1], kb);
  } else if (kind == OASIS_KV_FP8) {  // mixed tensor, FP8 row in nibble order
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t x = __byte_perm(w[2 * k], w[2 * k + 1], 0x5140);  // d0 d4 d1 d5
      const uint32_t y = __byte_perm(w[2 * k], w[2 * k + 1], 0x7362);  // d2 d6 d3 d7
      kb[2 * k][0] = f16x2_e4m3x2(x);
      kb[2 * k][1] = f16x2_e4m3x2(x >> 16);
      kb[2 * k + 1][0] = f16x2_e4m3x2(y);
      kb[2 * k + 1][1] = f16x2_e4m3x2(y >> 16);
    }
  } else {  // mixed tensor, bf16 row in nibble order
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      kb[2 * k][0] = f16x2_bf16x2(__byte_perm(w[4 * k], w[4 * k + 2], 0x5410));
      kb[2 * k][1] = f16x2_bf16x2(__byte_perm(w[4 * k], w[4 * k + 2], 0x7632));
      kb[2 * k + 1][0] = f16x2_bf16x2(__byte_perm(w[4 * k + 1], w[4 * k + 3], 0x5410));
      kb[2 * k + 1][1] = f16x2_bf16x2(__byte_perm(w[4 * k + 1], w[4 * k + 3], 0x7632));
    }
  }
}

// f16x2 pairs of dims (2m, 2m+1), m = 0..3, of one value row's 8-dim chunk (mixed
// tensors: 4 words a row)
__device__ __forceinline__ void value_row_pairs(const uint32_t (&r)[4], int kind, uint32_t (&G)[4]) {
  if (kind == OASIS_KV_BF16) {
#pragma unroll
    for (int m = 0; m < 4; ++m) G[m] = f16x2_bf16x2(r[m]);
  } else if (kind == OASIS_KV_FP8) {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      G[2 * m] = f16x2_e4m3x2(r[m]);
      G[2 * m + 1] = f16x2_e4m3x2(r[m] >> 16);
    }
  } else {
#pragma unroll
    for (int m = 0; m < 4; ++m) G[m] = f16x2_nibbles((r[0] >> (8 * m)) & 0xFFu);
  }
}
__device__ __forceinline__ void value_fragments_bf16(const uint32_t* r0, const uint32_t* r1, uint32_t (&F)[8]) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    F[2 * m] = __byte_perm(r0[m], r1[m], 0x5410);
    F[2 * m + 1] = __byte_perm(r0[m], r1[m], 0x7632);
  }
}
__device__ __forceinline__ void value_fragments_fp8(const uint32_t* r0, const uint32_t* r1, uint32_t (&F)[8]) {
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const uint32_t x = __byte_perm(r0[m], r1[m], 0x5140);  // dims 4m of both keys, then 4m+1
    const uint32_t y = __byte_perm(r0[m], r1[m], 0x7362);  // dims 4m+2, 4m+3
    F[4 * m] = f16x2_e4m3x2(x);
    F[4 * m + 1] = f16x2_e4m3x2(x >> 16);
    F[4 * m + 2] = f16x2_e4m3x2(y);
    F[4 * m + 3] = f16x2_e4m3x2(y >> 16);
  }
}
__device__ __forceinline__ void value_fragments_int4(uint32_t r0, uint32_t r1, uint32_t (&F)[8]) {
  const uint32_t x = __byte_perm(r0, r1, 0x5410);  // elements 0..3 of both keys
  const uint32_t y = __byte_perm(r0, r1, 0x7632);  // elements 4..7
  F[0] = nibble_pair(x, 4);
  F[1] = nibble_pair(x, 0);
  F[2] = nibble_pair(x, 12);
  F[3] = nibble_pair(x, 8);
  F[4] = nibble_pair(y, 4);
  F[5] = nibble_pair(y, 0);
  F[6] = nibble_pair(y, 12);
  F[7] = nibble_pair(y, 8);
}
// V^T fragments of two keys (r0: key 2c [+8], r1: key 2c+1 [+8]): F[e] = the pair
// (key 0, key 1) of dim 8g + e; bf16 pairs for a tensor of bf16 slots, else f16.
template <int VK, int VW>
__device__ __forceinline__ void value_fragments(const uint32_t (&r0)[VW], const uint32_t (&r1)[VW], int k0,
                                                int k1, uint32_t (&F)[8]) {
  if constexpr (VK == OASIS_KV_BF16) {
    value_fragments_bf16(r0, r1, F);
  } else if constexpr (VK == OASIS_KV_FP8) {
    value_fragments_fp8(r0, r1, F);
  } else if constexpr (VK == OASIS_KV_INT4) {
    value_fragments_int4(r0[0], r1[0], F);
  } else if (k0 != k1) {  // mixed tensor, two kinds: each row to f16 pairs, then interleave
    uint32_t G0[4], G1[4];
    value_row_pairs(r0, k0, G0);
    value_row_pairs(r1, k1, G1);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      F[2 * m] = __byte_perm(G0[m], G1[m], 0x5410);
      F[2 * m + 1] = __byte_perm(G0[m], G1[m], 0x7632);
    }
  } else if (k0 == OASIS_KV_INT4) {
    value_fragments_int4(r0[0], r1[0], F);
  } else if (k0 == OASIS_KV_FP8) {
    value_fragments_fp8(r0, r1, F);
  } else {
    value_fragments_bf16(r0, r1, F);
#pragma unroll
    for (int e = 0; e < 8; ++e) F[e] = f16x2_bf16x2(F[e]);
  }
}

// Pool bytes of (session b, token p, head h) in a tensor's pool of `kind`.
__device__ __forceinline__ const uint8_t* dec_item_rows(const KvTensor& t, const DecodeTensor& d, int kind,
                                                        int b, int p, int h) {
  const uint8_t* pool = kind == OASIS_KV_BF16 ? reinterpret_cast<const uint8_t*>(t.bf16)
                                              : (kind == OASIS_KV_FP8 ? t.fp8 : t.int4);
  return pool + (static_cast<long long>(b) * d.session_pages[kind] * OASIS_TOKENS + p) * dec_row_bytes(kind) +
         h * dec_head_bytes(kind);
}
// Scale / zero element index of (session b, token p, head h) for page 0 of the session:
// FP8 per (page, head), INT4 per (page, token, head).
__device__ __forceinline__ long long dec_item_scale(const DecodeTensor& d, int kind, int b, int p, int h) {
  if (kind == OASIS_KV_FP8) return static_cast<long long>(b) * d.session_pages[kind] * OASIS_HEADS + h;
  return (static_cast<long long>(b) * d.session_pages[kind] * OASIS_TOKENS + p) * OASIS_HEADS + h;
}
__device__ __forceinline__ uint32_t dec_slot_scale(int kind, uint32_t slot_page) {
  return kind == OASIS_KV_FP8 ? slot_page * OASIS_HEADS : slot_page * (OASIS_TOKENS * OASIS_HEADS);
}
// a slot's (multiplier, offset) from its raw scale bits: FP8 bf16 scale; INT4 f16 scale |
// f16 zero << 16; bf16 (1, 0); slots past n_past (dead, 0) - keys are masked anyway
__device__ __forceinline__ float2 dec_scale(uint32_t raw, int kind, bool live) {
  if (!live) return make_float2(0.0f, 0.0f);
  if (kind == OASIS_KV_FP8) return make_float2(__uint_as_float(raw << 16), 0.0f);
  if (kind == OASIS_KV_INT4) {
    const __half2 h = *reinterpret_cast<const __half2*>(&raw);
    return __half22float2(h);
  }
  return make_float2(1.0f, 0.0f);
}

// CTAs (of 4 warps) per SM the register budget is sized for: four (128 registers) for one
// storage kind per tensor; three (170) for two kind-uniform runs, which at 128 registers
// spilled inside the item loop (163 without: 4.40 against 4.66 ms for the incremental
// forward of 16 sessions over 23 INT4 + 8 bf16 frames); mixed tensors keep their row kinds
// and three row pointers live and take two (255)
__host__ __device__ constexpr int dec_min_ctas(int kk, int vk) {
  return kk == kDecMixed || vk == kDecMixed ? 2 : (kk >= kDecSplit ? 3 : 4);
}
// storage kind of key position j under template kind code `code`
__device__ __forceinline__ int dec_position_kind(int code, const DecodeTensor& d, int split, int j) {
  if (code == kDecMixed) return static_cast<int>((d.kinds >> (2 * j)) & 3ull);
  if (code >= kDecSplit) return j < split ? dec_split_a(code) : dec_split_b(code);
  return code;
}
template <int KK, int VK>
__global__ void __launch_bounds__(kDecThreads, dec_min_ctas(KK, VK))
    attn_decode_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                       const __grid_constant__ KvView kv, const __grid_constant__ DecodeLayout lay,
                       int q_pos, int n_past, float scale_log2) {
  pdl_trigger();
  constexpr int KW = KK == OASIS_KV_FP8 ? 4 : (KK == OASIS_KV_INT4 ? 2 : 8);  // words per key chunk
  constexpr int VW = VK == OASIS_KV_FP8 ? 2 : (VK == OASIS_KV_INT4 ? 1 : 4);  // words per value chunk
  constexpr bool kNibble = KK == OASIS_KV_INT4 || KK >= kDecMixed;  // key dim order
  constexpr bool kZeroK = dec_has(KK, OASIS_KV_INT4);               // keys may carry zeros
  constexpr bool kZeroV = dec_has(VK, OASIS_KV_INT4);
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const KvTensor& tk = kv.t[0];
  const KvTensor& tv = kv.t[1];
  const DecodeTensor& dk = lay.t[0];
  const DecodeTensor& dv = lay.t[1];
  auto kind_of = [&](const DecodeTensor& d, int tmpl, int j) { return dec_position_kind(tmpl, d, lay.split, j); };

  // ---- loop-invariant parts of this lane's addresses
  // key rows r = 0..3: key 8r + g, dims 16c..16c+15
  uint32_t koff[4];
  uint32_t kpack = 0;  // 2 bits per row: its kind (mixed tensors)
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int j = 8 * r + g, kind = kind_of(dk, KK, j);
    kpack |= static_cast<uint32_t>(kind) << (2 * r);
    koff[r] = dk.slot_page[j] * (OASIS_TOKENS * dec_row_bytes(kind)) + c * (dec_head_bytes(kind) / 4);
  }
  auto kkind = [&](int r) {
    if constexpr (KK >= kDecSplit) return 8 * r + g < lay.split ? dec_split_a(KK) : dec_split_b(KK);
    return KK == kDecMixed ? static_cast<int>((kpack >> (2 * r)) & 3u) : KK;
  };
  // value rows q = 0..7: key 16 (q >> 2) + 2c + 8 ((q >> 1) & 1) + (q & 1), dims 8g..8g+7
  uint32_t voff[8];
  uint32_t vpack = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int j = 16 * (q >> 2) + 2 * c + 8 * ((q >> 1) & 1) + (q & 1), kind = kind_of(dv, VK, j);
    vpack |= static_cast<uint32_t>(kind) << (2 * q);
    voff[q] = dv.slot_page[j] * (OASIS_TOKENS * dec_row_bytes(kind)) + g * (dec_head_bytes(kind) / 8);
  }
  auto vkind = [&](int q) {
    if constexpr (VK >= kDecSplit)
      return 16 * (q >> 2) + 8 * ((q >> 1) & 1) < lay.split ? dec_split_a(VK) : dec_split_b(VK);
    return VK == kDecMixed ? static_cast<int>((vpack >> (2 * q)) & 3u) : VK;
  };
  // scales of slot `lane`
  const bool slot_live = (lay.valid >> lane) & 1u;
  const int ks_kind = kind_of(dk, KK, lane), vs_kind = kind_of(dv, VK, lane);
  const uint32_t ks_off = dec_slot_scale(ks_kind, dk.slot_page[lane]);
  const uint32_t vs_off = dec_slot_scale(vs_kind, dv.slot_page[lane]);
  const bool live_key = lay.live_kv && n_past <= q_pos;
  uint32_t smask = 0;  // score i of lanes 0..3 (position 8 (i >> 1) + 2c + (i & 1)) is a cached key
#pragma unroll
  for (int i = 0; i < 8; ++i) smask |= ((lay.valid >> (8 * (i >> 1) + 2 * c + (i & 1))) & 1u) << i;

  const int warps_total = gridDim.x * kDecWarps;
  int it = blockIdx.x * kDecWarps + (threadIdx.x >> 5);
  pdl_wait();
  if (it >= lay.items) return;

  // ---- per-item loads (registers)
  uint32_t kr[4][KW], qraw[8], klraw[8], ks_raw;
  uint32_t vr[8][VW], vlraw[4], vs_raw;
  auto load_keys = [&](int item) {
    const int h = item & 15, tok = item >> 4;
    const int p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;
    const uint8_t* base0 = dec_has(KK, 0) ? dec_item_rows(tk, dk, 0, b, p, h) : nullptr;
    const uint8_t* base1 = dec_has(KK, 1) ? dec_item_rows(tk, dk, 1, b, p, h) : nullptr;
    const uint8_t* base2 = dec_has(KK, 2) ? dec_item_rows(tk, dk, 2, b, p, h) : nullptr;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int kind = kkind(r);
#pragma unroll
      for (int w = 0; w < KW; ++w) kr[r][w] = 0u;
      if ((lay.valid >> (8 * r + g)) & 1u) {
        const uint8_t* src = (kind == 0 ? base0 : (kind == 1 ? base1 : base2)) + koff[r];
        if (kind == OASIS_KV_BF16) {
          const uint4 x0 = ldg_stream_v4(src), x1 = ldg_stream_v4(src + 16);
          const uint32_t v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int w = 0; w < KW; ++w) kr[r][w] = v[w];
        } else if (kind == OASIS_KV_FP8) {
          const uint4 x = ldg_stream_v4(src);
          const uint32_t v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int w = 0; w < (KW < 4 ? KW : 4); ++w) kr[r][w] = v[w];
        } else {
          const uint2 x = ldg_stream_v2(src);
          kr[r][0] = x.x;
          kr[r][1] = x.y;
        }
      }
    }
    // the query frame's q (lanes 0..3: dims 16c..16c+15) and its own key
    const __nv_bfloat16* row = qkv + (static_cast<long long>(b) * OASIS_TOKENS + p) * kQkvLd + h * 64 + 16 * c;
#pragma unroll
    for (int w = 0; w < 8; ++w) qraw[w] = klraw[w] = 0u;
    if (g == 0) {
      const uint4 a = ldg_v4(row), a1 = ldg_v4(row + 8);
      qraw[0] = a.x; qraw[1] = a.y; qraw[2] = a.z; qraw[3] = a.w;
      qraw[4] = a1.x; qraw[5] = a1.y; qraw[6] = a1.z; qraw[7] = a1.w;
      if (live_key) {
        const uint4 k0 = ldg_v4(row + OASIS_HIDDEN), k1 = ldg_v4(row + OASIS_HIDDEN + 8);
        klraw[0] = k0.x; klraw[1] = k0.y; klraw[2] = k0.z; klraw[3] = k0.w;
        klraw[4] = k1.x; klraw[5] = k1.y; klraw[6] = k1.z; klraw[7] = k1.w;
      }
    }
    ks_raw = 0u;
    if (KK != OASIS_KV_BF16 && slot_live) {
      if (ks_kind == OASIS_KV_FP8) {
        ks_raw = ldg_u16(tk.fp8_scale + dec_item_scale(dk, OASIS_KV_FP8, b, p, h) + ks_off);
      } else if (ks_kind == OASIS_KV_INT4) {
        const long long e = dec_item_scale(dk, OASIS_KV_INT4, b, p, h) + ks_off;
        ks_raw = ldg_u16(tk.i4_scale + e) | (ldg_u16(tk.i4_zero + e) << 16);
      }
    }
  };
  auto load_values = [&](int item) {
    const int h = item & 15, tok = item >> 4;
    const int p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;
    const uint8_t* base0 = dec_has(VK, 0) ? dec_item_rows(tv, dv, 0, b, p, h) : nullptr;
    const uint8_t* base1 = dec_has(VK, 1) ? dec_item_rows(tv, dv, 1, b, p, h) : nullptr;
    const uint8_t* base2 = dec_has(VK, 2) ? dec_item_rows(tv, dv, 2, b, p, h) : nullptr;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int kind = vkind(q);
      const int j = 16 * (q >> 2) + 2 * c + 8 * ((q >> 1) & 1) + (q & 1);
#pragma unroll
      for (int w = 0; w < VW; ++w) vr[q][w] = 0u;
      if ((lay.valid >> j) & 1u) {
        const uint8_t* src = (kind == 0 ? base0 : (kind == 1 ? base1 : base2)) + voff[q];
        if (kind == OASIS_KV_BF16) {
          const uint4 x = ldg_stream_v4(src);
          const uint32_t v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int w = 0; w < VW; ++w) vr[q][w] = v[w];
        } else if (kind == OASIS_KV_FP8) {
          const uint2 x = ldg_stream_v2(src);
          vr[q][0] = x.x;
          if (VW > 1) vr[q][VW > 1 ? 1 : 0] = x.y;
        } else {
          vr[q][0] = ldg_stream_u32(src);
        }
      }
    }
    // the frame's own value (lanes c == 0: dims 8g..8g+7)
    vlraw[0] = vlraw[1] = vlraw[2] = vlraw[3] = 0u;
    if (c == 0 && live_key) {
      const uint4 v = ldg_v4(qkv + (static_cast<long long>(b) * OASIS_TOKENS + p) * kQkvLd + 2 * OASIS_HIDDEN +
                             h * 64 + 8 * g);
      vlraw[0] = v.x; vlraw[1] = v.y; vlraw[2] = v.z; vlraw[3] = v.w;
    }
    vs_raw = 0u;
    if (VK != OASIS_KV_BF16 && slot_live) {
      if (vs_kind == OASIS_KV_FP8) {
        vs_raw = ldg_u16(tv.fp8_scale + dec_item_scale(dv, OASIS_KV_FP8, b, p, h) + vs_off);
      } else if (vs_kind == OASIS_KV_INT4) {
        const long long e = dec_item_scale(dv, OASIS_KV_INT4, b, p, h) + vs_off;
        vs_raw = ldg_u16(tv.i4_scale + e) | (ldg_u16(tv.i4_zero + e) << 16);
      }
    }
  };

  load_keys(it);
  load_values(it);
  for (; it < lay.items; it += warps_total) {
    const int nx = it + warps_total;
    const int h = it & 15, tok = it >> 4;

    // ---- the query as row 0 of A (lanes 0..3 hold it; other rows are don't-care)
    uint32_t qa[4][2];
    if (KK == OASIS_KV_BF16) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = qraw[2 * ks];
        qa[ks][1] = qraw[2 * ks + 1];
      }
    } else if (!kNibble) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = f16x2_bf16x2(qraw[2 * ks]);
        qa[ks][1] = f16x2_bf16x2(qraw[2 * ks + 1]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        qa[2 * k][0] = pack_f16x2(bf16_lo(qraw[4 * k]), bf16_lo(qraw[4 * k + 2]));
        qa[2 * k][1] = pack_f16x2(bf16_hi(qraw[4 * k]), bf16_hi(qraw[4 * k + 2]));
        qa[2 * k + 1][0] = pack_f16x2(bf16_lo(qraw[4 * k + 1]), bf16_lo(qraw[4 * k + 3]));
        qa[2 * k + 1][1] = pack_f16x2(bf16_hi(qraw[4 * k + 1]), bf16_hi(qraw[4 * k + 3]));
      }
    }
    float qsum = 0.0f;
    if (kZeroK) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][0]));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][1]));
        qsum += (f0.x + f0.y) + (f1.x + f1.y);
      }
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
    }
    // the frame's own key on the CUDA cores (lanes 0..3, 16 dims each)
    float s_live = -INFINITY;
    if (live_key) {
      float d = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w)
        d = __fmaf_rn(bf16_hi(qraw[w]), bf16_hi(klraw[w]), __fmaf_rn(bf16_lo(qraw[w]), bf16_lo(klraw[w]), d));
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      s_live = d;
    }

    // ---- cached scores (n-tiles without a cached key are skipped: the warp agrees)
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
      if ((lay.valid >> (8 * nt)) & 0xFFu) {
        uint32_t kb[4][2];
        key_fragments<KK, KW>(kr[nt], kkind(nt), kb);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_16816<KK == OASIS_KV_BF16>(sacc[nt], qa[ks][0], 0u, qa[ks][1], 0u, kb[ks][0], kb[ks][1]);
      }
    }
    const float2 kscale = KK == OASIS_KV_BF16 ? make_float2(1.0f, 0.0f) : dec_scale(ks_raw, ks_kind, slot_live);
    if (nx < lay.items) load_keys(nx);  // the next item's keys, query, key scales

    // ---- softmax over the cached keys (lanes 0..3 hold keys 8nt + 2c + e) and the live key
    float sc[8];
    float mx = s_live;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = 8 * (i >> 1) + 2 * c + (i & 1);
      float s = sacc[i >> 1][i & 1];
      if (KK != OASIS_KV_BF16) {
        const float mul = __shfl_sync(0xffffffffu, kscale.x, j);
        s = kZeroK ? __fmaf_rn(s, mul, __shfl_sync(0xffffffffu, kscale.y, j) * qsum) : s * mul;
      }
      sc[i] = (smask >> i) & 1u ? s : -INFINITY;
      mx = fmaxf(mx, sc[i]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    // a finite floor: masked scores (-inf) then give 2^-inf = 0 with no select
    const float mxs = fmaxf(mx, -1e30f) * scale_log2;
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pr = ex2_ftz(__fmaf_rn(sc[i], scale_log2, -mxs));
      sum += pr;
      sc[i] = bf16_round(pr);  // the probability as the tensor-core path rounds it
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float p_live = ex2_ftz(__fmaf_rn(s_live, scale_log2, -mxs));  // 0 without the live key
    sum += p_live;
    const float pb_live = bf16_round(p_live);

    // ---- P' (value multipliers folded in, normalised by their max) as B column 0
    const float2 vscale = VK == OASIS_KV_BF16 ? make_float2(1.0f, 0.0f) : dec_scale(vs_raw, vs_kind, slot_live);
    float vmax = 1.0f, corr = 0.0f;
    if (VK != OASIS_KV_BF16) {
      vmax = vscale.x;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
      vmax = fmaxf(vmax, 1e-30f);
    }
    const float inv_vmax = 1.0f / vmax;
    uint32_t pb[2][2];
    {
      float pv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = 8 * (i >> 1) + 2 * c + (i & 1);
        pv[i] = sc[i];
        if (VK != OASIS_KV_BF16) {
          pv[i] = sc[i] * __shfl_sync(0xffffffffu, vscale.x, j) * inv_vmax;
          if (kZeroV) corr = __fmaf_rn(sc[i], __shfl_sync(0xffffffffu, vscale.y, j), corr);
        }
      }
#pragma unroll
      for (int kv2 = 0; kv2 < 2; ++kv2) {
        if (VK == OASIS_KV_BF16) {
          pb[kv2][0] = pack_bf16x2(pv[4 * kv2], pv[4 * kv2 + 1]);
          pb[kv2][1] = pack_bf16x2(pv[4 * kv2 + 2], pv[4 * kv2 + 3]);
        } else {
          pb[kv2][0] = pack_f16x2(pv[4 * kv2], pv[4 * kv2 + 1]);
          pb[kv2][1] = pack_f16x2(pv[4 * kv2 + 2], pv[4 * kv2 + 3]);
        }
      }
    }
    if (kZeroV) {
      corr += __shfl_xor_sync(0xffffffffu, corr, 1);
      corr += __shfl_xor_sync(0xffffffffu, corr, 2);
    }

    // ---- O^T = V^T P^T: m-tile mo rows g / g+8 are dims 8g + 2mo / 8g + 2mo + 1
    float oacc[4][4];
#pragma unroll
    for (int mo = 0; mo < 4; ++mo) oacc[mo][0] = oacc[mo][1] = oacc[mo][2] = oacc[mo][3] = 0.0f;
#pragma unroll
    for (int kv2 = 0; kv2 < 2; ++kv2) {
      if (!((lay.valid >> (16 * kv2)) & 0xFFFFu)) continue;  // no cached key in these 16
      uint32_t F[2][8];
#pragma unroll
      for (int pr = 0; pr < 2; ++pr)
        value_fragments<VK, VW>(vr[4 * kv2 + 2 * pr], vr[4 * kv2 + 2 * pr + 1], vkind(4 * kv2 + 2 * pr),
                                vkind(4 * kv2 + 2 * pr + 1), F[pr]);
#pragma unroll
      for (int mo = 0; mo < 4; ++mo)
        mma_16816<VK == OASIS_KV_BF16>(oacc[mo], F[0][2 * mo], F[0][2 * mo + 1], F[1][2 * mo], F[1][2 * mo + 1],
                                       pb[kv2][0], pb[kv2][1]);
    }
    const uint32_t vl[4] = {vlraw[0], vlraw[1], vlraw[2], vlraw[3]};
    if (nx < lay.items) load_values(nx);  // the next item's values, own value, value scales

    // ---- epilogue: lanes c == 0 hold dims 8g..8g+7 (column 0 of C)
    const float inv = __shfl_sync(0xffffffffu, 1.0f / sum, 0);
    const float corr0 = __shfl_sync(0xffffffffu, corr, 0);
    const float pl = __shfl_sync(0xffffffffu, pb_live, 0);
    if (c == 0) {
      uint32_t o[4];
#pragma unroll
      for (int mo = 0; mo < 4; ++mo) {
        const float a0 = __fmaf_rn(vmax, oacc[mo][0], corr0), a1 = __fmaf_rn(vmax, oacc[mo][2], corr0);
        o[mo] = pack_bf16x2(__fmaf_rn(pl, bf16_lo(vl[mo]), a0) * inv, __fmaf_rn(pl, bf16_hi(vl[mo]), a1) * inv);
      }
      *reinterpret_cast<uint4*>(out + static_cast<long long>(tok) * OASIS_HIDDEN + h * 64 + 8 * g) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ----------------------------------------------------------------------------------
// one query frame over FP8 or INT4 cached frames (all of them, or INT4 after a first
// n-tile of bf16 frames): one warp per (session, token, 4 or 8 heads)
// ----------------------------------------------------------------------------------
// The per-head kernel above leaves 15 of the 16 rows of its score tile empty and runs the
// softmax, the scale shuffles and the output on 4 of its 32 lanes; with FP8 / INT4 codes
// that scalar work, not HBM, sets its speed.  Here a warp takes 4 or 8 heads of a token.
// Head hh's query is row hh of the A operand (the lanes of row group g = hh supply it,
// every other row is zero) and its keys are the B columns, so the scores of all 8 heads
// accumulate in one tile, row g holding head 8 hg + g; every lane quad then takes the
// softmax, the scale folding and the live key of its own head.  P V runs per head as in
// the per-head kernel (V^T the A operand, column 0 of B the head's P' row, fetched from
// its lane quad by shuffle).  Fragment layouts, head-dim orders and the fp32 arithmetic
// of each head are those of attn_decode_kernel, so both give the same bits.  Heads go in
// pairs, the next head's rows loading while the current head's are used.
// Layouts: kDhgInt4 / kDhgFp8 - every position INT4 / FP8 (keys and values);
// kDhgBf16Int4 - key positions 0..7 bf16 (the newest frames of a progressive cache, placed
// first by the host), 8..31 INT4, the same for the values.
constexpr int kDhgWarps = 4;
constexpr int kDhgThreads = kDhgWarps * 32;
constexpr int kDhgInt4 = 0;
constexpr int kDhgBf16Int4 = 1;
constexpr int kDhgFp8 = 2;

// Four CTAs per SM (128 registers): the kernel is bound by loads in flight, and the
// sixteen warps beat twelve also where FP8 and the bf16 + INT4 layout spill 80-104 bytes
// at this budget (isolated 20-23 % faster than three CTAs at 156-162 registers)
template <int LAYOUT, int HPW>
__global__ void __launch_bounds__(kDhgThreads, 4)
    attn_decode_hg_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                          const __grid_constant__ KvView kv, const __grid_constant__ DecodeLayout lay,
                          int q_pos, int n_past, float scale_log2) {
  pdl_trigger();
  static_assert(HPW == 4 || HPW == 8, "4 or 8 heads per warp");
  constexpr int GROUPS = OASIS_HEADS / HPW;  // head groups of a token
  constexpr bool SPLIT = LAYOUT == kDhgBf16Int4;
  constexpr int BK = LAYOUT == kDhgFp8 ? OASIS_KV_FP8 : OASIS_KV_INT4;  // kind of n-tiles 1..3
  constexpr int K0 = SPLIT ? OASIS_KV_BF16 : BK;                         // kind of n-tile 0 (positions 0..7)
  constexpr int KW = BK == OASIS_KV_FP8 ? 4 : 2, VW = BK == OASIS_KV_FP8 ? 2 : 1;  // words per key / value chunk
  constexpr int K0W = SPLIT ? 8 : KW, V0W = SPLIT ? 4 : VW;  // the same for n-tile 0
  constexpr bool kNibble = BK == OASIS_KV_INT4;               // dim order of the keys (and query)
  constexpr bool kZero = BK == OASIS_KV_INT4;                 // scales carry zeros
  constexpr uint32_t RB = dec_row_bytes(BK), HB = dec_head_bytes(BK);
  constexpr uint32_t RB0 = dec_row_bytes(K0), HB0 = dec_head_bytes(K0);
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const KvTensor& tk = kv.t[0];
  const KvTensor& tv = kv.t[1];
  const DecodeTensor& dk = lay.t[0];
  const DecodeTensor& dv = lay.t[1];
  const uint8_t* kpool = BK == OASIS_KV_FP8 ? tk.fp8 : tk.int4;
  const uint8_t* vpool = BK == OASIS_KV_FP8 ? tv.fp8 : tv.int4;
  const uint8_t* kpool0 = SPLIT ? reinterpret_cast<const uint8_t*>(tk.bf16) : kpool;
  const uint8_t* vpool0 = SPLIT ? reinterpret_cast<const uint8_t*>(tv.bf16) : vpool;

  // This lane's rows (as attn_decode_kernel): key rows nt = 0..3 are key 8 nt + g, dims
  // 16c..16c+15; value rows q = 0..7 are key 16 (q >> 2) + 2c + 8 ((q >> 1) & 1) + (q & 1),
  // dims 8g..8g+7 (rows 0 and 1 lie in n-tile 0); score i is position 8 (i >> 1) + 2c +
  // (i & 1) (scores 0 and 1 in n-tile 0).  Their slot offsets are read from the parameter
  // space where they are used.
  auto koff = [&](int nt) {
    return nt == 0 ? dk.slot_page[g] * (OASIS_TOKENS * RB0) + c * (HB0 / 4)
                   : dk.slot_page[8 * nt + g] * (OASIS_TOKENS * RB) + c * (HB / 4);
  };
  auto vpos = [&](int q) { return 16 * (q >> 2) + 2 * c + 8 * ((q >> 1) & 1) + (q & 1); };
  auto voff = [&](int q) {
    return q < 2 ? dv.slot_page[vpos(q)] * (OASIS_TOKENS * RB0) + g * (HB0 / 8)
                 : dv.slot_page[vpos(q)] * (OASIS_TOKENS * RB) + g * (HB / 8);
  };
  auto spos = [&](int i) { return 8 * (i >> 1) + 2 * c + (i & 1); };
  uint32_t smask = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) smask |= ((lay.valid >> spos(i)) & 1u) << i;
  const bool live_key = lay.live_kv && n_past <= q_pos;
  const int items = lay.items;  // batch * 144 tokens * GROUPS head groups
  const int warps_total = gridDim.x * kDhgWarps;
  int it = blockIdx.x * kDhgWarps + (threadIdx.x >> 5);
  pdl_wait();
  if (it >= items) return;

  struct KHead {  // one head's key words of this lane: n-tile 0, n-tiles 1..3
    uint32_t n0[K0W];
    uint32_t n[3][KW];
  };
  struct VHead {  // one head's value words of this lane: rows 0, 1 (n-tile 0), rows 2..7
    uint32_t r0[2][V0W];
    uint32_t r[6][VW];
    uint32_t own[4];  // lanes c == 0: the frame's own value, dims 8g..8g+7
  };
  auto item_tok = [](int item) { return item / GROUPS; };
  auto item_h0 = [](int item) { return HPW * (item % GROUPS); };
  // head h0's rows of the item's (session, token) in a pool of row bytes `rb`
  auto row_base = [&](const uint8_t* pool, uint32_t pages, uint32_t rb, uint32_t hb, int item) {
    const int tok = item_tok(item), p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;
    return pool + (static_cast<long long>(b) * pages * OASIS_TOKENS + p) * rb + item_h0(item) * hb;
  };
  struct Bases {  // head h0's rows of an item: keys and values, n-tile 0 and the INT4 n-tiles
    const uint8_t *k0, *k, *v0, *v;
  };
  auto bases = [&](int item) {
    return Bases{row_base(kpool0, dk.session_pages[K0], RB0, HB0, item),
                 row_base(kpool, dk.session_pages[BK], RB, HB, item),
                 row_base(vpool0, dv.session_pages[K0], RB0, HB0, item),
                 row_base(vpool, dv.session_pages[BK], RB, HB, item)};
  };
  auto load_k = [&](const Bases& ib, int hh, KHead& k) {
    const uint8_t* b0 = ib.k0 + hh * HB0;
    const uint8_t* b = ib.k + hh * HB;
#pragma unroll
    for (int w = 0; w < K0W; ++w) k.n0[w] = 0u;
    if ((lay.valid >> g) & 1u) {
      const uint8_t* src = b0 + koff(0);
      if constexpr (SPLIT) {
        const uint4 x0 = ldg_stream_v4(src), x1 = ldg_stream_v4(src + 16);
        k.n0[0] = x0.x; k.n0[1] = x0.y; k.n0[2] = x0.z; k.n0[3] = x0.w;
        k.n0[4] = x1.x; k.n0[5] = x1.y; k.n0[6] = x1.z; k.n0[7] = x1.w;
      } else if constexpr (BK == OASIS_KV_FP8) {
        const uint4 x = ldg_stream_v4(src);
        k.n0[0] = x.x; k.n0[1] = x.y; k.n0[2] = x.z; k.n0[3] = x.w;
      } else {
        const uint2 x = ldg_stream_v2(src);
        k.n0[0] = x.x;
        k.n0[1] = x.y;
      }
    }
#pragma unroll
    for (int nt = 1; nt < 4; ++nt) {
#pragma unroll
      for (int w = 0; w < KW; ++w) k.n[nt - 1][w] = 0u;
      if ((lay.valid >> (8 * nt + g)) & 1u) {
        if constexpr (BK == OASIS_KV_FP8) {
          const uint4 x = ldg_stream_v4(b + koff(nt));
          k.n[nt - 1][0] = x.x; k.n[nt - 1][1] = x.y; k.n[nt - 1][2] = x.z; k.n[nt - 1][3] = x.w;
        } else {
          const uint2 x = ldg_stream_v2(b + koff(nt));
          k.n[nt - 1][0] = x.x;
          k.n[nt - 1][1] = x.y;
        }
      }
    }
  };
  auto load_v = [&](const Bases& ib, int item, int hh, VHead& v) {
    const uint8_t* b0 = ib.v0 + hh * HB0;
    const uint8_t* b = ib.v + hh * HB;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int w = 0; w < V0W; ++w) v.r0[q][w] = 0u;
      if ((lay.valid >> vpos(q)) & 1u) {
        const uint8_t* src = b0 + voff(q);
        if constexpr (SPLIT) {
          const uint4 x = ldg_stream_v4(src);
          v.r0[q][0] = x.x; v.r0[q][1] = x.y; v.r0[q][2] = x.z; v.r0[q][3] = x.w;
        } else if constexpr (BK == OASIS_KV_FP8) {
          const uint2 x = ldg_stream_v2(src);
          v.r0[q][0] = x.x;
          v.r0[q][1] = x.y;
        } else {
          v.r0[q][0] = ldg_stream_u32(src);
        }
      }
    }
#pragma unroll
    for (int q = 2; q < 8; ++q) {
#pragma unroll
      for (int w = 0; w < VW; ++w) v.r[q - 2][w] = 0u;
      if ((lay.valid >> vpos(q)) & 1u) {
        if constexpr (BK == OASIS_KV_FP8) {
          const uint2 x = ldg_stream_v2(b + voff(q));
          v.r[q - 2][0] = x.x;
          v.r[q - 2][1] = x.y;
        } else {
          v.r[q - 2][0] = ldg_stream_u32(b + voff(q));
        }
      }
    }
    v.own[0] = v.own[1] = v.own[2] = v.own[3] = 0u;
    if (c == 0 && live_key) {
      const uint4 x = ldg_v4(qkv + static_cast<long long>(item_tok(item)) * kQkvLd + 2 * OASIS_HIDDEN +
                             (item_h0(item) + hh) * 64 + 8 * g);
      v.own[0] = x.x; v.own[1] = x.y; v.own[2] = x.z; v.own[3] = x.w;
    }
  };
  // scale (| zero << 16) of score position i for the row head of an item: INT4 per
  // (page, token, head), FP8 per (page, head); bf16 positions carry none
  auto load_scales = [&](const KvTensor& t, const DecodeTensor& d, int item, uint32_t (&dst)[8]) {
    const int tok = item_tok(item), p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;
    const long long e0 = dec_item_scale(d, BK, b, p, item_h0(item) + (g < HPW ? g : g - HPW));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dst[i] = 0u;
      if ((!SPLIT || i >= 2) && ((smask >> i) & 1u)) {
        const uint32_t so = dec_slot_scale(BK, d.slot_page[spos(i)]);
        if constexpr (BK == OASIS_KV_FP8)
          dst[i] = ldg_u16(t.fp8_scale + e0 + so);
        else
          dst[i] = ldg_u16(t.i4_scale + e0 + so) | (ldg_u16(t.i4_zero + e0 + so) << 16);
      }
    }
  };
  auto scale_of = [&](uint32_t raw, int i, bool live) {
    return SPLIT && i < 2 ? dec_scale(raw, OASIS_KV_BF16, live) : dec_scale(raw, BK, live);
  };
  // the row head's query (dims 16c..16c+15) and own key
  uint32_t qraw[8], klraw[8], ksr[8], vsr[8];
  auto load_q = [&](int item) {
    const int tok = item_tok(item);
    // lanes of row groups g >= HPW take head h0 + g - HPW: a valid row whose scores are never read
    const int hr = item_h0(item) + (g < HPW ? g : g - HPW);
    const __nv_bfloat16* row = qkv + static_cast<long long>(tok) * kQkvLd + hr * 64 + 16 * c;
    const uint4 a = ldg_v4(row), a1 = ldg_v4(row + 8);
    qraw[0] = a.x; qraw[1] = a.y; qraw[2] = a.z; qraw[3] = a.w;
    qraw[4] = a1.x; qraw[5] = a1.y; qraw[6] = a1.z; qraw[7] = a1.w;
#pragma unroll
    for (int w = 0; w < 8; ++w) klraw[w] = 0u;
    if (live_key) {
      const uint4 k0 = ldg_v4(row + OASIS_HIDDEN), k1 = ldg_v4(row + OASIS_HIDDEN + 8);
      klraw[0] = k0.x; klraw[1] = k0.y; klraw[2] = k0.z; klraw[3] = k0.w;
      klraw[4] = k1.x; klraw[5] = k1.y; klraw[6] = k1.z; klraw[7] = k1.w;
    }
    load_scales(tk, dk, item, ksr);
  };

  KHead kh[2];
  VHead vh[2];
  Bases ib = bases(it);
  load_q(it);
  load_k(ib, 0, kh[0]);
  for (; it < items; it += warps_total) {
    const int nx = it + warps_total;
    const int tok = item_tok(it), h0 = item_h0(it);

    // ---- the row head's query as A fragments (row g) in the keys' dim order
    uint32_t qa[4][2];
    if (!kNibble) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = f16x2_bf16x2(qraw[2 * ks]);
        qa[ks][1] = f16x2_bf16x2(qraw[2 * ks + 1]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        qa[2 * k][0] = pack_f16x2(bf16_lo(qraw[4 * k]), bf16_lo(qraw[4 * k + 2]));
        qa[2 * k][1] = pack_f16x2(bf16_hi(qraw[4 * k]), bf16_hi(qraw[4 * k + 2]));
        qa[2 * k + 1][0] = pack_f16x2(bf16_lo(qraw[4 * k + 1]), bf16_lo(qraw[4 * k + 3]));
        qa[2 * k + 1][1] = pack_f16x2(bf16_hi(qraw[4 * k + 1]), bf16_hi(qraw[4 * k + 3]));
      }
    }
    float qsum = 0.0f;
    if (kZero) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][0]));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][1]));
        qsum += (f0.x + f0.y) + (f1.x + f1.y);
      }
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
      qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
    }
    float s_live = -INFINITY;
    if (live_key) {
      float d = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w)
        d = __fmaf_rn(bf16_hi(qraw[w]), bf16_hi(klraw[w]), __fmaf_rn(bf16_lo(qraw[w]), bf16_lo(klraw[w]), d));
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      s_live = d;
    }

    // ---- scores of the 8 heads in one tile: head hh's MMAs carry row hh of A only
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
    auto score_head = [&](int hh, const KHead& k) {
      const bool mine = g == hh;
      uint32_t a0[4], a2[4];
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        a0[ks] = mine ? qa[ks][0] : 0u;
        a2[ks] = mine ? qa[ks][1] : 0u;
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        if ((lay.valid >> (8 * nt)) & 0xFFu) {
          uint32_t kbf[4][2];
          if (nt == 0)
            key_fragments<SPLIT ? kDecMixed : BK, K0W>(k.n0, K0, kbf);
          else
            key_fragments<BK, KW>(k.n[nt - 1], BK, kbf);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_16816<false>(sacc[nt], a0[ks], 0u, a2[ks], 0u, kbf[ks][0], kbf[ks][1]);
        }
      }
    };
#pragma unroll 1
    for (int hp = 0; hp < HPW; hp += 2) {
      load_k(ib, hp + 1, kh[1]);
      score_head(hp, kh[0]);
      if (hp < HPW - 2) load_k(ib, hp + 2, kh[0]);
      score_head(hp + 1, kh[1]);
    }
    // the first head's values and the value scales load while the softmax runs
    load_v(ib, it, 0, vh[0]);
    load_scales(tv, dv, it, vsr);

    // ---- softmax of row g (head h0 + g) over the cached keys and the live key
    float sc[8];
    float mx = s_live;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 ks = scale_of(ksr[i], i, true);
      const float s = sacc[i >> 1][i & 1];
      const float sv = kZero ? __fmaf_rn(s, ks.x, ks.y * qsum) : s * ks.x;
      sc[i] = (smask >> i) & 1u ? sv : -INFINITY;
      mx = fmaxf(mx, sc[i]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mxs = fmaxf(mx, -1e30f) * scale_log2;
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pr = ex2_ftz(__fmaf_rn(sc[i], scale_log2, -mxs));
      sum += pr;
      sc[i] = bf16_round(pr);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float p_live = ex2_ftz(__fmaf_rn(s_live, scale_log2, -mxs));
    sum += p_live;
    const float pb_live = bf16_round(p_live);

    // ---- P' = p * value multiplier / the row's largest multiplier, and sum p * zero
    float vmax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) vmax = fmaxf(vmax, scale_of(vsr[i], i, (smask >> i) & 1u).x);
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
    vmax = fmaxf(vmax, 1e-30f);
    const float inv_vmax = 1.0f / vmax;
    float corr = 0.0f;
    uint32_t pbk[2][2];
    {
      float pv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 vs = scale_of(vsr[i], i, (smask >> i) & 1u);
        pv[i] = sc[i] * vs.x * inv_vmax;
        if (kZero) corr = __fmaf_rn(sc[i], vs.y, corr);
      }
#pragma unroll
      for (int kv2 = 0; kv2 < 2; ++kv2) {
        pbk[kv2][0] = pack_f16x2(pv[4 * kv2], pv[4 * kv2 + 1]);
        pbk[kv2][1] = pack_f16x2(pv[4 * kv2 + 2], pv[4 * kv2 + 3]);
      }
    }
    if (kZero) {
      corr += __shfl_xor_sync(0xffffffffu, corr, 1);
      corr += __shfl_xor_sync(0xffffffffu, corr, 2);
    }
    const float inv = 1.0f / sum;

    // ---- per head: O^T = V^T P'^T, then the live value, the multipliers and 1 / sum
    auto pv_head = [&](int hh, const VHead& v) {
      // column 0 of B: head hh's P' row from its lane quad (lanes 4 hh + c); the other
      // columns (lanes g > 0) give output columns that are not read
      uint32_t pb[2][2];
#pragma unroll
      for (int kv2 = 0; kv2 < 2; ++kv2) {
        pb[kv2][0] = __shfl_sync(0xffffffffu, pbk[kv2][0], 4 * hh + c);
        pb[kv2][1] = __shfl_sync(0xffffffffu, pbk[kv2][1], 4 * hh + c);
      }
      float oacc[4][4];
#pragma unroll
      for (int mo = 0; mo < 4; ++mo) oacc[mo][0] = oacc[mo][1] = oacc[mo][2] = oacc[mo][3] = 0.0f;
#pragma unroll
      for (int kv2 = 0; kv2 < 2; ++kv2) {
        if (!((lay.valid >> (16 * kv2)) & 0xFFFFu)) continue;
        uint32_t F[2][8];
        if (kv2 == 0)  // rows 0, 1: n-tile 0; rows 2, 3: n-tile 1
          value_fragments<SPLIT ? kDecMixed : BK, V0W>(v.r0[0], v.r0[1], K0, K0, F[0]);
        else
          value_fragments<BK, VW>(v.r[2], v.r[3], BK, BK, F[0]);
        value_fragments<BK, VW>(v.r[4 * kv2], v.r[4 * kv2 + 1], BK, BK, F[1]);
#pragma unroll
        for (int mo = 0; mo < 4; ++mo)
          mma_16816<false>(oacc[mo], F[0][2 * mo], F[0][2 * mo + 1], F[1][2 * mo], F[1][2 * mo + 1], pb[kv2][0],
                           pb[kv2][1]);
      }
      const float inv_h = __shfl_sync(0xffffffffu, inv, 4 * hh);
      const float corr_h = __shfl_sync(0xffffffffu, corr, 4 * hh);
      const float vmax_h = __shfl_sync(0xffffffffu, vmax, 4 * hh);
      const float pl_h = __shfl_sync(0xffffffffu, pb_live, 4 * hh);
      if (c == 0) {
        uint32_t o[4];
#pragma unroll
        for (int mo = 0; mo < 4; ++mo) {
          const float a0 = __fmaf_rn(vmax_h, oacc[mo][0], corr_h), a1 = __fmaf_rn(vmax_h, oacc[mo][2], corr_h);
          o[mo] = pack_bf16x2(__fmaf_rn(pl_h, bf16_lo(v.own[mo]), a0) * inv_h,
                              __fmaf_rn(pl_h, bf16_hi(v.own[mo]), a1) * inv_h);
        }
        *reinterpret_cast<uint4*>(out + static_cast<long long>(tok) * OASIS_HIDDEN + (h0 + hh) * 64 + 8 * g) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
    };
    const Bases cur = ib;
#pragma unroll 1
    for (int hp = 0; hp < HPW; hp += 2) {
      load_v(cur, it, hp + 1, vh[1]);
      pv_head(hp, vh[0]);
      if (hp < HPW - 2) {
        load_v(cur, it, hp + 2, vh[0]);
      } else if (nx < items) {
        ib = bases(nx);
        load_q(nx);            // the next item's query, own key and key scales
        load_k(ib, 0, kh[0]);  // and its first head's keys
      }
      pv_head(hp + 1, vh[1]);
    }
  }
}

// decode kernel for (key kind, value kind), each a storage kind or kDecMixed
using DecodeKernel = void (*)(const __nv_bfloat16*, __nv_bfloat16*, const KvView, const DecodeLayout, int, int,
                              float);
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
  if (kk >= kDecSplit && kk == vk) {
    switch (kk - kDecSplit) {
      case 1: return attn_decode_kernel<kDecSplit + 1, kDecSplit + 1>;  // bf16 | FP8
      case 2: return attn_decode_kernel<kDecSplit + 2, kDecSplit + 2>;  // bf16 | INT4
      case 3: return attn_decode_kernel<kDecSplit + 3, kDecSplit + 3>;  // FP8 | bf16
      case 5: return attn_decode_kernel<kDecSplit + 5, kDecSplit + 5>;  // FP8 | INT4
      case 6: return attn_decode_kernel<kDecSplit + 6, kDecSplit + 6>;  // INT4 | bf16
      case 7: return attn_decode_kernel<kDecSplit + 7, kDecSplit + 7>;  // INT4 | FP8
    }
  }
  switch (kk) {
    case OASIS_KV_BF16: return decode_kernel_v<OASIS_KV_BF16>(vk);
    case OASIS_KV_FP8: return decode_kernel_v<OASIS_KV_FP8>(vk);
    case OASIS_KV_INT4: return decode_kernel_v<OASIS_KV_INT4>(vk);
  }
  return decode_kernel_v<kDecMixed>(vk);
}

// ----------------------------------------------------------------------------------
// temporal attention of several query frames whose keys and values all come from cache
// slots of one kind per tensor (no live frames: the isolated sweep's case)
// ----------------------------------------------------------------------------------
// One warp per (session, token, head), its 16-query tiles in turn.  The key and value fragments come
// straight from the cache into registers and are converted there, as in the one-query-frame
// kernel (same fragment layouts and head-dim orders); the query tile is the A operand of the
// scores, whose accumulators are the A operand of P V (no shuffle), and the softmax of the
// 16 rows uses every lane (rows g and g + 8 of each lane quad).
constexpr int kWcWarps = 4;

struct WindowLayout {
  DecodeTensor t[2];  // keys, values by slot
  int items;          // batch * 144 tokens * 16 heads
  int m_tiles;        // 16-row query tiles per item (1 or 2)
};

// Loads of cached key / value chunks that stay in registers for every query tile: volatile,
// so the compiler keeps the values rather than issuing the load again for a later tile.
__device__ __forceinline__ uint4 ldg_keep_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldg_keep_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_keep_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// MT: query tiles per warp (1: windows of up to 16 query frames, sized for four CTAs per
// SM; 2: the second tile's rows load under the first tile's math, three CTAs per SM)
template <int KK, int VK, int MT>
__global__ void __launch_bounds__(kWcWarps * 32, MT == 1 ? 4 : 3)
    attn_window_cached_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                              const __grid_constant__ KvView kv, const __grid_constant__ WindowLayout lay,
                              int q_frames, int q_pos0, int n_past, float scale_log2) {
  pdl_trigger();
  constexpr int KW = KK == OASIS_KV_FP8 ? 4 : (KK == OASIS_KV_INT4 ? 2 : 8);
  constexpr int VW = VK == OASIS_KV_FP8 ? 2 : (VK == OASIS_KV_INT4 ? 1 : 4);
  constexpr bool kNibble = KK == OASIS_KV_INT4;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int item = blockIdx.x * kWcWarps + (threadIdx.x >> 5);
  const KvTensor& tk = kv.t[0];
  const KvTensor& tv = kv.t[1];
  const DecodeTensor& dk = lay.t[0];
  const DecodeTensor& dv = lay.t[1];
  pdl_wait();
  if (item >= lay.items) return;
  const int h = item & 15, tok = item >> 4;
  const int p = tok % OASIS_TOKENS, b = tok / OASIS_TOKENS;

  // ---- loads: keys 8r + g (dims 16c..), values 16kv + 2c + {0,1,8,9} (dims 8g..), query rows
  uint32_t kr[4][KW], vr[8][VW], q0[8], q1[8];
  {
    const uint8_t* kb = dec_item_rows(tk, dk, KK, b, p, h);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int j = 8 * r + g;
#pragma unroll
      for (int w = 0; w < KW; ++w) kr[r][w] = 0u;
      if (j < n_past) {
        const uint8_t* src = kb + dk.slot_page[j] * (OASIS_TOKENS * dec_row_bytes(KK)) + c * (dec_head_bytes(KK) / 4);
        if (KK == OASIS_KV_INT4) {
          const uint2 x = ldg_keep_v2(src);
          kr[r][0] = x.x;
          kr[r][KW > 1 ? 1 : 0] = x.y;
        } else {
#pragma unroll
          for (int w4 = 0; w4 < KW / 4; ++w4) {
            const uint4 x = ldg_keep_v4(src + 16 * w4);
            kr[r][4 * w4] = x.x; kr[r][4 * w4 + 1] = x.y; kr[r][4 * w4 + 2] = x.z; kr[r][4 * w4 + 3] = x.w;
          }
        }
      }
    }
    const uint8_t* vb = dec_item_rows(tv, dv, VK, b, p, h);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = 16 * (q >> 2) + 2 * c + 8 * ((q >> 1) & 1) + (q & 1);
#pragma unroll
      for (int w = 0; w < VW; ++w) vr[q][w] = 0u;
      if (j < n_past) {
        const uint8_t* src = vb + dv.slot_page[j] * (OASIS_TOKENS * dec_row_bytes(VK)) + g * (dec_head_bytes(VK) / 8);
        if (VW == 4) {
          const uint4 x = ldg_keep_v4(src);
          vr[q][0] = x.x; vr[q][VW > 1 ? 1 : 0] = x.y; vr[q][VW > 2 ? 2 : 0] = x.z; vr[q][VW > 3 ? 3 : 0] = x.w;
        } else if (VW == 2) {
          const uint2 x = ldg_keep_v2(src);
          vr[q][0] = x.x; vr[q][VW > 1 ? 1 : 0] = x.y;
        } else {
          vr[q][0] = ldg_keep_u32(src);
        }
      }
    }
  }
  // query rows t0 = 16 mt + g and t1 = t0 + 8 of query tile mt (zero past q_frames)
  auto load_q = [&](int mt) {
    const int t0 = 16 * mt + g, t1 = t0 + 8;
#pragma unroll
    for (int w = 0; w < 8; ++w) q0[w] = q1[w] = 0u;
    if (t0 < q_frames) {
      const uint4* src = reinterpret_cast<const uint4*>(
          qkv + (static_cast<long long>(b * q_frames + t0) * OASIS_TOKENS + p) * kQkvLd + h * 64 + 16 * c);
      const uint4 x0 = src[0], x1 = src[1];
      q0[0] = x0.x; q0[1] = x0.y; q0[2] = x0.z; q0[3] = x0.w; q0[4] = x1.x; q0[5] = x1.y; q0[6] = x1.z; q0[7] = x1.w;
    }
    if (t1 < q_frames) {
      const uint4* src = reinterpret_cast<const uint4*>(
          qkv + (static_cast<long long>(b * q_frames + t1) * OASIS_TOKENS + p) * kQkvLd + h * 64 + 16 * c);
      const uint4 x0 = src[0], x1 = src[1];
      q1[0] = x0.x; q1[1] = x0.y; q1[2] = x0.z; q1[3] = x0.w; q1[4] = x1.x; q1[5] = x1.y; q1[6] = x1.z; q1[7] = x1.w;
    }
  };
  load_q(0);
  // scales of slot `lane`
  const bool slot_live = lane < n_past;
  float2 kscale = make_float2(1.0f, 0.0f), vscale = make_float2(slot_live ? 1.0f : 0.0f, 0.0f);
  if (KK != OASIS_KV_BF16 && slot_live) {
    const long long e = dec_item_scale(dk, KK, b, p, h) + dec_slot_scale(KK, dk.slot_page[lane]);
    const uint32_t raw = KK == OASIS_KV_FP8
                             ? static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tk.fp8_scale) + e))
                             : static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tk.i4_scale) + e)) |
                                   (static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tk.i4_zero) + e)) << 16);
    kscale = dec_scale(raw, KK, true);
  }
  if (VK != OASIS_KV_BF16 && slot_live) {
    const long long e = dec_item_scale(dv, VK, b, p, h) + dec_slot_scale(VK, dv.slot_page[lane]);
    const uint32_t raw = VK == OASIS_KV_FP8
                             ? static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tv.fp8_scale) + e))
                             : static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tv.i4_scale) + e)) |
                                   (static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(tv.i4_zero) + e)) << 16);
    vscale = dec_scale(raw, VK, true);
  }

  float vmax = 1.0f, inv_vmax = 1.0f;
  if (VK != OASIS_KV_BF16) {
    vmax = vscale.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    vmax = fmaxf(vmax, 1e-30f);
    inv_vmax = 1.0f / vmax;
  }
  const float vmul = vscale.x * inv_vmax;  // slot `lane`'s value multiplier over the max
  for (int mt = 0; mt < (MT == 1 ? 1 : lay.m_tiles); ++mt) {
  // ---- the query tile as A (rows g, g + 8), in the keys' head-dim order
  uint32_t qa[4][4];
  if (KK == OASIS_KV_BF16) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qa[ks][0] = q0[2 * ks]; qa[ks][1] = q1[2 * ks]; qa[ks][2] = q0[2 * ks + 1]; qa[ks][3] = q1[2 * ks + 1];
    }
  } else if (!kNibble) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qa[ks][0] = f16x2_bf16x2(q0[2 * ks]); qa[ks][1] = f16x2_bf16x2(q1[2 * ks]);
      qa[ks][2] = f16x2_bf16x2(q0[2 * ks + 1]); qa[ks][3] = f16x2_bf16x2(q1[2 * ks + 1]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      qa[2 * k][0] = pack_f16x2(bf16_lo(q0[4 * k]), bf16_lo(q0[4 * k + 2]));
      qa[2 * k][1] = pack_f16x2(bf16_lo(q1[4 * k]), bf16_lo(q1[4 * k + 2]));
      qa[2 * k][2] = pack_f16x2(bf16_hi(q0[4 * k]), bf16_hi(q0[4 * k + 2]));
      qa[2 * k][3] = pack_f16x2(bf16_hi(q1[4 * k]), bf16_hi(q1[4 * k + 2]));
      qa[2 * k + 1][0] = pack_f16x2(bf16_lo(q0[4 * k + 1]), bf16_lo(q0[4 * k + 3]));
      qa[2 * k + 1][1] = pack_f16x2(bf16_lo(q1[4 * k + 1]), bf16_lo(q1[4 * k + 3]));
      qa[2 * k + 1][2] = pack_f16x2(bf16_hi(q0[4 * k + 1]), bf16_hi(q0[4 * k + 3]));
      qa[2 * k + 1][3] = pack_f16x2(bf16_hi(q1[4 * k + 1]), bf16_hi(q1[4 * k + 3]));
    }
  }
  float qs0 = 0.0f, qs1 = 0.0f;  // sum of each row's f16 query (INT4 zero term)
  if (KK == OASIS_KV_INT4) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][0]));
      const float2 a2 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][2]));
      const float2 bq = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][1]));
      const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&qa[ks][3]));
      qs0 += (a.x + a.y) + (a2.x + a2.y);
      qs1 += (bq.x + bq.y) + (b2.x + b2.y);
    }
    qs0 += __shfl_xor_sync(0xffffffffu, qs0, 1);
    qs0 += __shfl_xor_sync(0xffffffffu, qs0, 2);
    qs1 += __shfl_xor_sync(0xffffffffu, qs1, 1);
    qs1 += __shfl_xor_sync(0xffffffffu, qs1, 2);
  }

  // ---- scores: s[nt][e] row g, s[nt][2 + e] row g + 8, key 8nt + 2c + e.  Keys from
  // `vis` on are masked for every row of the tile (past the cache or the tile's last
  // window position): their n-tiles and P V k-steps are skipped (the warp agrees).
  const int vis = min(n_past, q_pos0 + 16 * mt + 16);
  float s[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
    if (8 * nt < vis) {
      uint32_t kb[4][2];
      key_fragments<KK, KW>(kr[nt], KK, kb);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_16816<KK == OASIS_KV_BF16>(s[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[ks][0], kb[ks][1]);
    }
  }
  const int qp0 = q_pos0 + 16 * mt + g, qp1 = qp0 + 8;  // window positions of the two rows
  float mx0 = -1e30f, mx1 = -1e30f;  // finite floor: a fully masked row gives 0, not NaN
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int nt = i >> 1, e = i & 1, j = 8 * nt + 2 * c + e;
    float a = s[nt][e], bb = s[nt][2 + e];
    if (KK != OASIS_KV_BF16) {
      const float mul = __shfl_sync(0xffffffffu, kscale.x, j);
      if (KK == OASIS_KV_INT4) {
        const float off = __shfl_sync(0xffffffffu, kscale.y, j);
        a = __fmaf_rn(a, mul, off * qs0);
        bb = __fmaf_rn(bb, mul, off * qs1);
      } else {
        a *= mul;
        bb *= mul;
      }
    }
    s[nt][e] = (j < n_past && j <= qp0) ? a : -INFINITY;
    s[nt][2 + e] = (j < n_past && j <= qp1) ? bb : -INFINITY;
    mx0 = fmaxf(mx0, s[nt][e]);
    mx1 = fmaxf(mx1, s[nt][2 + e]);
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float o0 = mx0 * scale_log2, o1 = mx1 * scale_log2;
  if (MT > 1 && mt + 1 < lay.m_tiles) load_q(mt + 1);  // the next tile's rows load under this tile's math
  float sum0 = 0.0f, sum1 = 0.0f;
  float corr0 = 0.0f, corr1 = 0.0f;
  uint32_t pa[2][4];  // P' as the A operand of P V, k-step kv: keys 16kv..16kv+15
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    float pr[4];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      pr[e] = ex2_ftz(__fmaf_rn(s[nt][e], scale_log2, -o0));
      pr[2 + e] = ex2_ftz(__fmaf_rn(s[nt][2 + e], scale_log2, -o1));
      sum0 += pr[e];
      sum1 += pr[2 + e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = bf16_round(pr[e]);  // P as the tensor-core path rounds it
    if (VK != OASIS_KV_BF16) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 8 * nt + 2 * c + e;
        const float m = __shfl_sync(0xffffffffu, vmul, j);
        if (VK == OASIS_KV_INT4) {
          const float z = __shfl_sync(0xffffffffu, vscale.y, j);
          corr0 = __fmaf_rn(pr[e], z, corr0);
          corr1 = __fmaf_rn(pr[2 + e], z, corr1);
        }
        pr[e] *= m;
        pr[2 + e] *= m;
      }
      pa[nt >> 1][2 * (nt & 1)] = pack_f16x2(pr[0], pr[1]);
      pa[nt >> 1][2 * (nt & 1) + 1] = pack_f16x2(pr[2], pr[3]);
    } else {
      pa[nt >> 1][2 * (nt & 1)] = pack_bf16x2(pr[0], pr[1]);
      pa[nt >> 1][2 * (nt & 1) + 1] = pack_bf16x2(pr[2], pr[3]);
    }
  }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
  if (VK == OASIS_KV_INT4) {
    corr0 += __shfl_xor_sync(0xffffffffu, corr0, 1);
    corr0 += __shfl_xor_sync(0xffffffffu, corr0, 2);
    corr1 += __shfl_xor_sync(0xffffffffu, corr1, 1);
    corr1 += __shfl_xor_sync(0xffffffffu, corr1, 2);
  }

  // ---- O = P' V: n-tile n column 2c / 2c + 1 are dims 16c + n / 16c + 8 + n
  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
  for (int kv2 = 0; kv2 < 2; ++kv2) {
    if (16 * kv2 >= vis) continue;  // every probability of these keys is 0
    uint32_t F[2][8];
#pragma unroll
    for (int pr = 0; pr < 2; ++pr)
      value_fragments<VK, VW>(vr[4 * kv2 + 2 * pr], vr[4 * kv2 + 2 * pr + 1], VK, VK, F[pr]);
#pragma unroll
    for (int n = 0; n < 8; ++n)
      mma_16816<VK == OASIS_KV_BF16>(o[n], pa[kv2][0], pa[kv2][1], pa[kv2][2], pa[kv2][3], F[0][n], F[1][n]);
  }
  const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
  const int t0 = 16 * mt + g, t1 = t0 + 8;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = half ? t1 : t0;
    if (t >= q_frames) continue;
    const float inv = half ? inv1 : inv0, corr = half ? corr1 : corr0;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // dims 16c + 2k, + 1: n-tiles 2k, 2k + 1 (mod 8) of column 2c (k < 4) or 2c + 1
      const int n = (2 * k) & 7, col = k >> 2;
      const float a0 = __fmaf_rn(vmax, o[n][2 * half + col], corr), a1 = __fmaf_rn(vmax, o[n + 1][2 * half + col], corr);
      w[k] = pack_bf16x2(a0 * inv, a1 * inv);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<long long>(b * q_frames + t) * OASIS_TOKENS + p) * OASIS_HIDDEN +
                                          h * 64 + 16 * c);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  }  // query tiles
}

using WindowKernel = void (*)(const __nv_bfloat16*, __nv_bfloat16*, const KvView, const WindowLayout, int, int,
                              int, float);
template <int KK, int MT>
WindowKernel window_kernel_v(int vk) {
  switch (vk) {
    case OASIS_KV_FP8: return attn_window_cached_kernel<KK, OASIS_KV_FP8, MT>;
    case OASIS_KV_INT4: return attn_window_cached_kernel<KK, OASIS_KV_INT4, MT>;
  }
  return attn_window_cached_kernel<KK, OASIS_KV_BF16, MT>;
}
template <int MT>
WindowKernel window_kernel_m(int kk, int vk) {
  switch (kk) {
    case OASIS_KV_FP8: return window_kernel_v<OASIS_KV_FP8, MT>(vk);
    case OASIS_KV_INT4: return window_kernel_v<OASIS_KV_INT4, MT>(vk);
  }
  return window_kernel_v<OASIS_KV_BF16, MT>(vk);
}
WindowKernel window_kernel(int kk, int vk, int m_tiles) {
  return m_tiles == 1 ? window_kernel_m<1>(kk, vk) : window_kernel_m<2>(kk, vk);
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
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attn_temporal)");
    configured = true;
  }
  if (q_frames == 1 && n_past > 0 && n_past < OASIS_MAX_FRAMES) {
    // one query frame over cached slots: the warp-per-head decode kernel
    DecodeLayout lay{};
    lay.live_kv = n_kv > n_past ? 1 : 0;
    lay.items = batch * OASIS_TOKENS * OASIS_HEADS;
    // key position of each cached slot
    int kinds[2][OASIS_MAX_FRAMES];
    bool present[2][3] = {{false, false, false}, {false, false, false}};
    for (int which = 0; which < 2; ++which)
      for (int s = 0; s < n_past; ++s) {
        kinds[which][s] = kv.t[which].kind[s];
        present[which][kinds[which][s]] = true;
      }
    int uniform[2];
    for (int which = 0; which < 2; ++which) {
      const bool* pr = present[which];
      uniform[which] = pr[0] + pr[1] + pr[2] == 1 ? (pr[0] ? 0 : (pr[1] ? 1 : 2)) : kDecMixed;
    }
    int pos_slot[OASIS_MAX_FRAMES];  // slot at each key position, -1: none
    int pos_kind[2][OASIS_MAX_FRAMES];
    for (int j = 0; j < OASIS_MAX_FRAMES; ++j) {
      pos_slot[j] = j < n_past ? j : -1;
      for (int which = 0; which < 2; ++which)
        pos_kind[which][j] = j < n_past ? kinds[which][j] : (uniform[which] == kDecMixed ? 0 : uniform[which]);
    }
    if (uniform[0] == kDecMixed || uniform[1] == kDecMixed) {
      // group the slots by (key kind, value kind), each group from an n-tile boundary,
      // when the groups fit the 4 n-tiles
      int combo_of[OASIS_MAX_FRAMES], count[9] = {0}, tiles = 0;
      for (int s = 0; s < n_past; ++s) {
        combo_of[s] = 3 * kinds[0][s] + kinds[1][s];
        ++count[combo_of[s]];
      }
      for (int cb = 0; cb < 9; ++cb) tiles += (count[cb] + 7) / 8;
      if (tiles <= OASIS_MAX_FRAMES / 8) {
        int next = 0;
        for (int cb = 0; cb < 9; ++cb) {
          if (!count[cb]) continue;
          const int start = next;
          for (int s = 0; s < n_past; ++s)
            if (combo_of[s] == cb) pos_slot[next++] = s;
          next = start + 8 * ((count[cb] + 7) / 8);
          for (int j = start; j < next; ++j) {
            if (j >= start + count[cb]) pos_slot[j] = -1;
            pos_kind[0][j] = cb / 3;
            pos_kind[1][j] = cb % 3;
          }
        }
        for (int j = next; j < OASIS_MAX_FRAMES; ++j) {  // trailing dead tiles: kinds of the last group
          pos_slot[j] = -1;
          pos_kind[0][j] = pos_kind[0][next - 1];
          pos_kind[1][j] = pos_kind[1][next - 1];
        }
      }
    }
    for (int j = 0; j < OASIS_MAX_FRAMES; ++j)
      if (pos_slot[j] >= 0 && pos_slot[j] <= q_pos0) lay.valid |= 1u << j;
    // two kind-uniform runs of tiles, the same for keys and values: the split kernels
    if (uniform[0] == kDecMixed && uniform[1] == kDecMixed) {
      int split = 0;
      while (split < OASIS_MAX_FRAMES && pos_kind[0][split] == pos_kind[0][0] && pos_kind[1][split] == pos_kind[1][0])
        ++split;
      bool two_runs = split % 8 == 0 && split < OASIS_MAX_FRAMES && pos_kind[0][0] == pos_kind[1][0] &&
                      pos_kind[0][split] == pos_kind[1][split] && pos_kind[0][split] != pos_kind[0][0];
      for (int j = split; two_runs && j < OASIS_MAX_FRAMES; ++j)
        two_runs = pos_kind[0][j] == pos_kind[0][split] && pos_kind[1][j] == pos_kind[1][split];
      if (two_runs) {
        uniform[0] = uniform[1] = dec_split_code(pos_kind[0][0], pos_kind[0][split]);
        lay.split = split;
      }
    }
    for (int which = 0; which < 2; ++which) {
      const KvTensor& t = kv.t[which];
      DecodeTensor& d = lay.t[which];
      const int n_kind[3] = {t.n_bf16, t.n_fp8, t.n_int4};
      for (int k = 0; k < 3; ++k) {
        d.session_pages[k] = static_cast<uint32_t>(kv.layers * n_kind[k]);
        // a slot's row offset (pages x 144 rows x row bytes) is a 32-bit lane register
        if (static_cast<unsigned long long>(kv.layers) * n_kind[k] * OASIS_TOKENS * dec_row_bytes(k) >= (1ull << 32))
          return fail(OASIS_ERR_UNSUPPORTED, "attn_decode_kernel: one session's pool exceeds 4 GiB");
      }
      for (int j = 0; j < OASIS_MAX_FRAMES; ++j) {
        d.kinds |= static_cast<unsigned long long>(pos_kind[which][j]) << (2 * j);
        if (pos_slot[j] >= 0) d.slot_page[j] = static_cast<uint32_t>(layer * n_kind[pos_kind[which][j]] + t.index[pos_slot[j]]);
      }
    }
    // keys and values all FP8, all INT4, or bf16 in n-tile 0 and INT4 after it: 4 or 8
    // heads per warp
    const bool hg_int4 = uniform[0] == OASIS_KV_INT4 && uniform[1] == OASIS_KV_INT4;
    const bool hg_split = uniform[0] == dec_split_code(OASIS_KV_BF16, OASIS_KV_INT4) && uniform[1] == uniform[0] &&
                          lay.split == 8;
    const bool hg_fp8 = uniform[0] == OASIS_KV_FP8 && uniform[1] == OASIS_KV_FP8;
    const bool hg = hg_int4 || hg_split || hg_fp8;
    // 8 heads per warp where the items fill at least two rounds of the resident warps
    // (three 4-warp CTAs per SM), else 4 (twice the items: less idle time in the last round)
    const bool hpw8 = batch * OASIS_TOKENS * 2 >= 2 * 3 * kDhgWarps * num_sms();
    DecodeKernel kern = !hg ? decode_kernel(uniform[0], uniform[1])
                        : hg_int4 ? (hpw8 ? attn_decode_hg_kernel<kDhgInt4, 8> : attn_decode_hg_kernel<kDhgInt4, 4>)
                        : hg_fp8  ? (hpw8 ? attn_decode_hg_kernel<kDhgFp8, 8> : attn_decode_hg_kernel<kDhgFp8, 4>)
                                  : (hpw8 ? attn_decode_hg_kernel<kDhgBf16Int4, 8> : attn_decode_hg_kernel<kDhgBf16Int4, 4>);
    const int threads = hg ? kDhgThreads : kDecThreads;
    const int warps = hg ? kDhgWarps : kDecWarps;
    if (hg) lay.items = batch * OASIS_TOKENS * (hpw8 ? 2 : 4);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess || per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    const int ctas = std::min((lay.items + warps - 1) / warps, per_sm * num_sms());
    cudaError_t e = launch_pdl(kern, dim3(ctas), dim3(threads), 0, stream,
                               static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out),
                               kv, lay, q_pos0, n_past, kScaleLog2);
    if (e != cudaSuccess) return cuda_status(e, "attn_decode_kernel");
    return OASIS_OK;
  }
  if (q_frames > 1 && n_past > 0 && n_kv == n_past) {
    // several query frames, every key and value from cache slots: the register-fragment
    // window kernel when each tensor's slots share one kind
    int uniform[2] = {-1, -1};
    for (int which = 0; which < 2; ++which) {
      const KvTensor& t = kv.t[which];
      uniform[which] = t.kind[0];
      for (int s = 1; s < n_past; ++s)
        if (t.kind[s] != uniform[which]) uniform[which] = -1;
    }
    if (uniform[0] >= 0 && uniform[1] >= 0) {
      WindowLayout lay{};
      lay.m_tiles = (q_frames + 15) / 16;
      lay.items = batch * OASIS_TOKENS * OASIS_HEADS;
      for (int which = 0; which < 2; ++which) {
        const KvTensor& t = kv.t[which];
        DecodeTensor& d = lay.t[which];
        const int n_kind[3] = {t.n_bf16, t.n_fp8, t.n_int4};
        for (int k = 0; k < 3; ++k) {
          d.session_pages[k] = static_cast<uint32_t>(kv.layers * n_kind[k]);
          if (static_cast<unsigned long long>(kv.layers) * n_kind[k] * OASIS_TOKENS * dec_row_bytes(k) >= (1ull << 32))
            return fail(OASIS_ERR_UNSUPPORTED, "attn_window_cached_kernel: one session's pool exceeds 4 GiB");
        }
        for (int s = 0; s < n_past; ++s)
          d.slot_page[s] = static_cast<uint32_t>(layer * n_kind[uniform[which]] + t.index[s]);
      }
      const int ctas = (lay.items + kWcWarps - 1) / kWcWarps;
      cudaError_t e = launch_pdl(window_kernel(uniform[0], uniform[1], lay.m_tiles), dim3(ctas), dim3(kWcWarps * 32), 0, stream,
                                 static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), kv, lay,
                                 q_frames, q_pos0, n_past, kScaleLog2);
      if (e != cudaSuccess) return cuda_status(e, "attn_window_cached_kernel");
      return OASIS_OK;
    }
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
