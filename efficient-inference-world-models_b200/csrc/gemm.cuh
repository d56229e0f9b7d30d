// tcgen05 / TMEM / TMA GEMM for the DiT projections, with fused epilogues.
//
//   D[m][n] = sum_k A[m][k] * B[n][k]        (A activations, B = nn.Linear weight)
//
// Persistent CTAs, one per SM, 10 warps:
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage (128-byte swizzle)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..9  epilogue, two warps per TMEM lane quarter splitting the columns:
//               tcgen05.ld of the fp32 accumulator, fused math in registers, then a
//               128B-swizzled shared-memory tile and a TMA tensor store (bf16 outputs) or
//               TMA reduce-add (the fp32 residual update), so global traffic leaves in
//               full lines asynchronously.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of one
// tile overlaps the main loop of the next; TMEM is released as soon as a tile's last
// tcgen05.ld has completed.
//
// CTA pairs (clusters of 2, tcgen05 cta_group::2) run 256 x BN tiles: each CTA stages
// its 128 rows of A and half of the BN rows of B, the leader issues M=256 MMAs that
// read both CTAs' shared memory and write each CTA's 128 accumulator rows into its own
// TMEM.  Per SM this halves the B bytes staged and read per MMA, which is what keeps
// the tensor pipe fed at N=256.
#pragma once

#include "common.cuh"
#include "ln.cuh"

namespace oasis {

enum EpiKind : int {
  kEpiStoreBF16 = 0,     // D bf16                                         (TMA store)
  kEpiStoreF32Bias = 1,  // D fp32 = acc + bias[n]                         (TMA store)
  kEpiQkvRope = 2,       // D bf16, RoPE on columns < rope_cols (q and k)  (TMA store)
  kEpiBiasGelu = 3,      // D bf16 = gelu_tanh(acc + bias[n])              (TMA store)
  kEpiGateResid = 4,     // resid fp32 += gate[m / 144][n] * (acc + bias[n]) (TMA reduce-add)
  kEpiAdaT = 5,          // swap-AB: out fp32 [n][m] = acc + bias[m]   (n < n_valid)
  kEpiFinal = 6,         // v fp32 unpatchified: token m, column (pi*2+qi)*16 + c
  kEpiAdaTSilu = 7,      // swap-AB: out bf16 [n][m] = silu(acc + bias[m])   (n < n_valid)
};

__host__ __device__ constexpr bool epi_uses_tma(int e) {
  return e == kEpiStoreBF16 || e == kEpiStoreF32Bias || e == kEpiQkvRope || e == kEpiBiasGelu ||
         e == kEpiGateResid;
}
__host__ __device__ constexpr bool epi_out_f32(int e) {
  return e == kEpiStoreF32Bias || e == kEpiGateResid;
}

struct EpiParams {
  void* out;            // output base (row-per-thread epilogues)
  long long ldd;        // output leading dim (elements)
  const float* bias;    // per-column bias (swap-AB epilogues: per-row)
  const float* gate;    // kEpiGateResid: gate rows, row stride gate_ld
  long long gate_ld;
  const float* rope;    // kEpiQkvRope: table [positions][32][2] (cos, sin)
  int rope_cols;        // columns < rope_cols are rotated (2048: q and k)
  int rope_div, rope_mod, rope_add;  // position(m) = (m / div) % mod + add
  int n_valid;          // swap-AB epilogues: number of valid B rows
  // kEpiGateResid with ln_out set: LayerNorm + modulate of the updated residual rows
  // into ln_out (bf16 [M][1024]) as the kernel's tail.  ln_count holds one zeroed
  // counter per 128-row block (ceil(M / 128)); the kernel leaves each at the number of
  // N tiles.
  __nv_bfloat16* ln_out;
  const float* ln_shift;  // per-frame rows, stride ln_mod_ld
  const float* ln_scale;
  long long ln_mod_ld;
  unsigned int* ln_count;
  // kEpiGateResid split along K (k_splits > 1, single-CTA tiles): every output tile is
  // computed by k_splits units over equal K ranges; split s adds gate * acc_s (split 0 also
  // gate * bias) into the residual.  The splits' reduce-adds of one tile are ordered by
  // split_flags (one zeroed counter per output tile and epilogue warp: split s issues its
  // reduce-adds after the counter reaches s and releases s + 1 once they completed), so
  // the fp32 sum is formed in the same order on every run.
  int k_splits;
  unsigned int* split_flags;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kEpiBufBytes = 32 * 128;  // 32 rows x 128 B: one TMA store box

// Per-CTA shared-memory plan.  A CTA pair (CTAS = 2) computes a 256 x BN tile: each
// CTA stages 128 rows of A and BN/2 rows of B per k-block and holds a 128 x BN
// accumulator in its own TMEM.
template <int BN, int CTAS = 1>
struct GemmShape {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = (BN / CTAS) * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes > 8 ? 8 : (192 * 1024) / kStageBytes;
  // two accumulator buffers of BN columns, allocated as a power of two >= 64
  static constexpr int kTmemCols = 2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512));
  static constexpr int kBarBytes = 1024;
  static constexpr int kEpiBytes = kEpiWarps * kEpiBufBytes;  // one TMA box per epilogue warp
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kEpiBytes + kBarBytes + 1024;  // +1 KB alignment slack
};

// GELU, tanh approximation (nn.GELU(approximate="tanh")); tanh from the SFU
// (tanh.approx.f32, ~2^-11 relative error, below the bf16 rounding of the output).
__device__ __forceinline__ float tanh_sfu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanh_sfu(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Named barrier 1 over the 8 epilogue warps (warps 2..9).
__device__ __forceinline__ void epilogue_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_or(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.or.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until *p >= target (another CTA of this grid publishes it); records a
// timeout in the device error word and returns false after kWaitTimeoutNs.
__device__ __forceinline__ bool wait_count_geq(const unsigned int* p, unsigned int target) {
  if (ld_acquire(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire(p) >= target) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      atomicOr(&g_dev_error, kDevErrTimeout);
      return false;
    }
  }
}

// Bounded wait until bit `bit` of *p is set (another CTA of this grid sets it); `have`
// holds the last value read, so bits already seen cost no further round trip.  Records a
// timeout in the device error word and returns false after kWaitTimeoutNs.
__device__ __forceinline__ bool wait_bit(const unsigned int* p, int bit, unsigned int& have) {
  if ((have >> bit) & 1u) return true;
  have = ld_acquire(p);
  if ((have >> bit) & 1u) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    have = ld_acquire(p);
    if ((have >> bit) & 1u) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      atomicOr(&g_dev_error, kDevErrTimeout);
      return false;
    }
  }
}

// Write 16-byte chunk `c` (0..7) of row `r` (0..31) of a 128B-swizzled 32 x 128 B box.
__device__ __forceinline__ void st_swizzled(uint8_t* buf, int r, int c, uint4 v) {
  *reinterpret_cast<uint4*>(buf + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

// Row-per-thread epilogues (lane = row m, 32 consecutive columns from n0): used where
// that layout is already the coalesced one (swap-AB writes out[n][m]: lanes hold
// consecutive m) or the output is tiny and scattered (kEpiFinal).
template <int EPI>
__device__ __forceinline__ void epilogue_rows(const EpiParams& p, int M, int m, int n0,
                                              const float (&v)[32]) {
  if (m >= M) return;
  if (EPI == kEpiAdaT) {
    const float b = p.bias ? p.bias[m] : 0.0f;
    float* out = static_cast<float*>(p.out);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = n0 + i;
      if (n < p.n_valid) out[static_cast<long long>(n) * p.ldd + m] = v[i] + b;
    }
  } else if (EPI == kEpiAdaTSilu) {
    const float b = p.bias[m];
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = n0 + i;
      const float y = v[i] + b;
      if (n < p.n_valid) out[static_cast<long long>(n) * p.ldd + m] = __float2bfloat16_rn(y / (1.0f + expf(-y)));
    }
  } else if (EPI == kEpiFinal) {
    // token m = (frame, hp, wp); column j = (pi*2 + qi)*16 + c
    const int f = m / OASIS_TOKENS;
    const int pp = m % OASIS_TOKENS;
    const int hp = pp / 16, wp = pp % 16;
    float* out = static_cast<float*>(p.out) + static_cast<long long>(f) * (16 * 18 * 32);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int j = n0 + i;
      const int c = j & 15;
      const int pq = j >> 4;
      const int pi = pq >> 1, qi = pq & 1;
      out[(c * 18 + hp * 2 + pi) * 32 + wp * 2 + qi] = v[i] + p.bias[j];
    }
  }
}

// Elementwise math of the TMA epilogues on one thread's row segment (row m, columns
// n0..n0+31), in registers.
template <int EPI>
__device__ __forceinline__ void epilogue_math(const EpiParams& p, int m, int n0, float (&v)[32],
                                              bool bias_on = true) {
  if (EPI == kEpiBiasGelu || EPI == kEpiStoreF32Bias) {
    if (EPI == kEpiStoreF32Bias && !p.bias) return;
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 b = b4[j];
      v[4 * j + 0] += b.x;
      v[4 * j + 1] += b.y;
      v[4 * j + 2] += b.z;
      v[4 * j + 3] += b.w;
    }
    if (EPI == kEpiBiasGelu) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
    }
  } else if (EPI == kEpiQkvRope) {
    if (n0 < p.rope_cols) {
      const int pos = (m / p.rope_div) % p.rope_mod + p.rope_add;
      const float4* tab = reinterpret_cast<const float4*>(p.rope) + pos * 16 + ((n0 & 63) >> 2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 cs = tab[i];  // (cos, sin) of two consecutive pairs
        const float a0 = bf16_round(v[4 * i + 0]), a1 = bf16_round(v[4 * i + 1]);
        const float b0 = bf16_round(v[4 * i + 2]), b1 = bf16_round(v[4 * i + 3]);
        // the reference rotates the bf16-rounded projection: (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)
        v[4 * i + 0] = a0 * cs.x - a1 * cs.y;
        v[4 * i + 1] = a1 * cs.x + a0 * cs.y;
        v[4 * i + 2] = b0 * cs.z - b1 * cs.w;
        v[4 * i + 3] = b1 * cs.z + b0 * cs.w;
      }
    }
  } else if (EPI == kEpiGateResid) {
    const float4* g4 = reinterpret_cast<const float4*>(
        p.gate + static_cast<long long>(m / OASIS_TOKENS) * p.gate_ld + n0);
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 g = g4[j];
      const float4 b = bias_on ? b4[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      v[4 * j + 0] = g.x * (v[4 * j + 0] + b.x);
      v[4 * j + 1] = g.y * (v[4 * j + 1] + b.y);
      v[4 * j + 2] = g.z * (v[4 * j + 2] + b.z);
      v[4 * j + 3] = g.w * (v[4 * j + 3] + b.w);
    }
  }
}

// L1 prefetch of the operands epilogue_math reads for this thread's row m and blocks
// half, half+2, ... of the tile at n0 (issued before the accumulator is ready, so the
// loads in the epilogue hit L1 instead of waiting on L2 after each TMEM load).
template <int EPI, int COLS, int NBLK>
__device__ __forceinline__ void epilogue_prefetch(const EpiParams& p, int M, int N, int m, int n0,
                                                  int half) {
  if (m >= M) return;
#pragma unroll
  for (int blk = half; blk < NBLK; blk += 2) {
    const int nb = n0 + blk * COLS;
    if (nb >= N) break;
    if (EPI == kEpiGateResid) {
      prefetch_l1(p.gate + static_cast<long long>(m / OASIS_TOKENS) * p.gate_ld + nb);
      prefetch_l1(p.bias + nb);
    } else if (EPI == kEpiBiasGelu || EPI == kEpiStoreF32Bias) {
      if (p.bias)
        for (int c = 0; c < COLS; c += 32) prefetch_l1(p.bias + nb + c);
    } else if (EPI == kEpiQkvRope) {
      if (nb < p.rope_cols) {
        const int pos = (m / p.rope_div) % p.rope_mod + p.rope_add;
        for (int c = 0; c < COLS; c += 32) prefetch_l1(p.rope + pos * 64 + ((nb + c) & 63));
      }
    }
  }
}

// Box geometry of an epilogue: bf16 TMA boxes are 64 columns (2 TMEM loads); fp32 boxes
// and row epilogues 32.
template <int BN, int EPI>
struct EpiGeom {
  static constexpr int COLS = (epi_uses_tma(EPI) && !epi_out_f32(EPI)) ? 64 : 32;
  static constexpr int NBLK = BN / COLS;
  // bytes one warp needs to stage all of its boxes of a tile at once
  static constexpr int kWarpTileBytes = ((NBLK + 1) / 2) * kEpiBufBytes;
};

// The epilogue of one accumulator tile by one epilogue warp (TMEM lane quarter
// `quarter`, column blocks half, half+2, ...).  taddr: the warp's TMEM lanes at the
// tile's accumulator; m0: this CTA's first row of the tile.  Boxes go through `buf`
// (one 4 KB box, reused after its TMA store has read it; nbuf counts its stores) or,
// when `staging` is set, each to its own 4 KB slot there (all stores in flight at once).
// `release()` is called once the warp's last TMEM load of the tile has completed.
template <int BN, int EPI, typename Release>
__device__ __forceinline__ void epilogue_tile(const EpiParams& ep, const CUtensorMap* tmD, int M,
                                              int N, uint32_t taddr, int m0, int n0, int quarter,
                                              int half, int lane, uint8_t* buf, int& nbuf,
                                              uint8_t* staging, Release release, int split = 0,
                                              unsigned int* split_flag = nullptr,
                                              bool publish = false) {
  using G = EpiGeom<BN, EPI>;
  bool ordered = split_flag == nullptr || split == 0;  // may issue its reduce-adds
  constexpr int COLS = G::COLS, NBLK = G::NBLK;
  const int m_row = m0 + quarter * 32 + lane;  // this thread's row
  const bool rows_live = m0 + quarter * 32 < M;
  // operand row for the math: lanes past M (their stores are clipped) read row M - 1's
  // gate, not a frame beyond the modulation rows
  const int m_op = min(m_row, M - 1);
  const int last_blk = (NBLK - 1 - half) >= 0 ? ((NBLK - 1 - half) / 2) * 2 + half : -1;
  if (last_blk < 0) {  // owns no columns of this tile
    release();
    if (publish && lane == 0) red_release_add(split_flag, 1u);
    return;
  }
#pragma unroll 1
  for (int blk = half; blk < NBLK; blk += 2) {
    const int nb = n0 + blk * COLS;
    float v[32], w[32];
    tmem_ld32(taddr + blk * COLS, v);
    if (COLS == 64) tmem_ld32(taddr + blk * COLS + 32, w);
    if (blk == last_blk) release();  // this warp's share of the accumulator is read
    if (!epi_uses_tma(EPI)) {
      if (EPI != kEpiFinal || nb < N) epilogue_rows<EPI>(ep, M, m_row, nb, v);
      continue;
    }
    if (!rows_live || nb >= N) continue;
    uint8_t* box = buf;
    if (staging) {
      box = staging + (blk >> 1) * kEpiBufBytes;
    } else if (nbuf > 0) {  // the previous store from buf must have read it
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
    }
    epilogue_math<EPI>(ep, m_op, nb, v, split == 0);
    if (COLS == 64) {
      epilogue_math<EPI>(ep, m_op, nb + 32, w, split == 0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        st_swizzled(box, lane, c, make_uint4(pack_bf16x2(v[8 * c + 0], v[8 * c + 1]),
                                             pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                                             pack_bf16x2(v[8 * c + 4], v[8 * c + 5]),
                                             pack_bf16x2(v[8 * c + 6], v[8 * c + 7])));
        st_swizzled(box, lane, 4 + c, make_uint4(pack_bf16x2(w[8 * c + 0], w[8 * c + 1]),
                                                 pack_bf16x2(w[8 * c + 2], w[8 * c + 3]),
                                                 pack_bf16x2(w[8 * c + 4], w[8 * c + 5]),
                                                 pack_bf16x2(w[8 * c + 6], w[8 * c + 7])));
      }
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_swizzled(box, lane, c, make_uint4(__float_as_uint(v[4 * c + 0]), __float_as_uint(v[4 * c + 1]),
                                             __float_as_uint(v[4 * c + 2]), __float_as_uint(v[4 * c + 3])));
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (!ordered) {  // the previous split's reduce-adds of these rows must be complete
        wait_count_geq(split_flag, static_cast<unsigned>(split));
        fence_async_global();
        ordered = true;
      }
      if (EPI == kEpiGateResid)
        tma_reduce_add_2d(tmD, box, nb, m0 + quarter * 32);
      else
        tma_store_2d(tmD, box, nb, m0 + quarter * 32);
      bulk_commit();
    }
    if (!staging) ++nbuf;
  }
  if (publish && lane == 0) {  // next split of this tile: these reduce-adds are complete
    bulk_wait<0>();
    fence_async_global();
    red_release_add(split_flag, 1u);
  }
}

// LayerNorm + modulate of the residual rows [c*R, c*R + R) of this CTA (c = blockIdx.x,
// R = ceil(M / gridDim.x) rounded to 4) into ep.ln_out, each 4-row group once the
// `target` tiles of its 128-row block have been counted in ep.ln_count.  Warp w
// (0..7) takes groups w, w+8, ...; a group never crosses a frame or a block (144 and
// 128 are multiples of 4).  A group's 16 KB are copied into `stage` (16 KB per warp,
// idle shared memory) in one round trip and reduced from there.  When `rows_done` is
// set, each finished group adds its row count to rows_done[block] (release).
// Returns false when a wait timed out.
__device__ __forceinline__ bool ln_rows_phase(const EpiParams& ep, int M, unsigned target, int w,
                                              int lane, float4* stage, unsigned int* rows_done) {
  const int R = ((M + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x) + 3) & ~3;
  const int r_begin = static_cast<int>(blockIdx.x) * R;
  const int r_end = min(M, r_begin + R);
  // rows per group: 4 where every warp gets at least one group of 4, else 2 or 1, so
  // that all eight warps share a short row range (8 rows at 1,152 rows over 144 CTAs);
  // groups of 1, 2 or 4 tile R (a multiple of 4) and never cross a frame or a block
  const int gr = R >= kEpiWarps * kLnRowsPerWarp ? kLnRowsPerWarp : (R >= 2 * kEpiWarps ? 2 : 1);
  for (int row0 = r_begin + w * gr; row0 < r_end; row0 += kEpiWarps * gr) {
    // the frame's shift/scale (written by an earlier kernel) load while the rows finish
    const long long f = row0 / OASIS_TOKENS;
    float4 a4[8], s4[8];
    ln_load_modulation(ep.ln_shift + f * ep.ln_mod_ld, ep.ln_scale + f * ep.ln_mod_ld, lane, a4, s4);
    int ok = 1;
    if (lane == 0) ok = wait_count_geq(ep.ln_count + row0 / kGemmBM, target);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    __syncwarp();  // the acquire by lane 0 orders the whole warp's loads
    const int nrows = min(gr, r_end - row0);
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(ep.out) +
                                                        static_cast<long long>(row0) * OASIS_HIDDEN);
    // rows in pairs, each pair one cp.async group: the second pair lands while the first
    // is normalised (each lane copies, and later reads, only its own columns)
    for (int r = 0; r < nrows; ++r) {
#pragma unroll
      for (int i = 0; i < 8; ++i) cp_async16(stage + r * 256 + lane + 32 * i, src + r * 256 + lane + 32 * i);
      if (r & 1 || r + 1 == nrows) cp_async_commit();
    }
    __nv_bfloat16* out0 = ep.ln_out + static_cast<long long>(row0) * OASIS_HIDDEN;
#pragma unroll 1
    for (int r0 = 0; r0 < nrows; r0 += 2) {
      if (r0 + 2 < nrows)
        cp_async_wait_group<1>();  // this pair has landed, the next may be in flight
      else
        cp_async_wait_group<0>();
      ln_modulate_rows_smem(stage + r0 * 256, min(2, nrows - r0), a4, s4, out0 + r0 * OASIS_HIDDEN, lane);
    }
    if (rows_done) {
      __syncwarp();
      if (lane == 0) red_release_add(rows_done + row0 / kGemmBM, static_cast<unsigned>(nrows));
    }
  }
  return true;
}

template <int BN, int EPI, int CTAS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmD, int M, int N, int K,
                        int prefetch_b, EpiParams ep) {
  static_assert(CTAS == 1 || CTAS == 2, "one CTA or a CTA pair per tile");
  using S = GemmShape<BN, CTAS>;
  constexpr int STAGES = S::kStages;
  constexpr int TILE_M = kGemmBM * CTAS;  // rows of one tile (the pair's MMA M)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* epi_smem = smem + STAGES * S::kStageBytes;  // 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + S::kEpiBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;       // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // A pair shares one tile: rank 0 (the leader) issues the MMAs for both CTAs, rank r
  // holds A rows [r*128, r*128+128) and B rows [r*BN/2, r*BN/2 + BN/2) of the tile.
  const uint32_t rank = CTAS == 2 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = static_cast<int>(blockIdx.x) / CTAS;
  const int num_units = static_cast<int>(gridDim.x) / CTAS;
  const int num_m = (M + TILE_M - 1) / TILE_M;
  const int num_n = (N + BN - 1) / BN;
  // kEpiGateResid may split K: unit = (output tile, split), the split fastest
  const int splits = (EPI == kEpiGateResid && CTAS == 1 && ep.k_splits > 1) ? ep.k_splits : 1;
  const int num_tiles = num_m * num_n * splits;
  const int num_kb = K / kGemmBK / splits;  // k-blocks of one unit
  auto unit_m0 = [&](int t) { return ((t / splits) % num_m) * TILE_M; };
  auto unit_n0 = [&](int t) { return ((t / splits) / num_m) * BN; };
  auto unit_kb0 = [&](int t) { return (t % splits) * num_kb; };
  const int a_row0 = static_cast<int>(rank) * kGemmBM;
  const int b_row0 = static_cast<int>(rank) * (BN / CTAS);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], CTAS * kEpiWarps);  // one arrival per epilogue warp of the pair
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (epi_uses_tma(EPI)) tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    if (CTAS == 2)
      tmem_alloc_pair<S::kTmemCols>(tmem_holder);
    else
      tmem_alloc<S::kTmemCols>(tmem_holder);
  }
  tc_fence_before();
  __syncthreads();
  if (CTAS == 2) cluster_sync_all();  // the peer's barriers are initialised before any use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // the leader's barriers as seen from either CTA of the pair
  const uint32_t lead_full = CTAS == 2 ? mapa_shared(smem_u32(full_bar), 0) : smem_u32(full_bar);
  const uint32_t lead_tempty =
      CTAS == 2 ? mapa_shared(smem_u32(tempty_bar), 0) : smem_u32(tempty_bar);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs of a pair load their own halves) ----------
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) last_phase[s] = -1;
      auto load = [&](void* dst, const CUtensorMap* map, int s, int c0, int c1) {
        if (CTAS == 2)
          tma_load_2d_pair(dst, map, lead_full + s * 8, c0, c1);
        else
          tma_load_2d(dst, map, &full_bar[s], c0, c1);
      };
      // The operand that is a weight (never written by an earlier kernel: B of the
      // projections, A of the swap-AB GEMMs) is fetched for the first stages before
      // waiting on the previous kernel, the other operand after.
      // prefetch_b: bit 0 = B is a weight, bit 1 = A is a weight.
      int pre = 0;
      const bool pre_a = (prefetch_b & 2) != 0;
      if (prefetch_b && unit < num_tiles) {
        const int m0 = unit_m0(unit);
        const int n0 = unit_n0(unit);
        const int kb0 = unit_kb0(unit);
        pre = num_kb < STAGES ? num_kb : STAGES;
        for (int kb = 0; kb < pre; ++kb) {
          if (leader) mbar_arrive_expect_tx(&full_bar[kb], CTAS * S::kStageBytes);
          if (pre_a)
            load(smem + kb * S::kStageBytes, &tmA, kb, (kb0 + kb) * kGemmBK, m0 + a_row0);
          else
            load(smem + kb * S::kStageBytes + S::kABytes, &tmB, kb, (kb0 + kb) * kGemmBK, n0 + b_row0);
        }
      }
      pdl_wait();
      for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units) {
        const int m0 = unit_m0(tile);
        const int n0 = unit_n0(tile);
        const int kb0 = unit_kb0(tile);
        for (int kb = 0; kb < num_kb; ++kb) {
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          const int kc = (kb0 + kb) * kGemmBK;
          if (pre > 0) {  // stage already armed and its weight tile in flight
            --pre;
            if (pre_a)
              load(sb, &tmB, stage, kc, n0 + b_row0);
            else
              load(sa, &tmA, stage, kc, m0 + a_row0);
          } else {
            // the stage is free once the MMAs that read it (in both CTAs) have completed
            if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], CTAS * S::kStageBytes);
            load(sa, &tmA, stage, kc, m0 + a_row0);
            load(sb, &tmB, stage, kc, n0 + b_row0);
          }
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // no TMA write may still be in flight when the CTA retires: the leader sees its
      // full barriers complete; the peer's copies count on the leader's barrier, so it
      // waits for the MMAs that consumed them to release its stages
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0) {
          if (CTAS == 1 || leader)
            mbar_wait(&full_bar[s], static_cast<uint32_t>(last_phase[s]));
          else
            mbar_wait(&empty_bar[s], static_cast<uint32_t>(last_phase[s]));
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (reads only shared memory and TMEM) ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(TILE_M, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(a_addr + k * 32), bd = umma_desc_sw128(b_addr + k * 32);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (CTAS == 2)
              umma_bf16_pair(d_tmem, ad, bd, idesc, accum);
            else
              umma_bf16(d_tmem, ad, bd, idesc, accum);
          }
          // frees the smem stage (of both CTAs) once these MMAs retire
          if (CTAS == 2)
            umma_commit_pair(&empty_bar[stage]);
          else
            umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        // accumulator ready for the epilogue (of both CTAs)
        if (CTAS == 2)
          umma_commit_pair(&tfull_bar[acc]);
        else
          umma_commit(&tfull_bar[acc]);
      }
      // all issued MMAs must retire before TMEM is released
      if (CTAS == 2)
        umma_commit_pair_local(drain_bar);
      else
        umma_commit(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue warps 2..9 ----------------
    pdl_wait();  // bias/gate/rope tables and the output buffers belong to earlier kernels
    const int quarter = warp & 3;        // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;    // which interleaved column blocks it owns
    uint8_t* buf = epi_smem + (warp - 2) * kEpiBufBytes;
    int nbuf = 0;  // TMA stores issued by this warp from buf
    int it = 0;
    using G = EpiGeom<BN, EPI>;
    // The last tile of a CTA has the operand stages to itself once its accumulator is
    // complete (no load is issued after its k-blocks and its MMAs have retired): each
    // warp stages all of its boxes there and issues their TMA stores back to back
    // instead of cycling one 4 KB buffer.
    static_assert(kEpiWarps * G::kWarpTileBytes <= STAGES * S::kStageBytes, "last-tile staging");
    for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units, ++it) {
      const int m0 = unit_m0(tile) + a_row0;  // this CTA's accumulator rows
      const int n0 = unit_n0(tile);
      const int split = tile % splits;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (epi_uses_tma(EPI))
        epilogue_prefetch<EPI, G::COLS, G::NBLK>(ep, M, N, m0 + quarter * 32 + lane, n0, half);
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      const bool last_tile = tile + num_units >= num_tiles;
      // one arrival per warp on the leader's tempty barrier once all its lanes have read
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (CTAS == 2)
            mbar_arrive_cluster(lead_tempty + acc * 8);
          else
            mbar_arrive(&tempty_bar[acc]);
        }
      };
      // split-K: this warp's counter of the output tile orders the splits' reduce-adds
      unsigned int* flag = splits > 1 ? ep.split_flags + (tile / splits) * kEpiWarps + half * 4 + quarter
                                      : nullptr;
      epilogue_tile<BN, EPI>(ep, &tmD, M, N, taddr, m0, n0, quarter, half, lane, buf, nbuf,
                             last_tile ? smem + (warp - 2) * G::kWarpTileBytes : nullptr, release,
                             split, flag, flag != nullptr && split + 1 < splits);
    }
    if (epi_uses_tma(EPI) && lane == 0) bulk_wait<0>();  // all stores complete before exit
    __syncwarp();
    if (EPI == kEpiGateResid && ep.ln_out) {
      // ---- tail: LayerNorm + modulate of the finished residual rows ----
      // publish: every 128-row block this CTA updated gets one count per tile, released
      // after all eight warps' reduce-adds have completed
      if (lane == 0) fence_async_global();
      epilogue_bar_sync();
      if (warp == 2 && lane == 0 && !*abort_flag) {
        const int nblk = (M + kGemmBM - 1) / kGemmBM;
        for (int tile = unit; tile < num_tiles; tile += num_units) {
          const int q = (unit_m0(tile) + a_row0) / kGemmBM;
          if (q < nblk) red_release_add(ep.ln_count + q, 1u);
        }
      }
      // consume, staging rows in the now idle operand stages (16 KB per warp)
      static_assert(kEpiWarps * kLnRowsPerWarp * OASIS_HIDDEN * 4 <= STAGES * S::kStageBytes, "LN staging");
      ln_rows_phase(ep, M, static_cast<unsigned>(num_n * splits), warp - 2, lane,
                    reinterpret_cast<float4*>(smem + (warp - 2) * (kLnRowsPerWarp * OASIS_HIDDEN * 4)),
                    nullptr);
    }
  }

  tc_fence_before();
  __syncthreads();
  // a pair frees its TMEM together, after both CTAs are done with it (and with each
  // other's barriers)
  if (CTAS == 2) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if (CTAS == 2)
      tmem_dealloc_pair<S::kTmemCols>(tmem_base);
    else
      tmem_dealloc<S::kTmemCols>(tmem_base);
  }
}

// ----------------------------------------------------------------------------------
// Chained projections in one persistent launch: the out-projection (+ LayerNorm tail),
// fc1, fc2 (+ LayerNorm tail) and the next sub-block's QKV of one token window run as
// successive ops of one grid of CTA pairs (256 x 256 tiles).  An op's A rows are
// loaded as soon as the 128-row block they come from is complete (row-block counters
// published with release / read with acquire), so one op's tail overlaps the next
// op's first tiles instead of a kernel boundary.  Dependencies only point to earlier
// ops and every CTA of the grid is resident, so every wait ends (each is also bounded).
// ----------------------------------------------------------------------------------
constexpr int kMaxChainOps = 4;

struct alignas(64) ChainOp {
  CUtensorMap a, b, d;
  EpiParams ep;                // ep.ln_out set (kEpiGateResid): LayerNorm phase after the op
  int M, N, K, epi;            // epi: kEpiGateResid, kEpiBiasGelu or kEpiQkvRope
  const unsigned int* wait;    // per 128-row block counters the A rows wait on, or null
  unsigned int wait_tiles;     // target: this many tiles, or (0) the block's row count
  unsigned int* tiles_done;    // +1 per finished tile and 128-row block (also ep.ln_count)
  unsigned int* rows_done;     // LayerNorm phase: + rows per finished group, or null
  int publish_bits;            // tiles_done[block] |= 1 << (n0 / 256) instead of += 1
  int wait_bits;               // `wait` holds such bitmasks: k-block kb of a tile needs bit
                               // kb * 64 / 256 of its block (the producing tile of those K
                               // columns), polled as the k loop reaches it
};

struct ChainParams {
  ChainOp op[kMaxChainOps];
  int n_ops;
  int prefetch_b;  // op 0's B (weights) may be fetched before the previous kernel ends
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_chain_kernel(const __grid_constant__ ChainParams P) {
  constexpr int BN = 256, CTAS = 2;
  using S = GemmShape<BN, CTAS>;
  constexpr int STAGES = S::kStages;
  constexpr int TILE_M = kGemmBM * CTAS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* epi_smem = smem + STAGES * S::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + S::kEpiBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;       // [1]
  uint64_t* ln_free_bar = drain_bar + 1;      // [1] epilogue warps -> producer: stages free again
  uint64_t* stored_bar = ln_free_bar + 1;     // [1] epilogue warps -> publisher: a tile's stores done
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stored_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert(kEpiWarps * kLnRowsPerWarp * OASIS_HIDDEN * 4 <= STAGES * S::kStageBytes, "LN staging");

  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int unit = static_cast<int>(blockIdx.x) / CTAS;
  const int num_units = static_cast<int>(gridDim.x) / CTAS;
  const int a_row0 = static_cast<int>(rank) * kGemmBM;
  const int b_row0 = static_cast<int>(rank) * (BN / CTAS);
  const int n_ops = P.n_ops;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], CTAS * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    mbar_init(ln_free_bar, kEpiWarps);
    mbar_init(stored_bar, kEpiWarps);
    *abort_flag = 0;
    mbar_fence_init();
    for (int o = 0; o < n_ops; ++o) {
      tma_prefetch_desc(&P.op[o].a);
      tma_prefetch_desc(&P.op[o].b);
      tma_prefetch_desc(&P.op[o].d);
    }
  }
  if (warp == 1) tmem_alloc_pair<S::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t lead_full = mapa_shared(smem_u32(full_bar), 0);
  const uint32_t lead_tempty = mapa_shared(smem_u32(tempty_bar), 0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) last_phase[s] = -1;
      int pre = 0;
      if (P.prefetch_b && n_ops > 0) {
        const ChainOp& op = P.op[0];
        const int num_m = (op.M + TILE_M - 1) / TILE_M;
        if (unit < num_m * (op.N / BN)) {
          const int n0 = (unit / num_m) * BN;
          const int num_kb = op.K / kGemmBK;
          pre = num_kb < STAGES ? num_kb : STAGES;
          for (int kb = 0; kb < pre; ++kb) {
            if (leader) mbar_arrive_expect_tx(&full_bar[kb], CTAS * S::kStageBytes);
            tma_load_2d_pair(smem + kb * S::kStageBytes + S::kABytes, &op.b, lead_full + kb * 8,
                             kb * kGemmBK, n0 + b_row0);
          }
        }
      }
      pdl_wait();
      uint32_t ln_phase = 0;
      for (int o = 0; o < n_ops && !*abort_flag; ++o) {
        const ChainOp& op = P.op[o];
        if (o > 0 && P.op[o - 1].ep.ln_out) {
          // the stages were lent to the previous op's LayerNorm phase
          if (!mbar_wait(ln_free_bar, ln_phase)) { *abort_flag = 1; break; }
          ln_phase ^= 1;
        }
        const int num_m = (op.M + TILE_M - 1) / TILE_M;
        const int num_tiles = num_m * (op.N / BN);
        const int num_kb = op.K / kGemmBK;
        for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units) {
          const int m0 = (tile % num_m) * TILE_M;
          const int n0 = (tile / num_m) * BN;
          const bool rows_in = m0 + a_row0 < op.M;
          unsigned int have = 0;  // wait_bits: the block's tile bits seen so far
          if (op.wait && !op.wait_bits) {  // this CTA's 128 A rows must be complete
            const int q = (m0 + a_row0) / kGemmBM;
            const unsigned target = op.wait_tiles ? op.wait_tiles
                                                  : static_cast<unsigned>(min(kGemmBM, op.M - q * kGemmBM));
            if (m0 + a_row0 < op.M && !wait_count_geq(op.wait + q, target)) { *abort_flag = 1; break; }
            fence_async_global();  // the acquired rows are read by TMA (async proxy)
          }
          for (int kb = 0; kb < num_kb; ++kb) {
            uint8_t* sa = smem + stage * S::kStageBytes;
            uint8_t* sb = sa + S::kABytes;
            if (op.wait_bits && rows_in && !((have >> ((kb * kGemmBK) / BN)) & 1u)) {
              // the A columns of this k-block come from one producer tile of the block
              if (!wait_bit(op.wait + (m0 + a_row0) / kGemmBM, (kb * kGemmBK) / BN, have)) {
                *abort_flag = 1;
                break;
              }
              fence_async_global();  // the acquired columns are read by TMA (async proxy)
            }
            if (pre > 0) {
              --pre;
              tma_load_2d_pair(sa, &op.a, lead_full + stage * 8, kb * kGemmBK, m0 + a_row0);
            } else {
              if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
              if (leader) mbar_arrive_expect_tx(&full_bar[stage], CTAS * S::kStageBytes);
              tma_load_2d_pair(sa, &op.a, lead_full + stage * 8, kb * kGemmBK, m0 + a_row0);
              tma_load_2d_pair(sb, &op.b, lead_full + stage * 8, kb * kGemmBK, n0 + b_row0);
            }
            last_phase[stage] = static_cast<int>(phase);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0) {
          if (leader)
            mbar_wait(&full_bar[s], static_cast<uint32_t>(last_phase[s]));
          else
            mbar_wait(&empty_bar[s], static_cast<uint32_t>(last_phase[s]));
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(TILE_M, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int o = 0; o < n_ops && !*abort_flag; ++o) {
        const ChainOp& op = P.op[o];
        const int num_tiles = ((op.M + TILE_M - 1) / TILE_M) * (op.N / BN);
        const int num_kb = op.K / kGemmBK;
        bool ok = true;
        for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units, ++it) {
          const int acc = it & 1;
          const uint32_t acc_phase = (it >> 1) & 1;
          if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
          for (int kb = 0; kb < num_kb; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + stage * S::kStageBytes);
            const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k)
              umma_bf16_pair(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                             idesc, (kb > 0 || k > 0) ? 1u : 0u);
            umma_commit_pair(&empty_bar[stage]);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          umma_commit_pair(&tfull_bar[acc]);
        }
        if (!ok) { *abort_flag = 1; break; }
      }
      umma_commit_pair_local(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue warps 2..9 ----------------
    pdl_wait();
    const int w = warp - 2;
    const int quarter = warp & 3;
    const int half = w >> 2;
    uint8_t* buf = epi_smem + w * kEpiBufBytes;
    int nbuf = 0;
    int it = 0;
    uint32_t stored_phase = 0;
    // (no bar.sync among the epilogue warps here: a warp that gives up on a timed-out
    // wait must not leave the others blocked; they meet on bounded mbarrier waits)
    for (int o = 0; o < n_ops && !*abort_flag; ++o) {
      const ChainOp& op = P.op[o];
      const int num_m = (op.M + TILE_M - 1) / TILE_M;
      const int num_n = op.N / BN;
      const int num_tiles = num_m * num_n;
      const int nblk = (op.M + kGemmBM - 1) / kGemmBM;
      // the stages are free for the last tile's boxes only if no later op is loading:
      // after the last op, or before a LayerNorm phase (the producer waits for it)
      const bool can_stage = o == n_ops - 1 || op.ep.ln_out != nullptr;
      for (int tile = unit; tile < num_tiles && !*abort_flag; tile += num_units, ++it) {
        const int m0 = (tile % num_m) * TILE_M + a_row0;
        const int n0 = (tile / num_m) * BN;
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        const int m_row = m0 + quarter * 32 + lane;
        switch (op.epi) {
          case kEpiGateResid:
            epilogue_prefetch<kEpiGateResid, 32, 8>(op.ep, op.M, op.N, m_row, n0, half);
            break;
          case kEpiBiasGelu:
            epilogue_prefetch<kEpiBiasGelu, 64, 4>(op.ep, op.M, op.N, m_row, n0, half);
            break;
          default:
            epilogue_prefetch<kEpiQkvRope, 64, 4>(op.ep, op.M, op.N, m_row, n0, half);
            break;
        }
        if (!mbar_wait(&tfull_bar[acc], acc_phase)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(acc * BN);
        const bool staged = can_stage && tile + num_units >= num_tiles;
        auto release = [&]() {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_tempty + acc * 8);
        };
        switch (op.epi) {
          case kEpiGateResid:
            epilogue_tile<BN, kEpiGateResid>(op.ep, &op.d, op.M, op.N, taddr, m0, n0, quarter, half,
                                             lane, buf, nbuf,
                                             staged ? smem + w * EpiGeom<BN, kEpiGateResid>::kWarpTileBytes
                                                    : nullptr,
                                             release);
            break;
          case kEpiBiasGelu:
            epilogue_tile<BN, kEpiBiasGelu>(op.ep, &op.d, op.M, op.N, taddr, m0, n0, quarter, half,
                                            lane, buf, nbuf,
                                            staged ? smem + w * EpiGeom<BN, kEpiBiasGelu>::kWarpTileBytes
                                                   : nullptr,
                                            release);
            break;
          default:
            epilogue_tile<BN, kEpiQkvRope>(op.ep, &op.d, op.M, op.N, taddr, m0, n0, quarter, half,
                                           lane, buf, nbuf,
                                           staged ? smem + w * EpiGeom<BN, kEpiQkvRope>::kWarpTileBytes
                                                  : nullptr,
                                           release);
            break;
        }
        if (op.tiles_done) {
          // publish the tile once all eight warps' stores to it have completed
          if (lane == 0) {
            bulk_wait<0>();
            fence_async_global();
            mbar_arrive(stored_bar);
          }
          nbuf = 0;  // buf is free again
          // every warp waits for the phase, so no warp can arrive for the next tile first
          if (lane == 0) {
            if (!mbar_wait(stored_bar, stored_phase)) {
              *abort_flag = 1;
            } else if (w == 0) {
              const int q = m0 / kGemmBM;
              if (q < nblk) {
                if (op.publish_bits)
                  red_release_or(op.tiles_done + q, 1u << (n0 / BN));
                else
                  red_release_add(op.tiles_done + q, 1u);
              }
            }
          }
          stored_phase ^= 1;
          __syncwarp();
        }
      }
      if (*abort_flag) break;
      if (op.ep.ln_out) {
        // LayerNorm phase in the (lent) operand stages, then hand them back
        if (!ln_rows_phase(op.ep, op.M, static_cast<unsigned>(num_n), w, lane,
                           reinterpret_cast<float4*>(smem + w * (kLnRowsPerWarp * OASIS_HIDDEN * 4)),
                           op.rows_done)) {
          *abort_flag = 1;
        }
        fence_async_smem();  // these generic writes precede the producer's TMA writes
        __syncwarp();
        if (lane == 0) mbar_arrive(ln_free_bar);
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair<S::kTmemCols>(tmem_base);
}

// Host side (gemm.cu).  A: [M][lda] bf16, B: [N][ldb] bf16; D described by its own
// tensor map for the TMA epilogues.
struct GemmOperands {
  CUtensorMap a, b, d;
  int M, N, K, bn;
  int ctas;    // 1: one CTA per 128 x bn tile; 2: CTA pairs on 256 x 256 tiles
  int splits;  // > 1: K split into this many equal ranges (residual epilogue only)
  bool has_d;
  bool b_is_weight;  // B is never written by another kernel: may be prefetched early
  bool a_is_weight;  // the same for A (swap-AB GEMMs)
};
int make_gemm_operands(GemmOperands* g, const void* A, long long lda, const void* B, long long ldb,
                       int M, int N, int K, int bn, int ctas = 1);
// Tile shape for an M x N x K projection on this GPU: CTA pairs on 256 x 256 tiles from
// 4,096 rows on, unless they take fewer than four waves with the last under 45 % full;
// otherwise single CTAs
// with the (tile N, K splits) of least estimated time (K splits only where allow_split:
// the residual epilogue, whose reduce-add is linear in the accumulator).
void choose_tiles(int M, int N, int K, bool allow_split, int* bn, int* ctas, int* splits);
// Counters (unsigned ints, zeroed before the launch) a split-K launch of `g` orders its
// reduce-adds with: one per output tile and epilogue warp.
size_t split_flag_count(const GemmOperands& g);
// Output tensor map for the TMA epilogues: D [M][N] with leading dim ldd, bf16 or fp32.
int set_gemm_output(GemmOperands* g, void* D, long long ldd, bool f32);
int launch_gemm(const GemmOperands& g, int epi, const EpiParams& ep, cudaStream_t stream,
                int max_ctas = 0);
// One step of a chained launch: operands from make_gemm_operands (CTA pairs, tile N
// 256, output map set), epilogue, and the row-block counters it waits on / publishes.
struct ChainStep {
  const GemmOperands* g;
  int epi;
  EpiParams ep;
  const unsigned int* wait;
  unsigned int wait_tiles;
  unsigned int* tiles_done;
  unsigned int* rows_done;
  bool publish_bits;  // tiles_done as per-block bitmasks of finished N tiles (at most 32)
  bool wait_bits;     // `wait` holds such bitmasks; each k-block waits for its producer tile
};
int launch_chain(const ChainStep* steps, int n, cudaStream_t stream);
int num_sms();

}  // namespace oasis
