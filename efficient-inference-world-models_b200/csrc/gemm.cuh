// tcgen05 / TMEM / TMA GEMM for the DiT projections, with fused epilogues.
//
//   D[m][n] = sum_k A[m][k] * B[n][k]        (A activations, B = nn.Linear weight)
//
// One persistent CTA per SM, 6 warps:
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage (128-byte swizzle)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, fused math, global stores
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of one
// tile overlaps the main loop of the next.
#pragma once

#include "common.cuh"

namespace oasis {

enum EpiKind : int {
  kEpiStoreBF16 = 0,     // D bf16
  kEpiStoreF32Bias = 1,  // D fp32 (+ bias[n])
  kEpiQkvRope = 2,       // D bf16, RoPE on columns < rope_cols (q and k), pairs (2i, 2i+1)
  kEpiBiasGelu = 3,      // D bf16 = gelu_tanh(acc + bias[n])
  kEpiGateResid = 4,     // resid fp32 [m][n] += gate[m / 144][n] * (acc + bias[n])
  kEpiAdaT = 5,          // swap-AB: out fp32 [n][m] = acc + bias[m]   (n < n_valid)
  kEpiFinal = 6,         // v fp32 unpatchified: token m, column (pi*2+qi)*16 + c
};

struct EpiParams {
  void* out;            // output base
  long long ldd;        // output leading dim (elements)
  const float* bias;    // per-column bias (kEpiAdaT: per-row)
  const float* gate;    // kEpiGateResid: gate rows, row stride gate_ld
  long long gate_ld;
  const float* rope;    // kEpiQkvRope: table [positions][32][2] (cos, sin)
  int rope_cols;        // columns < rope_cols are rotated (2048: q and k)
  int rope_div, rope_mod, rope_add;  // position(m) = (m / div) % mod + add
  int n_valid;          // kEpiAdaT: number of valid B rows
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;

template <int BN>
struct GemmShape {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes > 8 ? 8 : (192 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;  // power of two >= 64 for BN in {32..256}
  static constexpr int kBarBytes = 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;  // +1 KB align slack
};

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

// Epilogue for one thread: row m (global), 32 consecutive columns starting at n0.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const EpiParams& p, int M, int N, int m, int n0,
                                               float (&v)[32]) {
  if (EPI == kEpiAdaT) {
    // out[n][m]: lanes hold consecutive m -> coalesced across the warp for each n
    if (m >= M) return;
    const float b = p.bias ? p.bias[m] : 0.0f;
    float* out = static_cast<float*>(p.out);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = n0 + i;
      if (n < p.n_valid) out[static_cast<long long>(n) * p.ldd + m] = v[i] + b;
    }
    return;
  }
  if (m >= M) return;
  if (EPI == kEpiStoreBF16 || EPI == kEpiBiasGelu || EPI == kEpiQkvRope) {
    if (EPI == kEpiBiasGelu) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i] + p.bias[n0 + i]);
    }
    if (EPI == kEpiQkvRope) {
      if (n0 < p.rope_cols) {
        const int pos = (m / p.rope_div) % p.rope_mod + p.rope_add;
        const int pair0 = (n0 & 63) >> 1;  // 0 or 16
        const float2* tab = reinterpret_cast<const float2*>(p.rope) + pos * 32 + pair0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          // round the projection to bf16 first (the reference rotates the bf16 tensor)
          const float x0 = bf16_round(v[2 * i]);
          const float x1 = bf16_round(v[2 * i + 1]);
          const float2 cs = tab[i];
          v[2 * i] = x0 * cs.x - x1 * cs.y;
          v[2 * i + 1] = x1 * cs.x + x0 * cs.y;
        }
      }
    }
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + static_cast<long long>(m) * p.ldd + n0;
    uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      o4[j] = w;
    }
    return;
  }
  if (EPI == kEpiStoreF32Bias) {
    float* out = static_cast<float*>(p.out) + static_cast<long long>(m) * p.ldd + n0;
    float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 w;
      w.x = v[4 * j + 0] + (p.bias ? p.bias[n0 + 4 * j + 0] : 0.0f);
      w.y = v[4 * j + 1] + (p.bias ? p.bias[n0 + 4 * j + 1] : 0.0f);
      w.z = v[4 * j + 2] + (p.bias ? p.bias[n0 + 4 * j + 2] : 0.0f);
      w.w = v[4 * j + 3] + (p.bias ? p.bias[n0 + 4 * j + 3] : 0.0f);
      o4[j] = w;
    }
    return;
  }
  if (EPI == kEpiGateResid) {
    const float* g = p.gate + static_cast<long long>(m / OASIS_TOKENS) * p.gate_ld + n0;
    const float* b = p.bias + n0;
    float4* r4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) +
                                           static_cast<long long>(m) * p.ldd + n0);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 r = r4[j];
      const float4 gg = g4[j];
      const float4 bb = b4[j];
      r.x += gg.x * (v[4 * j + 0] + bb.x);
      r.y += gg.y * (v[4 * j + 1] + bb.y);
      r.z += gg.z * (v[4 * j + 2] + bb.z);
      r.w += gg.w * (v[4 * j + 3] + bb.w);
      r4[j] = r;
    }
    return;
  }
  if (EPI == kEpiFinal) {
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
    return;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                        EpiParams ep) {
  using S = GemmShape<BN>;
  constexpr int STAGES = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;       // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + kGemmBM - 1) / kGemmBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc<S::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) last_phase[s] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile % num_m) * kGemmBM;
        const int n0 = (tile / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sa, &tmA, &full_bar[stage], kb * kGemmBK, m0);
          tma_load_2d(sb, &tmB, &full_bar[stage], kb * kGemmBK, n0);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // make sure no TMA write is still in flight when the CTA retires
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0) mbar_wait(&full_bar[s], static_cast<uint32_t>(last_phase[s]));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++it) {
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
            umma_bf16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                      idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);  // frees the smem stage once these MMAs retire
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        umma_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
      }
      // all issued MMAs must retire before TMEM is released
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue warps 2..5 ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++it) {
      const int m0 = (tile % num_m) * kGemmBM;
      const int n0 = (tile / num_m) * BN;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        const int n_chunk = n0 + c * 32;
        if (EPI == kEpiAdaT || n_chunk < N) epilogue_chunk<EPI>(ep, M, N, m0 + row_in_tile, n_chunk, v);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<S::kTmemCols>(tmem_base);
}

// Host launcher (gemm.cu).  A: [M][lda] bf16, B: [N][ldb] bf16.
struct GemmOperands {
  CUtensorMap a, b;
  int M, N, K, bn;
};
int make_gemm_operands(GemmOperands* g, const void* A, long long lda, const void* B, long long ldb,
                       int M, int N, int K, int bn);
int launch_gemm(const GemmOperands& g, int epi, const EpiParams& ep, cudaStream_t stream,
                int max_ctas = 0);
int num_sms();

}  // namespace oasis
