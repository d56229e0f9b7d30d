// ViT latent decoder (`vae.decode` of the Oasis rollout, worldserve/models/oasis.py:237-245):
// latents (frames, 576, 16) -> RGB (frames, 3, 360, 640).  The projections run on the
// tcgen05 GEMMs of the DiT with the same fused epilogues (QKV with axial RoPE, residual
// reduce-add with the next LayerNorm as its tail, bias + GELU); attention over the 576
// tokens of a frame is a flash-attention kernel on mma.sync.
#include "launch.cuh"
#include "gemm.cuh"

namespace oasis {
namespace {

constexpr int kVaeTokens = 576;   // 18 x 32 latent tokens per frame
constexpr int kVaeImgH = 360, kVaeImgW = 640;
inline size_t vae_align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// z fp32 [M][16] -> bf16 [M][64] (columns 16..63 zero): the A operand of the latent
// projection, whose K is padded to one 64-wide k-block
__global__ void vae_latent_prep_kernel(const float* __restrict__ z, __nv_bfloat16* __restrict__ a, int M) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // one 8-column chunk
  if (i >= M * 8) return;
  const int row = i >> 3, ch = i & 7;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (ch < 2) {
    const float4* src = reinterpret_cast<const float4*>(z + static_cast<long long>(row) * 16 + ch * 8);
    const float4 x0 = src[0], x1 = src[1];
    v = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                   pack_bf16x2(x1.z, x1.w));
  }
  reinterpret_cast<uint4*>(a + static_cast<long long>(row) * 64)[ch] = v;
}

// predictor output fp32 [M][ld] (column (p*20 + q)*3 + c of token (h, w)) -> RGB
// [frames][3][360][640], pixel (h*20 + p, w*20 + q)
__global__ void vae_unpatchify_kernel(const float* __restrict__ y, int ld, float* __restrict__ out, int frames) {
  pdl_trigger();
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(frames) * 3 * kVaeImgH * kVaeImgW) return;
  const int x = static_cast<int>(i % kVaeImgW);
  long long r = i / kVaeImgW;
  const int yy = static_cast<int>(r % kVaeImgH);
  r /= kVaeImgH;
  const int c = static_cast<int>(r % 3);
  const long long f = r / 3;
  const int tok = (yy / 20) * 32 + x / 20, p = yy % 20, q = x % 20;
  out[i] = y[(f * kVaeTokens + tok) * ld + (p * 20 + q) * 3 + c];
}

// ----------------------------------------------------------------------------------
// attention over the 576 tokens of a frame (non-causal): one CTA per (64-query block,
// head, frame), one warp per 16 query rows; 64-key K/V tiles double-buffered through
// shared memory by cp.async; S and P V on mma.sync (bf16, fp32 accumulation) with an
// online softmax in registers.  q and k arrive post-RoPE from the QKV epilogue.
// KG key groups of 4 warps split the 9 key blocks (group g takes blocks g, g + KG, ...),
// each with its own K/V ring and named barrier; groups 1.. hand their running max, sum
// and O to group 0, which merges them (the exact rescaling of the online softmax) and
// writes the rows.  KG = 3 triples the warps per query row for a 1-frame decode, whose
// 144 CTAs leave each SM one CTA; larger decodes run KG = 1.
// ----------------------------------------------------------------------------------
constexpr int kVaTile = 64 * 72;  // bf16 elements of a 64-row tile, rows padded to 72 (conflict-free ldmatrix)
constexpr int kVaBlocks = kVaeTokens / 64;  // 9 key blocks (and query blocks)
constexpr int kVaGroupTiles = 4;            // per key group: 2 stages x (K, V)
// Q + KG groups' rings: 46,080 B (KG = 1), 119,808 B (KG = 3)
constexpr int va_smem(int kg) { return (1 + kVaGroupTiles * kg) * kVaTile * 2; }
constexpr int kVaExFloats = 36;             // per thread: o[8][4], m0, m1, l0, l1

__device__ __forceinline__ void va_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void va_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// barrier of key group g's 128 threads (id 0 is __syncthreads, the whole CTA when KG = 1)
template <int KG>
__device__ __forceinline__ void va_group_sync(int g) {
  if constexpr (KG == 1)
    __syncthreads();
  else
    asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory");
}

template <int KG>
__global__ void __launch_bounds__(128 * KG) attn_vae_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                            __nv_bfloat16* __restrict__ out, float scale_log2) {
  static_assert(KG >= 1 && KG <= 3, "1..3 key groups");
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm_va[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(sm_va);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int grp = warp >> 2, wq = warp & 3, gtid = tid & 127;
  // this group's ring: stage s has K at skv + 2s tiles, V at + (2s + 1)
  __nv_bfloat16* skv = sq + kVaTile + grp * kVaGroupTiles * kVaTile;
  const int g = lane >> 2, c = lane & 3;
  const int qb = blockIdx.x, h = blockIdx.y;
  const long long row0 = static_cast<long long>(blockIdx.z) * kVaeTokens;
  pdl_wait();
  // a 64 x 64 tile: 64 rows x 8 chunks of 16 B, copied by `n` threads from thread `t0` on
  auto load_tile = [&](__nv_bfloat16* dst, int col0, int tok0, int t0, int n) {
#pragma unroll
    for (int i = t0; i < 512; i += n) {
      const int r = i >> 3, ch = i & 7;
      cp_async16(dst + r * 72 + ch * 8, qkv + (row0 + tok0 + r) * (3 * OASIS_HIDDEN) + col0 + ch * 8);
    }
  };
  auto tile_addr = [&](const __nv_bfloat16* base, int row, int chunk) { return smem_u32(base + row * 72 + chunk * 8); };

  load_tile(sq, h * 64, qb * 64, tid, 128 * KG);
  load_tile(skv, OASIS_HIDDEN + h * 64, grp * 64, gtid, 128);
  load_tile(skv + kVaTile, 2 * OASIS_HIDDEN + h * 64, grp * 64, gtid, 128);
  va_commit();

  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -1e30f, m1 = -1e30f, l0 = 0.0f, l1 = 0.0f;

  int st = 0;
  for (int kb = grp; kb < kVaBlocks; kb += KG, st ^= 1) {
    if (kb + KG < kVaBlocks) {
      __nv_bfloat16* nx = skv + 2 * (st ^ 1) * kVaTile;
      load_tile(nx, OASIS_HIDDEN + h * 64, (kb + KG) * 64, gtid, 128);
      load_tile(nx + kVaTile, 2 * OASIS_HIDDEN + h * 64, (kb + KG) * 64, gtid, 128);
      va_commit();
      va_wait<1>();  // this thread's copies of block kb (and of Q) have landed
    } else {
      va_wait<0>();
    }
    if (kb == grp) {
      __syncthreads();  // Q (copied by every group) and each group's first block are in
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldsm_x4(tile_addr(sq, wq * 16 + (lane & 15), kk * 2 + (lane >> 4)), qa[kk][0], qa[kk][1], qa[kk][2],
                qa[kk][3]);
    } else {
      va_group_sync<KG>(grp);  // ... and those of the group's other threads
    }
    const __nv_bfloat16* sk = skv + 2 * st * kVaTile;
    const __nv_bfloat16* sv = sk + kVaTile;
    // S = Q K^T: n-tile j holds keys 8j..8j+7 of the block
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(tile_addr(sk, jp * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * jp], qa[kk], b0, b1);
        mma_bf16_16816(s[2 * jp + 1], qa[kk], b2, b3);
      }
    }
    // online softmax over rows g (s[.][0..1]) and g + 8 (s[.][2..3])
    float bm0 = -1e30f, bm1 = -1e30f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bm0 = fmaxf(bm0, fmaxf(s[j][0], s[j][1]));
      bm1 = fmaxf(bm1, fmaxf(s[j][2], s[j][3]));
    }
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
    const float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
    const float cr0 = exp2f((m0 - nm0) * scale_log2), cr1 = exp2f((m1 - nm1) * scale_log2);
    m0 = nm0;
    m1 = nm1;
    const float o0 = nm0 * scale_log2, o1 = nm1 * scale_log2;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(__fmaf_rn(s[j][0], scale_log2, -o0));
      s[j][1] = exp2f(__fmaf_rn(s[j][1], scale_log2, -o0));
      s[j][2] = exp2f(__fmaf_rn(s[j][2], scale_log2, -o1));
      s[j][3] = exp2f(__fmaf_rn(s[j][3], scale_log2, -o1));
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * cr0 + rs0;
    l1 = l1 * cr1 + rs1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= cr0;
      o[j][1] *= cr0;
      o[j][2] *= cr1;
      o[j][3] *= cr1;
    }
    // O += P V, P (bf16) straight from the score accumulators
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jd = 0; jd < 8; jd += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(tile_addr(sv, kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, jd + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16_16816(o[jd], pa, b0, b1);
        mma_bf16_16816(o[jd + 1], pa, b2, b3);
      }
    }
    va_group_sync<KG>(grp);  // the group's warps are done with this stage before it is refilled
  }
  if constexpr (KG > 1) {
    // groups 1.. leave their partial state in their own (now idle) ring; group 0 merges
    float* ex = reinterpret_cast<float*>(skv) + (wq * 32 + lane) * kVaExFloats;
    if (grp > 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(ex + 4 * j) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
      *reinterpret_cast<float4*>(ex + 32) = make_float4(m0, m1, l0, l1);
    }
    __syncthreads();
    if (grp > 0) return;
#pragma unroll
    for (int q = 1; q < KG; ++q) {
      const float* ey = reinterpret_cast<const float*>(sq + kVaTile + q * kVaGroupTiles * kVaTile) +
                        (wq * 32 + lane) * kVaExFloats;
      const float4 ml = *reinterpret_cast<const float4*>(ey + 32);
      const float nm0 = fmaxf(m0, ml.x), nm1 = fmaxf(m1, ml.y);
      const float a0 = exp2f((m0 - nm0) * scale_log2), b0 = exp2f((ml.x - nm0) * scale_log2);
      const float a1 = exp2f((m1 - nm1) * scale_log2), b1 = exp2f((ml.y - nm1) * scale_log2);
      m0 = nm0;
      m1 = nm1;
      l0 = l0 * a0 + ml.z * b0;
      l1 = l1 * a1 + ml.w * b1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 y = *reinterpret_cast<const float4*>(ey + 4 * j);
        o[j][0] = o[j][0] * a0 + y.x * b0;
        o[j][1] = o[j][1] * a0 + y.y * b0;
        o[j][2] = o[j][2] * a1 + y.z * b1;
        o[j][3] = o[j][3] * a1 + y.w * b1;
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  const long long r0 = row0 + qb * 64 + wq * 16 + g;
  __nv_bfloat16* o_row0 = out + r0 * OASIS_HIDDEN + h * 64;
  __nv_bfloat16* o_row1 = o_row0 + 8 * OASIS_HIDDEN;
#pragma unroll
  for (int jd = 0; jd < 8; ++jd) {
    *reinterpret_cast<uint32_t*>(o_row0 + jd * 8 + 2 * c) = pack_bf16x2(o[jd][0] * inv0, o[jd][1] * inv0);
    *reinterpret_cast<uint32_t*>(o_row1 + jd * 8 + 2 * c) = pack_bf16x2(o[jd][2] * inv1, o[jd][3] * inv1);
  }
}

// workspace layout of a decode of F frames (M = 576 F token rows)
struct VaeLayout {
  size_t zin, resid, hbuf, qkv, attn, mlp, pred, cnt, total;
  size_t cnt_words;   // LayerNorm-tail tile counters: 2 launches per block x ceil(M / 128)
  size_t flag_words;  // split-K order counters of one residual launch (<= 16 N tiles x 8 warps)
};
VaeLayout vae_layout(int F, int depth) {
  const size_t M = static_cast<size_t>(F) * kVaeTokens;
  VaeLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = vae_align256(off + bytes);
    return o;
  };
  L.zin = take(M * 64 * 2);
  L.resid = take(M * OASIS_HIDDEN * 4);
  L.hbuf = take(M * OASIS_HIDDEN * 2);
  L.qkv = take(M * 3 * OASIS_HIDDEN * 2);
  L.attn = take(M * OASIS_HIDDEN * 2);
  L.mlp = take(M * OASIS_MLP_HIDDEN * 2);
  L.pred = take(M * OASIS_VAE_PRED_LD * 4);
  L.cnt_words = static_cast<size_t>(2 * depth) * ((M + 127) / 128);
  L.flag_words = ((M + 127) / 128) * (OASIS_HIDDEN / 64) * kEpiWarps;
  // zeroed together per decode: the tile counters, then the split-K counters of every
  // residual launch (out-proj and fc2 of each block)
  L.cnt = take((L.cnt_words + static_cast<size_t>(2 * depth) * L.flag_words) * 4);
  L.total = off;
  return L;
}

}  // namespace
}  // namespace oasis

struct oasis_vae_plan {
  oasis_vae_weights_t w;
  int frames = 0, M = 0;
  uint8_t* ws = nullptr;
  oasis::VaeLayout L{};
  oasis::GemmOperands post, pred;
  oasis::GemmOperands qkv[OASIS_VAE_MAX_DEPTH], proj[OASIS_VAE_MAX_DEPTH], fc1[OASIS_VAE_MAX_DEPTH],
      fc2[OASIS_VAE_MAX_DEPTH];
};

namespace oasis {
namespace {

// A projection over the M token rows: tile shape from choose_tiles; the residual GEMMs
// (out-proj, fc2) may split K, their splits' reduce-adds ordered by counters.
int vae_proj(GemmOperands* g, const void* A, long long lda, const void* B, int M, int N, int K,
             bool residual = false) {
  int bn = 256, ctas = 1, splits = 1;
  choose_tiles(M, N, K, residual, &bn, &ctas, &splits);
  if (int st = make_gemm_operands(g, A, lda, B, K, M, N, K, bn, ctas)) return st;
  g->splits = splits;
  if (split_flag_count(*g) > vae_layout(M / kVaeTokens, 1).flag_words)
    return fail(OASIS_ERR_UNSUPPORTED, "oasis_vae_plan_create: split-K counters exceed their region");
  return OASIS_OK;
}

int vae_plan_init(oasis_vae_plan* p, const oasis_vae_weights_t* w, int frames, void* workspace, size_t ws_bytes) {
  if (!w || !workspace) return fail(OASIS_ERR_INVALID_ARG, "oasis_vae_plan_create: null argument");
  if (frames <= 0 || frames > 4096) return fail(OASIS_ERR_INVALID_ARG, "oasis_vae_plan_create: need 1 <= frames <= 4096");
  if (w->depth <= 0 || w->depth > OASIS_VAE_MAX_DEPTH)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_vae_plan_create: depth must be 1..12");
  const VaeLayout L = vae_layout(frames, w->depth);
  if (ws_bytes < L.total)
    return fail(OASIS_ERR_WORKSPACE, "oasis_vae_plan_create: workspace smaller than oasis_vae_workspace_size()");
  if (!aligned16(workspace)) return fail(OASIS_ERR_ALIGNMENT, "oasis_vae_plan_create: workspace alignment");
  p->w = *w;
  p->frames = frames;
  p->M = frames * kVaeTokens;
  p->ws = static_cast<uint8_t*>(workspace);
  p->L = L;
  const int M = p->M;
  uint8_t* ws = p->ws;
  int st = vae_proj(&p->post, ws + L.zin, 64, w->post_w, M, OASIS_HIDDEN, 64);
  if (!st) st = set_gemm_output(&p->post, ws + L.resid, OASIS_HIDDEN, true);
  for (int i = 0; i < w->depth && !st; ++i) {
    const oasis_vae_block_t& b = w->blk[i];
    st = vae_proj(&p->qkv[i], ws + L.hbuf, OASIS_HIDDEN, b.qkv_w, M, 3 * OASIS_HIDDEN, OASIS_HIDDEN);
    if (!st) st = set_gemm_output(&p->qkv[i], ws + L.qkv, 3 * OASIS_HIDDEN, false);
    if (!st) st = vae_proj(&p->proj[i], ws + L.attn, OASIS_HIDDEN, b.proj_w, M, OASIS_HIDDEN, OASIS_HIDDEN, true);
    if (!st) st = set_gemm_output(&p->proj[i], ws + L.resid, OASIS_HIDDEN, true);
    if (!st) st = vae_proj(&p->fc1[i], ws + L.hbuf, OASIS_HIDDEN, b.fc1_w, M, OASIS_MLP_HIDDEN, OASIS_HIDDEN);
    if (!st) st = set_gemm_output(&p->fc1[i], ws + L.mlp, OASIS_MLP_HIDDEN, false);
    if (!st) st = vae_proj(&p->fc2[i], ws + L.mlp, OASIS_MLP_HIDDEN, b.fc2_w, M, OASIS_HIDDEN, OASIS_MLP_HIDDEN, true);
    if (!st) st = set_gemm_output(&p->fc2[i], ws + L.resid, OASIS_HIDDEN, true);
  }
  if (!st) st = vae_proj(&p->pred, ws + L.hbuf, OASIS_HIDDEN, w->pred_w, M, OASIS_VAE_PRED_LD, OASIS_HIDDEN);
  if (!st) st = set_gemm_output(&p->pred, ws + L.pred, OASIS_VAE_PRED_LD, true);
  if (!st)
    for (GemmOperands* g : {&p->post, &p->pred}) g->b_is_weight = true;
  for (int i = 0; i < w->depth && !st; ++i)
    p->qkv[i].b_is_weight = p->proj[i].b_is_weight = p->fc1[i].b_is_weight = p->fc2[i].b_is_weight = true;
  return st;
}

int vae_run(oasis_vae_plan* p, const float* z, float* out, cudaStream_t s) {
  const oasis_vae_weights_t& w = p->w;
  const VaeLayout& L = p->L;
  const int M = p->M;
  uint8_t* ws = p->ws;
  float* resid = reinterpret_cast<float*>(ws + L.resid);
  auto* hbuf = reinterpret_cast<__nv_bfloat16*>(ws + L.hbuf);
  auto* cnt = reinterpret_cast<unsigned int*>(ws + L.cnt);
  const size_t nblk = (static_cast<size_t>(M) + 127) / 128;
  unsigned int* flags = cnt + L.cnt_words;
  cudaError_t ce = cudaMemsetAsync(cnt, 0, (L.cnt_words + static_cast<size_t>(2 * w.depth) * L.flag_words) * 4, s);
  if (ce != cudaSuccess) return cuda_status(ce, "cudaMemsetAsync(vae counters)");

  // latent projection into the fp32 residual, then the first LayerNorm (affine as
  // (1 + scale) x + shift with the same row for every frame)
  {
    const int chunks = M * 8;
    cudaError_t e = launch_pdl(vae_latent_prep_kernel, dim3((chunks + 255) / 256), dim3(256), 0, s, z,
                               reinterpret_cast<__nv_bfloat16*>(ws + L.zin), M);
    if (e != cudaSuccess) return cuda_status(e, "vae_latent_prep_kernel");
    EpiParams ep{};
    ep.out = resid;
    ep.ldd = OASIS_HIDDEN;
    ep.bias = w.post_b;
    if (int r = launch_gemm(p->post, kEpiStoreF32Bias, ep, s)) return r;
    if (int r = launch_ln_modulate(resid, w.blk[0].ln1_shift, w.blk[0].ln1_scale, 0, hbuf, M, kVaeTokens, s))
      return r;
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_vae_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, va_smem(1));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_vae_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, va_smem(3));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attn_vae)");
    configured = true;
  }
  for (int i = 0; i < w.depth; ++i) {
    const oasis_vae_block_t& b = w.blk[i];
    EpiParams eq{};  // q | k | v, RoPE on q and k at the token's grid position
    eq.out = ws + L.qkv;
    eq.ldd = 3 * OASIS_HIDDEN;
    eq.rope = w.rope;
    eq.rope_cols = 2 * OASIS_HIDDEN;
    eq.rope_div = 1;
    eq.rope_mod = kVaeTokens;
    eq.rope_add = 0;
    if (int r = launch_gemm(p->qkv[i], kEpiQkvRope, eq, s)) return r;
    // one frame (144 CTAs, one per SM): three key groups per CTA; from two frames on the
    // 120 KB CTAs would take two waves, and single-group CTAs (4 per SM) fill the SMs
    const bool split_keys = p->frames == 1;
    const dim3 grid(kVaBlocks, OASIS_HEADS, p->frames);
    const auto* q_in = reinterpret_cast<const __nv_bfloat16*>(ws + L.qkv);
    auto* a_out = reinterpret_cast<__nv_bfloat16*>(ws + L.attn);
    cudaError_t e = split_keys
                        ? launch_pdl(attn_vae_kernel<3>, grid, dim3(3 * 128), va_smem(3), s, q_in, a_out,
                                     0.125f * 1.4426950408889634f)
                        : launch_pdl(attn_vae_kernel<1>, grid, dim3(128), va_smem(1), s, q_in, a_out,
                                     0.125f * 1.4426950408889634f);
    if (e != cudaSuccess) return cuda_status(e, "attn_vae_kernel");
    EpiParams eo{};  // x += proj(attn) + b, then LayerNorm 2 into hbuf
    eo.out = resid;
    eo.ldd = OASIS_HIDDEN;
    eo.bias = b.proj_b;
    eo.gate = w.ones;
    eo.gate_ld = 0;
    eo.ln_out = hbuf;
    eo.ln_shift = b.ln2_shift;
    eo.ln_scale = b.ln2_scale;
    eo.ln_mod_ld = 0;
    eo.ln_count = cnt + (2 * static_cast<size_t>(i)) * nblk;
    eo.split_flags = flags + (2 * static_cast<size_t>(i)) * L.flag_words;
    if (int r = launch_gemm(p->proj[i], kEpiGateResid, eo, s)) return r;
    EpiParams e1{};
    e1.out = ws + L.mlp;
    e1.ldd = OASIS_MLP_HIDDEN;
    e1.bias = b.fc1_b;
    if (int r = launch_gemm(p->fc1[i], kEpiBiasGelu, e1, s)) return r;
    EpiParams e2{};  // x += fc2(h) + b, then the next block's LayerNorm 1 (or the final one)
    e2.out = resid;
    e2.ldd = OASIS_HIDDEN;
    e2.bias = b.fc2_b;
    e2.gate = w.ones;
    e2.gate_ld = 0;
    e2.ln_out = hbuf;
    const bool last = i + 1 == w.depth;
    e2.ln_shift = last ? w.norm_shift : w.blk[i + 1].ln1_shift;
    e2.ln_scale = last ? w.norm_scale : w.blk[i + 1].ln1_scale;
    e2.ln_mod_ld = 0;
    e2.ln_count = cnt + (2 * static_cast<size_t>(i) + 1) * nblk;
    e2.split_flags = flags + (2 * static_cast<size_t>(i) + 1) * L.flag_words;
    if (int r = launch_gemm(p->fc2[i], kEpiGateResid, e2, s)) return r;
  }
  EpiParams ep{};
  ep.out = ws + L.pred;
  ep.ldd = OASIS_VAE_PRED_LD;
  ep.bias = w.pred_b;
  if (int r = launch_gemm(p->pred, kEpiStoreF32Bias, ep, s)) return r;
  const long long px = static_cast<long long>(p->frames) * 3 * kVaeImgH * kVaeImgW;
  cudaError_t e = launch_pdl(vae_unpatchify_kernel, dim3(static_cast<unsigned>((px + 255) / 256)), dim3(256), 0, s,
                             reinterpret_cast<const float*>(ws + L.pred), OASIS_VAE_PRED_LD, out, p->frames);
  if (e != cudaSuccess) return cuda_status(e, "vae_unpatchify_kernel");
  return OASIS_OK;
}

}  // namespace
}  // namespace oasis

extern "C" size_t oasis_vae_workspace_size(int frames, int depth) {
  if (frames <= 0 || depth <= 0 || depth > OASIS_VAE_MAX_DEPTH) return 0;
  return oasis::vae_layout(frames, depth).total;
}

extern "C" int oasis_vae_plan_create(const oasis_vae_weights_t* w, int frames, void* workspace,
                                     size_t workspace_bytes, oasis_vae_plan_t** out) {
  using namespace oasis;
  if (!out) return fail(OASIS_ERR_INVALID_ARG, "oasis_vae_plan_create: null argument");
  *out = nullptr;
  oasis_vae_plan* p = new oasis_vae_plan();
  if (int st = vae_plan_init(p, w, frames, workspace, workspace_bytes)) {
    delete p;
    return st;
  }
  *out = p;
  return OASIS_OK;
}

extern "C" void oasis_vae_plan_destroy(oasis_vae_plan_t* plan) { delete plan; }

extern "C" int oasis_vae_decode(oasis_vae_plan_t* plan, const float* z, float* out, cudaStream_t stream) {
  using namespace oasis;
  if (!plan || !z || !out) return fail(OASIS_ERR_INVALID_ARG, "oasis_vae_decode: null argument");
  if (!aligned16(z) || !aligned16(out)) return fail(OASIS_ERR_ALIGNMENT, "oasis_vae_decode: alignment");
  return vae_run(plan, z, out, stream);
}
