/*
 * oasis_b200.h — C ABI of the B200-native Oasis-500M DiT denoising forward.
 *
 * One shared library (liboasis_b200.so, sm_100a) exports everything below.
 * Conventions for every entry point:
 *   - plain pointers and sizes; all buffers are DEVICE memory owned by the
 *     caller unless a parameter says "host";
 *   - work is enqueued on the given stream; nothing synchronises, allocates or
 *     frees device memory inside a call (all scratch comes from a caller-owned
 *     workspace), so the calls can be captured into CUDA graphs;
 *   - the return value is a status (OASIS_OK == 0); on failure
 *     oasis_last_error() returns a message for the calling host thread.  No
 *     call aborts the process and there is no CPU fallback.
 *
 * The reference ("worldserve") has no C ABI for this path: its operators are
 * Python monkey-patches over torch modules.  Each entry point names the
 * reference interface it replaces.
 */
#ifndef OASIS_B200_H
#define OASIS_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define OASIS_OK                 0
#define OASIS_ERR_INVALID_ARG    1  /* null pointer, bad size or shape          */
#define OASIS_ERR_ALIGNMENT      2  /* pointer/stride not 16-byte aligned       */
#define OASIS_ERR_WORKSPACE      3  /* workspace missing or too small           */
#define OASIS_ERR_CUDA           4  /* a CUDA runtime/driver call failed        */
#define OASIS_ERR_DEVICE_TIMEOUT 5  /* a bounded device-side wait gave up       */
#define OASIS_ERR_UNSUPPORTED    6  /* shape outside what the kernels support   */

/* Model geometry (Oasis-500M, open-oasis DiT-S/2). */
#define OASIS_HIDDEN      1024
#define OASIS_HEADS       16
#define OASIS_HEAD_DIM    64
#define OASIS_MLP_HIDDEN  4096
#define OASIS_TOKENS      144   /* 9 x 16 patches per frame */
#define OASIS_LATENT_C    16
#define OASIS_LATENT_H    18
#define OASIS_LATENT_W    32
#define OASIS_ACTION_DIM  25
#define OASIS_MAX_DEPTH   16
#define OASIS_MAX_FRAMES  32    /* sliding window */
#define OASIS_ADA_PER_SUB (6 * OASIS_HIDDEN)

/* Message describing the last failure on this host thread ("" if none). */
const char* oasis_last_error(void);
/* Library version string. */
const char* oasis_version(void);
/* Reads and clears the device-side error word set by bounded waits (synchronises
 * the device).  Returns OASIS_ERR_DEVICE_TIMEOUT if any kernel gave up a wait. */
int oasis_check_device_error(void);
/* Self-test of that failure path: launches one thread that waits, through the same
 * bounded wait the chained GEMM and the LayerNorm tails use, for a device word that
 * nothing ever sets.  After the 2 s limit the wait records a timeout in the device error
 * word and the kernel returns normally, so oasis_check_device_error then reports
 * OASIS_ERR_DEVICE_TIMEOUT (and clears it) while the context stays usable.  No
 * counterpart in the reference, whose waits are all on the host. */
int oasis_selftest_bounded_wait(cudaStream_t stream);

/* ------------------------------------------------------------------ weights */
/* One attention+MLP sub-block (spatial or temporal).  Linear weights are bf16
 * row-major [out][in] exactly as nn.Linear stores them; biases fp32. */
typedef struct {
  const void*  qkv_w;  /* bf16 [3072][1024], no bias (to_qkv)              */
  const void*  out_w;  /* bf16 [1024][1024]                                 */
  const float* out_b;  /* fp32 [1024]                                       */
  const void*  fc1_w;  /* bf16 [4096][1024]                                 */
  const float* fc1_b;  /* fp32 [4096]                                       */
  const void*  fc2_w;  /* bf16 [1024][4096]                                 */
  const float* fc2_b;  /* fp32 [1024]                                       */
} oasis_sub_weights_t;

typedef struct {
  int depth;                 /* number of SpatioTemporal blocks (16)            */
  const void*  patch_w;      /* bf16 [1024][64]: Conv2d(16,1024,2,2) weight as
                                [out][c*4 + pi*2 + qi]                          */
  const float* patch_b;      /* fp32 [1024]                                     */
  const void*  t_fc1_w;      /* bf16 [1024][256] timestep MLP first linear      */
  const float* t_fc1_b;      /* fp32 [1024]                                     */
  /* timestep MLP second linear with the external_cond (action) linear appended
   * along K: columns 0..1023 = t_embedder.mlp.2.weight, 1024..1048 =
   * external_cond.weight, 1049 = external_cond.bias (multiplied by an input of 1
   * when actions are given, 0 otherwise), 1050..1087 = 0; bias = mlp.2.bias     */
  const void*  t_fc2_w;      /* bf16 [1024][1088]                               */
  const float* t_fc2_b;      /* fp32 [1024]                                     */
  /* All adaLN modulation linears stacked row-wise: sub-block j = 2*i (spatial)
   * or 2*i+1 (temporal) owns rows [j*6144, (j+1)*6144) in chunk order
   * shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp; the final
   * layer's (shift, scale) follow at rows [2*depth*6144, +2048). */
  const void*  ada_w;        /* bf16 [2*depth*6144 + 2048][1024]                */
  const float* ada_b;        /* fp32 [2*depth*6144 + 2048]                      */
  const void*  final_w;      /* bf16 [64][1024]                                 */
  const float* final_b;      /* fp32 [64]                                       */
  oasis_sub_weights_t sub[2 * OASIS_MAX_DEPTH]; /* [2i] spatial, [2i+1] temporal */
  /* RoPE tables (cos, sin) interleaved per rotated pair, fp32:
   *   spatial  [144][32][2]  (pairs 0..15 from the H axis, 16..31 from W)
   *   temporal [OASIS_MAX_FRAMES][32][2]                                       */
  const float* rope_spatial;
  const float* rope_temporal;
} oasis_dit_weights_t;

/* ------------------------------------------------------------------ KV cache */
/* Storage kinds of a temporal-attention KV frame slot. */
#define OASIS_KV_BF16 0
#define OASIS_KV_FP8  1   /* e4m3fn codes + one bf16 scale per (frame, head)   */
#define OASIS_KV_INT4 2   /* packed nibbles (element 2i high) + fp16 scale/zero
                             per (token, head) group of 64                      */

/* Bits of the `tensors` argument of oasis_kv_migrate. */
#define OASIS_KV_KEYS   1
#define OASIS_KV_VALUES 2

/* One tensor (the keys or the values) of a temporal KV cache.  Logical slot s
 * (0 <= s < n_slots of the cache; 0 = oldest frame) is stored in the pool of kind
 * slot_kind[s], at frame index slot_index[s] of that pool (shared by all sessions and
 * layers).  Keys and values carry separate maps and pools, so each sits in its own
 * precision tier, as ProgressiveKVQuantizer ages them on separate thresholds
 * (worldserve/optimizations/system_level/kv_cache/progressive_quant.py:92-98,310-322).
 * Pools (row-major, leading dims first):
 *   bf16: bf16       [batch][layers][n_bf16][144][1024] bf16
 *   fp8 : fp8        [batch][layers][n_fp8][144][1024] e4m3fn codes
 *         fp8_scale  [batch][layers][n_fp8][16] bf16
 *   int4: int4       [batch][layers][n_int4][144][16][32] packed codes
 *         i4_scale, i4_zero  [batch][layers][n_int4][144][16] fp16
 * Unused pools may be NULL with count 0.  Every pool base must be 16-byte aligned. */
typedef struct {
  int n_bf16, n_fp8, n_int4;
  uint8_t slot_kind[OASIS_MAX_FRAMES];
  uint8_t slot_index[OASIS_MAX_FRAMES];
  void* bf16;
  uint8_t* fp8; void* fp8_scale;
  uint8_t* int4; void* i4_scale; void* i4_zero;
} oasis_kv_tensor_t;

/* Post-RoPE temporal K/V of past frames, for `batch` sessions x `layers` blocks and
 * `n_slots` frames (slot 0 = oldest). */
typedef struct {
  int batch, layers, n_slots;
  oasis_kv_tensor_t k, v;
} oasis_kv_cache_t;

/* ------------------------------------------------------------------ forward plan */
typedef struct oasis_plan oasis_plan_t;

/* Bytes of workspace a plan for `batch` sessions x `frames` input frames needs. */
size_t oasis_plan_workspace_size(int batch, int frames, int depth);

/* Builds a forward plan (TMA descriptors, launch shapes) for inputs of
 * `batch` sessions x `frames` frames.  `w` and `workspace` must outlive the plan.
 * Replaces: the open-oasis `dit(x, t, external_cond)` module call made by
 * worldserve/models/oasis.py:216 and benchmarks/optimised/oasis_dpmpp_modal.py:141. */
int oasis_plan_create(const oasis_dit_weights_t* w, int batch, int frames,
                      void* workspace, size_t workspace_bytes, oasis_plan_t** out);
void oasis_plan_destroy(oasis_plan_t* plan);

/* Full-window forward: x fp32 [B][T][16][18][32], t int64 [B][T], act fp32
 * [B][T][25] (may be NULL: no external conditioning) -> v fp32 [B][T][16][18][32].
 * If `cache` is non-NULL, the post-RoPE temporal K/V of window frames
 * 0..T-2 are also stored into cache slots 0..T-2, keys and values each in its slot's kind (FP8/INT4
 * quantised exactly like ProgressiveKVQuantizer.quantize_to_fp8 / quantize_to_int4,
 * worldserve/optimizations/system_level/kv_cache/progressive_quant.py:113-193,
 * at the granularity above).  Replaces DiT.forward plus the KV capture of
 * KVCacheManager.wire_to_model (kv_cache/manager.py:923-1138). */
int oasis_dit_forward(oasis_plan_t* plan, const float* x, const int64_t* t, const float* act,
                      float* v, const oasis_kv_cache_t* cache, cudaStream_t stream);

/* Incremental forward of the newest frame (plan built with frames == 1):
 * x fp32 [B][16][18][32], t [B], act [B][25] -> v [B][16][18][32], with temporal
 * attention over cache slots 0..n_past-1 (dequantised inside the attention
 * K/V loads) plus the frame's own K/V at window position n_past.  Replaces the
 * persistent past-frame reuse of PersistentTemporalAxialAttention
 * (kv_cache/oasis_temporal_persistent_wrapper.py:116-150) and
 * KVCacheManager.get_kv_for_attention (kv_cache/manager.py:416-480). */
int oasis_dit_forward_cached(oasis_plan_t* plan, const float* x, const int64_t* t,
                             const float* act, float* v, const oasis_kv_cache_t* cache,
                             int n_past, cudaStream_t stream);

/* Per-kernel-family device time of the forwards run since the last reset
 * (CUDA events on the plan's stream; only while enabled).  A forward captured into a
 * CUDA graph while enabled records its events as graph nodes: the times then come
 * from the last replay of that graph.  families: 0 GEMM
 * projections, 1 adaLN GEMM, 2 spatial attention, 3 temporal attention,
 * 4 LayerNorm/modulate, 5 embeddings+final, 6 KV quantise. */
int oasis_plan_set_timing(oasis_plan_t* plan, int enable);
int oasis_plan_get_timing(oasis_plan_t* plan, float* ms_per_family, int* launches_per_family,
                          int n_families);

/* Full-window forward (same arguments and results as oasis_dit_forward without a
 * cache) for callers that cannot allocate device memory: it takes only the weights,
 * inputs and outputs, and uses as scratch a fixed 17 MiB file-scope device array of
 * this library, which every GPU that loads the library holds until the process exits.
 * Limit: batch * frames <= OASIS_NOALLOC_MAX_FRAMES; larger shapes are rejected with
 * OASIS_ERR_UNSUPPORTED.  Each call looks up that array's device address on the current
 * device (cudaGetSymbolAddress; after a device reset it may have moved, and the cached
 * launch descriptors are rebuilt); the first call on a device also sets up those
 * descriptors, so make that first call before any stream capture.
 * Calls share the one array: calls that overlap on the GPU (other streams, other host
 * threads) race.  No scratch byte has to start at zero: every byte the forward reads
 * is written earlier in the same call.  No counterpart in the reference (it has no
 * C ABI and allocates through PyTorch). */
#define OASIS_NOALLOC_MAX_FRAMES 4
int oasis_dit_forward_noalloc(const oasis_dit_weights_t* w, int batch, int frames,
                              const float* x, const int64_t* t, const float* act, float* v,
                              cudaStream_t stream);

/* ------------------------------------------------------------------ operators */
/* D[m][n] = sum_k A[m][k] * B[n][k] on tcgen05 tensor cores (bf16 in, fp32
 * accumulate).  epilogue: 0 store bf16 D; 1 store fp32 D + bias[n] (bias may be
 * NULL).  A, B, D row-major with leading dims lda/ldb/ldd (elements); K % 64 == 0,
 * N % 16 == 0.  Replaces nn.Linear -> cuBLAS on the DiT projections. */
int oasis_gemm_bf16(const void* A, const void* B, void* D, const float* bias,
                    int M, int N, int K, int lda, int ldb, int ldd, int epilogue,
                    cudaStream_t stream);

/* Spatial attention over the 144 tokens of each frame: qkv bf16
 * [frames*144][3072] (q | k | v, post-RoPE, head h at columns h*64) -> out bf16
 * [frames*144][1024], non-causal, scale 1/8.  Replaces the SDPA of open-oasis
 * SpatialAxialAttention (its Triton replacement:
 * worldserve/optimizations/system_level/pipeline/triton_kernels.py:91-191). */
int oasis_attn_spatial(const void* qkv, void* out, int frames, cudaStream_t stream);

/* Causal temporal attention over `n_kv` frames for every (session, token, head).
 * Queries: q_frames frames per session at window positions q_pos0.. from
 * qkv bf16 [batch*q_frames*144][3072] (q | k | v, post-RoPE).  Keys/values:
 * positions 0..n_past-1 from `cache` (NULL if n_past == 0), positions
 * n_past..n_kv-1 from the k|v columns of qkv (frame j of the session at
 * position n_past + j).  out bf16 [batch*q_frames*144][1024].  Replaces the
 * causal SDPA of TemporalAxialAttention
 * (kv_cache/oasis_temporal_persistent_wrapper.py:139-150) and the split-attention
 * over precision groups (progressive_quant.py:497-575). */
int oasis_attn_temporal(const void* qkv, const oasis_kv_cache_t* cache, int layer,
                        void* out, int batch, int q_frames, int q_pos0, int n_past,
                        int n_kv, cudaStream_t stream);

/* Quantise K/V of `frames` frames per session into cache slots
 * slot0..slot0+frames-1 (keys and values each in its slot kind) for one layer, from
 * kv bf16 [batch*frames*144][ld] where K is at column k_col and V at v_col.
 * Replaces ProgressiveKVQuantizer.quantize_to_fp8 / quantize_to_int4 applied
 * per frame-head slice / per token-head group (progressive_quant.py:113-193). */
int oasis_kv_store(const void* kv, int ld, int k_col, int v_col, const oasis_kv_cache_t* cache,
                   int layer, int batch, int frames, int slot0, cudaStream_t stream);

/* Dequantise cache slots back to bf16 [batch][frames][144][1024] (K then V
 * buffers).  Replaces ProgressiveKVQuantizer.dequantize_fp8 / dequantize_int4
 * (progressive_quant.py:195-257); used by KV-manager retrieval calls. */
int oasis_kv_load(const oasis_kv_cache_t* cache, int layer, int slot0, int frames,
                  void* k_out, void* v_out, cudaStream_t stream);
/* Age promotion of one frame of a temporal KV cache (replaces the per-entry
 * _promote_to_fp8 / _promote_to_int4 steps of ProgressiveKVQuantizer.update_cache,
 * worldserve/optimizations/system_level/kv_cache/progressive_quant.py:263-350):
 * re-quantises logical slot src_slot into logical slot dst_slot, for every session and
 * layer, of the keys (tensors & OASIS_KV_KEYS) and/or the values (OASIS_KV_VALUES),
 * each through its own slot map.  Allowed per tensor: bf16 -> FP8, bf16 -> INT4,
 * FP8 -> INT4 (an FP8 entry is dequantised to fp16 first, as the reference does).  The
 * two slots of a tensor must map to different storage. */
int oasis_kv_migrate(const oasis_kv_cache_t* cache, int tensors, int src_slot, int dst_slot,
                     cudaStream_t stream);

/* DPM-Solver++ 2M v-prediction update of the newest frame of each session
 * (benchmarks/optimised/oasis_dpmpp_modal.py:143-164):
 *   x0 = sqrt(ab_t) x - sqrt(1-ab_t) v;  eps = sqrt(1-ab_t) x + sqrt(ab_t) v
 *   D  = first ? eps : (3 eps - eps_prev) / 2;  x <- sqrt(ab_next) x0 + sqrt(1-ab_next) D
 *   eps_prev <- eps
 * x/v fp32 with `n` elements per session at session strides x_stride/v_stride;
 * eps_prev fp32 [batch][n].  With first == 1 and eps_prev == NULL this is the
 * DDIM v-step of worldserve/models/oasis.py:218-228 (ab_next = alpha-bar of t_prev). */
int oasis_dpmpp2m_update(float* x, const float* v, float* eps_prev, int batch, int n,
                         long long x_stride, long long v_stride, float ab_t, float ab_next,
                         int first, cudaStream_t stream);

/* DPMSolverPPSampler.step (optimizations/model_level/samplers/dpm_solver_pp.py:85-143):
 *   out = x + h * (c0*d0 + c1*d1 + c2*d2) over n fp32 elements (d1/d2 may be NULL
 *   when their coefficient is 0).  Euler: (1,0,0); AB2: (1.5,-0.5,0);
 *   AB3: (23/12,-4/3,5/12). */
int oasis_ab_update(const float* x, const float* d0, const float* d1, const float* d2,
                    float* out, long long n, float h, float c0, float c1, float c2,
                    cudaStream_t stream);

/* ------------------------------------------------------------------ VAE decode */
/* The latent decoder behind `vae.decode(z)` of the Oasis rollout
 * (worldserve/models/oasis.py:237-245): z (frames, 576, 16) fp32 latents (already divided
 * by the VAE scale) -> RGB (frames, 3, 360, 640) fp32 in [-1, 1].  The decoder is a ViT of
 * width 1024 (16 heads x 64) over the 18 x 32 token grid, patch 20: Linear(16 -> 1024),
 * `depth` pre-norm blocks (affine LayerNorm eps 1e-6; bias-free QKV with axial RoPE;
 * non-causal attention; output projection; MLP 1024 -> 4096 -> 1024, GELU(tanh)), a final
 * affine LayerNorm and Linear(1024 -> 20*20*3) unpatchified to pixels (upstream open-oasis
 * vae.py is not in the reference tree; these are the restated choices). */
#define OASIS_VAE_MAX_DEPTH 12
#define OASIS_VAE_PRED_LD 1216 /* predictor rows: 1200 padded to a multiple of 64       */

typedef struct {
  /* LayerNorms as (1 + scale) * x_hat + shift: shift = bias, scale = weight - 1      */
  const float* ln1_shift; const float* ln1_scale;   /* fp32 [1024] each                */
  const void*  qkv_w;     /* bf16 [3072][1024] (no bias)                             */
  const void*  proj_w;    /* bf16 [1024][1024]                                       */
  const float* proj_b;    /* fp32 [1024]                                             */
  const float* ln2_shift; const float* ln2_scale;
  const void*  fc1_w;     /* bf16 [4096][1024]                                       */
  const float* fc1_b;     /* fp32 [4096]                                             */
  const void*  fc2_w;     /* bf16 [1024][4096]                                       */
  const float* fc2_b;     /* fp32 [1024]                                             */
} oasis_vae_block_t;

typedef struct {
  int depth;              /* decoder blocks (12)                                     */
  const void*  post_w;    /* bf16 [1024][64]: Linear(16 -> 1024) weight, K zero-padded */
  const float* post_b;    /* fp32 [1024]                                             */
  oasis_vae_block_t blk[OASIS_VAE_MAX_DEPTH];
  const float* norm_shift; const float* norm_scale; /* final LayerNorm              */
  const void*  pred_w;    /* bf16 [1216][1024]: Linear(1024 -> 1200), rows 1200.. zero;
                             output column (p*20 + q)*3 + c                          */
  const float* pred_b;    /* fp32 [1216]                                             */
  const float* rope;      /* fp32 [576][32][2] (cos, sin): pairs 0..15 H axis, 16..31 W */
  const float* ones;      /* fp32 [1024] of 1.0 (the residual gate of the epilogue)  */
} oasis_vae_weights_t;

typedef struct oasis_vae_plan oasis_vae_plan_t;

/* Workspace bytes of a decode of `frames` frames (0 on invalid arguments). */
size_t oasis_vae_workspace_size(int frames, int depth);
/* Plan for `frames` frames over caller-owned weights and workspace (encodes tensor maps
 * on the host; allocates no device memory). */
int oasis_vae_plan_create(const oasis_vae_weights_t* w, int frames, void* workspace,
                          size_t workspace_bytes, oasis_vae_plan_t** out);
void oasis_vae_plan_destroy(oasis_vae_plan_t* plan);
/* Decode: z fp32 [frames][576][16] -> out fp32 [frames][3][360][640] (16-byte aligned).
 * Enqueues on `stream`, allocates nothing; one decode per plan at a time. */
int oasis_vae_decode(oasis_vae_plan_t* plan, const float* z, float* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* OASIS_B200_H */
