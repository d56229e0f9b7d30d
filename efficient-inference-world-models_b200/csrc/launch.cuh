// Internal launcher interface shared by the translation units of the library.
#pragma once

#include "common.cuh"

namespace oasis {

// By-value view of one tensor (keys or values) of a KV cache, handed to the kernels.
struct KvTensor {
  int n_bf16, n_fp8, n_int4;
  uint8_t kind[OASIS_MAX_FRAMES];
  uint8_t index[OASIS_MAX_FRAMES];
  __nv_bfloat16* bf16;
  uint8_t* fp8; __nv_bfloat16* fp8_scale;
  uint8_t* int4; __half* i4_scale; __half* i4_zero;
};

// By-value view of a KV cache: t[0] the keys, t[1] the values.
struct KvView {
  int layers;
  KvTensor t[2];
};

// Frame page (144 x 1024 elements, or 144 x 16 groups) of pool frame `idx` of session b,
// layer `layer` in a pool of `n` frames.
__host__ __device__ __forceinline__ long long kv_page(int b, int layers, int layer, int n, int idx) {
  return (static_cast<long long>(b) * layers + layer) * n + idx;
}

// Fills `v` from `c` after checking that every slot of both tensors maps into a pool
// that exists (c == NULL gives an empty view).
int make_kv_view(const oasis_kv_cache_t* c, KvView* v);
// bf16 tensor map of rank 2 or 3 (dims innermost first, byte strides of dims 1..),
// 128-byte swizzled boxes.
int encode_bf16_sw128(CUtensorMap* map, const void* base, int rank, const long long* dims,
                      const long long* strides_bytes, const int* box);
int validate_slots(const oasis_kv_cache_t* c, int slot0, int frames);

int num_sms();

int launch_attn_spatial(const void* qkv, void* out, int frames, cudaStream_t stream);
int launch_attn_temporal(const void* qkv, const KvView& kv, int layer, void* out, int batch,
                         int q_frames, int q_pos0, int n_past, int n_kv, cudaStream_t stream);
// Store frames [0, frames) of each session (session rows strided by src_frames frames)
// into cache slots slot0.. of one layer.
int launch_kv_store(const void* kv, long long ld, int k_col, int v_col, const oasis_kv_cache_t* c,
                    int layer, int batch, int frames, int src_frames, int slot0,
                    cudaStream_t stream);

int launch_ln_modulate(const float* x, const float* shift, const float* scale, long long mod_ld,
                       void* out, int M, int rows_per_frame, cudaStream_t stream);
int launch_temb_prep(const int64_t* t, const float* act, void* emb, void* h1a, int F,
                     cudaStream_t stream);
int launch_patch_im2col(const float* x, void* cols, int F, cudaStream_t stream);

}  // namespace oasis
