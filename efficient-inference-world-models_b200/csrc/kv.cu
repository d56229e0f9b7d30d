// Temporal KV cache store (quantise) and load (dequantise) kernels.
//
// Quantisation follows ProgressiveKVQuantizer bit for bit
// (worldserve/optimizations/system_level/kv_cache/progressive_quant.py:113-193) on
// bf16 inputs, at the cache granularity:
//   FP8 : one per-tensor absmax scale per (session, layer, frame, head, K|V) slice of
//         144 x 64: scale = bf16(bf16(max|x| clamped to 1e-12) / 448),
//         code  = e4m3(bf16(x / scale))            (fp32 IEEE division, RNE)
//   INT4: one asymmetric group per (token, head) row of 64, in fp32:
//         scale = max(max - min, 1e-12) / 15, zero = min,
//         code  = clamp(rint((x - zero) / scale), 0, 15), element 2i in the high nibble;
//         scale/zero stored as fp16 after the codes are computed.
#include "launch.cuh"

namespace oasis {

struct KvStoreParams {
  const __nv_bfloat16* kv;  // [batch*frames*144][ld]
  long long ld;
  int k_col, v_col;
  int layer, frames, src_frames, slot0;
  int layers, n_bf16, n_fp8, n_int4;
  uint8_t kind[OASIS_MAX_FRAMES];
  uint8_t index[OASIS_MAX_FRAMES];
  __nv_bfloat16* k_bf16; __nv_bfloat16* v_bf16;
  uint8_t* k_fp8; uint8_t* v_fp8;
  __nv_bfloat16* k_fp8_scale; __nv_bfloat16* v_fp8_scale;
  uint8_t* k_int4; uint8_t* v_int4;
  __half* k_i4_scale; __half* k_i4_zero; __half* v_i4_scale; __half* v_i4_zero;
};

constexpr int kStoreThreads = 256;

// grid: (frames*batch, 2 [K,V], 16 heads); one CTA quantises one 144 x 64 slice.
__global__ void __launch_bounds__(kStoreThreads) kv_store_kernel(KvStoreParams p) {
  pdl_trigger();
  pdl_wait();
  const int fb = blockIdx.x;
  const int j = fb % p.frames;
  const int b = fb / p.frames;
  const bool is_v = blockIdx.y == 1;
  const int h = blockIdx.z;
  const int s = p.slot0 + j;
  const int kind = p.kind[s];
  const int idx = p.index[s];
  const __nv_bfloat16* src =
      p.kv + (static_cast<long long>(b * p.src_frames + j) * OASIS_TOKENS) * p.ld + (is_v ? p.v_col : p.k_col) + h * 64;

  if (kind == OASIS_KV_BF16) {
    const long long slot = (static_cast<long long>(b) * p.layers + p.layer) * p.n_bf16 + idx;
    __nv_bfloat16* dst = (is_v ? p.v_bf16 : p.k_bf16) + slot * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
    for (int i = threadIdx.x; i < OASIS_TOKENS * 8; i += kStoreThreads) {
      const int r = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(dst + r * OASIS_HIDDEN + c * 8) =
          *reinterpret_cast<const uint4*>(src + r * p.ld + c * 8);
    }
    return;
  }

  if (kind == OASIS_KV_FP8) {
    __shared__ float red[kStoreThreads / 32];
    // 144 rows x 8 chunks of 8 bf16 = 1152 chunks; <= 5 per thread, kept in registers
    uint4 chunk[5];
    float amax = 0.0f;
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = threadIdx.x + q * kStoreThreads;
      if (i < OASIS_TOKENS * 8) {
        const int r = i >> 3, c = i & 7;
        chunk[q] = *reinterpret_cast<const uint4*>(src + r * p.ld + c * 8);
        const uint32_t w[4] = {chunk[q].x, chunk[q].y, chunk[q].z, chunk[q].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(w[e])), fabsf(bf16_hi(w[e]))));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kStoreThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    // amax is a bf16 value; clamp(min=1e-12) happens in bf16
    amax = fmaxf(amax, __bfloat162float(__float2bfloat16_rn(1e-12f)));
    const float scale = bf16_round(__fdiv_rn(amax, 448.0f));
    const long long slot = (static_cast<long long>(b) * p.layers + p.layer) * p.n_fp8 + idx;
    uint8_t* dst = (is_v ? p.v_fp8 : p.k_fp8) + slot * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = threadIdx.x + q * kStoreThreads;
      if (i < OASIS_TOKENS * 8) {
        const int r = i >> 3, c = i & 7;
        const uint32_t w[4] = {chunk[q].x, chunk[q].y, chunk[q].z, chunk[q].w};
        uint32_t out[2] = {0, 0};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t c0 = float_to_e4m3(bf16_round(__fdiv_rn(bf16_lo(w[e]), scale)));
          const uint32_t c1 = float_to_e4m3(bf16_round(__fdiv_rn(bf16_hi(w[e]), scale)));
          out[e >> 1] |= (c0 | (c1 << 8)) << (16 * (e & 1));
        }
        *reinterpret_cast<uint2*>(dst + r * OASIS_HIDDEN + c * 8) = make_uint2(out[0], out[1]);
      }
    }
    if (threadIdx.x == 0)
      (is_v ? p.v_fp8_scale : p.k_fp8_scale)[slot * OASIS_HEADS + h] = __float2bfloat16_rn(scale);
    return;
  }

  // INT4: one warp per (token) row of this head: lane holds elements 2l, 2l+1
  const long long slot = (static_cast<long long>(b) * p.layers + p.layer) * p.n_int4 + idx;
  uint8_t* codes = is_v ? p.v_int4 : p.k_int4;
  __half* sc = is_v ? p.v_i4_scale : p.k_i4_scale;
  __half* zp = is_v ? p.v_i4_zero : p.k_i4_zero;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < OASIS_TOKENS; r += kStoreThreads / 32) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(src + r * p.ld + 2 * lane);
    const float x0 = bf16_lo(w), x1 = bf16_hi(w);
    float mn = fminf(x0, x1), mx = fmaxf(x0, x1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), 1e-12f), 15.0f);
    const float q0 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x0, mn), scale)), 0.0f), 15.0f);
    const float q1 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x1, mn), scale)), 0.0f), 15.0f);
    const long long grp = (slot * OASIS_TOKENS + r) * OASIS_HEADS + h;
    codes[grp * 32 + lane] = static_cast<uint8_t>((static_cast<uint32_t>(q0) << 4) | static_cast<uint32_t>(q1));
    if (lane == 0) {
      sc[grp] = __float2half_rn(scale);
      zp[grp] = __float2half_rn(mn);
    }
  }
}

// Dequantise slots [slot0, slot0+frames) of one layer to bf16 [batch][frames][144][1024].
// grid: (frames*batch, 2 [K,V]); 256 threads stride over the 144*1024 elements.
__global__ void __launch_bounds__(256) kv_load_kernel(KvStoreParams p) {
  pdl_trigger();
  pdl_wait();
  const int fb = blockIdx.x;
  const int j = fb % p.frames, b = fb / p.frames;
  const bool is_v = blockIdx.y == 1;
  const int s = p.slot0 + j;
  const int kind = p.kind[s], idx = p.index[s];
  if (kind != OASIS_KV_FP8 && kind != OASIS_KV_INT4) return;  // bf16 slots are copied by the host
  // p.k_bf16/v_bf16 carry the OUTPUT buffers here; the sources are the quantised pools
  __nv_bfloat16* dst = (is_v ? p.v_bf16 : p.k_bf16) +
                       (static_cast<long long>(b) * p.frames + j) * OASIS_TOKENS * OASIS_HIDDEN;
  for (int i = threadIdx.x; i < OASIS_TOKENS * OASIS_HIDDEN / 2; i += 256) {
    const int e = 2 * i;
    const int r = e / OASIS_HIDDEN, col = e % OASIS_HIDDEN, h = col / 64, d = col % 64;
    float x0, x1;
    if (kind == OASIS_KV_FP8) {
      const long long slot = (static_cast<long long>(b) * p.layers + p.layer) * p.n_fp8 + idx;
      const uint8_t* c = (is_v ? p.v_fp8 : p.k_fp8) + slot * OASIS_TOKENS * OASIS_HIDDEN + e;
      const float scale = __bfloat162float((is_v ? p.v_fp8_scale : p.k_fp8_scale)[slot * OASIS_HEADS + h]);
      x0 = e4m3_to_float(c[0]) * scale;
      x1 = e4m3_to_float(c[1]) * scale;
    } else {
      const long long slot = (static_cast<long long>(b) * p.layers + p.layer) * p.n_int4 + idx;
      const long long grp = (slot * OASIS_TOKENS + r) * OASIS_HEADS + h;
      const uint8_t byte = (is_v ? p.v_int4 : p.k_int4)[grp * 32 + d / 2];
      const float scale = __half2float((is_v ? p.v_i4_scale : p.k_i4_scale)[grp]);
      const float zero = __half2float((is_v ? p.v_i4_zero : p.k_i4_zero)[grp]);
      x0 = static_cast<float>(byte >> 4) * scale + zero;
      x1 = static_cast<float>(byte & 0xF) * scale + zero;
    }
    *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16x2(x0, x1);
  }
}

int fill_store_params(KvStoreParams* p, const oasis_kv_cache_t* c) {
  p->layers = c->layers;
  p->n_bf16 = c->n_bf16;
  p->n_fp8 = c->n_fp8;
  p->n_int4 = c->n_int4;
  for (int s = 0; s < OASIS_MAX_FRAMES; ++s) {
    p->kind[s] = c->slot_kind[s];
    p->index[s] = c->slot_index[s];
  }
  p->k_bf16 = static_cast<__nv_bfloat16*>(c->k_bf16);
  p->v_bf16 = static_cast<__nv_bfloat16*>(c->v_bf16);
  p->k_fp8 = c->k_fp8;
  p->v_fp8 = c->v_fp8;
  p->k_fp8_scale = static_cast<__nv_bfloat16*>(c->k_fp8_scale);
  p->v_fp8_scale = static_cast<__nv_bfloat16*>(c->v_fp8_scale);
  p->k_int4 = c->k_int4;
  p->v_int4 = c->v_int4;
  p->k_i4_scale = static_cast<__half*>(c->k_i4_scale);
  p->k_i4_zero = static_cast<__half*>(c->k_i4_zero);
  p->v_i4_scale = static_cast<__half*>(c->v_i4_scale);
  p->v_i4_zero = static_cast<__half*>(c->v_i4_zero);
  return OASIS_OK;
}

// Age promotion of one frame (ProgressiveKVQuantizer.update_cache, progressive_quant.py:
// 263-350) for every session and layer: the slot at (src_kind, src_idx) is re-quantised
// into (dst_kind, dst_idx) with the store kernel's arithmetic.  The source values are
// the bf16 entries, or for an FP8 entry promoted to INT4 the reference's dequantisation
// with its default fp16 target: fp16(e4m3 x scale), the product exact in fp32 and
// rounded once.  grid: (batch*layers, 2 [K,V], 16 heads); one CTA per 144 x 64 slice.
__global__ void __launch_bounds__(kStoreThreads)
    kv_migrate_kernel(KvStoreParams p, int src_kind, int src_idx, int dst_kind, int dst_idx) {
  pdl_trigger();
  pdl_wait();
  const int bl = blockIdx.x;  // session * layers + layer
  const bool is_v = blockIdx.y == 1;
  const int h = blockIdx.z;
  const __nv_bfloat16* sb = nullptr;
  const uint8_t* sf = nullptr;
  float fscale = 0.0f;
  if (src_kind == OASIS_KV_BF16) {
    sb = (is_v ? p.v_bf16 : p.k_bf16) + (static_cast<long long>(bl) * p.n_bf16 + src_idx) * OASIS_TOKENS *
                                            OASIS_HIDDEN + h * 64;
  } else {
    const long long slot = static_cast<long long>(bl) * p.n_fp8 + src_idx;
    sf = (is_v ? p.v_fp8 : p.k_fp8) + slot * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
    fscale = __bfloat162float((is_v ? p.v_fp8_scale : p.k_fp8_scale)[slot * OASIS_HEADS + h]);
  }
  // element (row r, column c) of the source slice as the value the reference quantises
  auto value = [&](int r, int c) -> float {
    if (sb) return __bfloat162float(sb[r * OASIS_HIDDEN + c]);
    return __half2float(__float2half_rn(e4m3_to_float(sf[r * OASIS_HIDDEN + c]) * fscale));
  };

  if (dst_kind == OASIS_KV_FP8) {  // only from bf16 (a full-precision entry)
    __shared__ float red[kStoreThreads / 32];
    float amax = 0.0f;
    for (int i = threadIdx.x; i < OASIS_TOKENS * 64; i += kStoreThreads)
      amax = fmaxf(amax, fabsf(value(i >> 6, i & 63)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kStoreThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    amax = fmaxf(amax, __bfloat162float(__float2bfloat16_rn(1e-12f)));
    const float scale = bf16_round(__fdiv_rn(amax, 448.0f));
    const long long slot = static_cast<long long>(bl) * p.n_fp8 + dst_idx;
    uint8_t* dst = (is_v ? p.v_fp8 : p.k_fp8) + slot * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
    for (int i = threadIdx.x; i < OASIS_TOKENS * 64; i += kStoreThreads) {
      const int r = i >> 6, c = i & 63;
      dst[r * OASIS_HIDDEN + c] =
          static_cast<uint8_t>(float_to_e4m3(bf16_round(__fdiv_rn(value(r, c), scale))));
    }
    if (threadIdx.x == 0)
      (is_v ? p.v_fp8_scale : p.k_fp8_scale)[slot * OASIS_HEADS + h] = __float2bfloat16_rn(scale);
    return;
  }

  // INT4: one warp per token row of this head; lane holds elements 2l, 2l+1
  const long long slot = static_cast<long long>(bl) * p.n_int4 + dst_idx;
  uint8_t* codes = is_v ? p.v_int4 : p.k_int4;
  __half* sc = is_v ? p.v_i4_scale : p.k_i4_scale;
  __half* zp = is_v ? p.v_i4_zero : p.k_i4_zero;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < OASIS_TOKENS; r += kStoreThreads / 32) {
    const float x0 = value(r, 2 * lane), x1 = value(r, 2 * lane + 1);
    float mn = fminf(x0, x1), mx = fmaxf(x0, x1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), 1e-12f), 15.0f);
    const float q0 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x0, mn), scale)), 0.0f), 15.0f);
    const float q1 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x1, mn), scale)), 0.0f), 15.0f);
    const long long grp = (slot * OASIS_TOKENS + r) * OASIS_HEADS + h;
    codes[grp * 32 + lane] = static_cast<uint8_t>((static_cast<uint32_t>(q0) << 4) | static_cast<uint32_t>(q1));
    if (lane == 0) {
      sc[grp] = __float2half_rn(scale);
      zp[grp] = __float2half_rn(mn);
    }
  }
}

int validate_slots(const oasis_kv_cache_t* c, int slot0, int frames) {
  if (slot0 < 0 || frames < 0 || slot0 + frames > c->n_slots || c->n_slots > OASIS_MAX_FRAMES)
    return fail(OASIS_ERR_INVALID_ARG, "KV slot range outside the cache");
  for (int s = slot0; s < slot0 + frames; ++s) {
    const int kind = c->slot_kind[s], idx = c->slot_index[s];
    const bool ok = (kind == OASIS_KV_BF16 && idx < c->n_bf16 && c->k_bf16 && c->v_bf16) ||
                    (kind == OASIS_KV_FP8 && idx < c->n_fp8 && c->k_fp8 && c->v_fp8 &&
                     c->k_fp8_scale && c->v_fp8_scale) ||
                    (kind == OASIS_KV_INT4 && idx < c->n_int4 && c->k_int4 && c->v_int4 &&
                     c->k_i4_scale && c->k_i4_zero && c->v_i4_scale && c->v_i4_zero);
    if (!ok) return fail(OASIS_ERR_INVALID_ARG, "KV cache slot " + std::to_string(s) + " is invalid");
  }
  return OASIS_OK;
}

int launch_kv_store(const void* kv, long long ld, int k_col, int v_col, const oasis_kv_cache_t* c,
                    int layer, int batch, int frames, int src_frames, int slot0,
                    cudaStream_t stream) {
  if (frames == 0) return OASIS_OK;
  KvStoreParams p{};
  fill_store_params(&p, c);
  p.kv = static_cast<const __nv_bfloat16*>(kv);
  p.ld = ld;
  p.k_col = k_col;
  p.v_col = v_col;
  p.layer = layer;
  p.frames = frames;
  p.src_frames = src_frames;
  p.slot0 = slot0;
  dim3 grid(frames * batch, 2, OASIS_HEADS);
  cudaError_t e = launch_pdl(kv_store_kernel, grid, dim3(kStoreThreads), 0, stream, p);
  if (e != cudaSuccess) return cuda_status(e, "kv_store_kernel");
  return OASIS_OK;
}

}  // namespace oasis

extern "C" int oasis_kv_store(const void* kv, int ld, int k_col, int v_col,
                              const oasis_kv_cache_t* cache, int layer, int batch, int frames,
                              int slot0, cudaStream_t stream) {
  using namespace oasis;
  if (!kv || !cache || batch <= 0 || batch > cache->batch || layer < 0 || layer >= cache->layers)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_kv_store: bad args");
  if (!aligned16(kv) || (ld % 8) || (k_col % 64) || (v_col % 64) || k_col + OASIS_HIDDEN > ld ||
      v_col + OASIS_HIDDEN > ld)
    return fail(OASIS_ERR_ALIGNMENT, "oasis_kv_store: kv rows must be 16-byte aligned, K/V columns 64-aligned");
  if (int s = validate_slots(cache, slot0, frames)) return s;
  return launch_kv_store(kv, ld, k_col, v_col, cache, layer, batch, frames, frames, slot0, stream);
}

extern "C" int oasis_kv_load(const oasis_kv_cache_t* cache, int layer, int slot0, int frames,
                             void* k_out, void* v_out, cudaStream_t stream) {
  using namespace oasis;
  if (!cache || !k_out || !v_out || layer < 0 || layer >= cache->layers)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_kv_load: bad args");
  if (int s = validate_slots(cache, slot0, frames)) return s;
  if (frames == 0) return OASIS_OK;
  // bf16 slots are plain copies; quantised slots go through the kernel
  KvStoreParams p{};
  fill_store_params(&p, cache);
  const size_t frame_bytes = static_cast<size_t>(OASIS_TOKENS) * OASIS_HIDDEN * 2;
  for (int b = 0; b < cache->batch; ++b) {
    for (int j = 0; j < frames; ++j) {
      const int s = slot0 + j;
      if (cache->slot_kind[s] != OASIS_KV_BF16) continue;
      const long long slot = (static_cast<long long>(b) * cache->layers + layer) * cache->n_bf16 +
                             cache->slot_index[s];
      const size_t off_out = (static_cast<size_t>(b) * frames + j) * frame_bytes;
      cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(k_out) + off_out,
                                      static_cast<uint8_t*>(cache->k_bf16) + slot * frame_bytes,
                                      frame_bytes, cudaMemcpyDeviceToDevice, stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(static_cast<uint8_t*>(v_out) + off_out,
                            static_cast<uint8_t*>(cache->v_bf16) + slot * frame_bytes, frame_bytes,
                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return cuda_status(e, "oasis_kv_load(copy)");
    }
  }
  bool any_quant = false;
  for (int j = 0; j < frames; ++j) any_quant |= cache->slot_kind[slot0 + j] != OASIS_KV_BF16;
  if (!any_quant) return OASIS_OK;
  p.layer = layer;
  p.frames = frames;
  p.slot0 = slot0;
  // output buffers ride in the bf16 fields; bf16 slots are skipped by the kernel
  p.k_bf16 = static_cast<__nv_bfloat16*>(k_out);
  p.v_bf16 = static_cast<__nv_bfloat16*>(v_out);
  for (int j = 0; j < frames; ++j)
    if (cache->slot_kind[slot0 + j] == OASIS_KV_BF16) p.kind[slot0 + j] = 0xFF;
  dim3 grid(frames * cache->batch, 2);
  cudaError_t e = launch_pdl(kv_load_kernel, grid, dim3(256), 0, stream, p);
  if (e != cudaSuccess) return cuda_status(e, "kv_load_kernel");
  return OASIS_OK;
}

extern "C" int oasis_kv_migrate(const oasis_kv_cache_t* cache, int src_slot, int dst_slot,
                                cudaStream_t stream) {
  using namespace oasis;
  if (!cache || src_slot == dst_slot) return fail(OASIS_ERR_INVALID_ARG, "oasis_kv_migrate: bad args");
  if (int s = validate_slots(cache, src_slot, 1)) return s;
  if (int s = validate_slots(cache, dst_slot, 1)) return s;
  const int sk = cache->slot_kind[src_slot], dk = cache->slot_kind[dst_slot];
  if (!((sk == OASIS_KV_BF16 && (dk == OASIS_KV_FP8 || dk == OASIS_KV_INT4)) ||
        (sk == OASIS_KV_FP8 && dk == OASIS_KV_INT4)))
    return fail(OASIS_ERR_INVALID_ARG, "oasis_kv_migrate: promotions are bf16->fp8, bf16->int4, fp8->int4");
  KvStoreParams p{};
  fill_store_params(&p, cache);
  dim3 grid(cache->batch * cache->layers, 2, OASIS_HEADS);
  cudaError_t e = launch_pdl(kv_migrate_kernel, grid, dim3(kStoreThreads), 0, stream, p, sk,
                             static_cast<int>(cache->slot_index[src_slot]), dk,
                             static_cast<int>(cache->slot_index[dst_slot]));
  if (e != cudaSuccess) return cuda_status(e, "kv_migrate_kernel");
  return OASIS_OK;
}
