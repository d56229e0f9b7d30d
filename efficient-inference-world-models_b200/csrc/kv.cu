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

constexpr int kStoreThreads = 256;

// FP8 quantisation of one 144 x 64 slice whose 1152 16-byte chunks (8 bf16 each) are held
// by the CTA's threads (<= 5 each, chunk i = thread + q * 256: row i / 8, chunk i % 8):
// scale = bf16(bf16(max|x| clamped to 1e-12) / 448), code = e4m3(bf16(x / scale)).
__device__ __forceinline__ void fp8_quantize_slice(const uint4 (&chunk)[5], uint8_t* dst,
                                                   __nv_bfloat16* scale_out) {
  __shared__ float red[kStoreThreads / 32];
  float amax = 0.0f;
#pragma unroll
  for (int q = 0; q < 5; ++q) {
    const int i = threadIdx.x + q * kStoreThreads;
    if (i < OASIS_TOKENS * 8) {
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
  if (threadIdx.x == 0) *scale_out = __float2bfloat16_rn(scale);
}

// INT4 quantisation of one (token, head) group of 64 held by a warp (lane l: elements
// 2l, 2l+1), asymmetric in fp32: scale = max(max - min, 1e-12) / 15, zero = min,
// code = clamp(rint((x - zero) / scale), 0, 15), element 2l in the high nibble; scale
// and zero stored as fp16 after the codes are computed.
__device__ __forceinline__ void int4_quantize_group(float x0, float x1, int lane, uint8_t* codes,
                                                    __half* scale_out, __half* zero_out) {
  float mn = fminf(x0, x1), mx = fmaxf(x0, x1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float scale = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), 1e-12f), 15.0f);
  const float q0 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x0, mn), scale)), 0.0f), 15.0f);
  const float q1 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x1, mn), scale)), 0.0f), 15.0f);
  codes[lane] = static_cast<uint8_t>((static_cast<uint32_t>(q0) << 4) | static_cast<uint32_t>(q1));
  if (lane == 0) {
    *scale_out = __float2half_rn(scale);
    *zero_out = __float2half_rn(mn);
  }
}

struct KvStoreSrc {
  const __nv_bfloat16* kv;  // [batch*src_frames*144][ld]
  long long ld;
  int k_col, v_col;
  int layer, frames, src_frames, slot0;
};

// grid: (frames*batch, 2 [K,V], 16 heads); one CTA quantises one 144 x 64 slice into
// its slot's kind of that tensor.
__global__ void __launch_bounds__(kStoreThreads)
    kv_store_kernel(const __grid_constant__ KvView kv, KvStoreSrc p) {
  pdl_trigger();
  pdl_wait();
  const int fb = blockIdx.x;
  const int j = fb % p.frames;
  const int b = fb / p.frames;
  const bool is_v = blockIdx.y == 1;
  const int h = blockIdx.z;
  const KvTensor& t = kv.t[is_v ? 1 : 0];
  const int s = p.slot0 + j;
  const int kind = t.kind[s];
  const int idx = t.index[s];
  const __nv_bfloat16* src =
      p.kv + (static_cast<long long>(b * p.src_frames + j) * OASIS_TOKENS) * p.ld + (is_v ? p.v_col : p.k_col) + h * 64;

  if (kind == OASIS_KV_BF16) {
    const long long page = kv_page(b, kv.layers, p.layer, t.n_bf16, idx);
    __nv_bfloat16* dst = t.bf16 + page * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
    for (int i = threadIdx.x; i < OASIS_TOKENS * 8; i += kStoreThreads) {
      const int r = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(dst + r * OASIS_HIDDEN + c * 8) =
          *reinterpret_cast<const uint4*>(src + r * p.ld + c * 8);
    }
    return;
  }
  if (kind == OASIS_KV_FP8) {
    uint4 chunk[5];
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = threadIdx.x + q * kStoreThreads;
      if (i < OASIS_TOKENS * 8)
        chunk[q] = *reinterpret_cast<const uint4*>(src + (i >> 3) * p.ld + (i & 7) * 8);
    }
    const long long page = kv_page(b, kv.layers, p.layer, t.n_fp8, idx);
    fp8_quantize_slice(chunk, t.fp8 + page * OASIS_TOKENS * OASIS_HIDDEN + h * 64,
                       t.fp8_scale + page * OASIS_HEADS + h);
    return;
  }
  // INT4: one warp per token row of this head
  const long long page = kv_page(b, kv.layers, p.layer, t.n_int4, idx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < OASIS_TOKENS; r += kStoreThreads / 32) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(src + r * p.ld + 2 * lane);
    const long long grp = (page * OASIS_TOKENS + r) * OASIS_HEADS + h;
    int4_quantize_group(bf16_lo(w), bf16_hi(w), lane, t.int4 + grp * 32, t.i4_scale + grp,
                        t.i4_zero + grp);
  }
}

// Dequantise slots [slot0, slot0+frames) of one layer to bf16 [batch][frames][144][1024]
// (keys into k_out, values into v_out).  grid: (frames*batch, 2 [K,V]); 256 threads
// stride over the 144*1024 elements.  bf16 slots are copied by the host launcher.
__global__ void __launch_bounds__(256)
    kv_load_kernel(const __grid_constant__ KvView kv, int layer, int slot0, int frames,
                   __nv_bfloat16* k_out, __nv_bfloat16* v_out) {
  pdl_trigger();
  pdl_wait();
  const int fb = blockIdx.x;
  const int j = fb % frames, b = fb / frames;
  const bool is_v = blockIdx.y == 1;
  const KvTensor& t = kv.t[is_v ? 1 : 0];
  const int s = slot0 + j;
  const int kind = t.kind[s], idx = t.index[s];
  if (kind != OASIS_KV_FP8 && kind != OASIS_KV_INT4) return;
  __nv_bfloat16* dst = (is_v ? v_out : k_out) + (static_cast<long long>(b) * frames + j) * OASIS_TOKENS * OASIS_HIDDEN;
  const long long page = kv_page(b, kv.layers, layer, kind == OASIS_KV_FP8 ? t.n_fp8 : t.n_int4, idx);
  for (int i = threadIdx.x; i < OASIS_TOKENS * OASIS_HIDDEN / 2; i += 256) {
    const int e = 2 * i;
    const int r = e / OASIS_HIDDEN, col = e % OASIS_HIDDEN, h = col / 64, d = col % 64;
    float x0, x1;
    if (kind == OASIS_KV_FP8) {
      const uint8_t* c = t.fp8 + page * OASIS_TOKENS * OASIS_HIDDEN + e;
      const float scale = __bfloat162float(t.fp8_scale[page * OASIS_HEADS + h]);
      x0 = e4m3_to_float(c[0]) * scale;
      x1 = e4m3_to_float(c[1]) * scale;
    } else {
      const long long grp = (page * OASIS_TOKENS + r) * OASIS_HEADS + h;
      const uint8_t byte = t.int4[grp * 32 + d / 2];
      const float scale = __half2float(t.i4_scale[grp]);
      const float zero = __half2float(t.i4_zero[grp]);
      x0 = __fmaf_rn(static_cast<float>(byte >> 4), scale, zero);
      x1 = __fmaf_rn(static_cast<float>(byte & 0xF), scale, zero);
    }
    *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16x2(x0, x1);
  }
}

// Age promotion of one frame (ProgressiveKVQuantizer.update_cache, progressive_quant.py:
// 263-350) for every session and layer of the tensors in `tensors` (bit 0 keys, bit 1
// values): logical slot src_slot is re-quantised into dst_slot of the same tensor, each
// through that tensor's slot map, with the store kernel's arithmetic.  The source
// values are the bf16 entries, or for an FP8 entry promoted to INT4 the reference's
// dequantisation with its default fp16 target: fp16(e4m3 x scale), the product exact in
// fp32 and rounded once.  grid: (batch*layers, number of tensors, 16 heads); one CTA
// per 144 x 64 slice.
__global__ void __launch_bounds__(kStoreThreads)
    kv_migrate_kernel(const __grid_constant__ KvView kv, int tensors, int src_slot, int dst_slot) {
  pdl_trigger();
  pdl_wait();
  const int bl = blockIdx.x;  // session * layers + layer
  // blockIdx.y counts the selected tensors: the keys first when they are selected
  const bool is_v = (tensors & OASIS_KV_KEYS) ? blockIdx.y == 1 : true;
  const KvTensor& t = kv.t[is_v ? 1 : 0];
  const int h = blockIdx.z;
  const int src_kind = t.kind[src_slot], src_idx = t.index[src_slot];
  const int dst_kind = t.kind[dst_slot], dst_idx = t.index[dst_slot];
  const __nv_bfloat16* sb = nullptr;
  const uint8_t* sf = nullptr;
  float fscale = 0.0f;
  if (src_kind == OASIS_KV_BF16) {
    sb = t.bf16 + (static_cast<long long>(bl) * t.n_bf16 + src_idx) * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
  } else {
    const long long page = static_cast<long long>(bl) * t.n_fp8 + src_idx;
    sf = t.fp8 + page * OASIS_TOKENS * OASIS_HIDDEN + h * 64;
    fscale = __bfloat162float(t.fp8_scale[page * OASIS_HEADS + h]);
  }
  // element (row r, column c) of the source slice as the value the reference quantises
  auto value = [&](int r, int c) -> float {
    if (sb) return __bfloat162float(sb[r * OASIS_HIDDEN + c]);
    return __half2float(__float2half_rn(e4m3_to_float(sf[r * OASIS_HIDDEN + c]) * fscale));
  };

  if (dst_kind == OASIS_KV_FP8) {  // only from bf16 (a full-precision entry)
    uint4 chunk[5];
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = threadIdx.x + q * kStoreThreads;
      if (i < OASIS_TOKENS * 8) chunk[q] = *reinterpret_cast<const uint4*>(sb + (i >> 3) * OASIS_HIDDEN + (i & 7) * 8);
    }
    const long long page = static_cast<long long>(bl) * t.n_fp8 + dst_idx;
    fp8_quantize_slice(chunk, t.fp8 + page * OASIS_TOKENS * OASIS_HIDDEN + h * 64,
                       t.fp8_scale + page * OASIS_HEADS + h);
    return;
  }
  // INT4: one warp per token row of this head
  const long long page = static_cast<long long>(bl) * t.n_int4 + dst_idx;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < OASIS_TOKENS; r += kStoreThreads / 32) {
    const long long grp = (page * OASIS_TOKENS + r) * OASIS_HEADS + h;
    int4_quantize_group(value(r, 2 * lane), value(r, 2 * lane + 1), lane, t.int4 + grp * 32,
                        t.i4_scale + grp, t.i4_zero + grp);
  }
}

namespace {

bool slot_ok(const oasis_kv_tensor_t& t, int s) {
  const int kind = t.slot_kind[s], idx = t.slot_index[s];
  switch (kind) {
    case OASIS_KV_BF16: return idx < t.n_bf16 && t.bf16;
    case OASIS_KV_FP8: return idx < t.n_fp8 && t.fp8 && t.fp8_scale;
    case OASIS_KV_INT4: return idx < t.n_int4 && t.int4 && t.i4_scale && t.i4_zero;
  }
  return false;
}

bool pools_aligned(const oasis_kv_tensor_t& t) {
  const void* p[] = {t.bf16, t.fp8, t.fp8_scale, t.int4, t.i4_scale, t.i4_zero};
  for (const void* q : p)
    if (q && !aligned16(q)) return false;
  return true;
}

KvTensor tensor_view(const oasis_kv_tensor_t& c) {
  KvTensor t{};
  t.n_bf16 = c.n_bf16;
  t.n_fp8 = c.n_fp8;
  t.n_int4 = c.n_int4;
  for (int s = 0; s < OASIS_MAX_FRAMES; ++s) {
    t.kind[s] = c.slot_kind[s];
    t.index[s] = c.slot_index[s];
  }
  t.bf16 = static_cast<__nv_bfloat16*>(c.bf16);
  t.fp8 = c.fp8;
  t.fp8_scale = static_cast<__nv_bfloat16*>(c.fp8_scale);
  t.int4 = c.int4;
  t.i4_scale = static_cast<__half*>(c.i4_scale);
  t.i4_zero = static_cast<__half*>(c.i4_zero);
  return t;
}

}  // namespace

int validate_slots(const oasis_kv_cache_t* c, int slot0, int frames) {
  if (slot0 < 0 || frames < 0 || slot0 + frames > c->n_slots || c->n_slots > OASIS_MAX_FRAMES)
    return fail(OASIS_ERR_INVALID_ARG, "KV slot range outside the cache");
  if (c->batch <= 0 || c->layers <= 0)
    return fail(OASIS_ERR_INVALID_ARG, "KV cache needs batch > 0 and layers > 0");
  if (!pools_aligned(c->k) || !pools_aligned(c->v))
    return fail(OASIS_ERR_ALIGNMENT, "KV cache pools must be 16-byte aligned");
  for (int s = slot0; s < slot0 + frames; ++s) {
    if (!slot_ok(c->k, s))
      return fail(OASIS_ERR_INVALID_ARG, "KV cache key slot " + std::to_string(s) + " is invalid");
    if (!slot_ok(c->v, s))
      return fail(OASIS_ERR_INVALID_ARG, "KV cache value slot " + std::to_string(s) + " is invalid");
  }
  return OASIS_OK;
}

int make_kv_view(const oasis_kv_cache_t* c, KvView* v) {
  *v = KvView{};
  if (!c) return OASIS_OK;
  if (int s = validate_slots(c, 0, c->n_slots)) return s;
  v->layers = c->layers;
  v->t[0] = tensor_view(c->k);
  v->t[1] = tensor_view(c->v);
  return OASIS_OK;
}

int launch_kv_store(const void* kv, long long ld, int k_col, int v_col, const oasis_kv_cache_t* c,
                    int layer, int batch, int frames, int src_frames, int slot0,
                    cudaStream_t stream) {
  if (frames == 0) return OASIS_OK;
  KvView view;
  if (int s = make_kv_view(c, &view)) return s;
  KvStoreSrc p{};
  p.kv = static_cast<const __nv_bfloat16*>(kv);
  p.ld = ld;
  p.k_col = k_col;
  p.v_col = v_col;
  p.layer = layer;
  p.frames = frames;
  p.src_frames = src_frames;
  p.slot0 = slot0;
  dim3 grid(frames * batch, 2, OASIS_HEADS);
  cudaError_t e = launch_pdl(kv_store_kernel, grid, dim3(kStoreThreads), 0, stream, view, p);
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
  if (!aligned16(k_out) || !aligned16(v_out)) return fail(OASIS_ERR_ALIGNMENT, "oasis_kv_load: output alignment");
  if (int s = validate_slots(cache, slot0, frames)) return s;
  if (frames == 0) return OASIS_OK;
  // bf16 slots are plain copies; quantised slots go through the kernel
  const size_t frame_bytes = static_cast<size_t>(OASIS_TOKENS) * OASIS_HIDDEN * 2;
  bool any_quant = false;
  for (int which = 0; which < 2; ++which) {
    const oasis_kv_tensor_t& t = which ? cache->v : cache->k;
    uint8_t* out = static_cast<uint8_t*>(which ? v_out : k_out);
    for (int j = 0; j < frames; ++j) {
      const int s = slot0 + j;
      if (t.slot_kind[s] != OASIS_KV_BF16) {
        any_quant = true;
        continue;
      }
      for (int b = 0; b < cache->batch; ++b) {
        const long long page = kv_page(b, cache->layers, layer, t.n_bf16, t.slot_index[s]);
        cudaError_t e = cudaMemcpyAsync(out + (static_cast<size_t>(b) * frames + j) * frame_bytes,
                                        static_cast<uint8_t*>(t.bf16) + page * frame_bytes, frame_bytes,
                                        cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return cuda_status(e, "oasis_kv_load(copy)");
      }
    }
  }
  if (!any_quant) return OASIS_OK;
  KvView view;
  if (int s = make_kv_view(cache, &view)) return s;
  dim3 grid(frames * cache->batch, 2);
  cudaError_t e = launch_pdl(kv_load_kernel, grid, dim3(256), 0, stream, view, layer, slot0, frames,
                             static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(v_out));
  if (e != cudaSuccess) return cuda_status(e, "kv_load_kernel");
  return OASIS_OK;
}

extern "C" int oasis_kv_migrate(const oasis_kv_cache_t* cache, int tensors, int src_slot,
                                int dst_slot, cudaStream_t stream) {
  using namespace oasis;
  if (!cache || src_slot == dst_slot || tensors < 1 || tensors > 3)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_kv_migrate: bad args");
  if (int s = validate_slots(cache, src_slot, 1)) return s;
  if (int s = validate_slots(cache, dst_slot, 1)) return s;
  for (int which = 0; which < 2; ++which) {
    if (!(tensors & (which ? OASIS_KV_VALUES : OASIS_KV_KEYS))) continue;
    const oasis_kv_tensor_t& t = which ? cache->v : cache->k;
    const int sk = t.slot_kind[src_slot], dk = t.slot_kind[dst_slot];
    if (!((sk == OASIS_KV_BF16 && (dk == OASIS_KV_FP8 || dk == OASIS_KV_INT4)) ||
          (sk == OASIS_KV_FP8 && dk == OASIS_KV_INT4)))
      return fail(OASIS_ERR_INVALID_ARG,
                  "oasis_kv_migrate: promotions are bf16->fp8, bf16->int4, fp8->int4");
  }
  KvView view;
  if (int s = make_kv_view(cache, &view)) return s;
  const int n_tensors = tensors == 3 ? 2 : 1;
  dim3 grid(cache->batch * cache->layers, n_tensors, OASIS_HEADS);
  cudaError_t e = launch_pdl(kv_migrate_kernel, grid, dim3(kStoreThreads), 0, stream, view, tensors,
                             src_slot, dst_slot);
  if (e != cudaSuccess) return cuda_status(e, "kv_migrate_kernel");
  return OASIS_OK;
}
