// LayerNorm (eps 1e-6, no affine) + adaLN modulate of one row by one warp:
//   out = bf16(LN(x) * (1 + scale) + shift)
// The standalone kernel (elementwise.cu) and the residual-GEMM tail (gemm.cuh) both
// call ln_modulate_row on rows they have loaded their own way, so both produce the
// same bits.  Lane l holds columns l*4 + i*128 (i = 0..7).
#pragma once

#include "common.cuh"

namespace oasis {

constexpr int kLnRowsPerWarp = 4;

// shift and 1 + scale of one frame, in the lane's column layout
__device__ __forceinline__ void ln_load_modulation(const float* shift, const float* scale, int lane,
                                                   float4 (&a4)[8], float4 (&s4)[8]) {
  const float4* sh = reinterpret_cast<const float4*>(shift);
  const float4* sc = reinterpret_cast<const float4*>(scale);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a4[i] = sh[lane + 32 * i];
    const float4 s = sc[lane + 32 * i];
    s4[i] = make_float4(1.0f + s.x, 1.0f + s.y, 1.0f + s.z, 1.0f + s.w);
  }
}

// y = ((x - mean) * rstd) * (1 + scale) + shift, the last product and sum fused
__device__ __forceinline__ float ln_out(float d, float rstd, float ops, float shift) {
  return __fmaf_rn(d * rstd, ops, shift);
}

// One row (lane holds columns 4 lane + 128 i); s4 holds 1 + scale (ln_load_modulation).
__device__ __forceinline__ void ln_modulate_row(const float4 (&v)[8], const float4 (&a4)[8],
                                                const float4 (&s4)[8], __nv_bfloat16* out_row,
                                                int lane) {
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum * (1.0f / OASIS_HIDDEN);
  float4 d[8];  // the centred row, kept for the output
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    d[i] = make_float4(v[i].x - mean, v[i].y - mean, v[i].z - mean, v[i].w - mean);
    sq += (d[i].x * d[i].x + d[i].y * d[i].y) + (d[i].z * d[i].z + d[i].w * d[i].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * (1.0f / OASIS_HIDDEN) + 1e-6f);
  uint2* o2 = reinterpret_cast<uint2*>(out_row);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 a = a4[i];
    const float4 s = s4[i];
    o2[lane + 32 * i] = make_uint2(pack_bf16x2(ln_out(d[i].x, rstd, s.x, a.x), ln_out(d[i].y, rstd, s.y, a.y)),
                                   pack_bf16x2(ln_out(d[i].z, rstd, s.z, a.z), ln_out(d[i].w, rstd, s.w, a.w)));
  }
}

// The same for rows staged in shared memory (row r at rows[r * 256 + lane + 32 i]),
// two rows per pass with their reductions interleaved so the shuffle chains overlap;
// shift and 1 + scale (a4/s4, ln_load_modulation) stay in registers.  Per row the
// arithmetic is the sequence of ln_modulate_row.
__device__ __forceinline__ void ln_modulate_rows_smem(const float4* rows, int nrows,
                                                      const float4 (&a4)[8], const float4 (&s4)[8],
                                                      __nv_bfloat16* out, int lane) {
#pragma unroll 1
  for (int r0 = 0; r0 < nrows; r0 += 2) {
    float4 v[2][8];
    float sum[2], sq[2], mean[2], rstd[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[r][i] = rows[(r0 + r) * 256 + lane + 32 * i];
      sum[r] = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[r] += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < 2; ++r) sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], o);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mean[r] = sum[r] * (1.0f / OASIS_HIDDEN);
      sq[r] = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // v becomes the centred row
        v[r][i] = make_float4(v[r][i].x - mean[r], v[r][i].y - mean[r], v[r][i].z - mean[r], v[r][i].w - mean[r]);
        sq[r] += (v[r][i].x * v[r][i].x + v[r][i].y * v[r][i].y) + (v[r][i].z * v[r][i].z + v[r][i].w * v[r][i].w);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < 2; ++r) sq[r] += __shfl_xor_sync(0xffffffffu, sq[r], o);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r0 + r >= nrows) break;  // the staged row beyond nrows is never stored
      rstd[r] = rsqrtf(sq[r] * (1.0f / OASIS_HIDDEN) + 1e-6f);
      uint2* o2 = reinterpret_cast<uint2*>(out + static_cast<long long>(r0 + r) * OASIS_HIDDEN);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 a = a4[i];
        const float4 s = s4[i];
        const float4 d = v[r][i];
        o2[lane + 32 * i] = make_uint2(pack_bf16x2(ln_out(d.x, rstd[r], s.x, a.x), ln_out(d.y, rstd[r], s.y, a.y)),
                                       pack_bf16x2(ln_out(d.z, rstd[r], s.z, a.z), ln_out(d.w, rstd[r], s.w, a.w)));
      }
    }
  }
}

}  // namespace oasis
