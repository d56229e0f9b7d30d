// LayerNorm (eps 1e-6, no affine) + adaLN modulate of one row by one warp:
//   out = bf16(LN(x) * (1 + scale) + shift)
// The standalone kernel (elementwise.cu) and the residual-GEMM tail (gemm.cuh) both
// call ln_modulate_row on rows they have loaded their own way, so both produce the
// same bits.  Lane l holds columns l*4 + i*128 (i = 0..7).
#pragma once

#include "common.cuh"

namespace oasis {

constexpr int kLnRowsPerWarp = 4;

// shift/scale of one frame, in the lane's column layout
__device__ __forceinline__ void ln_load_modulation(const float* shift, const float* scale, int lane,
                                                   float4 (&a4)[8], float4 (&s4)[8]) {
  const float4* sh = reinterpret_cast<const float4*>(shift);
  const float4* sc = reinterpret_cast<const float4*>(scale);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a4[i] = sh[lane + 32 * i];
    s4[i] = sc[lane + 32 * i];
  }
}

__device__ __forceinline__ void ln_modulate_row(const float4 (&v)[8], const float4 (&a4)[8],
                                                const float4 (&s4)[8], __nv_bfloat16* out_row,
                                                int lane) {
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum * (1.0f / OASIS_HIDDEN);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    sq += (a * a + b * b) + (c * c + d * d);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * (1.0f / OASIS_HIDDEN) + 1e-6f);
  uint2* o2 = reinterpret_cast<uint2*>(out_row);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 a = a4[i];
    const float4 s = s4[i];
    const float y0 = (v[i].x - mean) * rstd * (1.0f + s.x) + a.x;
    const float y1 = (v[i].y - mean) * rstd * (1.0f + s.y) + a.y;
    const float y2 = (v[i].z - mean) * rstd * (1.0f + s.z) + a.z;
    const float y3 = (v[i].w - mean) * rstd * (1.0f + s.w) + a.w;
    o2[lane + 32 * i] = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
  }
}

// The same for rows staged in shared memory (row r at rows[r * 256 + lane + 32 i]),
// two rows per pass with their reductions interleaved so the shuffle chains overlap;
// shift/scale (a4/s4, ln_load_modulation) stay in registers.  Per row the arithmetic
// is the sequence of ln_modulate_row.
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
      for (int i = 0; i < 8; ++i) {
        const float a = v[r][i].x - mean[r], b = v[r][i].y - mean[r], c = v[r][i].z - mean[r],
                    d = v[r][i].w - mean[r];
        sq[r] += (a * a + b * b) + (c * c + d * d);
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
        const float y0 = (v[r][i].x - mean[r]) * rstd[r] * (1.0f + s.x) + a.x;
        const float y1 = (v[r][i].y - mean[r]) * rstd[r] * (1.0f + s.y) + a.y;
        const float y2 = (v[r][i].z - mean[r]) * rstd[r] * (1.0f + s.z) + a.z;
        const float y3 = (v[r][i].w - mean[r]) * rstd[r] * (1.0f + s.w) + a.w;
        o2[lane + 32 * i] = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
      }
    }
  }
}

}  // namespace oasis
