// Memory-bound kernels around the GEMMs: LayerNorm + adaLN modulate, the inputs of the
// embedding GEMMs (timestep sinusoid, action columns, patch im2col), and the sampler
// updates.
#include "launch.cuh"
#include "ln.cuh"

namespace oasis {

// ----------------------------------------------------------------------------------
// LayerNorm (eps 1e-6, no affine) + modulate: out = bf16(LN(x) * (1 + scale[f]) + shift[f])
// x fp32 [M][1024]; frame f = row / rows_per_frame; shift/scale rows of the adaLN table.
// A CTA takes 16 rows of one frame (4 warps x 4 rows, ln_modulate_rows).  The forward
// runs this kernel only for the first LayerNorm; the others are the tail of the
// residual GEMM that produces their input.
// ----------------------------------------------------------------------------------
constexpr int kLnWarps = 4;
constexpr int kLnRowsPerCta = kLnRowsPerWarp * kLnWarps;

__global__ void __launch_bounds__(kLnWarps * 32)
    ln_modulate_kernel(const float* __restrict__ x, const float* __restrict__ shift,
                       const float* __restrict__ scale, long long mod_ld,
                       __nv_bfloat16* __restrict__ out, int M, int rows_per_frame) {
  pdl_trigger();
  pdl_wait();
  const int chunks = (rows_per_frame + kLnRowsPerCta - 1) / kLnRowsPerCta;
  const long long f = blockIdx.x / chunks;
  const int row0 = static_cast<int>(f * rows_per_frame) + (blockIdx.x % chunks) * kLnRowsPerCta +
                   (threadIdx.x >> 5) * kLnRowsPerWarp;
  const int row_end = min(static_cast<int>((f + 1) * rows_per_frame), M);
  if (row0 >= row_end) return;
  const int lane = threadIdx.x & 31;
  const int nrows = min(kLnRowsPerWarp, row_end - row0);
  float4 v[kLnRowsPerWarp][8];  // all rows in flight before any is reduced
#pragma unroll
  for (int r = 0; r < kLnRowsPerWarp; ++r) {
    if (r < nrows) {
      const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row0 + r) * OASIS_HIDDEN);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[r][i] = xr[lane + 32 * i];
    }
  }
  float4 a4[8], s4[8];
  ln_load_modulation(shift + f * mod_ld, scale + f * mod_ld, lane, a4, s4);
#pragma unroll
  for (int r = 0; r < kLnRowsPerWarp; ++r) {
    if (r >= nrows) break;
    ln_modulate_row(v[r], a4, s4, out + static_cast<long long>(row0 + r) * OASIS_HIDDEN, lane);
  }
}

int launch_ln_modulate(const float* x, const float* shift, const float* scale, long long mod_ld,
                       void* out, int M, int rows_per_frame, cudaStream_t stream) {
  const int frames = (M + rows_per_frame - 1) / rows_per_frame;
  const int chunks = (rows_per_frame + kLnRowsPerCta - 1) / kLnRowsPerCta;
  cudaError_t e = launch_pdl(ln_modulate_kernel, dim3(frames * chunks), dim3(kLnWarps * 32), 0, stream,
                             x, shift, scale, mod_ld, static_cast<__nv_bfloat16*>(out), M,
                             rows_per_frame);
  if (e != cudaSuccess) return cuda_status(e, "ln_modulate_kernel");
  return OASIS_OK;
}

// ----------------------------------------------------------------------------------
// conditioning inputs of the two timestep-MLP GEMMs
//   emb [F][256] bf16: sinusoidal timestep embedding [cos(t f_i) | sin(t f_i)],
//                      f_i = exp(-ln(10000) i / 128), computed in fp32
//   h1a [F][1088] bf16: columns 1024..1087 <- the 25 action values, a 1 for the action
//                      bias column (0 without actions), zeros (the first-linear GEMM
//                      writes columns 0..1023)
// ----------------------------------------------------------------------------------
__global__ void temb_prep_kernel(const int64_t* __restrict__ t, const float* __restrict__ act,
                                 __nv_bfloat16* __restrict__ emb, __nv_bfloat16* __restrict__ h1a,
                                 int F) {
  pdl_trigger();
  pdl_wait();
  const int f = blockIdx.x;
  const int i = threadIdx.x;  // 128 threads
  if (f >= F) return;
  const float freq = expf(-9.210340371976184f * static_cast<float>(i) / 128.0f);
  const float arg = static_cast<float>(t[f]) * freq;
  emb[f * 256 + i] = __float2bfloat16_rn(cosf(arg));
  emb[f * 256 + 128 + i] = __float2bfloat16_rn(sinf(arg));
  if (i < 64) {
    // 25 action values, then the constant input of the action bias column
    float a = 0.0f;
    if (act && i < OASIS_ACTION_DIM) a = act[f * OASIS_ACTION_DIM + i];
    if (act && i == OASIS_ACTION_DIM) a = 1.0f;
    h1a[static_cast<long long>(f) * (OASIS_HIDDEN + 64) + OASIS_HIDDEN + i] = __float2bfloat16_rn(a);
  }
}

int launch_temb_prep(const int64_t* t, const float* act, void* emb, void* h1a, int F,
                     cudaStream_t stream) {
  cudaError_t e = launch_pdl(temb_prep_kernel, dim3(F), dim3(128), 0, stream, t, act,
                             static_cast<__nv_bfloat16*>(emb), static_cast<__nv_bfloat16*>(h1a), F);
  if (e != cudaSuccess) return cuda_status(e, "temb_prep_kernel");
  return OASIS_OK;
}

// im2col of the 2x2 patch embedding: x fp32 [F][16][18][32] -> cols bf16 [F*144][64],
// column c*4 + pi*2 + qi (Conv2d weight order [out][c][pi][qi]).  One thread per
// (token, channel) writes its 4 patch values.
__global__ void patch_im2col_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ cols,
                                    int F) {
  pdl_trigger();
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(F) * OASIS_TOKENS * 16;
  if (i >= total) return;
  const int c = static_cast<int>(i & 15);
  const long long m = i >> 4;
  const int f = static_cast<int>(m / OASIS_TOKENS);
  const int pp = static_cast<int>(m % OASIS_TOKENS);
  const int hp = pp / 16, wp = pp % 16;
  const float* src = x + ((static_cast<long long>(f) * 16 + c) * 18 + hp * 2) * 32 + wp * 2;
  const float2 r0 = *reinterpret_cast<const float2*>(src);
  const float2 r1 = *reinterpret_cast<const float2*>(src + 32);
  uint2 w;
  w.x = pack_bf16x2(r0.x, r0.y);
  w.y = pack_bf16x2(r1.x, r1.y);
  *reinterpret_cast<uint2*>(cols + m * 64 + c * 4) = w;
}

int launch_patch_im2col(const float* x, void* cols, int F, cudaStream_t stream) {
  const long long total = static_cast<long long>(F) * OASIS_TOKENS * 16;
  cudaError_t e = launch_pdl(patch_im2col_kernel, dim3(static_cast<unsigned>((total + 255) / 256)),
                             dim3(256), 0, stream, x, static_cast<__nv_bfloat16*>(cols), F);
  if (e != cudaSuccess) return cuda_status(e, "patch_im2col_kernel");
  return OASIS_OK;
}

// ----------------------------------------------------------------------------------
// samplers
// ----------------------------------------------------------------------------------
// DPM-Solver++ 2M (v-prediction) on `n` elements per session; with first != 0 it is the
// DDIM v-step.  a = sqrt(ab_t), b = sqrt(1 - ab_t), c = sqrt(ab_next), d = sqrt(1 - ab_next).
__global__ void dpmpp2m_kernel(float* __restrict__ x, const float* __restrict__ v,
                               float* __restrict__ eps_prev, int n, long long xs, long long vs,
                               float a, float b, float c, float d, int first) {
  pdl_trigger();
  pdl_wait();
  const int sess = blockIdx.y;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= n) return;
  float4 xv = *reinterpret_cast<float4*>(x + sess * xs + i);
  const float4 vv = *reinterpret_cast<const float4*>(v + sess * vs + i);
  float* ep = eps_prev ? eps_prev + static_cast<long long>(sess) * n + i : nullptr;
  float4 pv = make_float4(0, 0, 0, 0);
  if (!first && ep) pv = *reinterpret_cast<float4*>(ep);
  float xs4[4] = {xv.x, xv.y, xv.z, xv.w};
  const float vs4[4] = {vv.x, vv.y, vv.z, vv.w};
  const float ps4[4] = {pv.x, pv.y, pv.z, pv.w};
  float es4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float x0 = a * xs4[k] - b * vs4[k];
    const float eps = b * xs4[k] + a * vs4[k];
    const float D = first ? eps : (3.0f * eps - ps4[k]) / 2.0f;
    es4[k] = eps;
    xs4[k] = c * x0 + d * D;
  }
  *reinterpret_cast<float4*>(x + sess * xs + i) = make_float4(xs4[0], xs4[1], xs4[2], xs4[3]);
  if (ep) *reinterpret_cast<float4*>(ep) = make_float4(es4[0], es4[1], es4[2], es4[3]);
}

__global__ void ab_update_kernel(const float* __restrict__ x, const float* __restrict__ d0,
                                 const float* __restrict__ d1, const float* __restrict__ d2,
                                 float* __restrict__ out, long long n, float h, float c0, float c1,
                                 float c2) {
  pdl_trigger();
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = c0 * d0[i];
  if (d1) acc += c1 * d1[i];
  if (d2) acc += c2 * d2[i];
  out[i] = x[i] + h * acc;
}

}  // namespace oasis

extern "C" int oasis_dpmpp2m_update(float* x, const float* v, float* eps_prev, int batch, int n,
                                    long long x_stride, long long v_stride, float ab_t,
                                    float ab_next, int first, cudaStream_t stream) {
  using namespace oasis;
  if (!x || !v || batch <= 0 || n <= 0) return fail(OASIS_ERR_INVALID_ARG, "oasis_dpmpp2m_update: bad args");
  if (!first && !eps_prev) return fail(OASIS_ERR_INVALID_ARG, "oasis_dpmpp2m_update: multistep needs eps_prev");
  if ((n % 4) || (x_stride % 4) || (v_stride % 4) || !aligned16(x) || !aligned16(v) ||
      (eps_prev && !aligned16(eps_prev)))
    return fail(OASIS_ERR_ALIGNMENT, "oasis_dpmpp2m_update: n/strides must be multiples of 4, 16-byte aligned");
  if (batch > 65535) return fail(OASIS_ERR_UNSUPPORTED, "oasis_dpmpp2m_update: batch too large");
  const float a = sqrtf(ab_t), b = sqrtf(1.0f - ab_t), c = sqrtf(ab_next), d = sqrtf(1.0f - ab_next);
  dim3 grid((n / 4 + 255) / 256, batch);
  cudaError_t e = launch_pdl(dpmpp2m_kernel, grid, dim3(256), 0, stream, x, v, eps_prev, n, x_stride,
                             v_stride, a, b, c, d, first);
  if (e != cudaSuccess) return cuda_status(e, "dpmpp2m_kernel");
  return OASIS_OK;
}

extern "C" int oasis_ab_update(const float* x, const float* d0, const float* d1, const float* d2,
                               float* out, long long n, float h, float c0, float c1, float c2,
                               cudaStream_t stream) {
  using namespace oasis;
  if (!x || !d0 || !out || n <= 0) return fail(OASIS_ERR_INVALID_ARG, "oasis_ab_update: bad args");
  if ((c1 != 0.0f && !d1) || (c2 != 0.0f && !d2))
    return fail(OASIS_ERR_INVALID_ARG, "oasis_ab_update: missing history for a non-zero coefficient");
  cudaError_t e = launch_pdl(ab_update_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256),
                             0, stream, x, d0, c1 != 0.0f ? d1 : nullptr, c2 != 0.0f ? d2 : nullptr,
                             out, n, h, c0, c1, c2);
  if (e != cudaSuccess) return cuda_status(e, "ab_update_kernel");
  return OASIS_OK;
}
