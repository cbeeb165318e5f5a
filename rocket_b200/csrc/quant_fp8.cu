// Per-token e4m3 quantization of bf16 activation rows for the FP8 GEMM:
//   s_r = amax(x_r) / 448 (1 for an all-zero row),  q_r = e4m3_rn_satfinite(x_r / s_r)
// One CTA per row: a vectorized amax pass, then the conversion pass (the row is still in
// L1 / L2).  The GEMM epilogue multiplies its accumulators by s_r and the weight row scale.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rkt {

namespace {

__global__ void __launch_bounds__(256) quantize_rows_fp8_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K,
                                                                uint8_t* __restrict__ out, int ldo,
                                                                float* __restrict__ row_scale) {
  pdl_enter();
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)r * ldx;
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      amax = fmaxf(amax, fabsf(__uint_as_float(w[i] << 16)));
      amax = fmaxf(amax, fabsf(__uint_as_float(w[i] & 0xffff0000u)));
    }
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  const float s = m > 0.f ? m / 448.f : 1.f;
  if (threadIdx.x == 0) row_scale[r] = s;
  uint8_t* orow = out + (size_t)r * ldo;
  for (int c = threadIdx.x * 8; c < K; c += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[2];
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
      const float2 a = make_float2(__uint_as_float(w[i] << 16) / s, __uint_as_float(w[i] & 0xffff0000u) / s);
      const float2 b = make_float2(__uint_as_float(w[i + 1] << 16) / s, __uint_as_float(w[i + 1] & 0xffff0000u) / s);
      const uint32_t lo = (uint32_t)__nv_cvt_float2_to_fp8x2(a, __NV_SATFINITE, __NV_E4M3);
      const uint32_t hi = (uint32_t)__nv_cvt_float2_to_fp8x2(b, __NV_SATFINITE, __NV_E4M3);
      o[i / 2] = lo | (hi << 16);
    }
    *reinterpret_cast<uint2*>(orow + c) = make_uint2(o[0], o[1]);
  }
}

}  // namespace

int launch_quantize_rows_fp8(const __nv_bfloat16* x, int ldx, int K, uint8_t* out, int ldo, float* row_scale, int rows,
                             cudaStream_t st) {
  if (rows == 0) return 0;
  if (K % 8 || ldx % 8 || ldo % 8) return -2;
  launch_pdl(quantize_rows_fp8_kernel, dim3(rows), dim3(256), 0, st, x, ldx, K, out, ldo, row_scale);
  return (int)cudaGetLastError();
}

}  // namespace rkt
