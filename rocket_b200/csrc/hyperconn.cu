// Manifold-constrained hyper-connections (mHC): HC parallel residual streams per
// token instead of one.  Around every sub-layer (attention / DeltaNet, MLP / MoE):
//
//   mix   = W_mix . rmsnorm(flatten(streams))               [2*HC + HC*HC]  (GEMM, ours)
//   pre_i = sigmoid(mix_i * s0 + b_i) + eps
//   post_i= 2 sigmoid(mix_{HC+i} * s1 + b_{HC+i})
//   comb  = row-softmax(mix_{2HC..} * s2 + b_{2HC..}) + eps, then Sinkhorn-Knopp
//           (columns once, then rows / columns for iters-1 rounds; +eps in every
//           denominator) -> doubly stochastic HC x HC
//   x     = sum_i pre_i * stream_i                          (sub-layer input)
//   y     = sub-layer(x)                                    (no residual add)
//   stream_i <- post_i * y + sum_j comb[j][i] * stream_j
//
// and the head reads the mean over streams.  The mix projection is a bf16 GEMM on
// the raw streams (the rms factor is a per-token scalar, applied here after the
// GEMM), so this file has only the memory-bound parts: one CTA per token for the
// split (sum of squares over HC*d, coefficients, collapse) and 8-column vector
// threads for the combine / broadcast / mean.
//
// Behavioural counterpart of the reference's hc_mix / hc_split / hc_combine /
// hc_head_mean kernels (engines/glm5-moe-nvfp4-2b/src/kernels.cu:205-318).
#include <cuda_bf16.h>

#include "kernels.h"

namespace rkt {

namespace {

__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

template <int HC>
__global__ void __launch_bounds__(256) hc_split_kernel(const __nv_bfloat16* __restrict__ streams,
                                                       const float* __restrict__ mix, int ld_mix,
                                                       const float* __restrict__ base, const float* __restrict__ scale,
                                                       float* __restrict__ coef, __nv_bfloat16* __restrict__ x, int d,
                                                       float norm_eps, float hc_eps, int iters) {
  constexpr int NC = HC + HC * HC;  // post + comb per token
  const int t = blockIdx.x;
  const __nv_bfloat16* s = streams + (size_t)t * HC * d;
  __shared__ float red[8];
  __shared__ float pre_sh[HC];
  // 1) sum of squares over the flattened streams
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < HC * d; c += blockDim.x * 8) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(s + c), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  // 2) coefficients (tiny: one thread)
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
    const float inv = rsqrtf(tot / (float)(HC * d) + norm_eps);
    const float* m = mix + (size_t)t * ld_mix;
    float* cf = coef + (size_t)t * NC;
    for (int i = 0; i < HC; ++i) pre_sh[i] = sigm(m[i] * inv * scale[0] + base[i]) + hc_eps;
    for (int i = 0; i < HC; ++i) cf[i] = 2.f * sigm(m[HC + i] * inv * scale[1] + base[HC + i]);
    float cm[HC][HC];
    for (int r = 0; r < HC; ++r) {
      float mx = -INFINITY;
      for (int c = 0; c < HC; ++c) {
        cm[r][c] = m[2 * HC + r * HC + c] * inv * scale[2] + base[2 * HC + r * HC + c];
        mx = fmaxf(mx, cm[r][c]);
      }
      float sum = 0.f;
      for (int c = 0; c < HC; ++c) {
        cm[r][c] = __expf(cm[r][c] - mx);
        sum += cm[r][c];
      }
      for (int c = 0; c < HC; ++c) cm[r][c] = cm[r][c] / sum + hc_eps;
    }
    for (int it = 0; it < iters; ++it) {
      if (it > 0) {
        for (int r = 0; r < HC; ++r) {
          float sum = 0.f;
          for (int c = 0; c < HC; ++c) sum += cm[r][c];
          for (int c = 0; c < HC; ++c) cm[r][c] /= (sum + hc_eps);
        }
      }
      for (int c = 0; c < HC; ++c) {
        float sum = 0.f;
        for (int r = 0; r < HC; ++r) sum += cm[r][c];
        for (int r = 0; r < HC; ++r) cm[r][c] /= (sum + hc_eps);
      }
    }
    for (int r = 0; r < HC; ++r)
      for (int c = 0; c < HC; ++c) cf[HC + r * HC + c] = cm[r][c];
  }
  __syncthreads();
  // 3) collapse: x = sum_i pre_i * stream_i
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(s + (size_t)i * d + c), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += pre_sh[i] * f[k];
    }
    *reinterpret_cast<uint4*>(x + (size_t)t * d + c) = pack8(acc);
  }
}

template <int HC>
__global__ void hc_combine_kernel(__nv_bfloat16* __restrict__ streams, const __nv_bfloat16* __restrict__ y,
                                  const float* __restrict__ coef, int d) {
  constexpr int NC = HC + HC * HC;
  const int t = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  __shared__ float cf[NC];
  if (threadIdx.x < NC) cf[threadIdx.x] = coef[(size_t)t * NC + threadIdx.x];
  __syncthreads();
  if (c >= d) return;
  __nv_bfloat16* s = streams + (size_t)t * HC * d;
  float yv[8], sv[HC][8];
  unpack8(*reinterpret_cast<const uint4*>(y + (size_t)t * d + c), yv);
#pragma unroll
  for (int j = 0; j < HC; ++j) unpack8(*reinterpret_cast<const uint4*>(s + (size_t)j * d + c), sv[j]);
#pragma unroll
  for (int i = 0; i < HC; ++i) {
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float a = cf[i] * yv[k];
#pragma unroll
      for (int j = 0; j < HC; ++j) a += cf[HC + j * HC + i] * sv[j][k];
      o[k] = a;
    }
    *reinterpret_cast<uint4*>(s + (size_t)i * d + c) = pack8(o);
  }
}

// mode 0: streams[t][i] = x[t] (embedding broadcast); mode 1: x[t] = mean_i streams[t][i]
template <int HC>
__global__ void hc_expand_mean_kernel(__nv_bfloat16* __restrict__ streams, __nv_bfloat16* __restrict__ x, int d,
                                      int mode) {
  const int t = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= d) return;
  __nv_bfloat16* s = streams + (size_t)t * HC * d;
  if (mode == 0) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)t * d + c);
#pragma unroll
    for (int i = 0; i < HC; ++i) *reinterpret_cast<uint4*>(s + (size_t)i * d + c) = v;
  } else {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(s + (size_t)i * d + c), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += f[k];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] *= 1.f / HC;
    *reinterpret_cast<uint4*>(x + (size_t)t * d + c) = pack8(acc);
  }
}

}  // namespace

int launch_hc_split(int hc, const __nv_bfloat16* streams, const float* mix, int ld_mix, const float* base,
                    const float* scale, float* coef, __nv_bfloat16* x, int T, int d, float norm_eps, float hc_eps,
                    int iters, cudaStream_t st) {
  if (T == 0) return 0;
  if (d % 8 || iters < 1) return -2;
  if (hc == 4)
    hc_split_kernel<4><<<T, 256, 0, st>>>(streams, mix, ld_mix, base, scale, coef, x, d, norm_eps, hc_eps, iters);
  else if (hc == 2)
    hc_split_kernel<2><<<T, 256, 0, st>>>(streams, mix, ld_mix, base, scale, coef, x, d, norm_eps, hc_eps, iters);
  else
    return -2;
  return (int)cudaGetLastError();
}

int launch_hc_combine(int hc, __nv_bfloat16* streams, const __nv_bfloat16* y, const float* coef, int T, int d,
                      cudaStream_t st) {
  if (T == 0) return 0;
  if (d % 8) return -2;
  const dim3 grid(T, (d / 8 + 127) / 128);
  if (hc == 4) hc_combine_kernel<4><<<grid, 128, 0, st>>>(streams, y, coef, d);
  else if (hc == 2) hc_combine_kernel<2><<<grid, 128, 0, st>>>(streams, y, coef, d);
  else return -2;
  return (int)cudaGetLastError();
}

int launch_hc_expand_mean(int hc, __nv_bfloat16* streams, __nv_bfloat16* x, int T, int d, int mode,
                          cudaStream_t st) {
  if (T == 0) return 0;
  if (d % 8) return -2;
  const dim3 grid(T, (d / 8 + 127) / 128);
  if (hc == 4) hc_expand_mean_kernel<4><<<grid, 128, 0, st>>>(streams, x, d, mode);
  else if (hc == 2) hc_expand_mean_kernel<2><<<grid, 128, 0, st>>>(streams, x, d, mode);
  else return -2;
  return (int)cudaGetLastError();
}

}  // namespace rkt
