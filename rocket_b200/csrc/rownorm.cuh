// Row RMSNorm arithmetic shared by the plain norm kernel (norm_rope.cu) and the fused
// landing kernels (ar_comm.cu).
//
// One row of D bf16 values (D % 8 == 0) is held by a 128-thread CTA in 16-byte chunks,
// chunk c = threadIdx.x + 128 * k.  Every floating-point step is an explicit rounding
// intrinsic (no contraction left to the compiler), so two kernels that call these
// helpers on the same row produce the same bits.  The multi-GPU exact-parity mode relies
// on this: the landing kernel that follows a fused combine must normalise exactly as
// the single-GPU step does.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rkt {

__device__ __forceinline__ float rn_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float rn_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// ss + the squares of one chunk's 8 values, in element order
__device__ __forceinline__ float rn_chunk_ss(uint4 v, float ss) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = rn_lo(u[i]), b = rn_hi(u[i]);
    ss = __fadd_rn(ss, __fmaf_rn(a, a, __fmul_rn(b, b)));
  }
  return ss;
}

// 1 / rms of the row from the 128 threads' partial sums (`red`: 4 floats of shared memory;
// every thread of the CTA must call this)
__device__ __forceinline__ float rn_inv(float ss, float* red, int D, float eps) {
#pragma unroll
  for (int off = 16; off; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float tot = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
  return rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), eps));
}

// bf16(x * inv * g) for one chunk, g = w (or 1 + w for zero-centred weights)
__device__ __forceinline__ uint4 rn_chunk_out(uint4 v, uint4 g, float inv, int zero_centered) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float g0 = rn_lo(gw[i]), g1 = rn_hi(gw[i]);
    if (zero_centered) {
      g0 = __fadd_rn(g0, 1.f);
      g1 = __fadd_rn(g1, 1.f);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(rn_lo(u[i]), inv), g0),
                                                   __fmul_rn(__fmul_rn(rn_hi(u[i]), inv), g1));
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- one-chunk-per-thread row kernels (blockDim >= D / 8): the row's chunks are staged
// in shared memory and threads < 128 sum the squares in the 128-thread chunk order above,
// so the norm equals rmsnorm_vec_kernel's bit for bit.  `red` holds 32 floats.
__device__ __forceinline__ float rn_inv_staged(const uint4* sx, int nch, float* red, int D, float eps) {
  float ss = 0.f;
  if (threadIdx.x < 128)
    for (int c = threadIdx.x; c < nch; c += 128) ss = rn_chunk_ss(sx[c], ss);
  return rn_inv(ss, red, D, eps);
}

// s[0..7] += w_j * row_j[c..c+8) over the slots j < k in order (rows p[j] < 0 skipped),
// the loads issued four slots at a time ahead of their fma chain
__device__ __forceinline__ void rn_slot_fma(const __nv_bfloat16* __restrict__ y, int ldy, const int* p, const float* w,
                                            int k, int c, float* s) {
  for (int j0 = 0; j0 < k; j0 += 4) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u;
      v[u] = (j < k && p[j] >= 0) ? *reinterpret_cast<const uint4*>(y + (size_t)p[j] * ldy + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u;
      if (j >= k || p[j] < 0) continue;
      const uint32_t vw[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      const float wj = w[j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s[2 * i] = __fmaf_rn(rn_lo(vw[i]), wj, s[2 * i]);
        s[2 * i + 1] = __fmaf_rn(rn_hi(vw[i]), wj, s[2 * i + 1]);
      }
    }
  }
}

}  // namespace rkt
