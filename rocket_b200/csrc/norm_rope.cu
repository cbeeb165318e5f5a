// RMSNorm, per-head q/k norm + RoPE + paged KV write, embedding gather, and
// the greedy-token finalize after the fused lm_head argmax.
//
// Reference counterparts: rmsnorm_kernel (engines/glm5-moe-nvfp4-2b/src/
// kernels.cu:153), rms_kernel<Hidden,Fused> (engines/qwen38-flash-next-nvfp4-2b/
// src/norm/residual_rmsnorm.cu:93), DFlash2 rms_rope (src/dflash2_engine.cu:81),
// kv_write_latent_kernel (src/kernels.cu:534), embedding_kernel
// (qwen38 src/output/token_output.cu:26), argmax_kernel (src/kernels.cu:1218).
//
// KV page layout (per layer): K [pages][kv_heads][page][D] and V transposed
// [pages][kv_heads][D][page], so both attention MMAs read K-major tiles.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "rownorm.cuh"
#include "kernels.h"

namespace rkt {

// out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * (w or 1+w).  One CTA per row.
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ w,
                               int D, float eps, int zero_centered, __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_enter();
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)r * ldx;
  float ss = 0.f;
  for (int c = threadIdx.x * 2; c < D; c += blockDim.x * 2) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(xr + c);
    const float a = __bfloat162float(v.x), b = __bfloat162float(v.y);
    ss += a * a + b * b;
  }
  __shared__ float red[32];
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int off = 16; off; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)D + eps);
  for (int c = threadIdx.x * 2; c < D; c += blockDim.x * 2) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(xr + c);
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(w + c);
    float g0 = __bfloat162float(g.x), g1 = __bfloat162float(g.y);
    if (zero_centered) {
      g0 += 1.f;
      g1 += 1.f;
    }
    *reinterpret_cast<__nv_bfloat162*>(out + (size_t)r * ldo + c) =
        __floats2bfloat162_rn(__bfloat162float(v.x) * inv * g0, __bfloat162float(v.y) * inv * g1);
  }
}

// Vectorized variant for D % 8 == 0, D <= 8 * 128 * CPT: 128 threads, each holds up to CPT
// 16-byte chunks of the row in registers (one read of x), chunk c = thread + 128 k.
template <int CPT>
__global__ void __launch_bounds__(128) rmsnorm_vec_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                          const __nv_bfloat16* __restrict__ w, int D, float eps,
                                                          int zero_centered, __nv_bfloat16* __restrict__ out,
                                                          int ldo) {
  pdl_enter();
  const int r = blockIdx.x;
  const int nch = D >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)r * ldx);
  uint4 v[CPT];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int c = threadIdx.x + 128 * k;
    if (c < nch) {
      v[k] = xr[c];
      ss = rn_chunk_ss(v[k], ss);
    }
  }
  __shared__ float red[4];
  const float inv = rn_inv(ss, red, D, eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)r * ldo);
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int c = threadIdx.x + 128 * k;
    if (c < nch) orow[c] = rn_chunk_out(v[k], wr[c], inv, zero_centered);
  }
}

// qkv row layout: [q: Hq*D | gate: Hq*D (if has_gate) | k: Hkv*D | v: Hkv*D].
// One CTA per token; warp w handles heads w, w+nwarps, ...  Each head: optional
// RMSNorm over D (qk_norm), RoPE rotate-half on the first `rot` dims, then
// q -> q_out[t, h, :], k/v -> paged cache at slot_mapping[t].
template <int PER>
__global__ void qk_rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, int ld, int Hq, int Hkv, int rot,
                                  int has_gate, const int* __restrict__ positions, const float* __restrict__ inv_freq,
                                  const __nv_bfloat16* __restrict__ qn_w, const __nv_bfloat16* __restrict__ kn_w,
                                  float eps, int zero_centered, __nv_bfloat16* __restrict__ q_out,
                                  __nv_bfloat16* __restrict__ gate_out, void* __restrict__ k_cache,
                                  void* __restrict__ v_cache, const int* __restrict__ slot_mapping,
                                  int page_size, int kv_fp8, float k_inv, float v_inv, int v_here) {
  pdl_enter();
  constexpr int D = PER * 32;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const __nv_bfloat16* row = qkv + (size_t)t * ld;
  const int nheads = Hq + Hkv;  // q heads then k heads get norm+rope
  const int qw = Hq * (has_gate ? 2 : 1);
  const int total = nheads + Hkv + (has_gate ? Hq : 0);
  auto col_of = [&](int h) {
    return h < Hq ? h * D
         : h < nheads ? (qw + (h - Hq)) * D
         : h < nheads + Hkv ? (qw + Hkv + (h - nheads)) * D
                            : (Hq + (h - nheads - Hkv)) * D;  // gate head
  };
  // the first head's row and the slot load before the angles are computed: a decode CTA
  // then waits on one memory round trip instead of two (position -> angles -> row)
  const int h0 = blockIdx.y * nwarps + warp;
  float x[PER];
  if (h0 < total) {
#pragma unroll
    for (int i = 0; i < PER; ++i) x[i] = __bfloat162float(row[col_of(h0) + lane + 32 * i]);
  }
  const int slot = slot_mapping ? slot_mapping[t] : -1;
  const float pos = (float)positions[t];
  // the token's rotation angles, once per CTA (every head of the token shares them)
  __shared__ float sn_sh[D / 2], cs_sh[D / 2];
  for (int i = threadIdx.x; i < rot / 2; i += blockDim.x) sincosf(pos * inv_freq[i], &sn_sh[i], &cs_sh[i]);
  __syncthreads();
  const int page = slot >= 0 ? slot / page_size : 0, off = slot >= 0 ? slot % page_size : 0;
  // grid (tokens, head groups): one warp per head, so decode-sized batches still fill the GPU
  for (int h = h0; h < total; h += gridDim.y * nwarps) {
    const bool is_q = h < Hq;
    const bool is_k = h >= Hq && h < nheads;
    const bool is_v = h >= nheads && h < nheads + Hkv;
    if (h != h0) {
      const int col0 = col_of(h);
#pragma unroll
      for (int i = 0; i < PER; ++i) x[i] = __bfloat162float(row[col0 + lane + 32 * i]);
    }
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? qn_w : kn_w;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) ss += x[i] * x[i];
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          float g = __bfloat162float(nw[lane + 32 * i]);
          if (zero_centered) g += 1.f;
          // round to bf16 like a separate norm kernel's output would be
          x[i] = __bfloat162float(__float2bfloat16(x[i] * inv * g));
        }
      }
      // rotate-half over [0, rot): element e pairs with e +- rot/2.  Lane l holds elements
      // l + 32 i, so when rot/2 is a multiple of 32 the partner is in this lane's registers
      const int half = rot / 2;
      const bool local = (half & 31) == 0;
      float y[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        const int pe = e < half ? e + half : e - half;
        const int pi = (pe >> 5) & (PER - 1), pl = pe & 31;
        float partner = 0.f;
        if (local) {
#pragma unroll
          for (int j = 0; j < PER; ++j)
            if (j == pi) partner = x[j];
        } else {
#pragma unroll
          for (int j = 0; j < PER; ++j) {
            const float v = __shfl_sync(0xffffffffu, x[j], pl);
            if (j == pi) partner = v;
          }
        }
        if (e < rot) {
          const int fi = e < half ? e : e - half;
          const float s = sn_sh[fi], c = cs_sh[fi];
          y[i] = e < half ? x[i] * c - partner * s : x[i] * c + partner * s;
        } else {
          y[i] = x[i];
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) x[i] = y[i];
    }
    if (is_q) {
#pragma unroll
      for (int i = 0; i < PER; ++i) q_out[((size_t)t * Hq + h) * D + lane + 32 * i] = __float2bfloat16(x[i]);
    } else if (is_k) {
      if (slot >= 0) {
        const int kh = h - Hq;
        const size_t base = (((size_t)page * Hkv + kh) * page_size + off) * D;
        if (kv_fp8) {
          uint8_t* dst = static_cast<uint8_t*>(k_cache) + base;
#pragma unroll
          for (int i = 0; i < PER; ++i)
            dst[lane + 32 * i] = (uint8_t)__nv_cvt_float_to_fp8(x[i] * k_inv, __NV_SATFINITE, __NV_E4M3);
        } else {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(k_cache) + base;
#pragma unroll
          for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = __float2bfloat16(x[i]);
        }
      }
    } else if (is_v) {
      if (slot >= 0 && v_here) {
        const int vh = h - nheads;
        const size_t base = ((size_t)page * Hkv + vh) * D * page_size + off;
        if (kv_fp8) {
          uint8_t* dst = static_cast<uint8_t*>(v_cache) + base;
#pragma unroll
          for (int i = 0; i < PER; ++i)
            dst[(size_t)(lane + 32 * i) * page_size] =
                (uint8_t)__nv_cvt_float_to_fp8(x[i] * v_inv, __NV_SATFINITE, __NV_E4M3);
        } else {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(v_cache) + base;
#pragma unroll
          for (int i = 0; i < PER; ++i) dst[(size_t)(lane + 32 * i) * page_size] = __float2bfloat16(x[i]);
        }
      }
    } else if (gate_out) {
      const int gh = h - nheads - Hkv;
#pragma unroll
      for (int i = 0; i < PER; ++i) gate_out[((size_t)t * Hq + gh) * D + lane + 32 * i] = __float2bfloat16(x[i]);
    }
  }
}

// Paged V write of a prefill-sized batch: the cache holds V transposed per page
// ([page][kv head][D][page_size]), so one token's V row lands in D different 128-byte
// rows.  A CTA takes 64 consecutive tokens of one kv head through shared memory and
// each warp then writes rows d with lanes on consecutive tokens: neighbouring slots of a
// page become one contiguous run per warp store instead of D scattered 2-byte writes.
template <int D>
__global__ void __launch_bounds__(256) v_cache_tile_kernel(const __nv_bfloat16* __restrict__ qkv, int ld, int T,
                                                           int v_col0, int Hkv, const int* __restrict__ slot_mapping,
                                                           int page_size, void* __restrict__ v_cache, int kv_fp8,
                                                           float v_inv) {
  pdl_enter();
  constexpr int TT = 64;
  __shared__ __nv_bfloat16 tile[TT][D + 8];
  __shared__ int slot_sh[TT];
  const int t0 = blockIdx.x * TT, h = blockIdx.y;
  const int col = v_col0 + h * D;
  for (int i = threadIdx.x; i < TT * (D / 8); i += blockDim.x) {
    const int r = i / (D / 8), c = i % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t0 + r < T) v = *reinterpret_cast<const uint4*>(qkv + (size_t)(t0 + r) * ld + col + c * 8);
    *reinterpret_cast<uint4*>(&tile[r][c * 8]) = v;
  }
  if (threadIdx.x < TT) slot_sh[threadIdx.x] = t0 + (int)threadIdx.x < T ? slot_mapping[t0 + threadIdx.x] : -1;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int d = warp; d < D; d += 8) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = hf * 32 + lane;
      const int slot = slot_sh[r];
      if (slot < 0) continue;
      const int page = slot / page_size, off = slot % page_size;
      const size_t idx = (((size_t)page * Hkv + h) * D + d) * page_size + off;
      if (kv_fp8)
        static_cast<uint8_t*>(v_cache)[idx] =
            (uint8_t)__nv_cvt_float_to_fp8(__bfloat162float(tile[r][d]) * v_inv, __NV_SATFINITE, __NV_E4M3);
      else
        static_cast<__nv_bfloat16*>(v_cache)[idx] = tile[r][d];
    }
  }
}

__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int D,
                             int vocab_lo, int vocab_hi, __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool mine = id >= vocab_lo && id < vocab_hi;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(mine ? id - vocab_lo : 0) * D);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * D);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) dst[c] = mine ? src[c] : make_uint4(0, 0, 0, 0);
}

// (orderable value << 32 | ~id) -> id; also resets the key for the next step.
__global__ void argmax_finalize_kernel(unsigned long long* __restrict__ keys, int T, int* __restrict__ out_ids,
                                       float* __restrict__ out_vals) {
  pdl_enter();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const unsigned long long k = keys[t];
  out_ids[t] = (int)(~(uint32_t)(k & 0xffffffffu));
  if (out_vals) {
    uint32_t b = (uint32_t)(k >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    out_vals[t] = __uint_as_float(b);
  }
  keys[t] = 0ull;
}

int launch_rmsnorm(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int rows, int D, float eps,
                   int zero_centered, __nv_bfloat16* out, int ldo, cudaStream_t st) {
  if (rows == 0) return 0;
  if (D % 2) return -2;
  const bool vec = D % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && ((uintptr_t)x & 15) == 0 &&
                   ((uintptr_t)out & 15) == 0 && ((uintptr_t)w & 15) == 0;
  if (vec && D <= 8 * 128 * 2) launch_pdl(rmsnorm_vec_kernel<2>, dim3(rows), dim3(128), 0, st, x, ldx, w, D, eps, zero_centered, out, ldo);
  else if (vec && D <= 8 * 128 * 8) launch_pdl(rmsnorm_vec_kernel<8>, dim3(rows), dim3(128), 0, st, x, ldx, w, D, eps, zero_centered, out, ldo);
  else launch_pdl(rmsnorm_kernel, dim3(rows), dim3(D >= 2048 ? 512 : 256), 0, st, x, ldx, w, D, eps, zero_centered, out, ldo);
  return (int)cudaGetLastError();
}

int launch_qk_rope_kv(const __nv_bfloat16* qkv, int ld, int T, int Hq, int Hkv, int D, int rot, int has_gate,
                      const int* positions, const float* inv_freq, const __nv_bfloat16* qn_w,
                      const __nv_bfloat16* kn_w, float eps, int zero_centered, __nv_bfloat16* q_out,
                      __nv_bfloat16* gate_out, void* k_cache, void* v_cache, const int* slot_mapping,
                      int page_size, int kv_fp8, float k_scale, float v_scale, cudaStream_t st) {
  if (T == 0) return 0;
  if (rot > D || rot % 2) return -2;
  const int total = Hq + 2 * Hkv + (has_gate ? Hq : 0);
  const dim3 grid(T, (total + 7) / 8);  // 8 warps = 8 heads per block
  // prefill-sized batches write V through the tile transpose kernel (coalesced page rows)
  const int v_tiled = (T >= 256 && v_cache && slot_mapping) ? 1 : 0;
#define RKT_ROPE(P) launch_pdl(qk_rope_kv_kernel<P>, dim3(grid), dim3(256), 0, st, qkv, ld, Hq, Hkv, rot, has_gate, positions, inv_freq, \
      qn_w, kn_w, eps, zero_centered, q_out, gate_out, k_cache, v_cache, slot_mapping, page_size, kv_fp8, \
      1.f / k_scale, 1.f / v_scale, 1 - v_tiled)
  if (D == 64) RKT_ROPE(2);
  else if (D == 128) RKT_ROPE(4);
  else if (D == 256) RKT_ROPE(8);
  else return -2;
#undef RKT_ROPE
  if (v_tiled) {
    const int v_col0 = (Hq * (has_gate ? 2 : 1) + Hkv) * D;
    const dim3 vg((T + 63) / 64, Hkv);
#define RKT_VT(DD) launch_pdl(v_cache_tile_kernel<DD>, dim3(vg), dim3(256), 0, st, qkv, ld, T, v_col0, Hkv, slot_mapping, \
      page_size, v_cache, kv_fp8, 1.f / v_scale)
    if (D == 64) RKT_VT(64);
    else if (D == 128) RKT_VT(128);
    else RKT_VT(256);
#undef RKT_VT
  }
  return (int)cudaGetLastError();
}

int launch_embed(const int* ids, const __nv_bfloat16* table, int T, int D, int vocab_lo, int vocab_hi,
                 __nv_bfloat16* out, cudaStream_t st) {
  if (T == 0) return 0;
  if (D % 8) return -2;
  launch_pdl(embed_kernel, dim3(T), dim3(128), 0, st, ids, table, D, vocab_lo, vocab_hi, out);
  return (int)cudaGetLastError();
}

int launch_argmax_finalize(unsigned long long* keys, int T, int* out_ids, float* out_vals, cudaStream_t st) {
  if (T == 0) return 0;
  launch_pdl(argmax_finalize_kernel, dim3((T + 127) / 128), dim3(128), 0, st, keys, T, out_ids, out_vals);
  return (int)cudaGetLastError();
}

}  // namespace rkt
