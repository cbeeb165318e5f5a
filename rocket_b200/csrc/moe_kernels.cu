// MoE routing, dispatch layout, NVFP4 activation quantization and combine.
//
// Reference counterparts: moe_router_kernel (engines/glm5-moe-nvfp4-2b/src/
// kernels.cu:931, sigma+bias top-8 serial on one thread), nvfp4_quantize_rows_kernel
// (:1048), moe_gather_rows / moe_scatter_add (:1104-1137, deterministic
// ascending-order accumulation).  Here routing is one warp per token, the
// per-expert layout is built on the device (no host round trip per layer, unlike
// src/model.cu:1976-1980), and the combine sums each token's k rows in slot
// order so the result does not depend on where rows landed in a segment.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"
#include "rownorm.cuh"

namespace rkt {

// ---------------------------------------------------------------- router
// logits [T, ld] fp32 (first E columns real).  For sigmoid routing the
// selection uses sigmoid(l)+bias, the weight the unbiased sigmoid (GLM-style);
// softmax routing selects and weights by the softmax probability.
// Writes ids/weights [T, k_out] where k_out = top_k + n_shared: the shared
// experts are appended as pseudo-experts E.. with weight 1 (or the sigmoid of
// logit column `shared_gate_col` when >= 0).  counts[e] += 1 per assignment.
// Under expert parallelism only experts [e_lo, e_hi) are local: their ids are
// rebased to 0.., the shared experts follow them when `shared_local`, and every
// other slot gets id -1 (skipped by dispatch and combine).
// One warp routes token `warp` (all 32 lanes call it); `counts` may be global or shared.
// Lane l holds experts l, l+32, ... in registers (every loop unrolled, no local memory)
// and keeps its own best remaining candidate; a selection round is one warp max of the
// order-preserving integer keys, one warp min of the tied expert ids (ties go to the
// lower id), and a rescan by the winning lane only.
__device__ __forceinline__ uint32_t route_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // monotone in x
}

__device__ __forceinline__ void route_token(int warp, int lane, const float* __restrict__ logits, int ld, int E,
                                            int top_k, int n_shared, int sigmoid_mode, int norm_topk, float scaling,
                                            const float* __restrict__ bias, int shared_gate_col, int e_lo, int e_hi,
                                            int shared_local, int* __restrict__ ids, float* __restrict__ weights,
                                            int* counts) {
  const float* l = logits + (size_t)warp * ld;
  constexpr int MAXV = 16;  // E <= 512
  // slots i with 32 * i >= E are empty for the whole warp: every loop stops there (a
  // warp-uniform branch), so 160 experts cost 5 slots per lane, not 16
  float score[MAXV], prob[MAXV];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (32 * i >= E) break;
    const int e = lane + 32 * i;
    const float x = e < E ? l[e] : -INFINITY;
    prob[i] = x;
    mx = fmaxf(mx, x);
  }
  if (!sigmoid_mode) {
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (32 * i >= E) break;
      const int e = lane + 32 * i;
      prob[i] = e < E ? __expf(prob[i] - mx) : 0.f;
      sum += prob[i];
    }
    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (32 * i >= E) break;
      prob[i] /= sum;
      score[i] = prob[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (32 * i >= E) break;
      const int e = lane + 32 * i;
      if (e < E) {
        prob[i] = 1.f / (1.f + __expf(-prob[i]));
        score[i] = prob[i] + (bias ? bias[e] : 0.f);
      } else {
        prob[i] = score[i] = 0.f;
      }
    }
  }
  // this lane's best remaining candidate (key 0: none)
  uint32_t taken = 0, key = 0;
  int slot = 0;
  auto rescan = [&]() {
    key = 0;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (32 * i >= E) break;
      const uint32_t k = route_key(score[i]);
      if (lane + 32 * i < E && !((taken >> i) & 1u) && k > key) {
        key = k;
        slot = i;
      }
    }
  };
  rescan();
  const int k_out = top_k + n_shared;
  float wsum = 0.f;
  float my_w = 0.f;
  int my_id = -1;
  for (int j = 0; j < top_k; ++j) {
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
    const uint32_t bi = __reduce_min_sync(0xffffffffu, (key == kmax && key) ? (uint32_t)(lane + 32 * slot) : 0xffffffffu);
    const int owner = (int)(bi & 31u);
    float w = 0.f;
    if (lane == owner) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        if (32 * i >= E) break;
        if (i == slot) w = prob[i];
      }
      taken |= 1u << slot;
      rescan();
    }
    w = __shfl_sync(0xffffffffu, w, owner);
    wsum += w;
    if (lane == j) {
      my_w = w;
      my_id = (int)bi;
    }
  }
  if (lane < top_k) {
    float w = my_w;
    if (norm_topk) w = w / wsum;
    w *= scaling;
    // expert parallelism: this rank owns experts [e_lo, e_hi); others become -1
    const int local = (my_id >= e_lo && my_id < e_hi) ? my_id - e_lo : -1;
    ids[(size_t)warp * k_out + lane] = local;
    weights[(size_t)warp * k_out + lane] = w;
    if (local >= 0) atomicAdd(&counts[local], 1);
  } else if (lane < k_out) {
    const int s = lane - top_k;
    float w = 1.f;
    if (shared_gate_col >= 0) w = 1.f / (1.f + __expf(-l[shared_gate_col]));
    const int local = shared_local ? (e_hi - e_lo) + s : -1;  // shared experts follow the local ones
    ids[(size_t)warp * k_out + lane] = local;
    weights[(size_t)warp * k_out + lane] = w;
    if (local >= 0) atomicAdd(&counts[local], 1);
  }
}


__global__ void router_topk_kernel(const float* __restrict__ logits, int ld, int T, int E, int top_k, int n_shared,
                                   int sigmoid_mode, int norm_topk, float scaling, const float* __restrict__ bias,
                                   int shared_gate_col, int e_lo, int e_hi, int shared_local,
                                   int* __restrict__ ids, float* __restrict__ weights, int* __restrict__ counts) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  route_token(warp, lane, logits, ld, E, top_k, n_shared, sigmoid_mode, norm_topk, scaling, bias, shared_gate_col,
              e_lo, e_hi, shared_local, ids, weights, counts);
}

// ---------------------------------------------------------------- plan
// One CTA.  From counts[E_tot] build segment offsets aligned to the tile's
// scale-atom height (32 rows for bn<=32, else 128), reset the
// dispatch cursors, build the GEMM block list for token tile `bn`, and zero
// the counts for the next use.
// One thread per expert (E_tot <= 1024): segment sizes (aligned to the token tile's
// scale-atom height) and block counts, exclusive prefix sums by warp shuffles plus a
// second-level scan of the warp totals, then each expert writes its own entries.
// Thread e (one per expert, blockDim >= E_tot) plans from `counts`: shared memory, or
// global (`zero`) when it also clears its count for the next router launch.
__device__ __forceinline__ void plan_experts(int* counts, bool zero, int E_tot, int bn, int* __restrict__ offsets,
                                             int* __restrict__ cursor, int* __restrict__ blk_expert,
                                             int* __restrict__ blk_row, int* __restrict__ blk_valid,
                                             int* __restrict__ num_blocks, int max_blocks,
                                             int* __restrict__ total_rows) {
  __shared__ int w_rows[32], w_blks[32];
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  const int align = bn <= 32 ? 32 : 128;
  // global counts are read and cleared for the next router launch in one atomic (they were
  // accumulated by other CTAs' atomics, which live in L2)
  const int cnt = e < E_tot ? (zero ? atomicExch(&counts[e], 0) : counts[e]) : 0;
  const int sz = (cnt + align - 1) / align * align;
  const int nb = (cnt + bn - 1) / bn;
  int a = sz, b = nb;  // inclusive scans within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
    if (lane >= o) {
      a += x;
      b += y;
    }
  }
  if (lane == 31) {
    w_rows[warp] = a;
    w_blks[warp] = b;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int x = lane < nw ? w_rows[lane] : 0, y = lane < nw ? w_blks[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, x, o), v = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) {
        x += u;
        y += v;
      }
    }
    w_rows[lane] = x;
    w_blks[lane] = y;
  }
  __syncthreads();
  const int off = (warp ? w_rows[warp - 1] : 0) + a - sz;  // exclusive
  const int boff = (warp ? w_blks[warp - 1] : 0) + b - nb;
  if (e < E_tot) {
    offsets[e] = off;
    cursor[e] = off;
    for (int i = 0; i < nb; ++i) {
      const int bi = boff + i;
      if (bi < max_blocks) {
        blk_expert[bi] = e;
        blk_row[bi] = off + i * bn;
        blk_valid[bi] = min(bn, cnt - i * bn);
      }
    }
  }
  if (e == E_tot - 1) {
    offsets[E_tot] = off + sz;
    *num_blocks = min(boff + nb, max_blocks);
    *total_rows = off + sz;
  }
}


__global__ void __launch_bounds__(1024) moe_plan_kernel(int* __restrict__ counts, int E_tot, int bn,
                                                        int* __restrict__ offsets, int* __restrict__ cursor,
                                                        int* __restrict__ blk_expert, int* __restrict__ blk_row,
                                                        int* __restrict__ blk_valid, int* __restrict__ num_blocks,
                                                        int max_blocks, int* __restrict__ total_rows) {
  pdl_enter();
  plan_experts(counts, true, E_tot, bn, offsets, cursor, blk_expert, blk_row, blk_valid, num_blocks, max_blocks,
               total_rows);
}

// Router top-k and plan in one launch: one token per warp over ceil(T / warps) CTAs, the
// per-expert counts accumulated by global atomics; the last CTA to finish (an atomic
// ticket after a fence) builds the segments and the block list from the counts and clears
// them and the ticket for the next launch.  Routing spreads over T / warps SMs instead of
// one, and no second launch or global count round trip through the host is needed.
__global__ void __launch_bounds__(1024) router_plan_kernel(
    const float* __restrict__ logits, int ld, int T, int E, int top_k, int n_shared, int sigmoid_mode, int norm_topk,
    float scaling, const float* __restrict__ bias, int shared_gate_col, int e_lo, int e_hi, int shared_local,
    int* __restrict__ ids, float* __restrict__ weights, int* __restrict__ counts, int* __restrict__ ticket, int E_tot,
    int bn, int* __restrict__ offsets, int* __restrict__ cursor, int* __restrict__ blk_expert,
    int* __restrict__ blk_row, int* __restrict__ blk_valid, int* __restrict__ num_blocks, int max_blocks,
    int* __restrict__ total_rows) {
  pdl_enter();
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t < T)
    route_token(t, lane, logits, ld, E, top_k, n_shared, sigmoid_mode, norm_topk, scaling, bias, shared_gate_col,
                e_lo, e_hi, shared_local, ids, weights, counts);
  __syncthreads();  // this CTA's count atomics are issued
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) *ticket = 0;
  plan_experts(counts, true, E_tot, bn, offsets, cursor, blk_expert, blk_row, blk_valid, num_blocks, max_blocks,
               total_rows);
}

// ---------------------------------------------------------------- recount
// counts[e] = number of entries of ids[0, n) equal to e, for e < E_tot (entries
// outside [0, E_tot) are skipped).  Used when routing ids were rewritten after
// the router ran (streamed experts map local expert ids onto device slots), so
// the plan's segment sizes follow the rewritten ids.  One CTA, shared-memory
// histogram, so no separate zeroing launch is needed.
__global__ void __launch_bounds__(1024) moe_recount_kernel(const int* __restrict__ ids, int n, int E_tot,
                                                           int* __restrict__ counts) {
  pdl_enter();
  __shared__ int h[1024];
  for (int e = threadIdx.x; e < E_tot; e += blockDim.x) h[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E_tot) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E_tot; e += blockDim.x) counts[e] = h[e];
}

// ---------------------------------------------------------------- NVFP4 quantize
__device__ __forceinline__ uint32_t e2m1_code(float q) {
  const float a = fabsf(q);
  uint32_t c = 0;
  c = a > 0.25f ? 1u : c;
  c = a >= 0.75f ? 2u : c;
  c = a > 1.25f ? 3u : c;
  c = a >= 1.75f ? 4u : c;
  c = a > 2.5f ? 5u : c;
  c = a >= 3.5f ? 6u : c;
  c = a > 5.0f ? 7u : c;
  return c | ((q < 0.f && c) ? 8u : 0u);
}

__device__ __forceinline__ float e4m3_round(float x, uint8_t* bits) {
  __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
  *bits = (uint8_t)b;
  __half_raw h = __nv_cvt_fp8_to_halfraw(b, __NV_E4M3);
  return __half2float(*reinterpret_cast<__half*>(&h));
}

// Scale atoms cover `sf_rows` (32 or 128) consecutive rows; in-atom byte
// (r % 32) * 16 + (r / 32) * 4 + s.
__device__ __forceinline__ size_t sf_atom_offset(int row, int sfi, int k_atoms, int sf_rows) {
  const int ar = row / sf_rows, r = row % sf_rows;
  return ((size_t)ar * k_atoms + (sfi >> 2)) * 512 + (size_t)((r & 31) * 16 + (r >> 5) * 4 + (sfi & 3));
}

// One CTA of 128 threads per source row.  Quantizes row x[src] (bf16, K) with
// a per-row tensor scale amax/2688 and writes it to `ncopy` destination rows:
//   mode 0: dst = src (identity layout)
//   mode 1: dst = pos[src] (row list, e.g. the GEMM1 output rows of assignments)
//   mode 2: dispatch: for j < ncopy, e = ids[src*ncopy+j]; dst = atomicAdd(cursor[e]);
//           pos[src*ncopy+j] = dst; row_weight[dst] = weights[src*ncopy+j];
//           row_meta[dst] = src << 8 | j (when given: the inverse map the combine push reads)
//   mode 3: weights: dst = src, tensor scale g_in[src / rows_per_g] instead of the row amax
// NT threads per row CTA: 128 with MAXB blocks per thread (prefill, many rows), or one
// 16-value block per thread (NT >= K / 16) when few rows must fill the GPU (decode)
template <int MAXB, int NT>
__global__ void __launch_bounds__(NT) quantize_nvfp4_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K,
                                                              int mode, int ncopy, const int* __restrict__ ids,
                                                              const float* __restrict__ weights,
                                                              int* __restrict__ cursor, int* __restrict__ pos,
                                                              uint8_t* __restrict__ packed, uint8_t* __restrict__ sf,
                                                              float* __restrict__ row_scale,
                                                              float* __restrict__ row_weight, int sf_rows,
                                                              const float* __restrict__ g_in, int rows_per_g,
                                                              int* __restrict__ row_meta) {
  pdl_enter();
  const int a = blockIdx.x;  // source row (mode 0/2/3) or assignment (mode 1)
  const int src = a;
  if (mode == 1 && pos[a] < 0) return;  // assignment owned by another rank
  const __nv_bfloat16* xr = x + (size_t)(mode == 1 ? pos[a] : src) * ldx;
  const int nblk = K / 16;
  // dispatch: the copy threads' expert ids and weights load alongside the row, and their
  // destination rows are claimed while the row's amax is reduced (a decode CTA otherwise
  // waited on row -> ids -> cursor one after another)
  int e_copy = -1;
  float w_copy = 0.f;
  if (mode == 2 && threadIdx.x < ncopy) {
    e_copy = ids[(size_t)src * ncopy + threadIdx.x];
    if (row_weight) w_copy = weights[(size_t)src * ncopy + threadIdx.x];
  }
  float v[MAXB][16];
  float bam[MAXB];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXB; ++i) {
    const int b = threadIdx.x + i * NT;
    bam[i] = 0.f;
    if (b < nblk) {
      const uint4* p4 = reinterpret_cast<const uint4*>(xr + b * 16);
      uint4 u0 = p4[0], u1 = p4[1];
      uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][2 * j] = bf16_bits_to_float(w[j] & 0xffff);
        v[i][2 * j + 1] = bf16_bits_to_float(w[j] >> 16);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) bam[i] = fmaxf(bam[i], fabsf(v[i][j]));
      amax = fmaxf(amax, bam[i]);
    }
  }
  __shared__ int dst_sh[16];
  int d_mine = -1;
  if (threadIdx.x < ncopy) {
    int d;
    if (mode == 2) {
      d = e_copy >= 0 ? atomicAdd(&cursor[e_copy], 1) : -1;
      pos[(size_t)src * ncopy + threadIdx.x] = d;
      if (row_weight && d >= 0) row_weight[d] = w_copy;
      if (row_meta && d >= 0) row_meta[d] = (src << 8) | (int)threadIdx.x;  // row -> (token, slot)
    } else if (mode == 1) {
      d = pos[a];
    } else {
      d = src;
    }
    dst_sh[threadIdx.x] = d;
    d_mine = d;
  }
  __shared__ float red[NT / 32];
  for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();  // also publishes dst_sh
  amax = red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) amax = fmaxf(amax, red[w]);  // a max: any order
  float g = amax > 0.f ? amax / 2688.0f : 1.0f;
  if (mode == 3) g = g_in[a / rows_per_g];  // weights: caller's tensor scale
  if (row_scale && d_mine >= 0) row_scale[d_mine] = g;
  const int K_atoms = K / 64;
#pragma unroll
  for (int i = 0; i < MAXB; ++i) {
    const int b = threadIdx.x + i * NT;
    if (b < nblk) {
      uint8_t sbits;
      const float s = e4m3_round(bam[i] / 6.0f / g, &sbits);
      const float denom = s * g;
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t c0 = denom > 0.f ? e2m1_code(__fdiv_rn(v[i][2 * j], denom)) : 0u;
        const uint32_t c1 = denom > 0.f ? e2m1_code(__fdiv_rn(v[i][2 * j + 1], denom)) : 0u;
        const uint32_t byte = c0 | (c1 << 4);
        if (j < 4) lo |= byte << (8 * j);
        else hi |= byte << (8 * (j - 4));
      }
      for (int c = 0; c < ncopy; ++c) {
        const int d = dst_sh[c];
        if (d < 0) continue;
        uint2* dp = reinterpret_cast<uint2*>(packed + (size_t)d * (K / 2) + b * 8);
        *dp = make_uint2(lo, hi);
        sf[sf_atom_offset(d, b, K_atoms, sf_rows)] = sbits;
      }
    }
  }
}

// ---------------------------------------------------------------- combine
// out[t] = (residual[t]) + sum_j y[pos[t*k+j]] * (apply_w ? w[t*k+j] : 1), slot order.
// out[t] = residual[t] + sum_j w[t][j] * y[pos[t][j]] in slot order j (deterministic).
// grid (tokens, column blocks of 8*blockDim): each thread owns 8 consecutive columns.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int ldy, const int* __restrict__ pos,
                                   const float* __restrict__ w, int k, int D, const __nv_bfloat16* __restrict__ residual,
                                   __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int t = blockIdx.x;
  __shared__ int p_sh[32];
  __shared__ float w_sh[32];
  if (threadIdx.x < k) {
    p_sh[threadIdx.x] = pos[(size_t)t * k + threadIdx.x];
    w_sh[threadIdx.x] = w ? w[(size_t)t * k + threadIdx.x] : 1.f;
  }
  __syncthreads();
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= D) return;
  float acc[8];
  if (residual) {
    const uint4 r = *reinterpret_cast<const uint4*>(residual + (size_t)t * D + c);
    const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] = __uint_as_float(rw[i] << 16);
      acc[2 * i + 1] = __uint_as_float(rw[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  }
  float s[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i] = 0.f;
  // explicit fma chain in slot order (the fused landing kernel repeats it bit for bit)
  rn_slot_fma(y, ldy, p_sh, w_sh, k, c, s);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(__fadd_rn(acc[2 * i], s[2 * i]), __fadd_rn(acc[2 * i + 1], s[2 * i + 1]));
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * D + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// moe_combine_kernel's row (residual + the slot fma chain, in the same order) followed by
// the next sub-layer's RMSNorm of the stored bf16 row: one CTA per token row, one 8-column
// chunk per thread, the row staged in shared memory for the norm (rn_inv_staged).
__global__ void __launch_bounds__(1024) moe_combine_norm_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy, const int* __restrict__ pos, const float* __restrict__ w, int k,
    int D, const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out,
    const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ norm_out, int ld_norm, float eps,
    int zero_centered) {
  pdl_enter();
  const int t = blockIdx.x;
  __shared__ int p_sh[32];
  __shared__ float w_sh[32];
  __shared__ uint4 sx[1024];
  __shared__ float red[32];
  if (threadIdx.x < k) {
    p_sh[threadIdx.x] = pos[(size_t)t * k + threadIdx.x];
    w_sh[threadIdx.x] = w ? w[(size_t)t * k + threadIdx.x] : 1.f;
  }
  __syncthreads();
  const int nch = D >> 3;
  const int ch = threadIdx.x;
  if (ch < nch) {
    const int c = ch * 8;
    float acc[8];
    if (residual) {
      const uint4 r = *reinterpret_cast<const uint4*>(residual + (size_t)t * D + c);
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = rn_lo(rw[i]);
        acc[2 * i + 1] = rn_hi(rw[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = 0.f;
    rn_slot_fma(y, ldy, p_sh, w_sh, k, c, s);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h =
          __floats2bfloat162_rn(__fadd_rn(acc[2 * i], s[2 * i]), __fadd_rn(acc[2 * i + 1], s[2 * i + 1]));
      o[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    sx[ch] = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(out + (size_t)t * D + c) = sx[ch];
  }
  __syncthreads();
  const float inv = rn_inv_staged(sx, nch, red, D, eps);
  if (ch < nch)
    reinterpret_cast<uint4*>(norm_out + (size_t)t * ld_norm)[ch] =
        rn_chunk_out(sx[ch], reinterpret_cast<const uint4*>(norm_w)[ch], inv, zero_centered);
}

// ---------------------------------------------------------------- launchers
int launch_moe_combine_norm(const __nv_bfloat16* y, int ldy, const int* pos, const float* w, int k, int T, int D,
                            const __nv_bfloat16* residual, __nv_bfloat16* out, const __nv_bfloat16* norm_w,
                            __nv_bfloat16* norm_out, int ld_norm, float eps, int zero_centered, cudaStream_t st) {
  if (T == 0) return 0;
  if (k > 32 || D % 8 || ldy % 8 || D > 8 * 1024 || !norm_w || !norm_out) return -2;
  const int threads = ((D / 8 + 31) / 32) * 32;
  launch_pdl(moe_combine_norm_kernel, dim3(T), dim3(threads < 128 ? 128 : threads), 0, st, y, ldy, pos, w, k, D,
             residual, out, norm_w, norm_out, ld_norm, eps, zero_centered);
  return (int)cudaGetLastError();
}

int launch_router_topk(const float* logits, int ld, int T, int E, int top_k, int n_shared, int sigmoid_mode,
                       int norm_topk, float scaling, const float* bias, int shared_gate_col, int e_lo, int e_hi,
                       int shared_local, int* ids, float* weights, int* counts, cudaStream_t st) {
  if (E > 512 || top_k + n_shared > 32) return -2;
  const int warps_per_block = 4;
  launch_pdl(router_topk_kernel, dim3((T + warps_per_block - 1) / warps_per_block), dim3(32 * warps_per_block), 0, st, 
      logits, ld, T, E, top_k, n_shared, sigmoid_mode, norm_topk, scaling, bias, shared_gate_col, e_lo, e_hi,
      shared_local, ids, weights, counts);
  return (int)cudaGetLastError();
}

int launch_router_plan(const float* logits, int ld, int T, int E, int top_k, int n_shared, int sigmoid_mode,
                       int norm_topk, float scaling, const float* bias, int shared_gate_col, int e_lo, int e_hi,
                       int shared_local, int* ids, float* weights, int* counts, int* ticket, int E_tot, int bn,
                       int* offsets, int* cursor, int* blk_expert, int* blk_row, int* blk_valid, int* num_blocks,
                       int max_blocks, int* total_rows, cudaStream_t st) {
  if (E > 512 || top_k + n_shared > 32 || E_tot < 1 || E_tot > 1024 || T < 0) return -2;
  // one thread per expert in the planning CTA, at least 8 warps (tokens) per CTA
  const int threads = E_tot <= 256 ? 256 : (E_tot + 31) / 32 * 32;
  const int per = threads / 32;
  const int grid = T > 0 ? (T + per - 1) / per : 1;  // T == 0 still writes an empty plan
  launch_pdl(router_plan_kernel, dim3(grid), dim3(threads), 0, st, logits, ld, T, E, top_k, n_shared, sigmoid_mode,
             norm_topk, scaling, bias, shared_gate_col, e_lo, e_hi, shared_local, ids, weights, counts, ticket, E_tot,
             bn, offsets, cursor, blk_expert, blk_row, blk_valid, num_blocks, max_blocks, total_rows);
  return (int)cudaGetLastError();
}

int launch_moe_plan(int* counts, int E_tot, int bn, int* offsets, int* cursor, int* blk_expert, int* blk_row,
                    int* blk_valid, int* num_blocks, int max_blocks, int* total_rows, cudaStream_t st) {
  if (E_tot < 1 || E_tot > 1024) return -2;
  const int threads = (E_tot + 31) / 32 * 32;
  launch_pdl(moe_plan_kernel, dim3(1), dim3(threads), 0, st, counts, E_tot, bn, offsets, cursor, blk_expert, blk_row, blk_valid,
                                         num_blocks, max_blocks, total_rows);
  return (int)cudaGetLastError();
}

int launch_moe_recount(const int* ids, int n, int E_tot, int* counts, cudaStream_t st) {
  if (E_tot < 1 || E_tot > 1024 || n < 0) return -2;
  launch_pdl(moe_recount_kernel, dim3(1), dim3(1024), 0, st, ids, n, E_tot, counts);
  return (int)cudaGetLastError();
}

int launch_quantize_nvfp4(const __nv_bfloat16* x, int ldx, int rows, int K, int mode, int ncopy, const int* ids,
                          const float* weights, int* cursor, int* pos, uint8_t* packed, uint8_t* sf,
                          float* row_scale, float* row_weight, int sf_rows, const float* g_in, int rows_per_g,
                          int* row_meta, cudaStream_t st) {
  if (mode == 3 && (!g_in || rows_per_g <= 0)) return -2;
  if (sf_rows != 32 && sf_rows != 128) return -2;
  if (K % 64 || ncopy > 16 || rows <= 0) return rows == 0 ? 0 : -2;
  const int nblk = K / 16;
#define RKT_QUANT(MB, NTH) launch_pdl(quantize_nvfp4_kernel<MB, NTH>, dim3(rows), dim3(NTH), 0, st, x, ldx, K, mode, \
                                      ncopy, ids, weights, cursor, pos, packed, sf, row_scale, row_weight, sf_rows,    \
                                      g_in, rows_per_g, row_meta)
  if (rows < 2 * num_sms() && nblk > 128 && nblk <= 1024) {
    // few rows: one block per thread so each row's divisions run in parallel
    if (nblk <= 256) RKT_QUANT(1, 256);
    else if (nblk <= 512) RKT_QUANT(1, 512);
    else RKT_QUANT(1, 1024);
  } else if (nblk <= 128)
    RKT_QUANT(1, 128);
  else if (nblk <= 256)
    RKT_QUANT(2, 128);
  else if (nblk <= 512)
    RKT_QUANT(4, 128);
  else if (nblk <= 1024)
    RKT_QUANT(8, 128);
  else
    return -2;
#undef RKT_QUANT
  return (int)cudaGetLastError();
}

int launch_moe_combine(const __nv_bfloat16* y, int ldy, const int* pos, const float* w, int k, int T, int D,
                       const __nv_bfloat16* residual, __nv_bfloat16* out, cudaStream_t st) {
  if (T == 0) return 0;
  if (k > 32 || D % 8 || ldy % 8) return -2;
  const int threads = 128;
  launch_pdl(moe_combine_kernel, dim3(dim3(T, (D / 8 + threads - 1) / threads)), dim3(threads), 0, st, y, ldy, pos, w, k, D, residual,
                                                                                   out);
  return (int)cudaGetLastError();
}

}  // namespace rkt
