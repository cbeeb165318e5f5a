// Landing kernel of the replicated-token multi-GPU decode path (models/ar_decode.py).
//
// Layout: every rank holds the residual rows of all T tokens.  Attention heads, the
// dense-MLP intermediate and the vocabulary are tensor parallel; routed experts are
// expert parallel.  Two kinds of collective end a sub-layer, and both are fused into
// the kernel that produces their data (gemm_sm100.cu epilogues):
//
//   all-reduce   (TP o_proj / dense down projection): EPI_AR_PUSH stores this rank's
//                bf16 partial rows into slot `rank` of every rank's buffer [world][T][d]
//   combine      (expert parallel MoE): EPI_COMBINE_ALL stores every expert output row
//                (token t, routing slot j) into comb[t][j] of every rank's buffer (the
//                exact layout, TP = 1); with TP > 1 moe_combine_push_kernel sums this
//                rank's slots first and pushes one partial row per token, an all-reduce
//
// and the last CTA of the producer publishes an epoch flag to every rank (comm.cuh).
// ar_land_kernel then waits for all ranks' epochs, sums the slots in a fixed order
// (ranks 0..N-1, or routing slots 0..k-1 with the fma chain of moe_combine_kernel),
// adds the residual, rounds to bf16 and, when a norm weight is given, applies the next
// sub-layer's RMSNorm with the shared row helpers (rownorm.cuh).  Every rank therefore
// lands identical bits and the replicated residual never diverges; with attention
// replicated (TP=1) a step reproduces the single-GPU step exactly.
//
// Two syncs per layer (attention all-reduce, MoE combine) replace the four of the
// sequence-parallel path; no dispatch all-to-all is needed because every rank already
// holds every token.  Only plain st.global reaches peer memory (from the GEMM epilogues)
// and only local memory is read here; waits are bounded (kWaitLimitNs) and report
// kErrPeerTimeout into the status word.
//
// Reference counterparts: the ExpertParallel row exchange with a host sync per MoE layer
// (engines/glm5-moe-nvfp4-2b/src/fabric/expert_parallel.h:51-130) and PairReduce's
// rank-ordered fp32 add (engines/qwen38-flash-next-nvfp4-2b/src/pair_reduce/
// pair_reduce.cu:53-190).  Here the exchange is inside the kernels, with no host step.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.cuh"
#include "common.cuh"
#include "fused_comm.h"
#include "rownorm.cuh"

namespace rkt {

// One CTA of 128 threads per token row t; thread i holds chunks i + 128 k (8 bf16 each).
template <int CPT>
__global__ void __launch_bounds__(128) ar_land_kernel(ArLandArgs a, PeerPtrs pp) {
  pdl_enter();
  const int t = blockIdx.x;
  const int D = a.d, nch = D >> 3;
  __shared__ float red[4];
  __shared__ bool ok_sh;
  if (threadIdx.x == 0) {
    ok_sh = true;
    if (a.wait_site >= 0) ok_sh = wait_peers(pp, a.wait_site, consumer_epoch(pp, a.wait_site), a.err);
  }
  __syncthreads();
  const bool ok = ok_sh;
  uint4 xv[CPT];
  float ss = 0.f;
  uint4* xrow = reinterpret_cast<uint4*>(a.x + (size_t)t * D);
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int c = threadIdx.x + 128 * k;
    if (c >= nch) continue;
    xv[k] = xrow[c];
    if (a.mode != LAND_NONE && ok) {
      const uint32_t u[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      float s[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i] = 0.f;
      if (a.mode == LAND_AR) {
        for (int r = 0; r < a.world; ++r) {
          const uint4 p = reinterpret_cast<const uint4*>(a.ar + ((size_t)r * a.ar_rows + t) * D)[c];
          const uint32_t q[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            s[2 * i] = __fadd_rn(s[2 * i], rn_lo(q[i]));
            s[2 * i + 1] = __fadd_rn(s[2 * i + 1], rn_hi(q[i]));
          }
        }
      } else {  // LAND_COMB: the fma chain of moe_combine_kernel, routing slots in order
        for (int j = 0; j < a.k_out; ++j) {
          const float wj = a.comb_w[(size_t)t * a.k_out + j];
          if (wj == 0.f) continue;
          const uint4 p = reinterpret_cast<const uint4*>(a.comb + ((size_t)t * a.k_out + j) * D)[c];
          const uint32_t q[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            s[2 * i] = __fmaf_rn(rn_lo(q[i]), wj, s[2 * i]);
            s[2 * i + 1] = __fmaf_rn(rn_hi(q[i]), wj, s[2 * i + 1]);
          }
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h =
            __floats2bfloat162_rn(__fadd_rn(rn_lo(u[i]), s[2 * i]), __fadd_rn(rn_hi(u[i]), s[2 * i + 1]));
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      xv[k] = make_uint4(o[0], o[1], o[2], o[3]);
      xrow[c] = xv[k];
    }
    ss = rn_chunk_ss(xv[k], ss);
  }
  if (a.norm_w) {
    const float inv = rn_inv(ss, red, D, a.eps);
    const uint4* wr = reinterpret_cast<const uint4*>(a.norm_w);
    uint4* orow = reinterpret_cast<uint4*>(a.xn + (size_t)t * D);
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      const int c = threadIdx.x + 128 * k;
      if (c < nch) orow[c] = rn_chunk_out(xv[k], wr[c], inv, a.zero_centered);
    }
  }
  if (a.wait_site >= 0 && last_block_done(arrival_counter(pp, a.wait_site)) && threadIdx.x == 0)
    consumer_commit(pp, a.wait_site, consumer_epoch(pp, a.wait_site));
}

// MoE combine + all-reduce push (tensor-parallel layout): row t of this rank's partial
// sum_j w[t][j] * y[pos[t][j]] over its local routing slots (the fma chain of
// moe_combine_kernel, slots in order; pos < 0 marks another rank's expert), rounded to
// bf16 and stored into slot `rank` of every rank's all-reduce buffer, so one row per
// token crosses NVLink instead of one per (token, slot).  The launch's last CTA publishes
// the epoch; ar_land_kernel (LAND_AR) sums the ranks in order.
// One CTA per token row with one 8-column chunk per thread (a single wave at decode sizes:
// each CTA pays one system-scope fence before the arrival count).
__global__ void __launch_bounds__(640) moe_combine_push_kernel(MoeCombinePushArgs a, PeerPtrs pp) {
  pdl_enter();
  const int t = blockIdx.x;
  __shared__ int p_sh[32];
  __shared__ float w_sh[32];
  if (threadIdx.x < a.k) {
    p_sh[threadIdx.x] = a.pos[(size_t)t * a.k + threadIdx.x];
    w_sh[threadIdx.x] = a.w[(size_t)t * a.k + threadIdx.x];
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < a.d; c += blockDim.x * 8) {
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = 0.f;
    rn_slot_fma(a.y, a.ldy, p_sh, w_sh, a.k, c, s);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(s[2 * i], s[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
    const uint64_t boff = a.ar_off + (((size_t)pp.rank * a.ar_rows + t) * a.d + c) * 2;
    for (int i = 0; i < pp.world; ++i) {
      const int rr = (pp.rank + i + (c >> 3)) % pp.world;  // spread the first store over the peers
      *reinterpret_cast<uint4*>(pp.base[rr] + boff) = ov;
    }
  }
  if (last_block_done(arrival_counter(pp, a.signal_site)) && threadIdx.x == 0) signal_peers(pp, a.signal_site);
}

int launch_moe_combine_push(const MoeCombinePushArgs& a, int peer_slot, int T, cudaStream_t st) {
  const PeerPtrs* pp = peer_get(peer_slot);
  if (!pp || a.d % 8 || a.ldy % 8 || a.k <= 0 || a.k > 32 || T < 0 || T > a.ar_rows || a.signal_site < 0 ||
      a.signal_site >= kSites)
    return -2;
  if (T == 0) return 0;
  const int threads = ((a.d / 8 + 31) / 32) * 32;
  launch_pdl(moe_combine_push_kernel, dim3(T), dim3(threads < 128 ? 128 : threads > 640 ? 640 : threads), 0, st, a,
             *pp);
  return (int)cudaGetLastError();
}

int launch_ar_land(const ArLandArgs& a, int peer_slot, int T, cudaStream_t st) {
  const PeerPtrs* pp = peer_get(peer_slot);
  if (!pp || a.d % 8 || a.d > 8 * 128 * 8 || T < 0) return -2;
  if (a.mode == LAND_AR && (!a.ar || a.world != pp->world || T > a.ar_rows)) return -2;
  if (a.mode == LAND_COMB && (!a.comb || !a.comb_w || a.k_out <= 0)) return -2;
  if (a.norm_w && !a.xn) return -2;
  if (T == 0) return 0;
  if (a.d <= 8 * 128 * 2)
    launch_pdl(ar_land_kernel<2>, dim3(T), dim3(128), 0, st, a, *pp);
  else
    launch_pdl(ar_land_kernel<8>, dim3(T), dim3(128), 0, st, a, *pp);
  return (int)cudaGetLastError();
}

}  // namespace rkt
