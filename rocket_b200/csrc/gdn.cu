// Gated DeltaNet (Qwen3-Next style linear attention) on sm_100a.
//
//   gdn_conv_prep_kernel   causal depthwise conv (kernel 4) + SiLU over the q|k|v
//                          channels of one token, per-head L2 norm of q and k
//                          (q additionally scaled by 1/sqrt(Dk)), beta = sigmoid(b),
//                          g = -exp(A_log) * softplus(a + dt_bias)
//   gdn_conv_state_kernel  keeps the last (K-1) raw conv inputs of every sequence with
//                          more than one token (the prep kernel shifts one-token ones)
//   gdn_scan_kernel        the gated delta rule over a sequence's tokens of this
//                          step, one CTA per (sequence, v head, 32 state columns), four
//                          threads per state column held in registers (fp32):
//                              S = exp(g) S ;  u = v - S^T k ;  S += beta k u^T ;  o = S^T q
//   gdn_norm_kernel        the gated RMSNorm  o * rsqrt(mean(o^2)+eps) * w * silu(z)
//   gdn_step_one_token_kernel  scan + gated norm of a step whose every sequence has one
//                          token (decode), the four column blocks of a head in one cluster
//
// The same scan serves decode (one token) and chunked prefill (many tokens of a
// sequence, staged 32 at a time in shared memory).  Sequences of one step are
// independent CTAs.
//
// Reference counterparts: kda_step / step_split (engines/glm5-moe-nvfp4-2b/src/
// kernels.cu:420, bench/kda_step_dropin.cuh: FP32 128x128 state held in
// registers, no cross-thread reduction in the update), kda_conv_kernel (:321) and
// the Qwen GDN decode kernels causal_conv_update / recurrent_gdn / gated_rmsnorm
// (engines/qwen38-flash-next-nvfp4-2b/src/linear_attention/gdn_core.cu:56-151).
#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"

namespace rkt {

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// proj row layout (local shard): [q Hk*Dk | k Hk*Dk | v Hv*Dv | z Hv*Dv | b Hv | a Hv]
// conv channels are the first C = 2*Hk*Dk + Hv*Dv entries.
// conv_state [slots][K-1][C] bf16 holds the raw inputs of the previous K-1 positions.
//
// grid (T, C / 128), 128 threads: one head's 128 channels of one token, one channel
// per thread (all conv taps loaded before use), then the head's L2 norm as a block
// reduction.  Blocks of head 0 also compute the token's gates.
// KT: the conv kernel size when known at compile time (4 in every shipped config), 0 for
// the runtime a.conv_k (at most 9): runtime-bounded tap loops cost indirect branches.
template <int KT>
__global__ void __launch_bounds__(128, 16) gdn_conv_prep_kernel(GdnArgs a) {
  pdl_enter();
  constexpr int KM = KT ? KT : 9;  // tap loop bound
  constexpr int Dh = 128;          // head dim (the launcher requires Dk == Dv == 128)
  __shared__ float red[4];
  const int t = blockIdx.x, hb = blockIdx.y;
  const int c = hb * 128 + threadIdx.x;
  // one row per sequence (T == S, decode): row t is sequence t, and the index loads below
  // are independent of one another instead of a chain behind a search
  const bool one_row = (int)gridDim.x == a.n_seqs;
  int seq = t;
  if (!one_row) {
    // sequence of row t: the last s with q_start[s] <= t (rows are grouped by sequence in order)
    int lo = 0, hi = a.n_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.q_start[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    seq = lo;
  }
  const int q0 = one_row ? t : a.q_start[seq];
  const int pos0 = a.positions[q0];  // absolute position of the chunk's first token
  const int tl = t - q0;             // token index within the sequence's chunk
  const int slot = a.state_slot[seq];
  const int C = (2 * a.Hk + a.Hv) * Dh;
  const int K = KT ? KT : a.conv_k;
  const __nv_bfloat16* row = a.proj + (size_t)t * a.ld_proj;
  float xin[KM];
#pragma unroll
  for (int j = 0; j < KM; ++j) {
    if (j >= K) break;
    const int rel = tl - (K - 1) + j;  // input at relative position rel
    if (rel >= 0) {
      xin[j] = __bfloat162float(a.proj[(size_t)(q0 + rel) * a.ld_proj + c]);
    } else if (a.conv_state) {
      // from the saved state: slot row (K-1) + rel  (rel in [-(K-1), -1]); loaded before the
      // position is known, and dropped before the first token of the sequence
      const float sv = __bfloat162float(a.conv_state[((size_t)slot * (K - 1) + (K - 1) + rel) * C + c]);
      xin[j] = pos0 + rel >= 0 ? sv : 0.f;
    } else {
      xin[j] = 0.f;
    }
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < KM; ++j) {
    if (j >= K) break;
    acc += xin[j] * __bfloat162float(a.conv_w[(size_t)c * K + j]);
  }
  const float y = acc / (1.f + __expf(-acc));  // SiLU
  if (t < a.spec_rows) {
    a.rx[(size_t)t * C + c] = row[c];
  } else if (a.conv_state && (one_row || a.q_len[seq] == 1)) {
    // a one-token sequence: only this thread reads channel c of the slot's state, so it
    // shifts the window in place (new row j = input j + 1 of this token's taps)
    __nv_bfloat16* stc = a.conv_state + (size_t)slot * (K - 1) * C + c;
#pragma unroll
    for (int j = 0; j < KM - 1; ++j) {
      if (j >= K - 1) break;
      stc[(size_t)j * C] = __float2bfloat16(xin[j + 1]);
    }
  }
  const int i = threadIdx.x;
  if (hb < 2 * a.Hk) {
    // per-head L2 norm of q and k (q additionally scaled by 1/sqrt(Dk))
    float ss = y * y;
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    float inv = rsqrtf(red[0] + red[1] + red[2] + red[3] + 1e-6f);
    if (hb < a.Hk) {
      inv *= rsqrtf((float)Dh);
      a.q[((size_t)t * a.Hk + hb) * Dh + i] = y * inv;
    } else {
      const size_t o = ((size_t)t * a.Hk + (hb - a.Hk)) * Dh + i;
      a.k[o] = y * inv;
      if (t < a.spec_rows) a.rk[o] = y * inv;
    }
  } else {
    const size_t o = ((size_t)t * a.Hv + (hb - 2 * a.Hk)) * Dh + i;
    a.v[o] = y;
    if (t < a.spec_rows) a.rv[o] = y;
  }
  // gates, spread over the token's blocks: block hb computes gate entries [hb*128, hb*128+128)
  {
    const int boff = 2 * (a.Hk + a.Hv) * Dh;
    const int h = hb * 128 + i;
    if (h < a.Hv) {
      const float bb = __bfloat162float(row[boff + h]);
      const float beta = 1.f / (1.f + __expf(-bb));
      a.beta[(size_t)t * a.Hv + h] = beta;
      if (t < a.spec_rows) a.rb[(size_t)t * a.Hv + h] = beta;
      if (!a.gate_ch) {
        const float av = __bfloat162float(row[boff + a.Hv + h]);
        const float g = -__expf(a.A_log[h]) * softplus(av + a.dt_bias[h]);
        a.g[(size_t)t * a.Hv + h] = g;
        if (t < a.spec_rows) a.rg[(size_t)t * a.Hv + h] = g;
      }
    }
    if (a.gate_ch) {
      // per-channel log decay (KDA): g = lb * sigmoid(exp(A_log[h]) * (f + dt_bias))
      const int n = a.Hv * Dh;
      const int nb = gridDim.y;
      for (int e = hb * 128 + i; e < n; e += nb * 128) {
        const int he = e / Dh;
        const float f = __bfloat162float(row[boff + a.Hv + e]);
        const float g = a.gate_lb / (1.f + __expf(-__expf(a.A_log[he]) * (f + a.dt_bias[e])));
        a.g[(size_t)t * n + e] = g;
        if (t < a.spec_rows) a.rg[(size_t)t * n + e] = g;
      }
    }
  }
}

// Sequences with more than one token of this step: shift their last K-1 raw conv
// inputs into the state (one-token sequences were shifted by the prep kernel, verify
// sequences are shifted by the commit).  grid (sequences, C / 256), one channel per thread.
__global__ void __launch_bounds__(256) gdn_conv_state_kernel(GdnArgs a) {
  pdl_enter();
  const int seq = blockIdx.x;
  const int q0 = a.q_start[seq], ql = a.q_len[seq];
  if (q0 < a.spec_rows || ql <= 1) return;
  const int C = 2 * a.Hk * a.Dk + a.Hv * a.Dv;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int K1 = a.conv_k - 1;
  __nv_bfloat16* st = a.conv_state + (size_t)a.state_slot[seq] * K1 * C + c;
  const bool fresh = a.positions[q0] == 0;  // a new sequence has no history
  // only taps j < K1 exist: for j >= K1, rel would point past the sequence's last row
  float old[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, nw[8];
  if (!fresh) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= K1) break;
      old[j] = __bfloat162float(st[(size_t)j * C]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j >= K1) break;
    // new state row j = input at relative position ql - K1 + j (before the chunk: old row K1 + rel)
    const int rel = ql - K1 + j;
    float x = 0.f;
    if (rel >= 0) {
      x = __bfloat162float(a.proj[(size_t)(q0 + rel) * a.ld_proj + c]);
    } else {
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m == K1 + rel) x = old[m];
    }
    nw[j] = x;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j >= K1) break;
    st[(size_t)j * C] = __float2bfloat16(nw[j]);
  }
}

// The recurrent state of a (slot, v head) is stored column-major, [Dv][Dk]: column j
// (the key-dimension vector that produces output j) is contiguous.  Columns evolve
// independently under the delta rule, so the scan splits them over CTAs:
//
// grid (sequences, Hv, D / kScanCols), 4 * kScanCols threads.  Four consecutive threads
// own state column j, a quarter of its rows each (32 fp32 registers, 16-byte vector
// loads); their partial dot products meet with two shuffles.  The raw outputs o go to
// an fp32 scratch; gdn_norm_kernel applies the gated RMSNorm over each head's outputs.
constexpr int kScanCols = 32;
// BATCH: stage a chunk with all of a thread's loads issued before its stores (prefill /
// verify chunks, where the per-token chain waits on the staging); off for one-token
// steps, whose state streaming wants the smaller register footprint (occupancy)
template <int D, bool CH, bool BATCH>
__global__ void __launch_bounds__(4 * kScanCols) gdn_scan_kernel(GdnArgs a) {
  pdl_enter();
  constexpr int TB = CH ? 16 : 32;  // tokens staged per round (static shared memory <= 48 KB)
  constexpr int R = D / 4;
  __shared__ float ks[TB][D], qs[TB][D];
  __shared__ float gs[CH ? TB : 1][CH ? D : 1];  // per-channel decays exp(g) (KDA)
  __shared__ float gb[TB][2];
  __shared__ float vs[TB][kScanCols];  // this CTA's value columns of the staged tokens
  const int seq = blockIdx.x, h = blockIdx.y;
  const int j = blockIdx.z * kScanCols + (threadIdx.x >> 2), part = threadIdx.x & 3;
  const int q0 = a.q_start[seq], ql = a.q_len[seq];
  const int slot = a.state_slot[seq];
  const int hk = h / (a.Hv / a.Hk);
  // thread `part` of column j holds the 16-byte chunks part, part + 4, part + 8, ... of the
  // column: the four threads of a column read 64 contiguous bytes per load instruction
  float* col = a.state + (((size_t)slot * a.Hv + h) * D + j) * D;  // [Dv][Dk]
  const bool fresh = a.positions[q0] == 0;  // a new sequence starts from a zero state
  auto kidx = [&](int i) { return 4 * (part + 4 * (i >> 2)) + (i & 3); };  // element i -> k index
  float S[R];
#pragma unroll
  for (int i = 0; i < R; i += 4) {
    const float4 v = fresh ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(col + kidx(i));
    S[i] = v.x;
    S[i + 1] = v.y;
    S[i + 2] = v.z;
    S[i + 3] = v.w;
  }
  for (int t0 = 0; t0 < ql; t0 += TB) {
    const int nt = min(TB, ql - t0);
    __syncthreads();
    if constexpr (!BATCH) {
      for (int e = threadIdx.x; e < nt * D; e += blockDim.x) {
        const int u = e / D, i = e % D;
        const size_t tok = q0 + t0 + u;
        ks[u][i] = a.k[(tok * a.Hk + hk) * D + i];
        qs[u][i] = a.q[(tok * a.Hk + hk) * D + i];
        if constexpr (CH) gs[u][i] = __expf(a.g[(tok * a.Hv + h) * D + i]);
      }
      if (threadIdx.x < nt) {
        const size_t tok = q0 + t0 + threadIdx.x;
        gb[threadIdx.x][0] = CH ? 1.f : __expf(a.g[tok * a.Hv + h]);
        gb[threadIdx.x][1] = a.beta[tok * a.Hv + h];
      }
      for (int e = threadIdx.x; e < nt * kScanCols; e += blockDim.x) {
        const int u = e / kScanCols, c = e % kScanCols;
        vs[u][c] = a.v[((size_t)(q0 + t0 + u) * a.Hv + h) * D + blockIdx.z * kScanCols + c];
      }
    } else
    // stage the chunk's k, q (and per-channel decay) rows, gates and this CTA's value
    // columns: every thread issues all of its 16-byte loads before its first store, so a
    // chunk costs one memory round trip instead of one per loaded vector
    {
      constexpr int NT = 4 * kScanCols;                 // threads
      constexpr int V4 = TB * (D / 4) / NT;             // float4 per thread per row array
      float4 kr[V4], qr[V4], gr[CH ? V4 : 1];
#pragma unroll
      for (int r = 0; r < V4; ++r) {
        const int e4 = threadIdx.x + r * NT, u = e4 / (D / 4), i4 = e4 % (D / 4);
        if (u < nt) {
          const size_t tok = q0 + t0 + u;
          kr[r] = reinterpret_cast<const float4*>(a.k + (tok * a.Hk + hk) * D)[i4];
          qr[r] = reinterpret_cast<const float4*>(a.q + (tok * a.Hk + hk) * D)[i4];
          if constexpr (CH) gr[r] = reinterpret_cast<const float4*>(a.g + (tok * a.Hv + h) * D)[i4];
        }
      }
      constexpr int VV = TB * kScanCols / NT;           // value floats per thread
      float vr[VV];
#pragma unroll
      for (int r = 0; r < VV; ++r) {
        const int e = threadIdx.x + r * NT, u = e / kScanCols, c = e % kScanCols;
        if (u < nt) vr[r] = a.v[((size_t)(q0 + t0 + u) * a.Hv + h) * D + blockIdx.z * kScanCols + c];
      }
      float gdec = 0.f, gbeta = 0.f;
      if (threadIdx.x < nt) {
        const size_t tok = q0 + t0 + threadIdx.x;
        gdec = CH ? 0.f : a.g[tok * a.Hv + h];
        gbeta = a.beta[tok * a.Hv + h];
      }
#pragma unroll
      for (int r = 0; r < V4; ++r) {
        const int e4 = threadIdx.x + r * NT, u = e4 / (D / 4), i4 = e4 % (D / 4);
        if (u < nt) {
          *reinterpret_cast<float4*>(&ks[u][i4 * 4]) = kr[r];
          *reinterpret_cast<float4*>(&qs[u][i4 * 4]) = qr[r];
          if constexpr (CH)
            *reinterpret_cast<float4*>(&gs[u][i4 * 4]) =
                make_float4(__expf(gr[r].x), __expf(gr[r].y), __expf(gr[r].z), __expf(gr[r].w));
        }
      }
#pragma unroll
      for (int r = 0; r < VV; ++r) {
        const int e = threadIdx.x + r * NT, u = e / kScanCols, c = e % kScanCols;
        if (u < nt) vs[u][c] = vr[r];
      }
      if (threadIdx.x < nt) {
        gb[threadIdx.x][0] = CH ? 1.f : __expf(gdec);
        gb[threadIdx.x][1] = gbeta;
      }
    }
    __syncthreads();
    for (int u = 0; u < nt; ++u) {
      const size_t tok = q0 + t0 + u;
      const float decay = gb[u][0], beta = gb[u][1];
      const float vj = vs[u][threadIdx.x >> 2];
      // the staged rows are indexed as shared arrays (not through generic pointers), so the
      // loads are shared-memory loads off the long-latency path
#define kk(i) ks[u][i]
#define qq(i) qs[u][i]
#define gg(i) gs[CH ? u : 0][i]
      // four partial sums per dot product: the per-token dependency chain is what bounds a
      // long prefill (one sequence's tokens are sequential), so keep it short
      float vq[4] = {0.f, 0.f, 0.f, 0.f};
      if constexpr (CH) {
        // per-channel decay: the prediction reads the decayed state
#pragma unroll
        for (int i = 0; i < R; ++i) vq[i & 3] += gg(kidx(i)) * S[i] * kk(kidx(i));
      } else {
#pragma unroll
        for (int i = 0; i < R; ++i) vq[i & 3] += S[i] * kk(kidx(i));
      }
      float vp = (vq[0] + vq[1]) + (vq[2] + vq[3]);
      vp += __shfl_xor_sync(0xffffffffu, vp, 1);
      vp += __shfl_xor_sync(0xffffffffu, vp, 2);
      const float upd = beta * (vj - decay * vp);
      float oq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < R; ++i) {
        S[i] = (CH ? gg(kidx(i)) : decay) * S[i] + kk(kidx(i)) * upd;
        oq[i & 3] += S[i] * qq(kidx(i));
      }
      float o = (oq[0] + oq[1]) + (oq[2] + oq[3]);
      o += __shfl_xor_sync(0xffffffffu, o, 1);
      o += __shfl_xor_sync(0xffffffffu, o, 2);
      if (part == 0) a.o_raw[(tok * a.Hv + h) * D + j] = o;
#undef kk
#undef qq
#undef gg
    }
  }
  if (q0 < a.spec_rows) return;  // verify sequence: the state advances in the commit
#pragma unroll
  for (int i = 0; i < R; i += 4)
    *reinterpret_cast<float4*>(col + kidx(i)) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
}

// One-token steps (T == S: every sequence has exactly one row, row s of sequence s): the
// scan of gdn_scan_kernel for that token followed by the gated RMSNorm of
// gdn_norm_kernel, in one persistent launch.
//
// Clusters of D / kScanCols CTAs (the column blocks of one head), 4 * kScanCols threads
// each, four threads per state column as in the scan.  Cluster c takes the (sequence,
// head) items c, c + G, c + 2G, ... (G clusters, as many as fit at once).  The decode
// step is a stream of 16 KB state tiles, so each item's tile is copied into shared
// memory with cp.async while the previous item computes (two stages; every thread
// copies exactly the 16-byte chunks it later reads, laid out so that a warp's reads are
// contiguous), and the item's k, q, v, gates, slot and position are loaded into registers
// one item ahead.  After the update each CTA stores its state columns from registers and
// reduces the squares of its 32 outputs in one warp; the head's RMS needs every column
// block, so each CTA delivers its partial sum into every CTA of the cluster with st.async
// (distributed shared memory, completing on the receiver's mbarrier; two slots and
// barriers alternate between items).  No cluster-wide barrier or release fence sits in
// the loop: a release would wait for the previous item's state stores.  Warp 0 applies an
// item's gated norm one item later, when the partials have long arrived, so the other
// warps do not wait on the exchange.
//
// Bit-identical to gdn_scan_kernel + gdn_norm_kernel: the per-column arithmetic is the
// same sequence of operations, the warp reduction of column block b is the norm kernel's
// warp b, and the four partials are added in the same order.
struct GdnItemRegs {  // one item's per-thread inputs, loaded an item ahead
  float kv, qv, gv, graw, beta, vj;
  int slot, fresh;
};

template <int D, bool CH>
__device__ __forceinline__ GdnItemRegs gdn_item_regs(const GdnArgs& a, int it, int blk, int e, int jl) {
  GdnItemRegs r;
  const int seq = it / a.Hv, h = it % a.Hv;
  const size_t tok = seq;
  const int hk = h / (a.Hv / a.Hk);
  r.kv = a.k[(tok * a.Hk + hk) * D + e];
  r.qv = a.q[(tok * a.Hk + hk) * D + e];
  r.gv = CH ? a.g[(tok * a.Hv + h) * D + e] : 0.f;
  r.graw = CH ? 0.f : a.g[tok * a.Hv + h];
  r.beta = a.beta[tok * a.Hv + h];
  r.vj = a.v[(tok * a.Hv + h) * D + blk * kScanCols + jl];
  r.slot = a.state_slot[seq];
  r.fresh = a.positions[tok] == 0;  // a new sequence starts from a zero state
  return r;
}

template <int D, bool CH>
__global__ void __cluster_dims__(1, 1, D / kScanCols) __launch_bounds__(4 * kScanCols, 5)
gdn_step_one_token_kernel(GdnArgs a) {
  pdl_enter();
  constexpr int R = D / 4;
  constexpr int NT = 4 * kScanCols;
  constexpr int NB = D / kScanCols;  // column blocks (CTAs) of one head
  static_assert(NT == D, "one staged element per thread");
  __shared__ __align__(16) float4 sbuf[2][R / 4][NT];  // state tiles: chunk c of thread t at [c][t]
  __shared__ __align__(16) float ks[D];
  __shared__ __align__(16) float qs[D];
  __shared__ __align__(16) float gs[CH ? D : 1];
  __shared__ float os[kScanCols];
  __shared__ float redv[2][NB];               // the column blocks' partial sums, two items in flight
  __shared__ __align__(8) uint64_t mbar[2];  // completes when the NB partials of an item have landed
  const int blk = blockIdx.z, G = gridDim.x, items = a.n_seqs * a.Hv;
  const int e = threadIdx.x, jl = e >> 2, part = e & 3;
  const int j = blk * kScanCols + jl;
  auto kidx = [&](int i) { return 4 * (part + 4 * (i >> 2)) + (i & 3); };
  auto column = [&](int it, int slot) {  // this thread's state column of item `it`, [Dv][Dk]
    return a.state + (((size_t)slot * a.Hv + it % a.Hv) * D + j) * D;
  };
  auto copy_state = [&](int stage, const float* col) {
#pragma unroll
    for (int c = 0; c < R / 4; ++c) {
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&sbuf[stage][c][e]);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(col + kidx(4 * c)) : "memory");
    }
  };
  int it = blockIdx.x;
  if (it >= items) return;  // the whole cluster shares `it`
  if (e == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_barrier_init();
  }
  // every CTA's barriers are initialized before any partial is delivered
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  bool failed = false;
  // warp 0 finishes an item's gated norm one item later (when its partials have arrived):
  // the previous item's index and this lane's raw output
  int it_p = -1, n_done = 0;
  float ov_p = 0.f;
  auto finish = [&](int m, int itm, float ovm) -> bool {
    const int b = m & 1;
    if (!mbar_wait(&mbar[b], (m >> 1) & 1, a.err)) return false;  // no partials: skip the rest
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NB; ++w) tot += redv[b][w];
    const int seq = itm / a.Hv, h = itm % a.Hv;
    const size_t tok = seq;
    const int jo = blk * kScanCols + e;
    const float z = __bfloat162float(a.proj[tok * a.ld_proj + a.z_off + (size_t)h * D + jo]);
    const float gz = a.out_sig ? 1.f / (1.f + __expf(-z)) : z / (1.f + __expf(-z));
    const float y = ovm * rsqrtf(tot / (float)D + a.eps) * __bfloat162float(a.norm_w[jo]) * gz;
    a.out[(tok * a.Hv + h) * D + jo] = __float2bfloat16(y);
    return true;
  };
  GdnItemRegs nx = gdn_item_regs<D, CH>(a, it, blk, e, jl);
  copy_state(0, column(it, nx.slot));
  asm volatile("cp.async.commit_group;" ::: "memory");
  int slot_n = it + G < items ? a.state_slot[(it + G) / a.Hv] : 0;  // slot of the next item
  for (int n = 0; it < items; ++n, it += G) {
    const GdnItemRegs cur = nx;
    const int itn = it + G;
    if (itn < items) {  // the next item's tile and inputs stream in while this one computes
      copy_state((n + 1) & 1, column(itn, slot_n));
      nx = gdn_item_regs<D, CH>(a, itn, blk, e, jl);
      slot_n = itn + G < items ? a.state_slot[(itn + G) / a.Hv] : 0;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    ks[e] = cur.kv;
    qs[e] = cur.qv;
    if constexpr (CH) gs[e] = __expf(cur.gv);
    const float decay = CH ? 1.f : __expf(cur.graw);
    const float beta = cur.beta, vj = cur.vj;
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // this item's tile has landed
    __syncthreads();
    float S[R];
#pragma unroll
    for (int c = 0; c < R / 4; ++c) {
      const float4 v = sbuf[n & 1][c][e];
      S[4 * c] = v.x;
      S[4 * c + 1] = v.y;
      S[4 * c + 2] = v.z;
      S[4 * c + 3] = v.w;
    }
    if (cur.fresh) {
#pragma unroll
      for (int i = 0; i < R; ++i) S[i] = 0.f;
    }
    float vq[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (CH) {
#pragma unroll
      for (int i = 0; i < R; ++i) vq[i & 3] += gs[kidx(i)] * S[i] * ks[kidx(i)];
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) vq[i & 3] += S[i] * ks[kidx(i)];
    }
    float vp = (vq[0] + vq[1]) + (vq[2] + vq[3]);
    vp += __shfl_xor_sync(0xffffffffu, vp, 1);
    vp += __shfl_xor_sync(0xffffffffu, vp, 2);
    const float upd = beta * (vj - decay * vp);
    float oq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < R; ++i) {
      S[i] = (CH ? gs[kidx(i)] : decay) * S[i] + ks[kidx(i)] * upd;
      oq[i & 3] += S[i] * qs[kidx(i)];
    }
    float o = (oq[0] + oq[1]) + (oq[2] + oq[3]);
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    o += __shfl_xor_sync(0xffffffffu, o, 2);
    const int seq = it / a.Hv, h = it % a.Hv;
    const size_t tok = seq;
    if (seq >= a.spec_rows) {  // a verify sequence's state advances in the commit
      float* col = column(it, cur.slot);
#pragma unroll
      for (int i = 0; i < R; i += 4)
        *reinterpret_cast<float4*>(col + kidx(i)) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
    }
    if (part == 0) os[jl] = o;
    __syncthreads();
    if (e < 32 && !failed) {  // warp 0: the gated norm of this column block
      const float ov = os[e];
      float ss = ov * ov;  // this column block's sum of squares (the norm kernel's warp blk)
#pragma unroll
      for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      // the previous item's norm first: its partials were sent an item ago, so the wait is
      // short, and its slot must be read before this item's partial goes out (a sibling
      // answers that with its next partial, which lands in the same slot)
      if (it_p >= 0) failed = !finish(n - 1, it_p, ov_p);
      // warp-uniform; every lane is past its reads of the slot (its output store used them)
      failed = __any_sync(0xffffffffu, failed);
      if (!failed && e == 0) {
        // the single arrival of this phase, then the partial into slot blk of every CTA
        const int b = n & 1;
        mbar_arrive_expect_tx(&mbar[b], NB * 4);
#pragma unroll
        for (int r = 0; r < NB; ++r) {
          uint32_t rs, rb;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rs) : "r"(smem_u32(&redv[b][blk])), "r"(r));
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(smem_u32(&mbar[b])), "r"(r));
          asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                       ::"r"(rs), "r"(__float_as_uint(ss)), "r"(rb) : "memory");
        }
      }
      ov_p = ov;
      it_p = it;
    }
    ++n_done;
  }
  if (e < 32 && !failed && it_p >= 0) finish(n_done - 1, it_p, ov_p);  // the last item's norm
  // no CTA leaves while a sibling may still deliver a partial into its shared memory
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Clusters of gdn_step_one_token_kernel that fit on the device at once (cached per
// device and variant); the persistent grid takes that many.
template <int D, bool CH>
static int one_token_clusters() {
  static int cached[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = cached[CH ? 1 : 0][dev & 63];
  if (!c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms(), 1, D / kScanCols);
    cfg.blockDim = dim3(4 * kScanCols);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)gdn_step_one_token_kernel<D, CH>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms();
    }
    c = n;
  }
  return c;
}

// grid (T, Hv), D threads: the gated RMSNorm  o * rsqrt(mean(o^2) + eps) * w * gate(z)
// of one head's outputs (gate = silu, or sigmoid for the KDA variant).
template <int D>
__global__ void __launch_bounds__(D) gdn_norm_kernel(GdnArgs a) {
  pdl_enter();
  const int t = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const float o = a.o_raw[((size_t)t * a.Hv + h) * D + j];
  float ss = o * o;
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __shared__ float red[D / 32];
  if ((j & 31) == 0) red[j >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < D / 32; ++w) tot += red[w];
  const float z = __bfloat162float(a.proj[(size_t)t * a.ld_proj + a.z_off + (size_t)h * D + j]);
  const float gz = a.out_sig ? 1.f / (1.f + __expf(-z)) : z / (1.f + __expf(-z));
  const float y = o * rsqrtf(tot / (float)D + a.eps) * __bfloat162float(a.norm_w[j]) * gz;
  a.out[((size_t)t * a.Hv + h) * D + j] = __float2bfloat16(y);
}

// grid (verify sequences, Hv, layers), 2*D threads: the scan of gdn_scan_kernel
// over the accepted tokens of a verify step, without outputs.
template <int D, bool CH>
__global__ void __launch_bounds__(2 * D) gdn_commit_scan_kernel(GdnCommitArgs a) {
  pdl_enter();
  constexpr int R = D / 2;
  const int seq = blockIdx.x, h = blockIdx.y, l = blockIdx.z;
  const int j = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int q0 = a.q_start[seq];
  const int n = a.n_acc[seq] + 1;
  const int hk = h / (a.Hv / a.Hk);
  float* col = a.state + l * a.state_layer_stride + (((size_t)a.state_slot[seq] * a.Hv + h) * D + j) * D + half * R;
  const float* rk = a.rk + (size_t)l * a.R * a.Hk * D;
  const float* rv = a.rv + (size_t)l * a.R * a.Hv * D;
  const float* rg = a.rg + (size_t)l * a.R * a.Hv * (CH ? D : 1);
  const float* rb = a.rb + (size_t)l * a.R * a.Hv;
  float S[R];
#pragma unroll
  for (int i = 0; i < R; i += 4) {
    const float4 v = *reinterpret_cast<const float4*>(col + i);
    S[i] = v.x;
    S[i + 1] = v.y;
    S[i + 2] = v.z;
    S[i + 3] = v.w;
  }
  for (int u = 0; u < n; ++u) {
    const size_t tok = q0 + u;
    const float beta = rb[tok * a.Hv + h];
    const float vj = rv[(tok * a.Hv + h) * D + j];
    const float* kk = rk + (tok * a.Hk + hk) * D + half * R;
    if constexpr (CH) {
      const float* gl = rg + (tok * a.Hv + h) * D + half * R;
      float dec[R];
      float vp = 0.f;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        dec[i] = __expf(gl[i]);
        vp += dec[i] * S[i] * kk[i];
      }
      vp += __shfl_xor_sync(0xffffffffu, vp, 1);
      const float upd = beta * (vj - vp);
#pragma unroll
      for (int i = 0; i < R; ++i) S[i] = dec[i] * S[i] + kk[i] * upd;
    } else {
      const float decay = __expf(rg[tok * a.Hv + h]);
      float vp = 0.f;
#pragma unroll
      for (int i = 0; i < R; ++i) vp += S[i] * kk[i];
      vp += __shfl_xor_sync(0xffffffffu, vp, 1);
      const float upd = beta * (vj - decay * vp);
#pragma unroll
      for (int i = 0; i < R; ++i) S[i] = decay * S[i] + kk[i] * upd;
    }
  }
#pragma unroll
  for (int i = 0; i < R; i += 4) *reinterpret_cast<float4*>(col + i) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
}

// grid (verify sequences, layers): conv state after the accepted tokens.
__global__ void gdn_commit_conv_kernel(GdnCommitArgs a) {
  pdl_enter();
  const int seq = blockIdx.x, l = blockIdx.y;
  const int q0 = a.q_start[seq];
  const int n = a.n_acc[seq] + 1;
  const int K1 = a.conv_k - 1;
  __nv_bfloat16* st = a.conv_state + l * a.conv_layer_stride + (size_t)a.state_slot[seq] * K1 * a.C;
  const __nv_bfloat16* rx = a.rx + (size_t)l * a.R * a.C;
  for (int c = threadIdx.x; c < a.C; c += blockDim.x) {
    __nv_bfloat16 old[8];
    for (int j = 0; j < K1; ++j) old[j] = st[(size_t)j * a.C + c];
    for (int j = 0; j < K1; ++j) {
      const int rel = n - K1 + j;  // new row j = input at relative position n - K1 + j
      st[(size_t)j * a.C + c] = rel >= 0 ? rx[(size_t)(q0 + rel) * a.C + c] : old[K1 + rel];
    }
  }
}

int launch_gdn_commit(const GdnCommitArgs& a, cudaStream_t st) {
  if (a.n_verify == 0 || a.n_layers == 0) return 0;
  if (a.D != 128 || a.conv_k > 9 || a.Hv % a.Hk) return -2;
  if (a.gate_ch) launch_pdl(gdn_commit_scan_kernel<128, true>, dim3(dim3(a.n_verify, a.Hv, a.n_layers)), dim3(256), 0, st, a);
  else launch_pdl(gdn_commit_scan_kernel<128, false>, dim3(dim3(a.n_verify, a.Hv, a.n_layers)), dim3(256), 0, st, a);
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  launch_pdl(gdn_commit_conv_kernel, dim3(dim3(a.n_verify, a.n_layers)), dim3(256), 0, st, a);
  return (int)cudaGetLastError();
}

int launch_gdn(const GdnArgs& a, int T, int S, cudaStream_t st) {
  if (T == 0) return 0;
  if (a.Dk != 128 || a.Dv != 128 || a.conv_k > 9 || a.Hv % a.Hk) return -2;
  const int C = 2 * a.Hk * a.Dk + a.Hv * a.Dv;
  if (a.conv_k == 4) launch_pdl(gdn_conv_prep_kernel<4>, dim3(dim3(T, C / 128)), dim3(128), 0, st, a);
  else launch_pdl(gdn_conv_prep_kernel<0>, dim3(dim3(T, C / 128)), dim3(128), 0, st, a);
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  // One scan for every shape (decode, verify, prefill chunks): results must not depend on
  // how a prompt was chunked, so the summation order of the state updates is fixed.
  const dim3 sg(S, a.Hv, 128 / kScanCols);
  if (T == S && a.one_token_kernel) {  // one token per sequence: scan + gated norm in one launch
    const int items = S * a.Hv;
    if (a.gate_ch)
      launch_pdl(gdn_step_one_token_kernel<128, true>, dim3(std::min(items, one_token_clusters<128, true>()), 1, 128 / kScanCols),
                 dim3(4 * kScanCols), 0, st, a);
    else
      launch_pdl(gdn_step_one_token_kernel<128, false>, dim3(std::min(items, one_token_clusters<128, false>()), 1, 128 / kScanCols),
                 dim3(4 * kScanCols), 0, st, a);
    return (int)cudaGetLastError();
  }
  if (!a.o_raw) return -2;
  if (T >= 8 * S) {  // prefill-sized chunks: batched staging (decode and verify keep the compact one)
    if (a.gate_ch) launch_pdl(gdn_scan_kernel<128, true, true>, dim3(sg), dim3(4 * kScanCols), 0, st, a);
    else launch_pdl(gdn_scan_kernel<128, false, true>, dim3(sg), dim3(4 * kScanCols), 0, st, a);
  } else {
    if (a.gate_ch) launch_pdl(gdn_scan_kernel<128, true, false>, dim3(sg), dim3(4 * kScanCols), 0, st, a);
    else launch_pdl(gdn_scan_kernel<128, false, false>, dim3(sg), dim3(4 * kScanCols), 0, st, a);
  }
  rc = (int)cudaGetLastError();
  if (rc) return rc;
  launch_pdl(gdn_norm_kernel<128>, dim3(dim3(T, a.Hv)), dim3(128), 0, st, a);
  rc = (int)cudaGetLastError();
  if (rc) return rc;
  if (a.conv_state && T > S) {  // T == S: every sequence has one token, shifted by the prep kernel
    launch_pdl(gdn_conv_state_kernel, dim3(dim3(S, (C + 255) / 256)), dim3(256), 0, st, a);
    rc = (int)cudaGetLastError();
  }
  return rc;
}

}  // namespace rkt
