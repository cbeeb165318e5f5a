// DSA-style sparse attention on the paged GQA cache (per query row t at position p_t):
//
//   dsa_index_kv_kernel   indexer key  k~ = layernorm(x Wk) * w + b  and compressor gate
//                         x Wg of every new token -> per-token index caches [pages, ps, Di]
//   dsa_score_kernel      pools of kpool consecutive tokens: pooled key = sum_i
//                         softmax_i(gate_i + ape_i) * key_i (per channel); pool score
//                         I = sum_h w_h(t) * relu(q_h(t) . pooled / sqrt(Di)) over the
//                         complete pools among the p_t + 1 visible tokens
//   dsa_select_kernel     the top_k / kpool best pools (exact: 4-pass 8-bit radix select
//                         on order-preserving keys; ties go to the lowest pool index),
//                         expanded to their tokens, plus the open tail (the tokens of
//                         the incomplete last pool) -- at most top_k + kpool - 1 tokens
//   dsa_attn_kernel       GQA attention of the row's G = Hq/Hkv heads over the selected
//                         tokens only: chunks of selected K / V staged in shared memory
//                         (V runs of 4 tokens as 8-byte loads), scores with lanes on
//                         tokens, softmax + PV with warps on heads; output gate
//                         sigmoid(gate) when the model has one
//
// The selection is deterministic (ascending pool order within each of the two
// passes), so the attention's summation order is too.  With p_t + 1 <= top_k every
// token is selected and the result equals dense attention.
//
// Behavioural counterpart of the reference's DSA indexer and sparse attention
// (engines/glm5-moe-nvfp4-2b/src/kernels.cu:767-928: indexer_pool / indexer_scores /
// indexer_select / indexer_expand; mla_fused_context_kernel :659), here on the GQA
// paged cache of this engine.  SIMT kernels: the indexer and the selected-token
// gather are latency-bound per row; not on the headline serving path.
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rkt {

namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ int seq_of(const int* q_start, int n_seqs, int t) {
  int lo = 0, hi = n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q_start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ unsigned order_key(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// grid T, Di threads
__global__ void dsa_index_kv_kernel(DsaArgs a) {
  const int t = blockIdx.x, c = threadIdx.x;
  const __nv_bfloat16* row = a.idx_proj + (size_t)t * a.ld_idx;
  const float x = bf(row[a.Hi * a.Di + c]);
  __shared__ float red[2][32];
  float s = x, s2 = x * x;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  if ((c & 31) == 0) {
    red[0][c >> 5] = s;
    red[1][c >> 5] = s2;
  }
  __syncthreads();
  float ts = 0.f, ts2 = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    ts += red[0][w];
    ts2 += red[1][w];
  }
  const float mean = ts / a.Di;
  const float var = fmaxf(ts2 / a.Di - mean * mean, 0.f);
  const float k = (x - mean) * rsqrtf(var + a.ln_eps) * a.k_norm_w[c] + a.k_norm_b[c];
  const size_t slot = (size_t)a.slots[t];
  if (!idx_ok((long long)slot, a.n_slots, a.err)) return;
  a.ik_cache[slot * a.Di + c] = __float2bfloat16(k);
  a.ig_cache[slot * a.Di + c] = row[a.Hi * a.Di + a.Di + c];
}

// grid (T, pool tiles of 8 warps x kPoolsPerWarp), 256 threads; Di == 128, Hi <= 32
constexpr int kPoolsPerWarp = 8;
__global__ void __launch_bounds__(256) dsa_score_kernel(DsaArgs a) {
  __shared__ float qT[128][33];  // [channel][head] (+1 pad)
  __shared__ float pk[8][128];
  __shared__ float wh[32];
  const int t = blockIdx.x;
  const int seq = seq_of(a.q_start, a.n_seqs, t);
  const int n_tok = a.positions[t] + 1;
  const int n_pools = n_tok / a.kpool;
  const int p_base = blockIdx.y * 8 * kPoolsPerWarp;
  if (p_base >= n_pools) return;
  const __nv_bfloat16* row = a.idx_proj + (size_t)t * a.ld_idx;
  for (int e = threadIdx.x; e < a.Hi * 128; e += blockDim.x) qT[e % 128][e / 128] = bf(row[e]);
  if (threadIdx.x < a.Hi) wh[threadIdx.x] = bf(row[a.Hi * 128 + 2 * 128 + threadIdx.x]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int* bt = a.block_table + (size_t)seq * a.bt_ld;
  const float scale = rsqrtf(128.f);
  for (int k = 0; k < kPoolsPerWarp; ++k) {
    const int p = p_base + warp * kPoolsPerWarp + k;
    if (p >= n_pools) break;
    float lg[8][4], kv[8][4];
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int i = 0; i < a.kpool; ++i) {
      const int tok = p * a.kpool + i;
      size_t slot = (size_t)bt[tok / a.page_size] * a.page_size + tok % a.page_size;
      if (!idx_ok((long long)slot, a.n_slots, a.err)) slot = 0;
      const uint2 gv = *reinterpret_cast<const uint2*>(a.ig_cache + slot * 128 + lane * 4);
      const uint2 kvv = *reinterpret_cast<const uint2*>(a.ik_cache + slot * 128 + lane * 4);
      const __nv_bfloat16* g4 = reinterpret_cast<const __nv_bfloat16*>(&gv);
      const __nv_bfloat16* k4 = reinterpret_cast<const __nv_bfloat16*>(&kvv);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        lg[i][c] = bf(g4[c]) + a.ape[i * 128 + lane * 4 + c];
        kv[i][c] = bf(k4[c]);
        mx[c] = fmaxf(mx[c], lg[i][c]);
      }
    }
    float num[4] = {0.f, 0.f, 0.f, 0.f}, den[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < a.kpool; ++i) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float e = __expf(lg[i][c] - mx[c]);
        den[c] += e;
        num[c] += e * kv[i][c];
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) pk[warp][lane * 4 + c] = num[c] / den[c];
    __syncwarp();
    float v = 0.f;
    if (lane < a.Hi) {
      float dot = 0.f;
#pragma unroll 8
      for (int c = 0; c < 128; ++c) dot += qT[c][lane] * pk[warp][c];
      v = wh[lane] * fmaxf(dot * scale, 0.f);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) a.scores[(size_t)t * a.ld_scores + p] = v;
    __syncwarp();
  }
}

// grid T, 512 threads
__global__ void __launch_bounds__(512) dsa_select_kernel(DsaArgs a) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_prefix;
  __shared__ int s_left, s_count;
  __shared__ int wsum[16];
  const int t = blockIdx.x;
  const int n_tok = a.positions[t] + 1;
  const int n_pools = n_tok / a.kpool;
  const int want = a.top_k / a.kpool;
  const float* sc = a.scores + (size_t)t * a.ld_scores;
  int* out = a.sel + (size_t)t * a.ld_sel;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int n_sel_pools;
  if (n_pools <= want) {
    for (int p = threadIdx.x; p < n_pools; p += blockDim.x)
      for (int i = 0; i < a.kpool; ++i) out[p * a.kpool + i] = p * a.kpool + i;
    n_sel_pools = n_pools;
  } else {
    if (threadIdx.x == 0) {
      s_prefix = 0u;
      s_left = want;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
      __syncthreads();
      const unsigned hi_mask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
      const unsigned pre = s_prefix;
      for (int p = threadIdx.x; p < n_pools; p += blockDim.x) {
        const unsigned k = order_key(sc[p]);
        if ((k & hi_mask) == pre) atomicAdd(&hist[(k >> shift) & 0xffu], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int left = s_left, b = 255;
        for (; b > 0; --b) {
          if ((int)hist[b] >= left) break;
          left -= (int)hist[b];
        }
        s_left = left;  // how many of the threshold key's ties are still wanted
        s_prefix = pre | ((unsigned)b << shift);
      }
      __syncthreads();
    }
    const unsigned thr = s_prefix;
    if (threadIdx.x == 0) s_count = 0;
    __syncthreads();
    // two ordered compaction passes: keys above the threshold, then ties (lowest index first)
    for (int pass = 0; pass < 2; ++pass) {
      for (int base = 0; base < n_pools; base += blockDim.x) {
        const int p = base + threadIdx.x;
        bool f = false;
        if (p < n_pools) {
          const unsigned k = order_key(sc[p]);
          f = pass == 0 ? k > thr : k == thr;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, f);
        if (lane == 0) wsum[warp] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
          if (w < warp) before += wsum[w];
          total += wsum[w];
        }
        const int rank = s_count + before + __popc(bal & ((1u << lane) - 1u));
        if (f && rank < want)
          for (int i = 0; i < a.kpool; ++i) out[rank * a.kpool + i] = p * a.kpool + i;
        __syncthreads();
        if (threadIdx.x == 0) s_count = min(want, s_count + total);
        __syncthreads();
      }
    }
    n_sel_pools = want;
  }
  // the open tail: tokens of the incomplete last pool
  const int tail0 = n_pools * a.kpool;
  for (int i = threadIdx.x; i < n_tok - tail0; i += blockDim.x) out[n_sel_pools * a.kpool + i] = tail0 + i;
  if (threadIdx.x == 0) a.n_sel[t] = n_sel_pools * a.kpool + (n_tok - tail0);
}

// grid (T, Hkv), 128 threads (4 warps); DPL = D / 32 dims per lane; G <= kMaxG heads
constexpr int kMaxG = 16;

// grid (T, Hkv), 128 threads.  Selected tokens are processed in chunks of CH = 128 / LPT:
//   1. the chunk's K rows ([page][g][off][:]) and V columns ([page][g][:][off], transposed
//      into [token][dim]) are staged in shared memory; V moves as 8-byte runs of 4 tokens
//      when the selection holds an aligned run (pools of 4 always are), else token by token
//   2. scores: LPT lanes per token, DPT = D / LPT dims each (registers), one shuffle round
//   3. softmax + PV: warp w owns heads w, w+4, ..; lanes own D/32 dims; online over chunks
// Each warp finishes its heads alone, so no cross-warp merge is needed.
template <int D>
__global__ void __launch_bounds__(128) dsa_attn_kernel(DsaArgs a) {
  constexpr int LPT = D == 256 ? 4 : 2;
  constexpr int DPT = D / LPT;
  constexpr int CH = 128 / LPT;
  constexpr int DPL = D / 32;
  constexpr int MG = D == 256 ? 8 : kMaxG;
  constexpr int HPW = MG / 4;          // heads per warp
  constexpr int KLD = D + 8;           // padded K row (bf16 elements)
  __shared__ __align__(16) __nv_bfloat16 ks[CH][KLD];
  __shared__ __align__(16) __nv_bfloat16 vs[CH][D];
  __shared__ float qs[MG][D];
  __shared__ float sc[MG][CH];
  __shared__ int tk[CH];
  const int t = blockIdx.x, g = blockIdx.y;
  const int G = a.Hq / a.Hkv;
  const int seq = seq_of(a.q_start, a.n_seqs, t);
  const int* bt = a.block_table + (size_t)seq * a.bt_ld;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x)
    qs[e / D][e % D] = bf(a.q[((size_t)t * a.Hq + g * G + e / D) * D + e % D]) * a.scale;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m[HPW], l[HPW], acc[HPW][DPL];
#pragma unroll
  for (int h = 0; h < HPW; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[h][d] = 0.f;
  }
  const int n = a.n_sel[t];
  const int n_vis = a.positions[t] + 1;
  const int* sel = a.sel + (size_t)t * a.ld_sel;
  const size_t kv_page = (size_t)a.Hkv * a.page_size * D;
  for (int c0 = 0; c0 < n; c0 += CH) {
    const int cn = min(CH, n - c0);
    __syncthreads();  // the previous chunk's tiles are consumed
    for (int s = threadIdx.x; s < CH; s += blockDim.x) {
      int tok = s < cn ? sel[c0 + s] : -1;
      if (tok >= 0 && !idx_ok(tok, n_vis, a.err)) tok = -1;
      if (tok >= 0 && !idx_ok((long long)bt[tok / a.page_size] * a.page_size, a.n_slots, a.err)) tok = -1;
      tk[s] = tok;
    }
    __syncthreads();
    // K rows: 16-byte pieces
    for (int e = threadIdx.x; e < CH * (D / 8); e += blockDim.x) {
      const int s = e / (D / 8), q8 = e % (D / 8);
      const int tok = tk[s];
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (tok >= 0) {
        const size_t page = (size_t)bt[tok / a.page_size];
        v = *reinterpret_cast<const uint4*>(a.k_cache + page * kv_page +
                                           ((size_t)g * a.page_size + tok % a.page_size) * D + q8 * 8);
      }
      *reinterpret_cast<uint4*>(&ks[s][q8 * 8]) = v;
    }
    // V columns, transposed to [token][dim]: aligned runs of 4 tokens move as 8 bytes per dim
    for (int e = threadIdx.x; e < (CH / 4) * D; e += blockDim.x) {
      const int r = e / D, d = e % D;
      const int s0 = r * 4;
      const int t0 = tk[s0];
      const bool run = t0 >= 0 && (t0 & 3) == 0 && tk[s0 + 1] == t0 + 1 && tk[s0 + 2] == t0 + 2 &&
                       tk[s0 + 3] == t0 + 3;
      if (run) {
        const size_t page = (size_t)bt[t0 / a.page_size];
        const uint2 w = *reinterpret_cast<const uint2*>(a.v_cache + page * kv_page +
                                                        ((size_t)g * D + d) * a.page_size + t0 % a.page_size);
        const __nv_bfloat16* w4 = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) vs[s0 + i][d] = w4[i];
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = tk[s0 + i];
          __nv_bfloat16 x = __float2bfloat16(0.f);
          if (tok >= 0) {
            const size_t page = (size_t)bt[tok / a.page_size];
            x = a.v_cache[page * kv_page + ((size_t)g * D + d) * a.page_size + tok % a.page_size];
          }
          vs[s0 + i][d] = x;
        }
      }
    }
    __syncthreads();
    // scores: token s = threadIdx.x / LPT, dims [part * DPT, +DPT)
    {
      const int s = threadIdx.x / LPT, part = threadIdx.x % LPT;
      float k[DPT];
#pragma unroll
      for (int d = 0; d < DPT; d += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(&ks[s][part * DPT + d]);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          k[d + 2 * i] = __uint_as_float(w[i] << 16);
          k[d + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
      }
      for (int j = 0; j < G; ++j) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < DPT; ++d) dot += qs[j][part * DPT + d] * k[d];
#pragma unroll
        for (int o = 1; o < LPT; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (part == 0) sc[j][s] = tk[s] >= 0 ? dot : -INFINITY;
      }
    }
    __syncthreads();
    // softmax + PV: warp w owns heads w + 4 h
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
      const int j = warp + 4 * h;
      if (j >= G) break;
      float cm = -INFINITY;
      for (int s = lane; s < CH; s += 32) cm = fmaxf(cm, sc[j][s]);
#pragma unroll
      for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      const float mn = fmaxf(m[h], cm);
      if (mn == -INFINITY) continue;  // nothing valid yet
      const float corr = __expf(m[h] - mn);
      float ps = 0.f;
      for (int s = lane; s < CH; s += 32) {
        const float p = __expf(sc[j][s] - mn);
        sc[j][s] = p;
        ps += p;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      __syncwarp();
      l[h] = l[h] * corr + ps;
      m[h] = mn;
      float o8[DPL];
#pragma unroll
      for (int d = 0; d < DPL; ++d) o8[d] = acc[h][d] * corr;
      for (int s = 0; s < CH; ++s) {
        const float p = sc[j][s];
        const __nv_bfloat16* vr = &vs[s][lane * DPL];
#pragma unroll
        for (int d = 0; d < DPL; ++d) o8[d] += p * bf(vr[d]);
      }
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[h][d] = o8[d];
    }
  }
#pragma unroll
  for (int h = 0; h < HPW; ++h) {
    const int j = warp + 4 * h;
    if (j >= G) break;
    const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
      const size_t oi = ((size_t)t * a.Hq + g * G + j) * D + lane * DPL + d;
      float o = acc[h][d] * inv;
      if (a.gate) o *= 1.f / (1.f + __expf(-bf(a.gate[oi])));
      a.out[oi] = __float2bfloat16(o);
    }
  }
}

}  // namespace

int launch_dsa_index_kv(const DsaArgs& a, int T, cudaStream_t st) {
  if (T == 0) return 0;
  if (a.Di != 128) return -2;
  dsa_index_kv_kernel<<<T, a.Di, 0, st>>>(a);
  return (int)cudaGetLastError();
}

int launch_dsa_attention(const DsaArgs& a, int T, int max_pools, cudaStream_t st) {
  if (T == 0) return 0;
  if (a.Di != 128 || a.Hi > 32 || a.Hi < 1 || a.kpool < 1 || a.kpool > 8 || a.top_k % a.kpool) return -2;
  if (a.out != nullptr && (a.Hq % a.Hkv || a.Hq / a.Hkv > (a.D == 256 ? 8 : kMaxG))) return -2;
  const int tiles = (max_pools + 8 * kPoolsPerWarp - 1) / (8 * kPoolsPerWarp);
  if (tiles > 0) {
    dsa_score_kernel<<<dim3(T, tiles), 256, 0, st>>>(a);
    int rc = (int)cudaGetLastError();
    if (rc) return rc;
  }
  dsa_select_kernel<<<T, 512, 0, st>>>(a);
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  if (a.out == nullptr) return 0;  // selection only (the MLA kernel attends over it)
  if (a.D == 64) dsa_attn_kernel<64><<<dim3(T, a.Hkv), 128, 0, st>>>(a);
  else if (a.D == 128) dsa_attn_kernel<128><<<dim3(T, a.Hkv), 128, 0, st>>>(a);
  else if (a.D == 256) dsa_attn_kernel<256><<<dim3(T, a.Hkv), 128, 0, st>>>(a);
  else return -2;
  return (int)cudaGetLastError();
}

}  // namespace rkt
