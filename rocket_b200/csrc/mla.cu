// Multi-head latent attention (MLA, NoPE) with the key/value up-projections absorbed:
//
//   c_t      = rmsnorm(x_t W_kva) * w                 512-wide latent, the only KV cached
//   q_h      = q_b(rmsnorm(q_a(x)))                   per head, `nope` wide   (GEMMs)
//   qa_h     = W_k[h]^T q_h * scale                   absorbed query, 512 wide
//   ctx_h    = sum_i softmax_i(qa_h . c_i) c_i        over the visible (or DSA-selected) tokens
//   o_h      = W_v[h] ctx_h                           `v` wide, then o_proj (GEMM)
//
//   mla_latent_write_kernel  rmsnorm of the latent rows + scatter into the paged cache
//   mla_absorb_kernel        qa for 16 tokens x one head per CTA (W_k[h] read once per tile)
//   mla_attn_kernel          one warp per head: 16 latent dims per lane, online softmax
//   mla_expand_kernel        o for 16 tokens x one head per CTA (W_v[h] stored [512][v])
//
// All heads of a token read the same latent rows (multi-query over the latent), so the
// attention reads 1 KB per visible token per token-CTA.  SIMT kernels (the benchmark
// serving configs use GQA layers).
//
// Behavioural counterpart of the reference's absorbed sparse MLA
// (engines/glm5-moe-nvfp4-2b/src/kernels.cu:566-760: mla_absorb_q, mla_fused_context,
// mla_expand_v; fuels/glm-5.3-flash/attention.yaml mla: NoPE, 512-wide cached latent).
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rkt {

namespace {

constexpr int kLat = 512;
constexpr int kTokTile = 16;

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

// grid T, 128 threads (4 latent values each)
__global__ void mla_latent_write_kernel(MlaArgs a) {
  const int t = blockIdx.x;
  const __nv_bfloat16* x = a.kv_lat + (size_t)t * a.ld_kv_lat;
  float v[4], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = bf(x[threadIdx.x * 4 + i]);
    ss += v[i] * v[i];
  }
  __shared__ float red[4];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / kLat + a.eps);
  if (!idx_ok(a.slots[t], a.n_slots, a.err)) return;
  __nv_bfloat16* dst = a.latent + (size_t)a.slots[t] * kLat;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = threadIdx.x * 4 + i;
    dst[c] = __float2bfloat16(v[i] * inv * bf(a.kv_norm_w[c]));
  }
}

// grid (H, ceil(T / 16)), 512 threads: thread c owns latent dim c for 16 tokens
__global__ void __launch_bounds__(512) mla_absorb_kernel(MlaArgs a, int T) {
  __shared__ float qs[kTokTile][256];
  const int h = blockIdx.x, t0 = blockIdx.y * kTokTile;
  const int nt = min(kTokTile, T - t0);
  for (int e = threadIdx.x; e < nt * a.nope; e += blockDim.x) {
    const int j = e / a.nope, d = e % a.nope;
    qs[j][d] = bf(a.q_nope[(size_t)(t0 + j) * a.ld_q + (size_t)h * a.nope + d]);
  }
  __syncthreads();
  const int c = threadIdx.x;
  float acc[kTokTile];
#pragma unroll
  for (int j = 0; j < kTokTile; ++j) acc[j] = 0.f;
  const __nv_bfloat16* w = a.wk + (size_t)h * a.nope * kLat + c;  // [h][d][c]
  for (int d = 0; d < a.nope; ++d) {
    const float wv = bf(w[(size_t)d * kLat]);
#pragma unroll
    for (int j = 0; j < kTokTile; ++j) acc[j] += wv * qs[j][d];
  }
  for (int j = 0; j < nt; ++j) a.q_abs[((size_t)(t0 + j) * a.H + h) * kLat + c] = acc[j] * a.scale;
}

// grid (T, ceil(H / 8)), 256 threads: warp = head, lane = 16 latent dims
__global__ void __launch_bounds__(256) mla_attn_kernel(MlaArgs a) {
  const int t = blockIdx.x;
  const int h = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (h >= a.H) return;
  const int seq = seq_of(a.q_start, a.n_seqs, a.row0 + t);
  const int* bt = a.block_table + (size_t)seq * a.bt_ld;
  const float* qa = a.q_abs + ((size_t)t * a.H + h) * kLat + lane * 16;
  float q[16], acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    q[i] = qa[i];
    acc[i] = 0.f;
  }
  const int n_tok = a.positions[t] + 1;
  const int n = a.sel ? a.n_sel[t] : n_tok;
  const int* sel = a.sel ? a.sel + (size_t)t * a.ld_sel : nullptr;
  float m = -INFINITY, l = 0.f;
  for (int s = 0; s < n; ++s) {
    const int tok = sel ? sel[s] : s;
    if (!idx_ok(tok, n_tok, a.err)) continue;
    const size_t slot = (size_t)bt[tok / a.page_size] * a.page_size + tok % a.page_size;
    if (!idx_ok((long long)slot, a.n_slots, a.err)) continue;
    const uint4* src = reinterpret_cast<const uint4*>(a.latent + slot * kLat + lane * 16);
    const uint4 u0 = src[0], u1 = src[1];
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float c[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      c[2 * i] = __uint_as_float(w[i] << 16);
      c[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) dot += q[i] * c[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float mn = fmaxf(m, dot);
    const float corr = __expf(m - mn), p = __expf(dot - mn);
    l = l * corr + p;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = acc[i] * corr + p * c[i];
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float* out = a.ctx + ((size_t)t * a.H + h) * kLat + lane * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = acc[i] * inv;
}

// grid (H, ceil(T / 16)), v threads: thread vd owns output dim vd for 16 tokens
__global__ void __launch_bounds__(512) mla_expand_kernel(MlaArgs a, int T) {
  extern __shared__ float cs[];  // [16][512]
  const int h = blockIdx.x, t0 = blockIdx.y * kTokTile;
  const int nt = min(kTokTile, T - t0);
  for (int e = threadIdx.x; e < nt * kLat; e += blockDim.x)
    cs[e] = a.ctx[((size_t)(t0 + e / kLat) * a.H + h) * kLat + e % kLat];
  __syncthreads();
  const int vd = threadIdx.x;
  if (vd >= a.v) return;
  float acc[kTokTile];
#pragma unroll
  for (int j = 0; j < kTokTile; ++j) acc[j] = 0.f;
  const __nv_bfloat16* w = a.wv_t + (size_t)h * kLat * a.v + vd;  // [h][c][vd]
  for (int c = 0; c < kLat; ++c) {
    const float wv = bf(w[(size_t)c * a.v]);
#pragma unroll
    for (int j = 0; j < kTokTile; ++j) acc[j] += wv * cs[j * kLat + c];
  }
  for (int j = 0; j < nt; ++j) a.out[(size_t)(t0 + j) * a.ld_out + (size_t)h * a.v + vd] = __float2bfloat16(acc[j]);
}

}  // namespace

int launch_mla_latent_write(const MlaArgs& a, int T, cudaStream_t st) {
  if (T == 0) return 0;
  mla_latent_write_kernel<<<T, 128, 0, st>>>(a);
  return (int)cudaGetLastError();
}

int launch_mla_attention(const MlaArgs& a, int T, cudaStream_t st) {
  if (T == 0) return 0;
  if (a.nope < 1 || a.nope > 256 || a.v < 1 || a.v > 512 || a.H < 1) return -2;
  const int tiles = (T + kTokTile - 1) / kTokTile;
  mla_absorb_kernel<<<dim3(a.H, tiles), 512, 0, st>>>(a, T);
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  mla_attn_kernel<<<dim3(T, (a.H + 7) / 8), 256, 0, st>>>(a);
  rc = (int)cudaGetLastError();
  if (rc) return rc;
  rc = ensure_smem_attr(mla_expand_kernel, kTokTile * kLat * 4);
  if (rc) return rc;
  const int thr = (a.v + 31) / 32 * 32;
  mla_expand_kernel<<<dim3(a.H, tiles), thr, kTokTile * kLat * 4, st>>>(a, T);
  return (int)cudaGetLastError();
}

}  // namespace rkt
