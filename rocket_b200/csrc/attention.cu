// Paged GQA flash attention on tcgen05 (sm_100a): one kernel for chunked
// prefill and decode.
//
// A CTA owns one (sequence, kv head, query block).  Its 128 MMA rows are
// (query token, q head of the group) pairs, so a decode step with 12 q heads
// per kv head fills 12 rows and a prefill block packs floor(128/G) tokens.
//   S = Q K^T   (M=128 rows, N=BN keys, K=D)      -> TMEM, double buffered
//   O += P V    (M=128 rows, N=D, K=BN keys)      -> TMEM accumulator
// K pages [page][kvh][64][D] and transposed V pages [page][kvh][D][64] are
// fetched with TMA (local memory only, no multicast).  Softmax runs one thread
// per row on TMEM loads; when the running max grows the thread rescales its
// row of O in TMEM (tcgen05.ld/st) before the next P V is issued.
//
// Warps 0-3: Q staging, softmax, epilogue.  Warp 4: TMA producer.  Warp 5:
// TMEM owner and MMA issuer.
//
// Split-K (flash-decode): a work item may cover a key-block range and write
// unnormalised O with (m, l) to a workspace; attn_combine_kernel merges.
//
// FP8 (e4m3) KV cache.  Decode kernel: everything e4m3 -- K pages land by TMA
// in the S^T MMA's A layout (SW128), V^T pages in the O^T MMA's A layout (SW64),
// the query rows are quantized per head (scale amax/448) and P^T is written as
// e4m3 of 256*P; both MMAs are kind::f8f6f4 with f32 accumulation, and the scales
// (query, K, V, 256) are applied to the f32 scores / outputs.  Generic kernel:
// TMA brings the pages into a staging buffer and two converter warps widen them
// to bf16 (times the K / V scale) in the swizzled layout the bf16 MMAs read.
//
// Reference counterparts: mla_fused_context_kernel (engines/glm5-moe-nvfp4-2b/
// src/kernels.cu:659, one warp per head, online softmax over a page-table
// gather) and qsa_sparse_splitk_block16 + qsa_merge_splitk (engines/
// qwen38-flash-next-nvfp4-2b/src/projection/cutlass_qkv.cu:601,759).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"

namespace rkt {

template <int D, int BN, bool F8 = false>
struct AttnCfg {
  static constexpr int kQ = (D / 64) * 16384;          // Q tile: D/64 column atoms of [128][128B]
  static constexpr int kK = BN * D * 2;                // K stage: D/64 atoms of [BN][128B]
  static constexpr int kV = BN * D * 2;                // V stage: BN/64 pages of [D][128B]
  static constexpr int kPBytes = (BN / 64) * 16384;    // P tile: BN/64 atoms of [128][128B]
  // P of block j is written over the K tile of j's stage once S = Q K^T has been read
  // out of TMEM (the next load into that stage waits for P V), when K is large enough
  static constexpr bool kPInK = kK >= kPBytes;
  static constexpr int kP = kPInK ? 0 : kPBytes;
  static constexpr int kStages = 2;
  static constexpr int kStgBlock = 2 * BN * D;         // fp8 block: K pages [64][D] then V pages [D][64]
  static constexpr int kStgBufs = 1;                   // (a second one does not fit next to Q and P here)
  static constexpr int kStg = F8 ? kStgBufs * kStgBlock : 0;
  static constexpr int kSmem = kQ + kStages * (kK + kV) + kP + kStg + 1024;
  static constexpr int kConv = 64;                     // converter threads (warps 6-7)
  static constexpr int kThreads = F8 ? 192 + kConv : 192;
  // O [0,D) S0 [D,D+BN) S1 [D+BN, D+2BN); a 256-column allocation lets two CTAs share an SM
  static constexpr int kTmemCols = D + 2 * BN <= 256 ? 256 : 512;
  static constexpr int kMinBlocks = (kTmemCols == 256 && !F8 && 2 * (kSmem + 2048) <= 233472) ? 2 : 1;
  static_assert(D + 2 * BN <= 512, "TMEM");
};

// 2^x with the MUFU instruction (flush-to-zero; 2^-inf = +0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 16 fp8 (e4m3) -> 16 bf16 scaled, as 8 packed words.  Bit placement: the e4m3
// exponent and mantissa bits shifted into a float's exponent / mantissa fields give
// 2^(e-127) * 1.m (or the matching subnormal), so one multiply by 2^120 * scale
// yields the e4m3 value (2^(e-7) * 1.m, subnormals 2^-6 * 0.m) times the scale.
// e4m3fn NaN (0x7f / 0xff) is never stored (writers saturate).
__device__ __forceinline__ void fp8x16_to_bf16(const uint4 v, float scale, uint32_t out[8]) {
  const float mul = scale * 1.329227995784916e36f;  // 2^120
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float f[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t x = (w[i] >> (8 * b)) & 0xffu;
      f[b] = __uint_as_float(((x & 0x80u) << 24) | ((x & 0x7fu) << 20)) * mul;
    }
    out[2 * i] = pack_bf16(f[0], f[1]);
    out[2 * i + 1] = pack_bf16(f[2], f[3]);
  }
}

// Widen one staged fp8 key block (BN keys) into the bf16 K / V operand tiles.
// Staging: K pages [BN/64][64 keys][D bytes], then V pages [BN/64][D][64 bytes].
// K tile: D/64 column atoms of [BN keys][128 B] (SW128); V tile: BN/64 pages of
// [D][128 B] (SW128) -- the layouts the bf16 TMA loads produce.  t: 0..NT-1.
template <int D, int BN, int NT>
__device__ __forceinline__ void convert_kv_block(const uint8_t* stg, uint8_t* sK, uint8_t* sV, float ks, float vs,
                                                 int t) {
  constexpr int QK = D / 16;  // 16-byte fp8 chunks per key row
  for (int it = t; it < BN * QK; it += NT) {
    const int key = it / QK, q = it % QK;
    const uint4 v = *reinterpret_cast<const uint4*>(stg + (size_t)key * D + q * 16);
    uint32_t o[8];
    fp8x16_to_bf16(v, ks, o);
    const int d0 = q * 16, c = d0 >> 6, ch = (d0 & 63) >> 3, r = key & 63;
    uint8_t* dst = sK + c * (BN * 128) + (key >> 6) * 8192;
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, ch)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, ch + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
  const uint8_t* sv = stg + BN * D;
  for (int it = t; it < (BN / 64) * D * 4; it += NT) {
    const int pg = it / (D * 4), rem = it % (D * 4), d = rem >> 2, q = rem & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(sv + (size_t)pg * (D * 64) + d * 64 + q * 16);
    uint32_t o[8];
    fp8x16_to_bf16(v, vs, o);
    uint8_t* dst = sV + pg * (D * 128);
    *reinterpret_cast<uint4*>(dst + sw128_offset(d, 2 * q)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + sw128_offset(d, 2 * q + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// TMA of one fp8 key block into the staging buffer (K pages, then V pages).
template <int D, int BN>
__device__ __forceinline__ void load_kv_block_fp8(uint8_t* stg, const CUtensorMap* tmK, const CUtensorMap* tmV,
                                                  uint64_t* bar, const int* bt, int kb, int seq_pages, int Hkv,
                                                  int kvh) {
  for (int pg = 0; pg < BN / 64; ++pg) {
    const int pidx = kb * (BN / 64) + pg;
    const int page = bt[pidx < seq_pages ? pidx : 0];
    tma_load_2d(stg + pg * (64 * D), tmK, bar, 0, (page * Hkv + kvh) * 64);
    tma_load_2d(stg + BN * D + pg * (D * 64), tmV, bar, 0, (page * Hkv + kvh) * D);
  }
}

template <int D, int BN, bool F8>
__global__ void __launch_bounds__(AttnCfg<D, BN, F8>::kThreads, AttnCfg<D, BN, F8>::kMinBlocks)
    attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnArgs p) {
  pdl_enter();
  using C = AttnCfg<D, BN, F8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::kQ;
  uint8_t* sP0 = sKV + C::kStages * (C::kK + C::kV);  // P tile when it does not live in K
  uint8_t* sStg = sP0 + C::kP;  // fp8 staging (F8 only)
  // P tile of block j
  auto p_tile = [&](int j) -> uint8_t* { return C::kPInK ? sKV + (j & 1) * (C::kK + C::kV) : sP0; };
  // p_full[j & 1] / o_done[j & 1] complete with block j's P / P V.  The softmax waits for a
  // P V only when it rescales O (or reuses a single P buffer), so it may run a block ahead
  // of the MMA warp; a barrier per block parity keeps every parity wait at most one phase
  // behind (S of block j is issued after the MMA warp consumed P of j-2, and block j-2's
  // P V is done once S of j is)
  __shared__ __align__(8) uint64_t q_full, p_full[2], o_done[2];
  __shared__ __align__(8) uint64_t kv_full[2], kv_empty[2], s_full[2];
  __shared__ __align__(8) uint64_t conv_full[2], stg_free[C::kStgBufs];  // F8: stage converted / staging free
  __shared__ uint32_t tmem_sh;

  const int w = blockIdx.x;
  if (w >= *p.num_work) return;
  const int kvh = blockIdx.y;
  const int seq = p.w_seq[w];
  const int tok0 = p.w_tok0[w];
  const int q_start = p.q_start[seq], q_len = p.q_len[seq], kv_len = p.kv_len[seq];
  const int G = p.Hq / p.Hkv;
  const int tpb = 128 / G;                         // query tokens per block
  const int ntok = min(tpb, q_len - tok0);
  const int last_qpos = kv_len - q_len + tok0 + ntok - 1;
  const int kv_hi = min(kv_len, last_qpos + 1);
  const int kb_total = (kv_hi + BN - 1) / BN;
  const int kb_chunk = (kb_total + p.num_splits - 1) / p.num_splits;
  const int kb0 = min(kb_total, (int)blockIdx.z * kb_chunk);
  const int nb = min(kb_total, kb0 + kb_chunk) - kb0;
  const int* bt = p.block_table + (size_t)seq * p.max_pages;
  const int seq_pages = (kv_len + 63) / 64;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&q_full, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_full[s], 128);
      mbar_init(&o_done[s], 1);
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&conv_full[s], C::kConv);
    }
    for (int b = 0; b < C::kStgBufs; ++b) mbar_init(&stg_free[b], C::kConv);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc<C::kTmemCols>(&tmem_sh);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t tO = tmem, tS0 = tmem + D;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (F8) {
      if (elect_one() && nb > 0) {
        bool ok = true;
        for (int j = 0; j < nb && ok; ++j) {
          const int s = j & 1;
          // the TMA fills a staging buffer; the converter waits for the bf16 stage instead
          const int b = j % C::kStgBufs;  // the converter must have drained this staging buffer
          if (j >= C::kStgBufs) ok = mbar_wait(&stg_free[b], ((j / C::kStgBufs) - 1) & 1, p.err);
          if (!ok) break;
          mbar_arrive_expect_tx(&kv_full[s], C::kStgBlock);
          load_kv_block_fp8<D, BN>(sStg + b * C::kStgBlock, &tmK, &tmV, &kv_full[s], bt, kb0 + j, seq_pages, p.Hkv,
                                   kvh);
        }
      }
    } else if (nb > 0) {
      // the warp fetches the page ids of up to 32 / (BN / 64) blocks in one parallel load and
      // hands them to lane 0 by shuffles: no block-table round trip before a block's loads
      constexpr int PPB = BN / 64, BPB = 32 / PPB;
      bool ok = true;
      for (int j0 = 0; j0 < nb && ok; j0 += BPB) {
        const int pidx = (kb0 + j0) * PPB + lane;
        const int my_page = bt[pidx < seq_pages ? pidx : 0];
        const int jn = min(nb, j0 + BPB);
        for (int j = j0; j < jn; ++j) {
          const int s = j & 1;
          int pg_id[PPB];
#pragma unroll
          for (int pg = 0; pg < PPB; ++pg) pg_id[pg] = __shfl_sync(0xffffffffu, my_page, (j - j0) * PPB + pg);
          if (lane == 0) {
            if (j >= 2) ok = mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, p.err);
            if (ok) {
              uint8_t* sK = sKV + s * (C::kK + C::kV);
              uint8_t* sV = sK + C::kK;
              mbar_arrive_expect_tx(&kv_full[s], C::kK + C::kV);
#pragma unroll
              for (int pg = 0; pg < PPB; ++pg) {
                const int page = pg_id[pg];
                const int krow = (page * p.Hkv + kvh) * 64;
                for (int c = 0; c < D / 64; ++c)
                  tma_load_2d(sK + c * (BN * 128) + pg * 8192, &tmK, &kv_full[s], c * 64, krow);
                tma_load_2d(sV + pg * (D * 128), &tmV, &kv_full[s], 0, (page * p.Hkv + kvh) * D);
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one() && nb > 0) {
      bool ok = mbar_wait(&q_full, 0, p.err);
      const uint32_t id_s = idesc_bf16(128, BN);
      const uint32_t id_o = idesc_bf16(128, D);
      auto issue_qk = [&](int j) {
        const int s = j & 1;
        uint8_t* sK = sKV + s * (C::kK + C::kV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk >> 2, wi = kk & 3;
          mma_bf16(tS0 + s * BN, desc_sw128_kmajor(sQ + c * 16384) + 2 * wi,
                   desc_sw128_kmajor(sK + c * (BN * 128)) + 2 * wi, id_s, kk ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
      };
      uint64_t* ready = F8 ? conv_full : kv_full;  // F8: wait for the converted stage
      if (ok) ok = mbar_wait(&ready[0], 0, p.err);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb) {
          ok = mbar_wait(&ready[(j + 1) & 1], ((j + 1) >> 1) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          issue_qk(j + 1);
        }
        ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        uint8_t* sV = sKV + (j & 1) * (C::kK + C::kV) + C::kK;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const int c = kk >> 2, wi = kk & 3;
          mma_bf16(tO, desc_sw128_kmajor(p_tile(j) + c * 16384) + 2 * wi, desc_sw128_kmajor(sV + c * (D * 128)) + 2 * wi,
                   id_o, (j | kk) ? 1u : 0u);
        }
        tc_commit(&o_done[j & 1]);
        tc_commit(&kv_empty[j & 1]);
      }
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------------------------------------ fp8 converter (F8 only)
    if constexpr (F8) {
      const int t = threadIdx.x - 192;
      bool ok = true;
      for (int j = 0; j < nb && ok; ++j) {
        const int s = j & 1, b = j % C::kStgBufs;
        ok = mbar_wait(&kv_full[s], (j >> 1) & 1, p.err);
        if (ok && j >= 2) ok = mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, p.err);  // bf16 stage free
        if (!ok) break;
        uint8_t* sK = sKV + s * (C::kK + C::kV);
        convert_kv_block<D, BN, C::kConv>(sStg + b * C::kStgBlock, sK, sK + C::kK, p.k_scale, p.v_scale, t);
        fence_proxy_async();  // generic-proxy writes -> visible to the tensor core
        mbar_arrive(&conv_full[s]);
        mbar_arrive(&stg_free[b]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax rows
    const int r = threadIdx.x;  // 0..127 = TMEM lane
    const int ti = r / G;
    const bool row_ok = r < tpb * G && ti < ntok;
    const int head = kvh * G + (r % G);
    const int qtok = q_start + tok0 + ti;  // global token row
    const int qpos = kv_len - q_len + tok0 + ti;
    // stage Q row r into the swizzled tile
    {
      const uint4* src = reinterpret_cast<const uint4*>(p.q + ((size_t)qtok * p.Hq + head) * D);
#pragma unroll
      for (int u = 0; u < D / 8; ++u) {
        const uint4 v = row_ok ? src[u] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sQ + (u >> 3) * 16384 + sw128_offset(r, u & 7)) = v;
      }
      fence_proxy_async();
      mbar_arrive(&q_full);
    }
    const float sl2 = p.scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int s = j & 1;
      if (ok) ok = mbar_wait(&s_full[s], (j >> 1) & 1, p.err);
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tS0 + s * BN + c * 32 + lane_off, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(v[i]);
      }
      const int kbase = (kb0 + j) * BN;
      // raw scores; the scale is folded into the exponent's fma below.  Blocks wholly inside
      // the row's causal window skip the per-key mask; four independent max chains.
      if (!(row_ok && kbase + BN <= kv_len && kbase + BN - 1 <= qpos)) {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int kidx = kbase + i;
          if (!(row_ok && kidx < kv_len && kidx <= qpos)) sv[i] = -INFINITY;
        }
      }
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN; ++i) mq[i & 3] = fmaxf(mq[i & 3], sv[i]);
      const float bmax = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
      // lazy rescale: the exponent base moves on the first finite block max, or when a block
      // max passes it by more than 2^8 (P <= 256 in bf16 and the fp32 O / l stay exact
      // enough); otherwise O keeps accumulating without a rescale or its wait
      const float mx = (m == -INFINITY || bmax > m + 8.f) ? fmaxf(m, bmax) : m;
      const float alpha = (mx == -INFINITY || mx == m) ? 1.f : exp2f(m - mx);
      const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha < 1.f);
      // O rescale needs block j-1's P V done; so does a single P buffer (head_dim < 128), which
      // block j overwrites (with P in K's stage, block j-2's P V finished before the refill)
      if ((rescale || (!C::kPInK && j > 0)) && ok) ok = mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err);
      // tcgen05.ld/st are warp-collective: rescale when any lane of the warp needs it
      // (lanes whose max did not grow multiply by alpha = 1)
      if (rescale) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + c * 32 + lane_off, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32(tO + c * 32 + lane_off, v);
        }
        tmem_st_wait();
      }
      float rq[4] = {0.f, 0.f, 0.f, 0.f};
      uint8_t* sPj = p_tile(j);
      const float nmx = mx == -INFINITY ? 0.f : -mx;  // a fully masked row: every e is 0
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = ex2_approx(fmaf(sv[c * 8 + i], sl2, nmx));  // 2^(s*scale - base); -inf -> 0
          rq[i & 3] += e[i];
        }
        uint4 pk = make_uint4(pack_bf16(e[0], e[1]), pack_bf16(e[2], e[3]), pack_bf16(e[4], e[5]),
                              pack_bf16(e[6], e[7]));
        *reinterpret_cast<uint4*>(sPj + (c >> 3) * 16384 + sw128_offset(r, c & 7)) = pk;
      }
      l = l * alpha + ((rq[0] + rq[1]) + (rq[2] + rq[3]));
      m = mx;
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    // ------------------------------------------------------------ epilogue
    if (nb > 0 && ok) ok = mbar_wait(&o_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1, p.err);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (p.num_splits > 1) {
      const size_t rowid = (size_t)qtok * p.Hq + head;
      const size_t R = (size_t)p.total_tokens * p.Hq;
      const int split = blockIdx.z;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        if (nb > 0) {
          tmem_ld32(tO + c * 32 + lane_off, v);
          tmem_ld_wait();
        }
        if (row_ok) {
          float* dst = p.ws_o + ((size_t)split * R + rowid) * D + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) dst[i] = nb > 0 ? __uint_as_float(v[i]) : 0.f;
        }
      }
      if (row_ok) {
        p.ws_ml[((size_t)split * R + rowid) * 2 + 0] = m;
        p.ws_ml[((size_t)split * R + rowid) * 2 + 1] = l;
      }
    } else {
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        if (nb > 0) {
          tmem_ld32(tO + c * 32 + lane_off, v);
          tmem_ld_wait();
        }
        if (row_ok) {
          const size_t base = ((size_t)qtok * p.Hq + head) * D + c * 32;
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float a = nb > 0 ? __uint_as_float(v[2 * i]) * inv : 0.f;
            float b = nb > 0 ? __uint_as_float(v[2 * i + 1]) * inv : 0.f;
            if (p.gate) {
              const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(p.gate + base + 2 * i);
              a *= 1.f / (1.f + __expf(-__bfloat162float(g.x)));
              b *= 1.f / (1.f + __expf(-__bfloat162float(g.y)));
            }
            o[i] = pack_bf16(a, b);
          }
          uint4* dst = reinterpret_cast<uint4*>(p.out + base);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc<C::kTmemCols>(tmem);
}


// ---------------------------------------------------------------------------
// Decode specialization (every sequence has one query token).  Keys sit on the
// MMA's M axis and the G <= 16 query heads of a kv head on N (padded to 16):
//   S^T = K Q^T   (M=128 keys, N=16 heads, K=D)
//   O^T += V^T P^T (M=128 dims per half, N=16 heads, K=128 keys)
// A softmax thread owns one key of the block (16 scores), the per-head block
// max is a redux + smem reduction, the running row sums stay per thread and are
// reduced once at the end.  Work item = (sequence, kv head, key split).
//
// Pipelining (one persistent CTA per SM):
//  * S, P and O are double buffered (S and P per key block, O per work item), each
//    buffer with its own completion barrier, so softmax of block g overlaps the
//    P V MMA of block g-1 and only waits for the MMA of block g-2 before reusing a
//    P buffer;
//  * the next item's Q is staged right after the current item's last softmax, so
//    the MMA warp starts the next item's S while the softmax warps drain this O;
//  * lazy rescale (bf16): the running max moves only when a block's max exceeds it
//    by more than 2^8; below that P stays <= 256 and O keeps accumulating, so most
//    blocks skip the O rescale and its wait on the previous P V.
template <int D, bool F8 = false>
struct DecCfg {
  static constexpr int kBN = 128;                   // keys per block (2 pages)
  // F8: K, V, Q and P all e4m3 (kind::f8f6f4 MMAs); Q / P rows are D = 128 / 128 bytes
  static constexpr int kEl = F8 ? 1 : 2;
  static constexpr int kQbuf = F8 ? 2048 : (D / 64) * 2048;  // Q: [16 rows][128B] atoms
  static constexpr int kQ = 2 * kQbuf;
  static constexpr int kK = kBN * D * kEl;
  static constexpr int kV = kBN * D * kEl;
  static constexpr int kPbuf = F8 ? 2048 : 2 * 2048;  // P^T as [16 heads][128 keys]
  static constexpr int kP = 2 * kPbuf;
  static constexpr int kStages = F8 ? 4 : 3;
  static constexpr int kSmem = kQ + kStages * (kK + kV) + kP + 1024;
  static constexpr int kThreads = 320;  // softmax warps 0-3, TMA 4, MMA 5, epilogue 6-9
  static constexpr int kOcols = 16 * (D / 128 > 0 ? D / 128 : 1);
  static constexpr int kTmemCols = 32 + 2 * kOcols <= 64 ? 64 : 128;  // S^T x2 [0,32), O^T x2
  static constexpr float kLazy = F8 ? 0.f : 8.f;    // log2 headroom before the max moves
  static_assert(32 + 2 * kOcols <= kTmemCols, "TMEM");
  static_assert(!F8 || D == 128, "fp8 decode: head_dim 128");
};

__device__ __forceinline__ void soft_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The softmax warps' barrier with an OR of one predicate over its 128 threads.
__device__ __forceinline__ bool soft_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// GH: query heads per kv head rounded up to 4 (the per-head loops run over GH, the MMA's
// N stays 16 with P rows >= GH zero)
template <int D, bool F8, int GH>
__global__ void __launch_bounds__(DecCfg<D, F8>::kThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnArgs p) {
  pdl_enter();
  using C = DecCfg<D, F8>;
  constexpr int BN = C::kBN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::kQ;
  uint8_t* sP = sKV + C::kStages * (C::kK + C::kV);
  __shared__ __align__(8) uint64_t q_full[2], p_full[2], o_done[2];
  __shared__ __align__(8) uint64_t kv_full[C::kStages], kv_empty[C::kStages], s_full[2];
  // item hand-offs: softmax -> epilogue (row sums and max ready / consumed), MMA ->
  // epilogue (an item's last P V done) and epilogue -> MMA (its O buffer drained)
  __shared__ __align__(8) uint64_t ep_full[2], ep_free[2], o_final[2], o_free[2];
  __shared__ uint32_t tmem_sh;
  __shared__ float red[4][16];
  __shared__ float ep_l[2][4][16], ep_m[2][16];

  // Persistent: CTA b handles work items b, b + gridDim.x, ...; an item is a
  // (work item, kv head, key split) triple.  Every role walks the same item list, and
  // the KV pipeline (stages, S / P buffers, phases) runs on one global block counter g,
  // so the TMA producer streams the next item's keys while the current one finishes.
  // Barrier phases: buffer b of S / P / O is used by every other block (item), so the
  // k-th use of a buffer waits on parity k & 1, and no buffer can run two uses ahead of
  // its waiter (each reuse needs the previous use consumed).
  const int G = p.Hq / p.Hkv;
  const int n_items = (*p.num_work) * p.Hkv * p.num_splits;
  struct Item {
    int kvh, split, q_start, kv_len, kb0, nb, seq_pages;
    const int* bt;
  };
  auto item = [&](int it) {
    Item x;
    x.split = it % p.num_splits;
    const int rest = it / p.num_splits;
    x.kvh = rest % p.Hkv;
    const int seq = p.w_seq[rest / p.Hkv];
    x.q_start = p.q_start[seq];
    x.kv_len = p.kv_len[seq];
    const int kb_total = (x.kv_len + BN - 1) / BN;
    const int kb_chunk = (kb_total + p.num_splits - 1) / p.num_splits;
    x.kb0 = min(kb_total, x.split * kb_chunk);
    x.nb = min(kb_total, x.kb0 + kb_chunk) - x.kb0;
    x.bt = p.block_table + (size_t)seq * p.max_pages;
    x.seq_pages = (x.kv_len + 63) / 64;
    return x;
  };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 128);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_done[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&ep_full[b], 128);
      mbar_init(&ep_free[b], 128);
      mbar_init(&o_final[b], 1);
      mbar_init(&o_free[b], 128);
    }
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc<C::kTmemCols>(&tmem_sh);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t tS0 = tmem, tO0 = tmem + 32;

  if (warp == 4) {
    // TMA producer.  The warp fetches the page ids of up to 16 key blocks in one parallel
    // load (lane l: page l of the batch) and hands them to lane 0 by shuffles, so a block's
    // loads never wait on a block-table round trip; lane 0 alone waits and issues.
    bool ok = true;
    int jg = 0;  // global key-block counter of this CTA
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const Item x = item(it);
      for (int j0 = 0; j0 < x.nb && ok; j0 += 16) {
        const int pidx = (x.kb0 + j0) * (BN / 64) + lane;  // BN / 64 = 2 pages per block
        const int my_page = x.bt[pidx < x.seq_pages ? pidx : 0];
        const int jn = min(x.nb, j0 + 16);
        for (int j = j0; j < jn; ++j, ++jg) {
          const int s = jg % C::kStages;
          int pg_id[BN / 64];
#pragma unroll
          for (int pg = 0; pg < BN / 64; ++pg) pg_id[pg] = __shfl_sync(0xffffffffu, my_page, (j - j0) * (BN / 64) + pg);
          if (lane == 0) {
            if (jg >= C::kStages) ok = mbar_wait(&kv_empty[s], ((jg / C::kStages) - 1) & 1, p.err);
            if (ok) {
              uint8_t* sK = sKV + s * (C::kK + C::kV);
              uint8_t* sV = sK + C::kK;
              mbar_arrive_expect_tx(&kv_full[s], C::kK + C::kV);
#pragma unroll
              for (int pg = 0; pg < BN / 64; ++pg) {
                const int page = pg_id[pg];
                const int krow = (page * p.Hkv + x.kvh) * 64;
                if constexpr (F8) {
                  // e4m3 pages straight into the MMA operand layouts: K [128 keys][128 B] SW128,
                  // V^T pages [D][64 B] SW64
                  tma_load_2d(sK + pg * 8192, &tmK, &kv_full[s], 0, krow);
                  tma_load_2d(sV + pg * (D * 64), &tmV, &kv_full[s], 0, (page * p.Hkv + x.kvh) * D);
                } else {
                  for (int c = 0; c < D / 64; ++c)
                    tma_load_2d(sK + c * (BN * 128) + pg * 8192, &tmK, &kv_full[s], c * 64, krow);
                  tma_load_2d(sV + pg * (D * 128), &tmV, &kv_full[s], 0, (page * p.Hkv + x.kvh) * D);
                }
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (elect_one()) {
      bool ok = true;
      int jg = 0, qi = 0;  // global key-block / non-empty-item counters
      const uint32_t id16 = F8 ? idesc_f8(128, 16) : idesc_bf16(128, 16);
      auto issue_qk = [&](int g, const uint8_t* q) {
        const int s = g % C::kStages;
        uint8_t* sK = sKV + s * (C::kK + C::kV);
        if constexpr (F8) {
#pragma unroll
          for (int kk = 0; kk < D / 32; ++kk)  // 32 e4m3 = 32 B of K per MMA
            mma_f8(tS0 + (g & 1) * 16, desc_sw128_kmajor(sK) + 2 * kk, desc_sw128_kmajor(q) + 2 * kk, id16,
                   kk ? 1u : 0u);
        } else {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int c = kk >> 2, wi = kk & 3;
            mma_bf16(tS0 + (g & 1) * 16, desc_sw128_kmajor(sK + c * (BN * 128)) + 2 * wi,
                     desc_sw128_kmajor(q + c * 2048) + 2 * wi, id16, kk ? 1u : 0u);
          }
        }
        tc_commit(&s_full[g & 1]);
      };
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const Item x = item(it);
        if (x.nb == 0) continue;
        const uint8_t* q = sQ + (qi & 1) * C::kQbuf;
        const uint32_t tO = tO0 + (qi & 1) * C::kOcols;
        // the softmax warps staged this item's Q after the previous item's last block
        ok = mbar_wait(&q_full[qi & 1], (qi >> 1) & 1, p.err);
        const int qcur = qi++;
        // this item's O buffer was drained by the epilogue warps (item qcur - 2)
        if (qcur >= 2 && ok) ok = mbar_wait(&o_free[qcur & 1], ((qcur >> 1) - 1) & 1, p.err);
        if (ok) ok = mbar_wait(&kv_full[jg % C::kStages], (jg / C::kStages) & 1, p.err);
        if (ok) {
          tc_fence_after();
          issue_qk(jg, q);
        }
        for (int j = 0; j < x.nb && ok; ++j) {
          const int g = jg + j;
          if (j + 1 < x.nb) {
            ok = mbar_wait(&kv_full[(g + 1) % C::kStages], ((g + 1) / C::kStages) & 1, p.err);
            if (!ok) break;
            tc_fence_after();
            issue_qk(g + 1, q);
          }
          ok = mbar_wait(&p_full[g & 1], (g >> 1) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          uint8_t* sV = sKV + (g % C::kStages) * (C::kK + C::kV) + C::kK;
          const uint8_t* pb = sP + (g & 1) * C::kPbuf;
          if constexpr (F8) {
#pragma unroll
            for (int pg = 0; pg < BN / 64; ++pg)
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)  // 64 keys per page, 32 per MMA
                mma_f8(tO, desc_sw64_kmajor(sV + pg * (D * 64)) + 2 * kk, desc_sw128_kmajor(pb) + pg * 4 + kk * 2,
                       id16, (j | pg | kk) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              const int c = kk >> 2, wi = kk & 3;  // c = page within the block
#pragma unroll
              for (int h = 0; h < D / 128 || h == 0; ++h) {
                mma_bf16(tO + h * 16, desc_sw128_kmajor(sV + c * (D * 128) + h * 16384) + 2 * wi,
                         desc_sw128_kmajor(pb + c * 2048) + 2 * wi, id16, (j | kk) ? 1u : 0u);
                if (D < 128) break;
              }
            }
          }
          tc_commit(&o_done[g & 1]);
          tc_commit(&kv_empty[g % C::kStages]);
        }
        if (ok) tc_commit(&o_final[qcur & 1]);  // the item's O is complete
        jg += x.nb;
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    const int t = threadIdx.x;  // key within the block
    __shared__ float qsc[2][16];  // F8: per-head scale of the e4m3 query rows, per Q buffer
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    // Q of item `it` into buffer b (rows >= G zero); every softmax thread calls it
    auto stage_q = [&](int it, int b) {
      const Item x = item(it);
      const int qtok = x.q_start;
      uint8_t* q = sQ + b * C::kQbuf;
      if constexpr (F8) {
        // e4m3 [16 heads][128 B] (one SW128 atom column), scale amax/448 per head
        if (t < 16) {
          float am = 0.f;
          if (t < G) {
            const __nv_bfloat162* src =
                reinterpret_cast<const __nv_bfloat162*>(p.q + ((size_t)qtok * p.Hq + x.kvh * G + t) * D);
            for (int i = 0; i < D / 2; ++i) {
              const float2 f = __bfloat1622float2(src[i]);
              am = fmaxf(am, fmaxf(fabsf(f.x), fabsf(f.y)));
            }
          }
          qsc[b][t] = am > 0.f ? am / 448.f : 1.f;
        }
        soft_bar();
        for (int u = t; u < 16 * (D / 16); u += 128) {
          const int h = u / (D / 16), ch = u % (D / 16);
          uint32_t w[4] = {0, 0, 0, 0};
          if (h < G) {
            const __nv_bfloat162* src =
                reinterpret_cast<const __nv_bfloat162*>(p.q + ((size_t)qtok * p.Hq + x.kvh * G + h) * D + ch * 16);
            const float inv = 1.f / qsc[b][h];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float2 f = __bfloat1622float2(src[i]);
              f.x *= inv;
              f.y *= inv;
              const uint32_t pr = (uint32_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
              w[i >> 1] |= pr << (16 * (i & 1));
            }
          }
          *reinterpret_cast<uint4*>(q + sw128_offset(h, ch)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        for (int u = t; u < 16 * (D / 8); u += 128) {
          const int h = u / (D / 8), ch = u % (D / 8);
          uint4 v = make_uint4(0, 0, 0, 0);
          if (h < G) v = reinterpret_cast<const uint4*>(p.q + ((size_t)qtok * p.Hq + x.kvh * G + h) * D)[ch];
          *reinterpret_cast<uint4*>(q + (ch >> 3) * 2048 + sw128_offset(h, ch & 7)) = v;
        }
      }
      fence_proxy_async();
      mbar_arrive(&q_full[b]);
    };
    auto next_busy = [&](int it) {  // first item >= it of this CTA with key blocks
      for (; it < n_items; it += gridDim.x)
        if (item(it).nb > 0) return it;
      return n_items;
    };
    // P rows >= GH stay zero in both buffers (the MMA's N is 16); every block's P writes
    // come after its OR barrier, so they follow all of this zeroing
    if (GH < 16) {
      for (int i = t; i < C::kP / 16; i += 128) reinterpret_cast<uint4*>(sP)[i] = make_uint4(0, 0, 0, 0);
      fence_proxy_async();
    }
    int jg = 0, qi = 0, ei = 0;  // key blocks / non-empty items / items of this CTA
    {
      const int first = next_busy(blockIdx.x);
      if (first < n_items) stage_q(first, 0);
    }
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item(it);
      const int nb = x.nb, kb0 = x.kb0, kv_len = x.kv_len;
      const int ob = qi & 1;
      const uint32_t tO = tO0 + ob * C::kOcols;
      const float sl2 = p.scale * 1.4426950408889634f;
      float smul[GH];  // score multiplier per head (F8: query and key scales folded in)
#pragma unroll
      for (int h = 0; h < GH; ++h) smul[h] = F8 ? sl2 * qsc[ob][h] * p.k_scale : sl2;
      float m[GH], lp[GH];
#pragma unroll
      for (int h = 0; h < GH; ++h) {
        m[h] = -INFINITY;
        lp[h] = 0.f;
      }
      for (int j = 0; j < nb; ++j) {
        const int g = jg + j;
        if (ok) ok = mbar_wait(&s_full[g & 1], (g >> 1) & 1, p.err);
        tc_fence_after();
        uint32_t v[16];
        tmem_ld16(tS0 + (g & 1) * 16 + lane_off, v);
        tmem_ld_wait();
        const int key = (kb0 + j) * BN + t;
        const bool valid = key < kv_len;
        float s[GH];
        bool need = false;
#pragma unroll
        for (int h = 0; h < GH; ++h) {
          s[h] = (valid && h < G) ? __uint_as_float(v[h]) * smul[h] : -INFINITY;
          // the base moves on the first block, or when a score passes it by more than
          // kLazy: each thread checks its own key and one OR barrier makes it CTA-uniform,
          // so most blocks skip the per-head max reductions altogether
          need |= s[h] > m[h] + C::kLazy;
        }
        need = soft_bar_or(need);
        float alpha[GH];
        bool grow = false;
#pragma unroll
        for (int h = 0; h < GH; ++h) alpha[h] = 1.f;
        if (need) {
          // warp max per head in one redux.sync each, on an order-preserving integer image
          float bm[GH];
#pragma unroll
          for (int h = 0; h < GH; ++h) {
            const uint32_t b = __float_as_uint(s[h]);
            const uint32_t o = __reduce_max_sync(0xffffffffu, (b & 0x80000000u) ? ~b : (b | 0x80000000u));
            bm[h] = __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
          }
          if (lane < GH) {
            float xv = bm[0];
#pragma unroll
            for (int h = 1; h < GH; ++h) xv = lane == h ? bm[h] : xv;
            red[warp][lane] = xv;
          }
          soft_bar();
#pragma unroll
          for (int h = 0; h < GH; ++h) {
            const float b = fmaxf(fmaxf(red[0][h], red[1][h]), fmaxf(red[2][h], red[3][h]));
            const float mn = (m[h] == -INFINITY || b > m[h] + C::kLazy) ? fmaxf(m[h], b) : m[h];
            alpha[h] = (mn == -INFINITY || mn == m[h]) ? 1.f : exp2f(m[h] - mn);
            grow |= alpha[h] < 1.f;
            m[h] = mn;
          }
          // the next block's OR barrier orders these reads of `red` before its rewrite
        }
        // every thread holds the same m/alpha, so this branch is CTA-uniform
        if (j > 0 && grow) {
          // O holds blocks < g: wait for block g-1's P V before rescaling it in TMEM
          if (ok) ok = mbar_wait(&o_done[(g - 1) & 1], ((g - 1) >> 1) & 1, p.err);
          tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < (D >= 128 ? D / 128 : 1); ++hh) {
            uint32_t o[16];
            tmem_ld16(tO + hh * 16 + lane_off, o);
            tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < GH; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
            asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                         ::"r"(tO + hh * 16 + lane_off), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]),
                         "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7]), "r"(o[8]), "r"(o[9]), "r"(o[10]),
                         "r"(o[11]), "r"(o[12]), "r"(o[13]), "r"(o[14]), "r"(o[15])
                         : "memory");
          }
          tmem_st_wait();
        }
        // P buffer g & 1 was last read by block g-2's P V
        if (g >= 2 && ok) ok = mbar_wait(&o_done[g & 1], ((g - 2) >> 1) & 1, p.err);
        uint8_t* pb = sP + (g & 1) * C::kPbuf;
        // P^T [16 heads][128 keys]: this thread writes column t of head rows < GH (rows
        // >= GH were zeroed once at the start; F8: e4m3 of 256*P, one 128-B row per head,
        // the 256 is divided out at the end)
        const int c = t >> 6, kin = t & 63;
#pragma unroll
        for (int h = 0; h < GH; ++h) {
          const float e = (s[h] == -INFINITY) ? 0.f : ex2_approx(s[h] - m[h]);
          lp[h] = lp[h] * alpha[h] + e;
          if constexpr (F8) {
            pb[sw128_offset(h, t >> 4) + (t & 15)] = (uint8_t)__nv_cvt_float_to_fp8(e * 256.f, __NV_SATFINITE, __NV_E4M3);
          } else {
            const __nv_bfloat16 b = __float2bfloat16(e);
            *reinterpret_cast<__nv_bfloat16*>(pb + c * 2048 + sw128_offset(h, kin >> 3) + (kin & 7) * 2) = b;
          }
        }
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(&p_full[g & 1]);
        if (j == nb - 1) {
          // hand the MMA warp the next item's Q before draining this item's O
          const int nx = next_busy(it + gridDim.x);
          if (nx < n_items) stage_q(nx, (qi + 1) & 1);
        }
      }
      // ---------------- hand the item's row sums and max to the epilogue warps, which
      // drain O while these warps run the next item
      {
        const int eb = ei & 1;
        if (ei >= 2 && ok) ok = mbar_wait(&ep_free[eb], ((ei >> 1) - 1) & 1, p.err);
#pragma unroll
        for (int h = 0; h < GH; ++h)
          for (int off = 16; off; off >>= 1) lp[h] += __shfl_xor_sync(0xffffffffu, lp[h], off);
        if (lane < GH) {
          float xs = lp[0], xm = m[0];
#pragma unroll
          for (int h = 1; h < GH; ++h) {
            xs = lane == h ? lp[h] : xs;
            xm = lane == h ? m[h] : xm;
          }
          ep_l[eb][warp][lane] = xs;
          if (warp == 0) ep_m[eb][lane] = xm;
        }
        mbar_arrive(&ep_full[eb]);
      }
      jg += nb;
      if (nb > 0) ++qi;
      ++ei;
    }
  } else {
    // ---------------- epilogue warps 6-9: thread d = (warp & 3) * 32 + lane reads TMEM lane
    // d of the item's O (head dim d) once the MMA warp committed its last P V
    const int d = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const size_t R = (size_t)p.total_tokens * p.Hq;
    bool ok = true;
    int ei = 0, qi = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item(it);
      const int nb = x.nb, eb = ei & 1, kvh = x.kvh, qtok = x.q_start;
      if (ok) ok = mbar_wait(&ep_full[eb], (ei >> 1) & 1, p.err);
      uint32_t o[16];
      if (nb > 0) {
        if (ok) ok = mbar_wait(&o_final[qi & 1], (qi >> 1) & 1, p.err);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
        tc_fence_after();
        tmem_ld16(tO0 + (qi & 1) * C::kOcols + lane_off, o);
        tmem_ld_wait();
      }
#pragma unroll
      for (int h = 0; h < GH; ++h) {
        if (h >= G) break;
        const float L = ep_l[eb][0][h] + ep_l[eb][1][h] + ep_l[eb][2][h] + ep_l[eb][3][h];
        // F8: O accumulated 256*P times e4m3 V; undo both scales here
        const float ov = nb > 0 ? __uint_as_float(o[h]) * (F8 ? p.v_scale * (1.f / 256.f) : 1.f) : 0.f;
        const size_t rowid = (size_t)qtok * p.Hq + kvh * G + h;
        if (p.num_splits > 1) {
          p.ws_o[((size_t)x.split * R + rowid) * D + d] = ov;
          if (d == 0) {
            p.ws_ml[((size_t)x.split * R + rowid) * 2 + 0] = ep_m[eb][h];
            p.ws_ml[((size_t)x.split * R + rowid) * 2 + 1] = L;
          }
        } else {
          float xo = L > 0.f ? ov / L : 0.f;
          if (p.gate) xo *= 1.f / (1.f + __expf(-__bfloat162float(p.gate[rowid * D + d])));
          p.out[rowid * D + d] = __float2bfloat16(xo);
        }
      }
      tc_fence_before();  // the O reads precede the MMAs that reuse the buffer
      mbar_arrive(&ep_free[eb]);
      if (nb > 0) {
        mbar_arrive(&o_free[qi & 1]);
        ++qi;
      }
      ++ei;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc<C::kTmemCols>(tmem);
}

// Tensor maps of the paged caches: bf16 tiles land swizzled (SW128) in the operand
// layout; fp8 pages land unswizzled in the staging buffer (whole page rows).
static int make_kv_maps(CUtensorMap* tk, CUtensorMap* tv, const void* k_cache, const void* v_cache, int num_pages,
                        int Hkv, int D, bool f8) {
  if (f8) {
    int rc = make_tmap_2d(tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, (uint64_t)num_pages * Hkv * 64,
                          (uint64_t)D, D, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    return make_tmap_2d(tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 64, (uint64_t)num_pages * Hkv * D, 64, 64, D,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  int rc = make_tmap_2d(tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)num_pages * Hkv * 64,
                        (uint64_t)D * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return make_tmap_2d(tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, (uint64_t)num_pages * Hkv * D, 128, 64, D,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, bool F8>
static int attn_decode_launch_t(const AttnArgs& a, const void* k_cache, const void* v_cache, int num_pages,
                                int grid_work, cudaStream_t st) {
  using C = DecCfg<D, F8>;
  static_assert(C::kSmem <= 232448, "shared memory");
  CUtensorMap tk, tv;
  int rc;
  if (F8) {  // e4m3 pages land in the MMA operand layouts: K rows 128 B (SW128), V^T rows 64 B (SW64)
    rc = make_tmap_2d(&tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, (uint64_t)num_pages * a.Hkv * 64,
                      (uint64_t)D, D, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = make_tmap_2d(&tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 64, (uint64_t)num_pages * a.Hkv * D, 64, 64,
                        D, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    rc = make_kv_maps(&tk, &tv, k_cache, v_cache, num_pages, a.Hkv, D, false);
  }
  if (rc) return rc;
  const int G = a.Hq / a.Hkv;
  auto kern = G <= 4   ? attn_decode_kernel<D, F8, 4>
              : G <= 8  ? attn_decode_kernel<D, F8, 8>
              : G <= 12 ? attn_decode_kernel<D, F8, 12>
                        : attn_decode_kernel<D, F8, 16>;
  rc = ensure_smem_attr(kern, C::kSmem);
  if (rc) return rc;
  // persistent: one CTA per SM (shared memory allows one), each walks its share of items
  const int items = grid_work * a.Hkv * a.num_splits;
  launch_pdl(kern, dim3(dim3(items < num_sms() ? items : num_sms())), dim3(C::kThreads), C::kSmem, st, tk, tv, a);
  return (int)cudaGetLastError();
}

// Merge split-K partials: out = sum_s 2^(m_s-M) O_s / sum_s 2^(m_s-M) l_s.  One warp per
// (token, head) row, each lane four consecutive head dims per 128-wide pass (16-byte
// partial loads, 8-byte output stores); the sums run over the splits in order.
// SM > 0: at most SM splits and D <= 128 -- every load of the row ((m, l) and O of each
// split, the gate) is issued before the first use, one memory round trip instead of two
// (the O loads waited on (m, l)); same arithmetic in the same order as SM = 0.
template <int SM>
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ ws_o,
                                                           const float* __restrict__ ws_ml, int splits, size_t R,
                                                           int D, const __nv_bfloat16* __restrict__ gate,
                                                           __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  if constexpr (SM > 0) {
    const int d = lane * 4;
    const bool act = d < D;
    float2 ml[SM];
    float4 o[SM];
#pragma unroll
    for (int s = 0; s < SM; ++s) {
      if (s < splits) {
        ml[s] = *reinterpret_cast<const float2*>(ws_ml + (s * R + row) * 2);
        if (act) o[s] = *reinterpret_cast<const float4*>(ws_o + (s * R + row) * D + d);
      }
    }
    uint2 g = make_uint2(0u, 0u);
    if (gate && act) g = *reinterpret_cast<const uint2*>(gate + row * D + d);
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < SM; ++s)
      if (s < splits) M = fmaxf(M, ml[s].x);
    float L = 0.f;
#pragma unroll
    for (int s = 0; s < SM; ++s)
      if (s < splits && ml[s].x != -INFINITY) L += exp2f(ml[s].x - M) * ml[s].y;
    const float inv = L > 0.f ? 1.f / L : 0.f;
    if (!act) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < SM; ++s) {
      if (s >= splits || ml[s].x == -INFINITY) continue;
      const float wgt = exp2f(ml[s].x - M);
      acc.x += wgt * o[s].x;
      acc.y += wgt * o[s].y;
      acc.z += wgt * o[s].z;
      acc.w += wgt * o[s].w;
    }
    float v[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
    if (gate) {
      const float gf[4] = {__uint_as_float(g.x << 16), __uint_as_float(g.x & 0xffff0000u),
                           __uint_as_float(g.y << 16), __uint_as_float(g.y & 0xffff0000u)};
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] *= 1.f / (1.f + __expf(-gf[i]));
    }
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(out + row * D + d) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    return;
  }
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ws_ml[(s * R + row) * 2]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = ws_ml[(s * R + row) * 2];
    if (ms != -INFINITY) L += exp2f(ms - M) * ws_ml[(s * R + row) * 2 + 1];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = lane * 4; d < D; d += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      const float ms = ws_ml[(s * R + row) * 2];
      if (ms == -INFINITY) continue;
      const float wgt = exp2f(ms - M);
      const float4 o = *reinterpret_cast<const float4*>(ws_o + (s * R + row) * D + d);
      acc.x += wgt * o.x;
      acc.y += wgt * o.y;
      acc.z += wgt * o.z;
      acc.w += wgt * o.w;
    }
    float v[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
    if (gate) {
      const uint2 g = *reinterpret_cast<const uint2*>(gate + row * D + d);
      const float gf[4] = {__uint_as_float(g.x << 16), __uint_as_float(g.x & 0xffff0000u),
                           __uint_as_float(g.y << 16), __uint_as_float(g.y & 0xffff0000u)};
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] *= 1.f / (1.f + __expf(-gf[i]));
    }
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(out + row * D + d) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
  }
}

template <int D, int BN, bool F8>
static int attn_launch_t(const AttnArgs& a, const void* k_cache, const void* v_cache, int num_pages, int grid_work,
                         cudaStream_t st) {
  using C = AttnCfg<D, BN, F8>;
  static_assert(C::kSmem <= 232448, "shared memory");
  CUtensorMap tk, tv;
  int rc = make_kv_maps(&tk, &tv, k_cache, v_cache, num_pages, a.Hkv, D, F8);
  if (rc) return rc;
  auto kern = attn_kernel<D, BN, F8>;
  rc = ensure_smem_attr(kern, C::kSmem);
  if (rc) return rc;
  dim3 grid(grid_work, a.Hkv, a.num_splits);
  launch_pdl(kern, dim3(grid), dim3(C::kThreads), C::kSmem, st, tk, tv, a);
  return (int)cudaGetLastError();
}

int launch_attention(const AttnArgs& a, const void* k_cache, const void* v_cache, int num_pages, int grid_work,
                     cudaStream_t st) {
  if (a.page_size != 64 || grid_work <= 0) return grid_work == 0 ? 0 : -2;
  int rc;
  const bool f8 = a.kv_fp8 != 0;
  if (a.decode && a.Hq / a.Hkv <= 16 && a.D == 128) {
    rc = f8 ? attn_decode_launch_t<128, true>(a, k_cache, v_cache, num_pages, grid_work, st)
            : attn_decode_launch_t<128, false>(a, k_cache, v_cache, num_pages, grid_work, st);
  } else if (f8) {
    switch (a.D) {  // fp8 KV: head_dim <= 128 (a 256-wide fp8 stage does not fit next to the bf16 stages)
      case 64: rc = attn_launch_t<64, 128, true>(a, k_cache, v_cache, num_pages, grid_work, st); break;
      case 128: rc = attn_launch_t<128, 128, true>(a, k_cache, v_cache, num_pages, grid_work, st); break;
      default: return -2;
    }
  } else {
    switch (a.D) {
      case 64: rc = attn_launch_t<64, 128, false>(a, k_cache, v_cache, num_pages, grid_work, st); break;
      case 128:  // 64-key blocks in a 256-column TMEM allocation: two CTAs per SM overlap MMA and softmax
        rc = a.block_n == 128 ? attn_launch_t<128, 128, false>(a, k_cache, v_cache, num_pages, grid_work, st)
                              : attn_launch_t<128, 64, false>(a, k_cache, v_cache, num_pages, grid_work, st);
        break;
      case 256: rc = attn_launch_t<256, 64, false>(a, k_cache, v_cache, num_pages, grid_work, st); break;
      default: return -2;
    }
  }
  if (rc) return rc;
  if (a.num_splits > 1) {
    const size_t R = (size_t)a.total_tokens * a.Hq;
    if (a.D % 4) return -2;
    if (a.num_splits <= 4 && a.D <= 128)
      launch_pdl(attn_combine_kernel<4>, dim3((unsigned)((R + 7) / 8)), dim3(256), 0, st, a.ws_o, a.ws_ml,
                 a.num_splits, R, a.D, a.gate, a.out);
    else
      launch_pdl(attn_combine_kernel<0>, dim3((unsigned)((R + 7) / 8)), dim3(256), 0, st, a.ws_o, a.ws_ml,
                 a.num_splits, R, a.D, a.gate, a.out);
    rc = (int)cudaGetLastError();
  }
  return rc;
}

}  // namespace rkt
