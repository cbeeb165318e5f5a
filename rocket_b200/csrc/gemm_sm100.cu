// Persistent tcgen05 GEMM for sm_100a: out[token, n] = sum_k X[token, k] * W[n, k].
//
// Orientation ("weights as A"): the MMA's M=128 rows are 128 weight rows
// (output features) and its N columns are tokens.  A decode step that routes
// 3 tokens to an expert therefore runs an N=16 MMA instead of wasting a
// 128-row token tile; prefill runs N=128/256 tiles.  The accumulator lives in
// TMEM (lane = output feature, column = token).
//
// Operand formats:
//   BF16  kind::f16, K-tile 64 elements (128 B rows, 128-byte swizzle)
//   FP8   kind::f8f6f4 e4m3 x e4m3, K-tile 128 elements (the same 128 B rows; the tensor
//         maps treat byte pairs as bf16 elements), per-weight-row and per-token scales
//         applied in the epilogue (the reference's FP8-row weights)
//   NVF4  kind::mxf4nvf4.block_scale.scale_vec::4X: packed e2m1 A and B, one
//         ue4m3 scale per 16 elements for both, K-tile 256 elements (128 B
//         rows).  Scales are staged in smem in 512-byte atoms (128 rows x 4)
//         and moved to TMEM with tcgen05.cp.32x128b.warpx4.
//
// Work units are (token block, 128-row weight tile, K split).  Each CTA is
// persistent: a TMA warp streams operand tiles of all its units through one
// smem ring, an MMA warp accumulates each unit into one of two TMEM
// accumulators, and four epilogue warps drain the other accumulator, so weight
// streaming never stops at unit boundaries (short-K GEMMs such as the MoE down
// projection stay bandwidth bound).  Split-K units write fp32 partials to a
// workspace reduced by splitk_reduce_kernel in a fixed order (deterministic).
//
// Grouped mode (MoE): the token rows of expert e occupy a segment of the
// gathered activation buffer aligned to the token tile's scale-atom height
// (32 rows for BN=32, 128 otherwise: a scale atom always starts at TMEM lane 0
// since the MMA's scale-factor TMEM address must be column aligned).  A
// device-side block list (expert, first row, valid rows) defines the units, so
// no host sync is needed.
//
// Reference counterparts: CUTLASS NVFP4 grouped GEMM
// (engines/glm5-moe-nvfp4-2b/src/moe_grouped.cu:29-303) and the SIMT/cuBLAS
// BF16 GEMMs (src/kernels.cu:57-138, 1286-1425).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdio.h>

#include "comm.cuh"
#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"
#include "rownorm.cuh"

#include <cstdlib>

namespace rkt {
const PeerPtrs* peer_get(int slot);
}

namespace rkt {

// Warps 0-3: epilogue group 0, warp 4: TMA, warp 5: MMA / TMEM, warps 6-9: epilogue
// group 1 (when the config has two accumulators and shared memory for a second staging
// tile): the groups drain alternate units, so short-K units (small experts) are not
// bound by one group's epilogue.
constexpr int kEpiStaticBytes = 32 * (128 + 4) * 4 + 4 * 32 * 8;  // staging tile + argmax keys per group

template <bool NVF4, int BN, int STAGES>
struct GemmCfg {
  static constexpr int kA = 128 * 128;               // A tile bytes per stage
  static constexpr int kB = BN * 128;                // B tile bytes per stage
  static constexpr int kSFA = NVF4 ? 2048 : 0;       // 4 atoms of 512 B
  static constexpr int kSFB = NVF4 ? (BN > 128 ? 4096 : 2048) : 0;
  static constexpr int kStage = kA + kB + kSFA + kSFB;
  static constexpr int kSmem = STAGES * kStage + 1024;  // + alignment slack
  static constexpr int kKT = NVF4 ? 256 : 64;         // K elements per stage
  static constexpr int kSfCols = NVF4 ? (16 + (BN > 128 ? 32 : 16)) : 0;  // TMEM cols per stage
  // two accumulators (epilogue of unit i overlaps the MMAs of unit i+1) when TMEM allows
  static constexpr int kAccBufs = (2 * BN + STAGES * kSfCols <= 512) ? 2 : 1;
  static constexpr int kColsNeeded = kAccBufs * BN + STAGES * kSfCols;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                 : kColsNeeded <= 256 ? 256 : 512;
  static_assert(kColsNeeded <= 512, "TMEM budget");
  static constexpr int kEpiGroups = (kAccBufs == 2 && kSmem + 2 * kEpiStaticBytes + 2048 <= 232448) ? 2 : 1;
  static constexpr int kThreads = 64 + 128 * kEpiGroups;
};

__device__ __forceinline__ uint32_t orderable_f32(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// named barrier of one epilogue group (ids 1 and 2; id 0 is __syncthreads)
__device__ __forceinline__ void epi_bar(int grp) { asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory"); }

struct Unit {
  int expert, row0, valid, m_tile, split, kt0, kt1;
};

template <int BN>
__device__ __forceinline__ Unit decode_unit(const GemmArgs& p, int u, int m_tiles, int num_kt) {
  Unit w;
  const int split = u % p.splits;
  const int rest = u / p.splits;
  w.m_tile = rest % m_tiles;
  const int b = rest / m_tiles;
  w.split = split;
  w.kt0 = (int)((long)split * num_kt / p.splits);
  w.kt1 = (int)((long)(split + 1) * num_kt / p.splits);
  if (p.grouped) {
    w.expert = p.block_expert[b];
    w.row0 = p.block_row[b];
    w.valid = p.block_valid[b];
  } else {
    w.expert = 0;
    w.row0 = b * BN;
    w.valid = min(BN, p.m_tokens - w.row0);
  }
  return w;
}

template <bool NVF4, int BN, int STAGES>
__global__ void __launch_bounds__(GemmCfg<NVF4, BN, STAGES>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  pdl_enter();
  using C = GemmCfg<NVF4, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ __align__(16) float stage_all[C::kEpiGroups][32][128 + 4];  // epilogue staging [token][feature]
  __shared__ unsigned long long amax_all[C::kEpiGroups][4][32];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = p.n_w / 128;
  const int num_kt = p.k / C::kKT;
  const int n_blocks = p.grouped ? *p.num_blocks : (p.m_tokens + BN - 1) / BN;
  const int n_units = n_blocks * m_tiles * p.splits;
  // CTAs without units still run to the end: the last-CTA signal counts every CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc<C::kTmemCols>(&tmem_base_sh);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int k_atoms = p.k / 64;  // 512-byte scale atoms per row block

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      bool ok = true;
      // all-gather -> GEMM: token rows pushed by the peers must have landed
      if (p.wait_site >= 0 && (int)blockIdx.x < n_units)
        ok = wait_peers(p.pp, p.wait_site, consumer_epoch(p.pp, p.wait_site), p.err);
      int it = 0;  // global k-tile counter across this CTA's units
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Unit w = decode_unit<BN>(p, u, m_tiles, num_kt);
        const int w_row0 = w.expert * p.n_w + w.m_tile * 128;
        const int b_boxes = (w.valid + 31) >> 5;
        const uint32_t tx = C::kA + b_boxes * 4096 + C::kSFA + (NVF4 ? (w.valid > 128 ? 4096 : 2048) : 0);
        for (int kt = w.kt0; kt < w.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES) ok = mbar_wait(&empty_bar[s], ((it / STAGES) - 1) & 1, p.err);
          if (!ok) break;
          uint8_t* st = smem + s * C::kStage;
          mbar_arrive_expect_tx(&full_bar[s], tx);
          const int kx = NVF4 ? kt * 128 : kt * 64;  // x coordinate in tensor-map elements
          tma_load_2d(st, &tmA, &full_bar[s], kx, w_row0);
          for (int b = 0; b < b_boxes; ++b)
            tma_load_2d(st + C::kA + b * 4096, &tmB, &full_bar[s], kx, w.row0 + b * 32);
          if constexpr (NVF4) {
            const uint8_t* sfa =
                p.sfa + ((size_t)(w.expert * m_tiles + w.m_tile) * k_atoms + kt * 4) * 512;
            bulk_load(st + C::kA + C::kB, sfa, 2048, &full_bar[s]);
            // token scale atoms hold 32 rows for BN=32 tiles, 128 rows otherwise
            const uint8_t* sfb = p.sfb + ((size_t)(w.row0 / (BN <= 32 ? 32 : 128)) * k_atoms + kt * 4) * 512;
            bulk_load(st + C::kA + C::kB + C::kSFA, sfb, 2048, &full_bar[s]);
            if (w.valid > 128)
              bulk_load(st + C::kA + C::kB + C::kSFA + 2048, sfb + (size_t)k_atoms * 512, 2048, &full_bar[s]);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      bool ok = true;
      int it = 0, i = 0;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++i) {
        const Unit w = decode_unit<BN>(p, u, m_tiles, num_kt);
        const int n_mma = min(BN, max(16, (w.valid + 15) & ~15));
        const uint32_t idesc = NVF4 ? idesc_nvf4(128, n_mma) : (p.f8 ? idesc_f8(128, n_mma) : idesc_bf16(128, n_mma));
        const int ab = i % C::kAccBufs;
        const int use = i / C::kAccBufs;
        if (use >= 1) ok = mbar_wait(&acc_empty[ab], (use - 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + ab * BN;
        for (int kt = w.kt0; kt < w.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          ok = mbar_wait(&full_bar[s], (it / STAGES) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          uint8_t* st = smem + s * C::kStage;
          const uint64_t adesc = desc_sw128_kmajor(st);
          const uint64_t bdesc = desc_sw128_kmajor(st + C::kA);
          const uint32_t first = kt == w.kt0 ? 1u : 0u;
          if constexpr (NVF4) {
            const uint32_t sfa_t = tmem + C::kAccBufs * BN + s * C::kSfCols;
            const uint32_t sfb_t = sfa_t + 16;
            const uint8_t* sfa_s = st + C::kA + C::kB;
            const uint8_t* sfb_s = sfa_s + C::kSFA;
#pragma unroll
            for (int a = 0; a < 4; ++a) {
              tmem_cp_32x128b_x4(sfa_t + a * 4, desc_sf_rows16(sfa_s + a * 512));
              if (BN > 128) {
                tmem_cp_32x128b_x4(sfb_t + a * 8, desc_sf_rows16(sfb_s + a * 512));
                tmem_cp_32x128b_x4(sfb_t + a * 8 + 4, desc_sf_rows16(sfb_s + 2048 + a * 512));
              } else {
                tmem_cp_32x128b_x4(sfb_t + a * 4, desc_sf_rows16(sfb_s + a * 512));
              }
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              // 64 fp4 = 32 bytes per MMA along K: +2 in the >>4 start-address field
              mma_nvf4(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, sfa_t + kk * 4, sfb_t + kk * (BN > 128 ? 8 : 4),
                       (first && kk == 0) ? 0u : 1u);
            }
          } else if (p.f8) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              // 32 e4m3 = 32 bytes per MMA along K (the same byte layout as the bf16 tiles)
              mma_f8(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              // 16 bf16 = 32 bytes per MMA along K
              mma_bf16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
            }
          }
          tc_commit(&empty_bar[s]);
        }
        tc_commit(&acc_full[ab]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps 0-3
    // Each thread owns one weight row (output feature) of the tile for 32 token
    // columns at a time; values are scaled, staged in smem as [token][feature]
    // fp32, and written back as 16-byte chunks of token rows (local or peer).
    const int grp = warp < 4 ? 0 : 1;            // warps 6-9 form group 1
    const int r = (warp & 3) * 32 + lane;         // weight row within the 128-row tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float(*stage)[128 + 4] = stage_all[grp];
    unsigned long long(*amax_sh)[32] = amax_all[grp];
    bool ok = true;
    // group g drains units i = g, g + G, ... (accumulator buffer i % kAccBufs)
    for (int u = blockIdx.x + grp * gridDim.x, i = grp; u < n_units;
         u += C::kEpiGroups * gridDim.x, i += C::kEpiGroups) {
      const Unit w = decode_unit<BN>(p, u, m_tiles, num_kt);
      const int ab = i % C::kAccBufs;
      if (ok) ok = mbar_wait(&acc_full[ab], (i / C::kAccBufs) & 1, p.err);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
      tc_fence_after();
      const int n = w.m_tile * 128 + r;
      const int n0 = w.m_tile * 128;
      // weight tensor scale of this output row (gate and up rows of a fused w13 keep their own)
      const float wg = p.w_global ? p.w_global[(size_t)w.expert * p.n_w + n] : 1.0f;
      const uint32_t acc = tmem + ab * BN + lane_off;
      const bool partial = p.splits > 1 && p.epi != EPI_REDUCE_SCATTER;
      for (int c0 = 0; c0 < w.valid; c0 += 32) {
        uint32_t v[32];
        if (ok) {
          tmem_ld32(acc + c0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0;
        }
        const int cn = min(32, w.valid - c0);
        if (p.epi == EPI_ARGMAX) {
          // per token: max over this tile's 128 vocab rows, ties to the lower id;
          // vocab-parallel ranks add their shard offset so ids are global
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(v[j]) * wg;
            if (p.row_scale && j < cn) x *= p.row_scale[w.row0 + c0 + j];
            unsigned long long key =
                n < p.n_valid ? ((unsigned long long)orderable_f32(x) << 32) | (uint32_t)(~(uint32_t)(n + p.n_offset))
                              : 0ull;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
              unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
              key = o > key ? o : key;
            }
            if (lane == 0) amax_sh[warp & 3][j] = key;
          }
          epi_bar(grp);
          if (r < cn) {
            unsigned long long k = amax_sh[0][r];
            for (int q = 1; q < 4; ++q) k = amax_sh[q][r] > k ? amax_sh[q][r] : k;
            atomicMax(reinterpret_cast<unsigned long long*>(p.out) + w.row0 + c0 + r, k);
          }
          epi_bar(grp);
          continue;
        }
        // ---- stage scaled values: stage[j][r], j = token column within the chunk
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = __uint_as_float(v[j]) * wg;
          if (p.row_scale && j < cn) x *= p.row_scale[w.row0 + c0 + j];
          if (p.epi == EPI_MOE_DOWN && p.row_weight && j < cn) x *= p.row_weight[w.row0 + c0 + j];
          stage[j][r] = x;
        }
        epi_bar(grp);
        if (p.epi == EPI_SWIGLU) {
          // tile rows [0,64) are gate rows, [64,128) the matching up rows: 64 outputs per token,
          // 8 chunks of 8 bf16 per token row
          for (int c = r; c < 32 * 8; c += 128) {
            const int j = c >> 3, q = c & 7;
            if (j < cn) {
              const int row = w.row0 + c0 + j;
              uint32_t o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float h0 = silu(stage[j][q * 8 + 2 * e]) * stage[j][64 + q * 8 + 2 * e];
                const float h1 = silu(stage[j][q * 8 + 2 * e + 1]) * stage[j][64 + q * 8 + 2 * e + 1];
                __nv_bfloat162 hb = __floats2bfloat162_rn(h0, h1);
                o[e] = *reinterpret_cast<uint32_t*>(&hb);
              }
              *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo +
                                        w.m_tile * 64 + q * 8) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        } else if (partial || p.epi == EPI_STORE_F32 || p.epi == EPI_REDUCE_SCATTER) {
          // fp32 rows: 32 chunks of 4 floats per token row
          for (int c = r; c < 32 * 32; c += 128) {
            const int j = c >> 5, q = c & 31;
            if (j < cn) {
              const int row = w.row0 + c0 + j;
              const float4 val = *reinterpret_cast<const float4*>(&stage[j][q * 4]);
              float* dst;
              if (partial) {
                dst = p.ws + ((size_t)w.split * p.ws_rows + row) * p.n_w + n0 + q * 4;
              } else if (p.epi == EPI_REDUCE_SCATTER) {
                // o_proj -> reduce-scatter: this rank's fp32 partial of token row t goes to
                // the owner of t, slot (rank * splits + split); the owner sums slots in order
                const int owner = row / p.t_r, lt = row - owner * p.t_r;
                const int slot = p.pp.rank * p.splits + w.split;
                dst = reinterpret_cast<float*>(p.pp.base[owner] + p.rs_off) + ((size_t)slot * p.t_r + lt) * p.n_w +
                      n0 + q * 4;
              } else {
                dst = reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + n0 + q * 4;
              }
              *reinterpret_cast<float4*>(dst) = val;
            }
          }
        } else {
          // bf16 rows: 16 chunks of 8 per token row (store / residual / combine push)
          for (int c = r; c < 32 * 16; c += 128) {
            const int j = c >> 4, q = c & 15;
            if (j >= cn) continue;
            const int row = w.row0 + c0 + j;
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = stage[j][q * 8 + e];
            __nv_bfloat16* dst;
            if (p.epi == EPI_AR_PUSH || p.epi == EPI_COMBINE_ALL) {
              // replicated-token layout: the row goes to every rank (this one included); the
              // landing kernel on each rank sums the slots in a fixed order
              size_t off;
              if (p.epi == EPI_AR_PUSH) {
                off = ((size_t)p.pp.rank * p.ar_rows + row) * p.n_w + n0 + q * 8;
              } else {
                const int mt = p.meta[row];
                if (mt < 0) continue;
                off = ((size_t)(mt >> 8) * p.k_out + (mt & 255)) * p.n_w + n0 + q * 8;
              }
              uint32_t o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 hb = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
                o[e] = *reinterpret_cast<uint32_t*>(&hb);
              }
              const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
              const uint64_t boff = (p.epi == EPI_AR_PUSH ? p.ar_off : p.comb_off) + off * 2;
              // start at a different rank per chunk so the CTAs spread their stores over the links
              for (int i = 0; i < p.pp.world; ++i) {
                int rr = p.pp.rank + i + c;
                rr %= p.pp.world;
                *reinterpret_cast<uint4*>(p.pp.base[rr] + boff) = ov;
              }
              continue;
            } else if (p.epi == EPI_COMBINE_PUSH) {
              // down projection -> combine: expert output row goes back to its source rank
              const int rr = row - w.expert * p.seg_rows;
              const int src = rr / p.cap, slot = rr - src * p.cap;
              if (slot >= p.counts[w.expert * kMaxRanks + src]) continue;
              const int mt = p.meta[row];
              dst = reinterpret_cast<__nv_bfloat16*>(p.pp.base[src] + p.comb_off) +
                    ((size_t)(mt >> 8) * p.k_out + (mt & 255)) * p.n_w + n0 + q * 8;
            } else {
              dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + n0 + q * 8;
              if (p.epi == EPI_RESIDUAL_BF16) {
                const uint4 rv = *reinterpret_cast<const uint4*>(p.residual + (size_t)row * p.ld_res + n0 + q * 8);
                const uint32_t r4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  y[2 * e] += bf16_bits_to_float(r4[e] & 0xffff);
                  y[2 * e + 1] += bf16_bits_to_float(r4[e] >> 16);
                }
              }
            }
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 hb = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
              o[e] = *reinterpret_cast<uint32_t*>(&hb);
            }
            *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        epi_bar(grp);  // stage is rewritten by the next chunk
      }
      // accumulator drained: hand it back to the MMA warp
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc<C::kTmemCols>(tmem);
  if (p.wait_site >= 0 || p.signal_site >= 0) {
    const int site = p.signal_site >= 0 ? p.signal_site : p.wait_site;
    if (last_block_done(arrival_counter(p.pp, site)) && threadIdx.x == 0) {
      if (p.wait_site >= 0) consumer_commit(p.pp, p.wait_site, consumer_epoch(p.pp, p.wait_site));
      if (p.signal_site >= 0) signal_peers(p.pp, p.signal_site);
    }
  }
}

// out[row, n] = sum_s ws[s][row][n] (+ residual), fixed order -> deterministic.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int rows, int n_w, int ws_rows,
                                     int epi, const __nv_bfloat16* __restrict__ residual, int ld_res, void* out,
                                     int ldo) {
  pdl_enter();
  const int row = blockIdx.y;
  for (int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4; n < n_w; n += gridDim.x * blockDim.x * 4) {
    float4 a = *reinterpret_cast<const float4*>(ws + (size_t)row * n_w + n);
    for (int s0 = 1; s0 < splits; s0 += 4) {  // loads four splits ahead of their adds (split order kept)
      float4 b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (s0 + u < splits) b[u] = *reinterpret_cast<const float4*>(ws + ((size_t)(s0 + u) * ws_rows + row) * n_w + n);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (s0 + u >= splits) continue;
        a.x += b[u].x;
        a.y += b[u].y;
        a.z += b[u].z;
        a.w += b[u].w;
      }
    }
    if (epi == EPI_STORE_F32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)row * ldo + n) = a;
    } else {
      if (epi == EPI_RESIDUAL_BF16) {
        const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(residual + (size_t)row * ld_res + n);
        const __nv_bfloat162 r0 = rp[0], r1 = rp[1];
        a.x += __bfloat162float(r0.x);
        a.y += __bfloat162float(r0.y);
        a.z += __bfloat162float(r1.x);
        a.w += __bfloat162float(r1.y);
      }
      __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(out) +
                                                              (size_t)row * ldo + n);
      op[0] = __floats2bfloat162_rn(a.x, a.y);
      op[1] = __floats2bfloat162_rn(a.z, a.w);
    }
  }
}

// a, b += the partials of splits 1.. (in split order) at ws + row * n_w + n, the loads
// issued four splits at a time ahead of their adds
__device__ __forceinline__ void splits_sum8(const GemmArgs& p, int row, int n, float4& a, float4& b) {
  for (int s0 = 1; s0 < p.splits; s0 += 4) {
    float4 e[4], f[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (s0 + u < p.splits) {
        const float* ws = p.ws + ((size_t)(s0 + u) * p.ws_rows + row) * p.n_w + n;
        e[u] = reinterpret_cast<const float4*>(ws)[0];
        f[u] = reinterpret_cast<const float4*>(ws)[1];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (s0 + u >= p.splits) continue;
      a.x += e[u].x; a.y += e[u].y; a.z += e[u].z; a.w += e[u].w;
      b.x += f[u].x; b.y += f[u].y; b.z += f[u].z; b.w += f[u].w;
    }
  }
}

// Split-K reduce + residual + RMSNorm (EPI_RESIDUAL_BF16 with a norm weight): one CTA per
// row, one 8-column chunk per thread.  The row sum repeats splitk_reduce_kernel's
// arithmetic (splits in order, then the residual), the bf16 row is stored and staged in
// shared memory, and the norm of the stored bits follows rmsnorm_vec_kernel's order
// (rn_inv_staged), so both outputs equal the two kernels' exactly.
__global__ void __launch_bounds__(1024) splitk_reduce_norm_kernel(GemmArgs p) {
  pdl_enter();
  const int row = blockIdx.x;
  const int nch = p.n_w >> 3;
  __shared__ uint4 sx[1024];
  __shared__ float red[32];
  const int ch = threadIdx.x;
  if (ch < nch) {
    const int n = ch * 8;
    const float* w0 = p.ws + (size_t)row * p.n_w + n;
    float4 a = reinterpret_cast<const float4*>(w0)[0], b = reinterpret_cast<const float4*>(w0)[1];
    splits_sum8(p, row, n, a, b);
    const uint4 r = *reinterpret_cast<const uint4*>(p.residual + (size_t)row * p.ld_res + n);
    const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
    const float v[8] = {a.x + rn_lo(rw[0]), a.y + rn_hi(rw[0]), a.z + rn_lo(rw[1]), a.w + rn_hi(rw[1]),
                        b.x + rn_lo(rw[2]), b.y + rn_hi(rw[2]), b.z + rn_lo(rw[3]), b.w + rn_hi(rw[3])};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
      o[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    sx[ch] = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + n) = sx[ch];
  }
  __syncthreads();
  const float inv = rn_inv_staged(sx, nch, red, p.n_w, p.norm_eps);
  if (ch < nch)
    reinterpret_cast<uint4*>(p.norm_out + (size_t)row * p.ld_norm)[ch] =
        rn_chunk_out(sx[ch], reinterpret_cast<const uint4*>(p.norm_w)[ch], inv, p.norm_zc);
}

// Split-K reduce of an EPI_AR_PUSH GEMM: row `row` of the fp32 partials summed in split
// order (deterministic), rounded to bf16 and stored into slot `rank` of every rank's
// all-reduce buffer; the launch's last CTA publishes the epoch to every rank.
// One CTA per row, one 8-column chunk per thread (a single wave at decode sizes: one
// system-scope fence per CTA before the arrival count).
__global__ void __launch_bounds__(640) splitk_reduce_push_kernel(GemmArgs p) {
  pdl_enter();
  const int row = blockIdx.x;
  for (int n = threadIdx.x * 8; n < p.n_w; n += blockDim.x * 8) {
    const float* w0 = p.ws + (size_t)row * p.n_w + n;
    float4 a = reinterpret_cast<const float4*>(w0)[0], b = reinterpret_cast<const float4*>(w0)[1];
    splits_sum8(p, row, n, a, b);
    uint32_t o[4];
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 hb = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
      o[e] = *reinterpret_cast<uint32_t*>(&hb);
    }
    const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
    const uint64_t boff = p.ar_off + (((size_t)p.pp.rank * p.ar_rows + row) * p.n_w + n) * 2;
    for (int i = 0; i < p.pp.world; ++i) {
      const int rr = (p.pp.rank + i + (n >> 3)) % p.pp.world;
      *reinterpret_cast<uint4*>(p.pp.base[rr] + boff) = ov;
    }
  }
  if (last_block_done(arrival_counter(p.pp, p.signal_site)) && threadIdx.x == 0) signal_peers(p.pp, p.signal_site);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  auto enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

static int g_pdl = -1;  // -1: not read yet

#ifdef RKT_PDL
constexpr bool kPdlBuilt = true;
#else
constexpr bool kPdlBuilt = false;  // kernels have no griddepcontrol.wait: PDL launches would race
#endif

bool pdl_supported() { return kPdlBuilt; }

bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = getenv("ROCKET_PDL");
    g_pdl = (kPdlBuilt && e && e[0] == '1') ? 1 : 0;
  }
  return g_pdl == 1;
}

void set_pdl(bool on) { g_pdl = (on && kPdlBuilt) ? 1 : 0; }

int ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({func, dev});
  if (it != done.end() && it->second >= bytes) return 0;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return (int)e;
  done[{func, dev}] = bytes;
  return 0;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <bool NVF4, int BN, int STAGES>
static int launch_t(const GemmArgs& p, const void* A, const void* B, int b_rows, int max_blocks, cudaStream_t st) {
  using C = GemmCfg<NVF4, BN, STAGES>;
  CUtensorMap ta, tb;
  const int E = p.grouped ? p.num_experts : 1;
  int rc;
  if (NVF4) {
    rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.k / 2, (uint64_t)E * p.n_w, p.k / 2, 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.k / 2, b_rows, p.ldb_bytes, 128, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.k, (uint64_t)E * p.n_w, (uint64_t)p.k * 2, 64,
                      128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.k, b_rows, p.ldb_bytes, 64, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  auto kern = gemm_kernel<NVF4, BN, STAGES>;
  rc = ensure_smem_attr(kern, C::kSmem);
  if (rc) return rc;
  // persistent grid: one CTA per SM, never more than the largest possible unit count
  const long units = (long)max_blocks * (p.n_w / 128) * p.splits;
  const int grid = (int)(units < num_sms() ? units : num_sms());
  launch_pdl(kern, dim3(grid), dim3(C::kThreads), C::kSmem, st, ta, tb, p);
  return (int)cudaGetLastError();
}

int gemm_launch(const GemmArgs& p_in, const void* A, const void* B, int b_rows, int grid_y, int bn, cudaStream_t st) {
  GemmArgs p = p_in;
  if (p.f8) {
    // e4m3 rows move through the bf16 tile path byte for byte: a 128-byte swizzle row holds
    // 128 e4m3 = 64 "bf16" elements, so the maps and k tiles are built on k / 2
    if (p.nvf4 || p.k % 128) return -2;
    p.k /= 2;
  }
  if (p.n_w % 128 || p.k % (p.nvf4 ? 256 : 64) || grid_y <= 0) return -2;
  if (p.splits < 1) p.splits = 1;
  if (p.peer_slot >= 0) {
    const PeerPtrs* pp = peer_get(p.peer_slot);
    if (!pp) return -4;
    p.pp = *pp;
  } else if (p.wait_site >= 0 || p.signal_site >= 0 || p.epi == EPI_REDUCE_SCATTER || p.epi == EPI_COMBINE_PUSH ||
             p.epi == EPI_AR_PUSH || p.epi == EPI_COMBINE_ALL) {
    return -4;
  }
  if (p.epi == EPI_COMBINE_ALL && p.splits > 1) return -3;
  if (p.epi == EPI_AR_PUSH && p.splits > 1 && (!p.ws || p.n_w % 8 || p.signal_site < 0)) return -3;
  if (p.epi == EPI_AR_PUSH && p.m_tokens > p.ar_rows) return -3;
  if (p.epi == EPI_COMBINE_ALL && (!p.meta || !p.grouped)) return -3;
  if (p.splits > 1 && p.epi != EPI_REDUCE_SCATTER) {
    if (!p.ws || p.grouped || p.epi == EPI_SWIGLU || p.epi == EPI_ARGMAX || p.epi == EPI_MOE_DOWN) return -3;
    if (p.ws_rows < p.m_tokens || p.n_w % 4) return -3;
  }
  int rc;
  // a split-K all-reduce push: the GEMM writes fp32 partials, the reduce kernel pushes and signals
  const bool ar_split = p.epi == EPI_AR_PUSH && p.splits > 1;
  const GemmArgs p_out = p;
  if (ar_split) p.signal_site = -1;
  if (p.nvf4) {
    if (bn <= 32) rc = launch_t<true, 32, 7>(p, A, B, b_rows, grid_y, st);
    else if (bn <= 128) rc = launch_t<true, 128, 5>(p, A, B, b_rows, grid_y, st);
    else rc = launch_t<true, 256, 3>(p, A, B, b_rows, grid_y, st);
  } else {
    if (bn <= 32) rc = launch_t<false, 32, 8>(p, A, B, b_rows, grid_y, st);
    else if (bn <= 64) rc = launch_t<false, 64, 8>(p, A, B, b_rows, grid_y, st);  // decode: 8 weight stages in flight
    else if (bn <= 128) rc = launch_t<false, 128, 6>(p, A, B, b_rows, grid_y, st);
    else rc = launch_t<false, 256, 4>(p, A, B, b_rows, grid_y, st);
  }
  const bool norm = p.norm_w && p.epi == EPI_RESIDUAL_BF16;
  if (!rc && norm && p.splits == 1)  // no split reduce to fold the norm into: a second launch
    return launch_rmsnorm(reinterpret_cast<const __nv_bfloat16*>(p.out), p.ldo, p.norm_w, p.m_tokens, p.n_w,
                          p.norm_eps, p.norm_zc, p.norm_out, p.ld_norm, st);
  if (rc || p.splits == 1 || p.epi == EPI_REDUCE_SCATTER) return rc;
  if (norm) {
    if (p.n_w % 8 || p.n_w > 8 * 1024 || !p.residual || !p.norm_out) return -2;
    const int th = ((p.n_w / 8 + 31) / 32) * 32;
    launch_pdl(splitk_reduce_norm_kernel, dim3(p.m_tokens), dim3(th < 128 ? 128 : th), 0, st, p);
    return (int)cudaGetLastError();
  }
  if (ar_split) {
    const int th = ((p.n_w / 8 + 31) / 32) * 32;
    launch_pdl(splitk_reduce_push_kernel, dim3(p.m_tokens), dim3(th < 128 ? 128 : th > 640 ? 640 : th), 0, st,
               p_out);
    return (int)cudaGetLastError();
  }
  dim3 grid((p.n_w / 4 + 255) / 256, p.m_tokens);
  launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, st, p.ws, p.splits, p.m_tokens, p.n_w, p.ws_rows, p.epi, p.residual,
                                             p.ld_res, p.out, p.ldo);
  return (int)cudaGetLastError();
}

}  // namespace rkt
