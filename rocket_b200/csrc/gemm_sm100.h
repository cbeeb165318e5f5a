// Host interface of the sm_100a tcgen05 GEMM (see gemm_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm_types.h"

namespace rkt {

enum GemmEpilogue : int {
  EPI_STORE_BF16 = 0,     // out[row, n] = acc * w_global[e, n] * row_scale[row]         (bf16)
  EPI_STORE_F32 = 1,      // same, fp32
  EPI_SWIGLU = 2,         // tile rows = [64 gate | 64 up]; out[row, tile*64+i] = silu(g)*u (bf16)
  EPI_MOE_DOWN = 3,       // EPI_STORE_BF16 * row_weight[row]                            (bf16)
  EPI_RESIDUAL_BF16 = 4,  // out = residual + acc                                         (bf16)
  EPI_ARGMAX = 5,         // atomicMax of (orderable(acc), ~n) into u64 out[row]
  EPI_REDUCE_SCATTER = 6, // fp32 partial of token row t -> owner rank t / t_r, slot (rank*splits+split)
  EPI_COMBINE_PUSH = 7,   // expert output row -> its source rank's combine slot (token, j)  (bf16)
  EPI_AR_PUSH = 8,        // bf16 partial row -> slot `rank` of every rank's all-reduce buffer
  EPI_COMBINE_ALL = 9,    // expert output row (token, j) = meta[row] -> comb[token][j] on every rank (bf16)
};

struct GemmArgs {
  int nvf4 = 0;          // 1: NVFP4 block-scaled operands, 0: bf16
  int f8 = 0;            // 1: e4m3 operands (kind::f8f6f4); scales in w_global (per weight row) and
                         //    row_scale (per token); k counts e4m3 elements (multiple of 128)
  int n_w = 0;           // weight rows per expert (output features), multiple of 128
  int k = 0;             // contraction length
  int grouped = 0;       // 1: block list drives grid.y
  int num_experts = 1;
  int m_tokens = 0;      // non-grouped: token rows
  const int* block_expert = nullptr;
  const int* block_row = nullptr;
  const int* block_valid = nullptr;
  const int* num_blocks = nullptr;
  uint64_t ldb_bytes = 0;         // row stride of the token operand in bytes
  const uint8_t* sfa = nullptr;   // weight scale atoms [E][n_w/128][k/64][512]
  const uint8_t* sfb = nullptr;   // token scale atoms  [rows/128][k/64][512]
  const float* w_global = nullptr;  // [E*n_w] weight tensor scale per output row
  const float* row_scale = nullptr; // [rows] activation row scales
  const float* row_weight = nullptr;  // [rows] router weight (EPI_MOE_DOWN)
  const __nv_bfloat16* residual = nullptr;
  int ld_res = 0;
  // optional RMSNorm of the stored bf16 rows (EPI_RESIDUAL_BF16): norm_out = RMSNorm(out) * norm_w,
  // in the split-K reduce kernel when the GEMM splits K, else as a second launch
  const __nv_bfloat16* norm_w = nullptr;
  __nv_bfloat16* norm_out = nullptr;
  int ld_norm = 0, norm_zc = 0;
  float norm_eps = 1e-6f;
  int epi = EPI_STORE_BF16;
  void* out = nullptr;
  int ldo = 0;
  int n_valid = 1 << 30;   // EPI_ARGMAX: rows >= n_valid are padding
  int n_offset = 0;        // EPI_ARGMAX: id of row 0 (vocab shard offset)
  int splits = 1;          // split-K factor (non-grouped; fp32 partials + fixed-order reduce)
  // ---- fused collectives (peer memory; see comm.cuh / fused_comm.cu)
  int peer_slot = -1;      // registered PeerPtrs (copied into pp at launch)
  PeerPtrs pp;
  int wait_site = -1;      // TMA producer waits for this epoch before its first token load
  int signal_site = -1;    // the launch's last CTA publishes this epoch after all pushes
  uint64_t rs_off = 0;     // EPI_REDUCE_SCATTER: partial buffer offset in the symmetric heap
  int t_r = 0;             //   tokens per rank
  uint64_t comb_off = 0;   // EPI_COMBINE_PUSH: combine buffer offset in the symmetric heap
  int k_out = 0, seg_rows = 0, cap = 0;
  const int* counts = nullptr;  // [experts][kMaxRanks] rows received per source
  const int* meta = nullptr;    // [rows] (token << 8 | slot j) of every received row (-1: padding)
  uint64_t ar_off = 0;     // EPI_AR_PUSH: all-reduce buffer offset ([world][ar_rows][n_w] bf16)
  int ar_rows = 0;         //   row capacity of one rank's slot
  float* ws = nullptr;     // split-K workspace [splits][ws_rows][n_w] fp32
  int ws_rows = 0;
  int* err = nullptr;
};

// Launch.  A: weights ([E*n_w, k] bf16 or [E*n_w, k/2] packed e2m1);
// B: tokens ([b_rows, k] bf16 or [b_rows, k/2] packed).  grid_y = token blocks
// (non-grouped: ceil(m/bn); grouped: upper bound of the block list).
// bn selects the token tile (32, 128 or 256).  Returns 0 or an error code.
int gemm_launch(const GemmArgs& p, const void* A, const void* B, int b_rows, int grid_y, int bn, cudaStream_t st);

int num_sms();

// Programmatic dependent launch of the hot kernels (common.cuh launch_pdl); off unless
// ROCKET_PDL=1 or set_pdl(true).
bool pdl_supported();  // built with RKT_PDL (the kernels carry the device-side waits)
bool pdl_enabled();
void set_pdl(bool on);

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz);

}  // namespace rkt
