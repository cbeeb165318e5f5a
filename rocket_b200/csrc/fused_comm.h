// Host interface of the fused-collective kernels (fused_comm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm_types.h"

namespace rkt {

enum LandMode : int { LAND_NONE = 0, LAND_RS = 1, LAND_COMB = 2, LAND_AR = 3 };
enum LandOut : int { OUT_LOCAL = 0, OUT_AG = 1, OUT_AG_NV = 2 };

struct SpLandArgs {
  __nv_bfloat16* x = nullptr;            // [T_r, d] residual rows of this rank (in/out)
  const __nv_bfloat16* norm_w = nullptr; // [d]
  int d = 0, t_r = 0, mode = LAND_NONE, out = OUT_LOCAL, zero_centered = 0;
  float eps = 1e-6f;
  const float* rs = nullptr;             // LAND_RS: [n_part][T_r][d] fp32 (local view)
  int n_part = 0;
  const __nv_bfloat16* comb = nullptr;   // LAND_COMB: [T_r][k_out][d] bf16 (local view)
  const float* comb_w = nullptr;         //   [T_r][k_out] routing weights
  int k_out = 0;
  __nv_bfloat16* xn_local = nullptr;     // OUT_LOCAL destination [T_r, d]
  uint64_t ag_off = 0;                   // OUT_AG: bf16 gather buffer [T, d]
  uint64_t agq_off = 0, agsf_off = 0, agrs_off = 0;  // OUT_AG_NV: packed / scale atoms / row scales
  int wait_site = -1, signal_site = -1;
  int* err = nullptr;
};

// Replicated-token landing (ar_comm.cu): one CTA per token row.
struct ArLandArgs {
  __nv_bfloat16* x = nullptr;            // [T, d] residual rows (in/out, identical on every rank)
  const __nv_bfloat16* norm_w = nullptr; // [d] next RMSNorm weight, or null: no normalised output
  __nv_bfloat16* xn = nullptr;           // [T, d] normalised rows (when norm_w)
  int d = 0, mode = LAND_NONE, zero_centered = 0;
  float eps = 1e-6f;
  const __nv_bfloat16* ar = nullptr;     // LAND_AR: [world][ar_rows][d] bf16 partial rows (local view)
  int ar_rows = 0, world = 0;
  const __nv_bfloat16* comb = nullptr;   // LAND_COMB: [T][k_out][d] bf16 expert rows (local view)
  const float* comb_w = nullptr;         //   [T][k_out] routing weights
  int k_out = 0;
  int wait_site = -1;
  int* err = nullptr;
};

struct MoeCombinePushArgs {
  const __nv_bfloat16* y = nullptr;      // [rows, ldy] expert output rows (local)
  int ldy = 0, d = 0, k = 0;
  const int* pos = nullptr;              // [T][k] row of (token, slot), < 0: not on this rank
  const float* w = nullptr;              // [T][k] routing weights
  uint64_t ar_off = 0;                   // byte offset of the all-reduce buffer [world][ar_rows][d]
  int ar_rows = 0, signal_site = -1;
};

struct MoeSpArgs {
  const float* logits = nullptr;         // [T_r, ld] router logits of local tokens
  int ld_logits = 0, E = 0, top_k = 0, n_shared = 0, sigmoid = 0, norm_topk = 1, shared_gate_col = -1;
  float scaling = 1.f;
  const float* bias = nullptr;
  const __nv_bfloat16* xn = nullptr;     // [T_r, k] normed MoE input (local)
  int k = 0;
  float* comb_w = nullptr;               // [T_r][k_out] routing weights (local)
  int* cnt_local = nullptr;              // [E] per-expert row counter (zero between launches)
  int seg_rows = 0, cap = 0;             // owner segment height per expert, rows per source
  int blk_rows = 128;                    // owner plan block height (the grouped GEMM's token tile)
  uint64_t xq_off = 0, sf_off = 0, rs_off = 0, meta_off = 0, cnt_off = 0;  // symmetric heap offsets
  int signal_site = -1;
  // owner plan outputs (local)
  int* blk_expert = nullptr;
  int* blk_row = nullptr;
  int* blk_valid = nullptr;
  int* num_blocks = nullptr;
  int* row_list = nullptr;
  int* num_rows = nullptr;
  int* err = nullptr;
};

int peer_register(int slot, const uint64_t* bases, int rank, int world, uint64_t flag_off, uint32_t* counters);
const PeerPtrs* peer_get(int slot);
int ipc_get_handle(const void* ptr, void* out64);
int ipc_open(const void* handle64, void** out);
int ipc_close(void* ptr);
// Bounded wait for *flag == expect (at most limit_ns <= kWaitLimitNs); a timeout sets
// kErrPeerTimeout in *err and returns.
// Copy `bytes` (multiple of 16, 16-byte aligned) from local memory to dst (local or peer).
int launch_p2p_copy(const void* src, void* dst, size_t bytes, int blocks, cudaStream_t st);
int launch_flag_wait(const uint32_t* flag, uint32_t expect, unsigned long long limit_ns, int* err, cudaStream_t st);

int launch_sp_land(const SpLandArgs& a, int peer_slot, int t_r, cudaStream_t st);
int launch_ar_land(const ArLandArgs& a, int peer_slot, int T, cudaStream_t st);
int launch_moe_combine_push(const MoeCombinePushArgs& a, int peer_slot, int T, cudaStream_t st);
int launch_moe_dispatch_sp(const MoeSpArgs& a, int peer_slot, int t_r, cudaStream_t st);
int launch_moe_owner_plan_sp(const MoeSpArgs& a, int peer_slot, cudaStream_t st);
int launch_quantize_rows_list(const __nv_bfloat16* x, int ldx, int K, const int* rows, const int* n_rows,
                              uint8_t* packed, uint8_t* sf, float* row_scale, int sf_rows, int max_rows,
                              cudaStream_t st);

}  // namespace rkt
