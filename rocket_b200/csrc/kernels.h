// Launchers of the framework's sm_100a kernels (raw pointers, no torch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rkt {

// ---------------------------------------------------------------- attention
struct AttnArgs {
  const __nv_bfloat16* q = nullptr;     // [T, Hq, D] (RoPE applied)
  __nv_bfloat16* out = nullptr;         // [T, Hq, D]
  const __nv_bfloat16* gate = nullptr;  // optional [T, Hq, D]: out *= sigmoid(gate)
  int Hq = 0, Hkv = 0, D = 0, page_size = 64;
  const int* block_table = nullptr;     // [S, max_pages]
  int max_pages = 0;
  const int* q_start = nullptr;         // [S] first token row of the sequence's queries
  const int* q_len = nullptr;           // [S]
  const int* kv_len = nullptr;          // [S] keys visible (incl. this step's)
  const int* w_seq = nullptr;           // [W] work item -> sequence
  const int* w_tok0 = nullptr;          // [W] first query (within the sequence) of the block
  const int* num_work = nullptr;        // device scalar W
  float scale = 1.f;
  int num_splits = 1;
  int decode = 0;                       // every sequence has q_len == 1 (decode kernel)
  int total_tokens = 0;                 // rows of q (for split workspaces)
  float* ws_o = nullptr;                // [splits, T*Hq, D] fp32
  float* ws_ml = nullptr;               // [splits, T*Hq, 2]
  int* err = nullptr;
  int kv_fp8 = 0;                       // caches hold e4m3 bytes: value = byte * k_scale / v_scale
  int block_n = 0;                      // generic kernel key block, D=128 bf16: 0/64 = 64 keys, two CTAs per SM; 128
  float k_scale = 1.f, v_scale = 1.f;
};
int launch_attention(const AttnArgs& a, const void* k_cache, const void* v_cache, int num_pages, int grid_work,
                     cudaStream_t st);

// ---------------------------------------------------------------- gated DeltaNet
struct GdnArgs {
  const __nv_bfloat16* proj = nullptr;  // [T, ld_proj]: q|k|v|z|b|a (local heads)
  int ld_proj = 0, z_off = 0;
  const __nv_bfloat16* conv_w = nullptr;  // [C, conv_k], C = 2*Hk*Dk + Hv*Dv
  __nv_bfloat16* conv_state = nullptr;    // [slots, conv_k-1, C]
  int conv_k = 4, Hk = 0, Hv = 0, Dk = 128, Dv = 128;
  const float* A_log = nullptr;           // [Hv]
  const float* dt_bias = nullptr;         // [Hv]
  const __nv_bfloat16* norm_w = nullptr;  // [Dv]
  float eps = 1e-6f;
  float* q = nullptr;                     // [T, Hk, Dk] scratch
  float* k = nullptr;                     // [T, Hk, Dk]
  float* v = nullptr;                     // [T, Hv, Dv]
  float* beta = nullptr;                  // [T, Hv]
  float* g = nullptr;                     // [T, Hv]
  float* state = nullptr;                 // [slots, Hv, Dk, Dv] fp32 recurrent state
  __nv_bfloat16* out = nullptr;           // [T, Hv*Dv]
  float* o_raw = nullptr;                 // [T, Hv, Dv] fp32 scan outputs before the gated norm
  const int* positions = nullptr;         // [T] absolute positions
  const int* q_start = nullptr;           // [S]
  const int* q_len = nullptr;             // [S]
  const int* state_slot = nullptr;        // [S]
  int n_seqs = 0;
  // Speculative verify: rows [0, spec_rows) belong to verify sequences.  Their
  // sequences keep the recurrent and conv state untouched (the scan starts from
  // it and does not write it back); k, v, g, beta and the raw conv inputs of
  // those rows are retained so that launch_gdn_commit can advance the state
  // over the accepted tokens only.
  int spec_rows = 0;
  float* rk = nullptr;                    // [spec_rows, Hk, Dk]
  float* rv = nullptr;                    // [spec_rows, Hv, Dv]
  float* rg = nullptr;                    // [spec_rows, Hv]  (log decay)
  float* rb = nullptr;                    // [spec_rows, Hv]  (beta)
  __nv_bfloat16* rx = nullptr;            // [spec_rows, C]   raw conv inputs
  // Kimi-style (KDA) variant: a log decay per (head, key channel) instead of per head,
  //   g[t,h,i] = gate_lb * sigmoid(exp(A_log[h]) * (f[t,h,i] + dt_bias[h*Dk+i]))
  // where the projection's "a" block is f [Hv*Dk]; g / rg are then [.., Hv, Dk].
  // out_sig: the output gate is sigmoid(z) instead of silu(z).
  int gate_ch = 0;
  float gate_lb = -5.f;
  int out_sig = 0;
  // T == S (one token per sequence): the fused one-token scan + gated norm kernel; 0 keeps
  // the scan and norm launches (the two paths give bit-identical results)
  int one_token_kernel = 1;
  int* err = nullptr;  // status word (bounded waits of the one-token kernel)
};
int launch_gdn(const GdnArgs& a, int T, int S, cudaStream_t st);

// Commit of a verify step for every DeltaNet layer at once: advance the state of
// each verify sequence s over its first n_acc[s] + 1 tokens (from the retained
// per-layer inputs) and shift its conv state the same way.
struct GdnCommitArgs {
  int n_layers = 0, Hk = 0, Hv = 0, D = 128, conv_k = 4, C = 0;
  float* state = nullptr;                 // [n_layers][slots][Hv][D][D]
  size_t state_layer_stride = 0;          // floats
  __nv_bfloat16* conv_state = nullptr;    // [n_layers][slots][conv_k-1][C]
  size_t conv_layer_stride = 0;           // elements
  const float* rk = nullptr; const float* rv = nullptr;  // [n_layers][R][H][D]
  const float* rg = nullptr; const float* rb = nullptr;  // [n_layers][R][Hv]
  const __nv_bfloat16* rx = nullptr;                     // [n_layers][R][C]
  int R = 0;                              // retained rows per layer
  const int* q_start = nullptr;           // [S]
  const int* state_slot = nullptr;        // [S]
  const int* n_acc = nullptr;             // [S] accepted drafts; the state advances n_acc + 1 tokens
  int n_verify = 0;                       // verify sequences (the first n_verify of the step)
  int gate_ch = 0;                        // rg holds per-channel log decays [.., Hv, D]
};
int launch_gdn_commit(const GdnCommitArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- speculative decoding
struct SpecAcceptArgs {
  int T = 0, S = 0, K = 0;                // rows, sequences, drafts per verify sequence
  const int* ids = nullptr;               // [T] fed tokens (verify rows: last token, then K drafts)
  const int* q_start = nullptr;           // [S]
  const int* q_len = nullptr;             // [S]
  const int* pos = nullptr;               // [T]
  const int* verify = nullptr;            // [S] 1 = verify sequence
  const int* sample = nullptr;            // [S] 1 = the sequence samples this step
  const int* y = nullptr;                 // [n_out] target argmax of each sampled row
  const int* out_idx = nullptr;           // [T] sampled index of a row, -1 if none
  const int* next_tok = nullptr;          // [T] known next token of a row, -1 = take the row's y
  const int* block_table = nullptr;       // [S][max_pages]
  int max_pages = 0, page_size = 64, dummy_page = 0;
  int* n_acc = nullptr;                   // [S]
  int* mtp_ids = nullptr;                 // [T] token paired with each row's hidden state in the draft pass
  long long* mtp_rows = nullptr;          // [S] row whose draft-pass output proposes the first draft
  int* d_pos = nullptr;                   // [K-1][d_ld] positions of the later draft steps
  int* d_slots = nullptr;                 // [K-1][d_ld]
  int* d_kvlen = nullptr;                 // [K-1][S]
  int d_ld = 0;                           // row stride of d_pos / d_slots / d_kvlen (>= S)
};
int launch_spec_accept(const SpecAcceptArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- MoE
int launch_router_topk(const float* logits, int ld, int T, int E, int top_k, int n_shared, int sigmoid_mode,
                       int norm_topk, float scaling, const float* bias, int shared_gate_col, int e_lo, int e_hi,
                       int shared_local, int* ids, float* weights, int* counts, cudaStream_t st);
int launch_router_plan(const float* logits, int ld, int T, int E, int top_k, int n_shared, int sigmoid_mode,
                       int norm_topk, float scaling, const float* bias, int shared_gate_col, int e_lo, int e_hi,
                       int shared_local, int* ids, float* weights, int* counts, int* ticket, int E_tot, int bn,
                       int* offsets, int* cursor, int* blk_expert, int* blk_row, int* blk_valid, int* num_blocks,
                       int max_blocks, int* total_rows, cudaStream_t st);
int launch_moe_plan(int* counts, int E_tot, int bn, int* offsets, int* cursor, int* blk_expert, int* blk_row,
                    int* blk_valid, int* num_blocks, int max_blocks, int* total_rows, cudaStream_t st);
int launch_moe_recount(const int* ids, int n, int E_tot, int* counts, cudaStream_t st);
int launch_quantize_nvfp4(const __nv_bfloat16* x, int ldx, int rows, int K, int mode, int ncopy, const int* ids,
                          const float* weights, int* cursor, int* pos, uint8_t* packed, uint8_t* sf,
                          float* row_scale, float* row_weight, int sf_rows, const float* g_in, int rows_per_g,
                          int* row_meta, cudaStream_t st);
int launch_moe_combine(const __nv_bfloat16* y, int ldy, const int* pos, const float* w, int k, int T, int D,
                       const __nv_bfloat16* residual, __nv_bfloat16* out, cudaStream_t st);
// moe_combine followed by the next sub-layer's RMSNorm of the stored rows (one kernel)
int launch_moe_combine_norm(const __nv_bfloat16* y, int ldy, const int* pos, const float* w, int k, int T, int D,
                            const __nv_bfloat16* residual, __nv_bfloat16* out, const __nv_bfloat16* norm_w,
                            __nv_bfloat16* norm_out, int ld_norm, float eps, int zero_centered, cudaStream_t st);

// ---------------------------------------------------------------- DSA sparse attention
struct DsaArgs {
  // indexer projection rows [T, ld_idx]: q_idx [Hi*Di] | k_idx [Di] | gate [Di] | head weights [Hi]
  const __nv_bfloat16* idx_proj = nullptr;
  int ld_idx = 0, Hi = 32, Di = 128, kpool = 4, top_k = 2048;
  float ln_eps = 1e-6f;
  const float* k_norm_w = nullptr;        // [Di]
  const float* k_norm_b = nullptr;        // [Di]
  const float* ape = nullptr;             // [kpool, Di] per-slot gate offsets
  __nv_bfloat16* ik_cache = nullptr;      // [pages * page_size, Di] indexer keys (one layer)
  __nv_bfloat16* ig_cache = nullptr;      // [pages * page_size, Di] compressor gates
  const int* slots = nullptr;             // [T] cache slot of each new token
  const int* positions = nullptr;         // [T]
  const int* q_start = nullptr;           // [S]
  int n_seqs = 0;
  const int* block_table = nullptr;       // [S, bt_ld]
  int bt_ld = 0, page_size = 64;
  float* scores = nullptr;                // [T, ld_scores] pool scores (scratch)
  int ld_scores = 0;
  int* sel = nullptr;                     // [T, ld_sel] selected token positions
  int ld_sel = 0;
  int* n_sel = nullptr;                   // [T]
  const __nv_bfloat16* q = nullptr;       // [T, Hq, D] (after norm / RoPE)
  const __nv_bfloat16* k_cache = nullptr; // [pages, Hkv, page_size, D]  (one layer)
  const __nv_bfloat16* v_cache = nullptr; // [pages, Hkv, D, page_size]
  const __nv_bfloat16* gate = nullptr;    // [T, Hq, D] output gate or null
  __nv_bfloat16* out = nullptr;           // [T, Hq, D]
  int Hq = 0, Hkv = 0, D = 128;
  float scale = 1.f;
  long long n_slots = 0;                  // cache slots (pages * page_size): debug bounds checks
  int* err = nullptr;
};
int launch_dsa_index_kv(const DsaArgs& a, int T, cudaStream_t st);
int launch_dsa_attention(const DsaArgs& a, int T, int max_pools, cudaStream_t st);

// ---------------------------------------------------------------- MLA (absorbed, NoPE)
struct MlaArgs {
  const __nv_bfloat16* kv_lat = nullptr;   // [T, ld_kv_lat] latent before its norm (x W_kva)
  int ld_kv_lat = 0;
  const __nv_bfloat16* kv_norm_w = nullptr;  // [512]
  float eps = 1e-6f;
  __nv_bfloat16* latent = nullptr;         // [pages * page_size, 512] latent cache (one layer)
  const int* slots = nullptr;              // [T]
  const __nv_bfloat16* q_nope = nullptr;   // [T, ld_q] heads x nope
  int ld_q = 0;
  const __nv_bfloat16* wk = nullptr;       // [H, nope, 512]
  const __nv_bfloat16* wv_t = nullptr;     // [H, 512, v]
  float* q_abs = nullptr;                  // [T, H, 512]
  float* ctx = nullptr;                    // [T, H, 512]
  __nv_bfloat16* out = nullptr;            // [T, ld_out] heads x v
  int ld_out = 0;
  int H = 0, nope = 0, v = 0;
  float scale = 1.f;
  const int* positions = nullptr;          // [T]
  const int* q_start = nullptr;            // [S]
  int n_seqs = 0;
  const int* block_table = nullptr;
  int bt_ld = 0, page_size = 64;
  const int* sel = nullptr;                // DSA selection [T, ld_sel] (null: every visible token)
  int ld_sel = 0;
  const int* n_sel = nullptr;
  int row0 = 0;                            // global index of row 0 (rows -> sequences via q_start)
  long long n_slots = 0;                   // latent cache rows: debug bounds checks
  int* err = nullptr;
};
int launch_mla_latent_write(const MlaArgs& a, int T, cudaStream_t st);
int launch_mla_attention(const MlaArgs& a, int T, cudaStream_t st);

// ---------------------------------------------------------------- FP8 activations
int launch_quantize_rows_fp8(const __nv_bfloat16* x, int ldx, int K, uint8_t* out, int ldo, float* row_scale, int rows,
                             cudaStream_t st);

// ---------------------------------------------------------------- probes
int launch_stamp(unsigned long long* out, int slot, cudaStream_t st);
// kind 0 copy a<-b, 1 read b (a: 4-byte sink), 2 triad a = b + 3c (fp32), 3 gather 64-byte rows a[r] = b[idx[r]];
// bytes: size of one stream (copy / read / triad) or of the gathered output
int launch_bw(int kind, void* a, const void* b, const void* c, const int* idx, size_t bytes, cudaStream_t st);

// ---------------------------------------------------------------- hyper-connections (mHC)
int launch_hc_split(int hc, const __nv_bfloat16* streams, const float* mix, int ld_mix, const float* base,
                    const float* scale, float* coef, __nv_bfloat16* x, int T, int d, float norm_eps, float hc_eps,
                    int iters, cudaStream_t st);
int launch_hc_combine(int hc, __nv_bfloat16* streams, const __nv_bfloat16* y, const float* coef, int T, int d,
                      cudaStream_t st);
int launch_hc_expand_mean(int hc, __nv_bfloat16* streams, __nv_bfloat16* x, int T, int d, int mode,
                          cudaStream_t st);

// ---------------------------------------------------------------- norm / rope / embed
int launch_rmsnorm(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int rows, int D, float eps,
                   int zero_centered, __nv_bfloat16* out, int ldo, cudaStream_t st);
int launch_qk_rope_kv(const __nv_bfloat16* qkv, int ld, int T, int Hq, int Hkv, int D, int rot, int has_gate,
                      const int* positions, const float* inv_freq, const __nv_bfloat16* qn_w,
                      const __nv_bfloat16* kn_w, float eps, int zero_centered, __nv_bfloat16* q_out,
                      __nv_bfloat16* gate_out, void* k_cache, void* v_cache, const int* slot_mapping,
                      int page_size, int kv_fp8, float k_scale, float v_scale, cudaStream_t st);
int launch_embed(const int* ids, const __nv_bfloat16* table, int T, int D, int vocab_lo, int vocab_hi,
                 __nv_bfloat16* out, cudaStream_t st);
int launch_argmax_finalize(unsigned long long* keys, int T, int* out_ids, float* out_vals, cudaStream_t st);

}  // namespace rkt
