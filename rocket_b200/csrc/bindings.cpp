// Python bindings of the sm_100a kernels.  Every op checks devices, dtypes and
// contiguity, launches on the current torch stream and raises on a launch
// error; there is no fallback path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "fused_comm.h"
#include "gemm_sm100.h"
#include "kernels.h"

namespace {

using at::Tensor;
using c10::optional;

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda() && (t).is_contiguous(), #t " must be a contiguous CUDA tensor")

template <typename T>
T* ptr(const optional<Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Per-device status word (ops.err_flag registers it): kernels without an explicit error
// argument OR their error bits into it.
static int* g_err[64] = {};
void set_err_flag(Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.device().index() < 64, "set_err_flag: int32 CUDA word");
  g_err[t.device().index()] = t.data_ptr<int>();
}
int* err_ptr(const c10::Device& d) { return d.index() >= 0 && d.index() < 64 ? g_err[d.index()] : nullptr; }

void check_rc(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }

// out[token, n] = X[token] . W[n]  (see gemm_sm100.cu).  `w` is [E*n_w, k] bf16
// or [E*n_w, k/2] uint8; `x` is [rows, k] bf16 or [rows, k/2] uint8.
void gemm(const Tensor& w, const Tensor& x, Tensor& out, int64_t epi, int64_t n_w, int64_t k, int64_t m_tokens,
          int64_t bn, const optional<Tensor>& sfa, const optional<Tensor>& sfb, const optional<Tensor>& w_global,
          const optional<Tensor>& row_scale, const optional<Tensor>& row_weight, const optional<Tensor>& residual,
          const optional<Tensor>& blk_expert, const optional<Tensor>& blk_row, const optional<Tensor>& blk_valid,
          const optional<Tensor>& num_blocks, int64_t grid_y, int64_t num_experts, int64_t n_valid,
          const optional<Tensor>& err, int64_t n_offset, int64_t splits, const optional<Tensor>& ws,
          const optional<py::dict>& fused) {
  CHECK_CUDA(w);
  TORCH_CHECK(x.is_cuda() && x.stride(-1) == 1, "x must be CUDA, unit inner stride");
  const c10::cuda::CUDAGuard g(w.device());
  rkt::GemmArgs a;
  a.nvf4 = w.scalar_type() == at::kByte;
  a.f8 = w.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(a.nvf4 ? x.scalar_type() == at::kByte
                     : a.f8 ? x.scalar_type() == at::kFloat8_e4m3fn
                            : (w.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16),
              "operand dtypes: both bf16, both e4m3 or both packed uint8");
  a.n_w = (int)n_w;
  a.k = (int)k;
  a.m_tokens = (int)m_tokens;
  a.grouped = blk_expert.has_value() ? 1 : 0;
  a.num_experts = (int)num_experts;
  a.block_expert = ptr<int>(blk_expert);
  a.block_row = ptr<int>(blk_row);
  a.block_valid = ptr<int>(blk_valid);
  a.num_blocks = ptr<int>(num_blocks);
  a.ldb_bytes = (uint64_t)x.stride(0) * x.element_size();
  a.sfa = ptr<uint8_t>(sfa);
  a.sfb = ptr<uint8_t>(sfb);
  if (a.nvf4) TORCH_CHECK(a.sfa && a.sfb, "NVFP4 GEMM needs both scale tensors");
  a.w_global = ptr<float>(w_global);
  a.row_scale = ptr<float>(row_scale);
  a.row_weight = ptr<float>(row_weight);
  a.residual = ptr<__nv_bfloat16>(residual);
  a.ld_res = residual.has_value() ? (int)residual->stride(0) : 0;
  a.epi = (int)epi;
  a.out = out.data_ptr();
  a.ldo = out.dim() > 1 ? (int)out.stride(0) : 1;
  a.n_valid = (int)n_valid;
  a.n_offset = (int)n_offset;
  a.splits = (int)splits;
  a.ws = ptr<float>(ws);
  a.ws_rows = ws.has_value() && splits > 1 ? (int)(ws->numel() / ((int64_t)splits * n_w)) : 0;
  if (fused.has_value()) {
    const py::dict& f = *fused;
    auto gi = [&](const char* k, int64_t dflt) { return f.contains(k) ? f[k].cast<int64_t>() : dflt; };
    a.peer_slot = (int)gi("peer_slot", -1);
    a.wait_site = (int)gi("wait_site", -1);
    a.signal_site = (int)gi("signal_site", -1);
    a.rs_off = (uint64_t)gi("rs_off", 0);
    a.t_r = (int)gi("t_r", 0);
    a.comb_off = (uint64_t)gi("comb_off", 0);
    a.k_out = (int)gi("k_out", 0);
    a.seg_rows = (int)gi("seg_rows", 0);
    a.cap = (int)gi("cap", 0);
    if (f.contains("counts")) a.counts = f["counts"].cast<Tensor>().data_ptr<int>();
    if (f.contains("meta")) a.meta = reinterpret_cast<const int*>(gi("meta", 0));
    a.ar_off = (uint64_t)gi("ar_off", 0);
    a.ar_rows = (int)gi("ar_rows", 0);
    if (f.contains("norm_w")) {  // RMSNorm of the stored rows (EPI_RESIDUAL_BF16)
      const Tensor nw = f["norm_w"].cast<Tensor>();
      Tensor no = f["norm_out"].cast<Tensor>();
      TORCH_CHECK(nw.scalar_type() == at::kBFloat16 && no.scalar_type() == at::kBFloat16 && nw.numel() == n_w &&
                      no.size(-1) == n_w && no.stride(-1) == 1 && no.size(0) >= m_tokens,
                  "gemm norm: weight [n] and output [m, n] bf16");
      a.norm_w = reinterpret_cast<const __nv_bfloat16*>(nw.data_ptr());
      a.norm_out = reinterpret_cast<__nv_bfloat16*>(no.data_ptr());
      a.ld_norm = (int)no.stride(0);
      a.norm_eps = (float)f["norm_eps"].cast<double>();
      a.norm_zc = (int)gi("norm_zc", 0);
    }
  }
  a.err = ptr<int>(err);
  const int b_rows = (int)x.size(0);
  int gy = (int)grid_y;
  // the token tile gemm_launch picks for `bn` (NVFP4 has no 64-row variant)
  const int tile = bn <= 32 ? 32 : bn <= 64 ? (a.nvf4 ? 128 : 64) : bn <= 128 ? 128 : 256;
  if (!a.grouped) gy = (int)((m_tokens + tile - 1) / tile);
  if (gy == 0) return;
  check_rc(rkt::gemm_launch(a, w.data_ptr(), x.data_ptr(), b_rows, gy, (int)bn, cur_stream()), "gemm");
}

void router_topk(const Tensor& logits, int64_t E, int64_t top_k, int64_t n_shared, bool sigmoid_mode, bool norm_topk,
                 double scaling, const optional<Tensor>& bias, int64_t shared_gate_col, int64_t e_lo, int64_t e_hi,
                 bool shared_local, Tensor& ids, Tensor& weights, Tensor& counts) {
  CHECK_CUDA(logits);
  const c10::cuda::CUDAGuard g(logits.device());
  check_rc(rkt::launch_router_topk(logits.data_ptr<float>(), (int)logits.stride(0), (int)logits.size(0), (int)E,
                                   (int)top_k, (int)n_shared, sigmoid_mode, norm_topk, (float)scaling, ptr<float>(bias),
                                   (int)shared_gate_col, (int)e_lo, (int)e_hi, shared_local, ids.data_ptr<int>(),
                                   weights.data_ptr<float>(),
                                   counts.data_ptr<int>(), cur_stream()),
           "router_topk");
}

void router_plan(const Tensor& logits, int64_t E, int64_t top_k, int64_t n_shared, bool sigmoid_mode, bool norm_topk,
                 double scaling, const optional<Tensor>& bias, int64_t shared_gate_col, int64_t e_lo, int64_t e_hi,
                 bool shared_local, Tensor& ids, Tensor& weights, Tensor& counts, Tensor& ticket, int64_t E_tot,
                 int64_t bn, Tensor& offsets, Tensor& cursor, Tensor& blk_expert, Tensor& blk_row, Tensor& blk_valid,
                 Tensor& num_blocks, Tensor& total_rows) {
  CHECK_CUDA(logits);
  TORCH_CHECK(counts.numel() >= E_tot && ticket.numel() >= 1, "router_plan: counts [E_tot] and ticket [1]");
  const c10::cuda::CUDAGuard g(logits.device());
  check_rc(rkt::launch_router_plan(logits.data_ptr<float>(), (int)logits.stride(0), (int)logits.size(0), (int)E,
                                   (int)top_k, (int)n_shared, sigmoid_mode, norm_topk, (float)scaling, ptr<float>(bias),
                                   (int)shared_gate_col, (int)e_lo, (int)e_hi, shared_local, ids.data_ptr<int>(),
                                   weights.data_ptr<float>(), counts.data_ptr<int>(), ticket.data_ptr<int>(),
                                   (int)E_tot, (int)bn, offsets.data_ptr<int>(),
                                   cursor.data_ptr<int>(), blk_expert.data_ptr<int>(), blk_row.data_ptr<int>(),
                                   blk_valid.data_ptr<int>(), num_blocks.data_ptr<int>(), (int)blk_expert.size(0),
                                   total_rows.data_ptr<int>(), cur_stream()),
           "router_plan");
}

void moe_plan(Tensor& counts, int64_t E_tot, int64_t bn, Tensor& offsets, Tensor& cursor, Tensor& blk_expert,
              Tensor& blk_row, Tensor& blk_valid, Tensor& num_blocks, Tensor& total_rows) {
  const c10::cuda::CUDAGuard g(counts.device());
  check_rc(rkt::launch_moe_plan(counts.data_ptr<int>(), (int)E_tot, (int)bn, offsets.data_ptr<int>(),
                                cursor.data_ptr<int>(), blk_expert.data_ptr<int>(), blk_row.data_ptr<int>(),
                                blk_valid.data_ptr<int>(), num_blocks.data_ptr<int>(), (int)blk_expert.size(0),
                                total_rows.data_ptr<int>(), cur_stream()),
           "moe_plan");
}

void moe_recount(const Tensor& ids, int64_t n, int64_t E_tot, Tensor& counts) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids: int32 CUDA contiguous");
  TORCH_CHECK(counts.is_cuda() && counts.scalar_type() == at::kInt && counts.numel() >= E_tot, "counts");
  TORCH_CHECK(n <= ids.numel(), "n exceeds ids");
  const c10::cuda::CUDAGuard g(ids.device());
  check_rc(rkt::launch_moe_recount(ids.data_ptr<int>(), (int)n, (int)E_tot, counts.data_ptr<int>(), cur_stream()),
           "moe_recount");
}

void quantize_nvfp4(const Tensor& x, int64_t rows, int64_t mode, int64_t ncopy, const optional<Tensor>& ids,
                    const optional<Tensor>& weights, const optional<Tensor>& cursor, const optional<Tensor>& pos,
                    Tensor& packed, Tensor& sf, const optional<Tensor>& row_scale, const optional<Tensor>& row_weight,
                    int64_t sf_rows, const optional<Tensor>& g_in, int64_t rows_per_g,
                    const optional<Tensor>& row_meta) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "x: bf16 CUDA");
  const c10::cuda::CUDAGuard g(x.device());
  check_rc(rkt::launch_quantize_nvfp4(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
                                      (int)rows, (int)x.size(1), (int)mode, (int)ncopy, ptr<int>(ids),
                                      ptr<float>(weights), ptr<int>(cursor), ptr<int>(pos),
                                      packed.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(), ptr<float>(row_scale),
                                      ptr<float>(row_weight), (int)sf_rows, ptr<float>(g_in), (int)rows_per_g,
                                      ptr<int>(row_meta), cur_stream()),
           "quantize_nvfp4");
}

void moe_combine(const Tensor& y, const Tensor& pos, const optional<Tensor>& w, int64_t k, int64_t T,
                 const optional<Tensor>& residual, Tensor& out, const optional<Tensor>& norm_w,
                 const optional<Tensor>& norm_out, double eps, int64_t zero_centered) {
  const c10::cuda::CUDAGuard g(y.device());
  if (norm_w.has_value()) {  // the next sub-layer's RMSNorm of the combined rows, same kernel
    TORCH_CHECK(norm_out.has_value() && norm_out->scalar_type() == at::kBFloat16 && norm_out->stride(-1) == 1 &&
                    norm_w->numel() == out.size(1),
                "moe_combine: norm weight [d] and bf16 output rows");
    check_rc(rkt::launch_moe_combine_norm(reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), (int)y.stride(0),
                                          pos.data_ptr<int>(), ptr<float>(w), (int)k, (int)T, (int)out.size(1),
                                          ptr<__nv_bfloat16>(residual),
                                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                          ptr<__nv_bfloat16>(norm_w), ptr<__nv_bfloat16>(norm_out),
                                          (int)norm_out->stride(0), (float)eps, (int)zero_centered, cur_stream()),
             "moe_combine_norm");
    return;
  }
  check_rc(rkt::launch_moe_combine(reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), (int)y.stride(0),
                                   pos.data_ptr<int>(), ptr<float>(w), (int)k, (int)T, (int)out.size(1),
                                   ptr<__nv_bfloat16>(residual), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                   cur_stream()),
           "moe_combine");
}

// mHC: streams [T, hc, d] bf16, mix [T, ld] f32 (raw W_mix . streams), coef [T, hc + hc*hc] f32
void hc_split(int64_t hc, const Tensor& streams, const Tensor& mix, const Tensor& base, const Tensor& scale,
              Tensor& coef, Tensor& x, int64_t T, double norm_eps, double hc_eps, int64_t iters) {
  CHECK_CUDA(streams);
  CHECK_CUDA(coef);
  const c10::cuda::CUDAGuard g(streams.device());
  TORCH_CHECK(mix.scalar_type() == at::kFloat && mix.stride(1) == 1 && base.scalar_type() == at::kFloat &&
              scale.scalar_type() == at::kFloat && coef.scalar_type() == at::kFloat, "hc_split: fp32 mix/base/scale/coef");
  TORCH_CHECK(streams.size(-1) == x.size(-1) && x.stride(0) == x.size(-1), "hc_split: x [T, d] contiguous");
  TORCH_CHECK(mix.size(1) >= 2 * hc + hc * hc && base.numel() >= 2 * hc + hc * hc && scale.numel() >= 3,
              "hc_split: mix / base / scale too small");
  check_rc(rkt::launch_hc_split((int)hc, reinterpret_cast<const __nv_bfloat16*>(streams.data_ptr()),
                                mix.data_ptr<float>(), (int)mix.stride(0), base.data_ptr<float>(),
                                scale.data_ptr<float>(), coef.data_ptr<float>(),
                                reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), (int)T, (int)x.size(-1),
                                (float)norm_eps, (float)hc_eps, (int)iters, cur_stream()),
           "hc_split");
}

void hc_combine(int64_t hc, Tensor& streams, const Tensor& y, const Tensor& coef, int64_t T) {
  CHECK_CUDA(streams);
  const c10::cuda::CUDAGuard g(streams.device());
  TORCH_CHECK(y.stride(0) == y.size(-1) && y.size(-1) == streams.size(-1), "hc_combine: y [T, d] contiguous");
  check_rc(rkt::launch_hc_combine((int)hc, reinterpret_cast<__nv_bfloat16*>(streams.data_ptr()),
                                  reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), coef.data_ptr<float>(),
                                  (int)T, (int)y.size(-1), cur_stream()),
           "hc_combine");
}

void hc_expand_mean(int64_t hc, Tensor& streams, Tensor& x, int64_t T, int64_t mode) {
  CHECK_CUDA(streams);
  const c10::cuda::CUDAGuard g(streams.device());
  TORCH_CHECK(x.stride(0) == x.size(-1) && x.size(-1) == streams.size(-1), "hc_expand_mean: x [T, d] contiguous");
  check_rc(rkt::launch_hc_expand_mean((int)hc, reinterpret_cast<__nv_bfloat16*>(streams.data_ptr()),
                                      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), (int)T, (int)x.size(-1),
                                      (int)mode, cur_stream()),
           "hc_expand_mean");
}

// DSA sparse attention: index caches + selection + sparse GQA attention of one layer
static rkt::DsaArgs dsa_args(const Tensor& idx_proj, int64_t Hi, int64_t Di, int64_t kpool, int64_t top_k,
                             const Tensor& k_norm_w, const Tensor& k_norm_b, const Tensor& ape, Tensor& ik_cache,
                             Tensor& ig_cache, const Tensor& slots, const Tensor& positions, const Tensor& q_start,
                             int64_t n_seqs, const Tensor& block_table, int64_t page_size) {
  TORCH_CHECK(idx_proj.scalar_type() == at::kBFloat16 && idx_proj.stride(1) == 1, "dsa: idx_proj bf16 rows");
  TORCH_CHECK(idx_proj.size(1) >= Hi * Di + 2 * Di + Hi, "dsa: idx_proj too narrow");
  TORCH_CHECK(ik_cache.scalar_type() == at::kBFloat16 && ig_cache.scalar_type() == at::kBFloat16 &&
              ik_cache.is_contiguous() && ig_cache.is_contiguous() && ik_cache.size(-1) == Di, "dsa: index caches");
  TORCH_CHECK(k_norm_w.scalar_type() == at::kFloat && k_norm_b.scalar_type() == at::kFloat &&
              ape.scalar_type() == at::kFloat && ape.numel() >= kpool * Di, "dsa: fp32 k_norm / ape");
  rkt::DsaArgs a;
  a.idx_proj = reinterpret_cast<const __nv_bfloat16*>(idx_proj.data_ptr());
  a.ld_idx = (int)idx_proj.stride(0);
  a.Hi = (int)Hi;
  a.Di = (int)Di;
  a.kpool = (int)kpool;
  a.top_k = (int)top_k;
  a.k_norm_w = k_norm_w.data_ptr<float>();
  a.k_norm_b = k_norm_b.data_ptr<float>();
  a.ape = ape.data_ptr<float>();
  a.ik_cache = reinterpret_cast<__nv_bfloat16*>(ik_cache.data_ptr());
  a.ig_cache = reinterpret_cast<__nv_bfloat16*>(ig_cache.data_ptr());
  a.slots = slots.data_ptr<int>();
  a.positions = positions.data_ptr<int>();
  a.q_start = q_start.data_ptr<int>();
  a.n_seqs = (int)n_seqs;
  a.block_table = block_table.data_ptr<int>();
  a.bt_ld = (int)block_table.stride(0);
  a.page_size = (int)page_size;
  a.n_slots = ik_cache.size(0);
  a.err = err_ptr(idx_proj.device());
  return a;
}

void dsa_index_kv(const Tensor& idx_proj, int64_t Hi, int64_t Di, int64_t kpool, int64_t top_k,
                  const Tensor& k_norm_w, const Tensor& k_norm_b, const Tensor& ape, Tensor& ik_cache,
                  Tensor& ig_cache, const Tensor& slots, const Tensor& positions, const Tensor& q_start,
                  int64_t n_seqs, const Tensor& block_table, int64_t page_size, int64_t T) {
  const c10::cuda::CUDAGuard g(idx_proj.device());
  rkt::DsaArgs a = dsa_args(idx_proj, Hi, Di, kpool, top_k, k_norm_w, k_norm_b, ape, ik_cache, ig_cache, slots,
                            positions, q_start, n_seqs, block_table, page_size);
  check_rc(rkt::launch_dsa_index_kv(a, (int)T, cur_stream()), "dsa_index_kv");
}

void dsa_attention(const Tensor& idx_proj, int64_t Hi, int64_t Di, int64_t kpool, int64_t top_k,
                   const Tensor& k_norm_w, const Tensor& k_norm_b, const Tensor& ape, Tensor& ik_cache,
                   Tensor& ig_cache, const Tensor& slots, const Tensor& positions, const Tensor& q_start,
                   int64_t n_seqs, const Tensor& block_table, int64_t page_size, Tensor& scores, Tensor& sel,
                   Tensor& n_sel, const Tensor& q, const Tensor& k_cache, const Tensor& v_cache,
                   const optional<Tensor>& gate, Tensor& out, int64_t Hq, int64_t Hkv, int64_t D, double scale,
                   int64_t T) {
  const c10::cuda::CUDAGuard g(idx_proj.device());
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16 && v_cache.scalar_type() == at::kBFloat16,
              "dsa_attention: bf16 KV cache only");
  TORCH_CHECK(scores.scalar_type() == at::kFloat && sel.scalar_type() == at::kInt && n_sel.scalar_type() == at::kInt,
              "dsa_attention: scratch dtypes");
  TORCH_CHECK(sel.size(1) >= top_k + kpool - 1, "dsa_attention: sel rows too short");
  rkt::DsaArgs a = dsa_args(idx_proj, Hi, Di, kpool, top_k, k_norm_w, k_norm_b, ape, ik_cache, ig_cache, slots,
                            positions, q_start, n_seqs, block_table, page_size);
  a.scores = scores.data_ptr<float>();
  a.ld_scores = (int)scores.stride(0);
  a.sel = sel.data_ptr<int>();
  a.ld_sel = (int)sel.stride(0);
  a.n_sel = n_sel.data_ptr<int>();
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.gate = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.scale = (float)scale;
  check_rc(rkt::launch_dsa_attention(a, (int)T, (int)scores.size(1), cur_stream()), "dsa_attention");
}

// DSA selection only (pool scores + top-k): MLA layers attend over it with their own kernel
void dsa_select(const Tensor& idx_proj, int64_t Hi, int64_t Di, int64_t kpool, int64_t top_k,
                const Tensor& k_norm_w, const Tensor& k_norm_b, const Tensor& ape, Tensor& ik_cache,
                Tensor& ig_cache, const Tensor& slots, const Tensor& positions, const Tensor& q_start,
                int64_t n_seqs, const Tensor& block_table, int64_t page_size, Tensor& scores, Tensor& sel,
                Tensor& n_sel, int64_t T) {
  const c10::cuda::CUDAGuard g(idx_proj.device());
  TORCH_CHECK(sel.size(1) >= top_k + kpool - 1, "dsa_select: sel rows too short");
  rkt::DsaArgs a = dsa_args(idx_proj, Hi, Di, kpool, top_k, k_norm_w, k_norm_b, ape, ik_cache, ig_cache, slots,
                            positions, q_start, n_seqs, block_table, page_size);
  a.scores = scores.data_ptr<float>();
  a.ld_scores = (int)scores.stride(0);
  a.sel = sel.data_ptr<int>();
  a.ld_sel = (int)sel.stride(0);
  a.n_sel = n_sel.data_ptr<int>();
  check_rc(rkt::launch_dsa_attention(a, (int)T, (int)scores.size(1), cur_stream()), "dsa_select");
}

// MLA: latent write (rmsnorm + scatter) then absorbed attention + value expansion
void mla_latent_write(const Tensor& kv_lat, const Tensor& kv_norm_w, double eps, Tensor& latent,
                      const Tensor& slots, int64_t T) {
  const c10::cuda::CUDAGuard g(kv_lat.device());
  TORCH_CHECK(kv_lat.stride(1) == 1 && kv_lat.size(1) >= 512 && latent.size(-1) == 512 && latent.is_contiguous(),
              "mla_latent_write: 512-wide latent");
  rkt::MlaArgs a;
  a.kv_lat = reinterpret_cast<const __nv_bfloat16*>(kv_lat.data_ptr());
  a.ld_kv_lat = (int)kv_lat.stride(0);
  a.kv_norm_w = reinterpret_cast<const __nv_bfloat16*>(kv_norm_w.data_ptr());
  a.eps = (float)eps;
  a.latent = reinterpret_cast<__nv_bfloat16*>(latent.data_ptr());
  a.slots = slots.data_ptr<int>();
  a.n_slots = latent.size(0);
  a.err = err_ptr(kv_lat.device());
  check_rc(rkt::launch_mla_latent_write(a, (int)T, cur_stream()), "mla_latent_write");
}

void mla_attention(const Tensor& q_nope, const Tensor& wk, const Tensor& wv_t, const Tensor& latent, Tensor& q_abs,
                   Tensor& ctx, Tensor& out, int64_t H, int64_t nope, int64_t v, double scale,
                   const Tensor& positions, const Tensor& q_start, int64_t n_seqs, const Tensor& block_table,
                   int64_t page_size, const optional<Tensor>& sel, const optional<Tensor>& n_sel, int64_t T,
                   int64_t row0) {
  const c10::cuda::CUDAGuard g(q_nope.device());
  TORCH_CHECK(wk.is_contiguous() && wv_t.is_contiguous() && wk.numel() == H * nope * 512 && wv_t.numel() == H * 512 * v,
              "mla_attention: W_k [H, nope, 512], W_v^T [H, 512, v]");
  TORCH_CHECK(q_abs.numel() >= T * H * 512 && ctx.numel() >= T * H * 512, "mla_attention: scratch too small");
  rkt::MlaArgs a;
  a.q_nope = reinterpret_cast<const __nv_bfloat16*>(q_nope.data_ptr());
  a.ld_q = (int)q_nope.stride(0);
  a.wk = reinterpret_cast<const __nv_bfloat16*>(wk.data_ptr());
  a.wv_t = reinterpret_cast<const __nv_bfloat16*>(wv_t.data_ptr());
  a.latent = reinterpret_cast<__nv_bfloat16*>(latent.data_ptr());
  a.q_abs = q_abs.data_ptr<float>();
  a.ctx = ctx.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = (int)out.stride(0);
  a.H = (int)H;
  a.nope = (int)nope;
  a.v = (int)v;
  a.scale = (float)scale;
  a.positions = positions.data_ptr<int>();
  a.q_start = q_start.data_ptr<int>();
  a.n_seqs = (int)n_seqs;
  a.block_table = block_table.data_ptr<int>();
  a.bt_ld = (int)block_table.stride(0);
  a.page_size = (int)page_size;
  a.row0 = (int)row0;
  a.n_slots = latent.size(0);
  a.err = err_ptr(q_nope.device());
  if (sel) {
    TORCH_CHECK(n_sel, "mla_attention: sel needs n_sel");
    a.sel = sel->data_ptr<int>();
    a.ld_sel = (int)sel->stride(0);
    a.n_sel = n_sel->data_ptr<int>();
  }
  check_rc(rkt::launch_mla_attention(a, (int)T, cur_stream()), "mla_attention");
}

void quantize_rows_fp8(const Tensor& x, Tensor& out, Tensor& row_scale, int64_t rows) {
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "quantize_rows_fp8: bf16 rows");
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.stride(1) == 1 && out.size(1) >= x.size(1),
              "quantize_rows_fp8: e4m3 output rows");
  TORCH_CHECK(row_scale.scalar_type() == at::kFloat && row_scale.numel() >= rows && x.size(0) >= rows &&
              out.size(0) >= rows, "quantize_rows_fp8: row scales");
  check_rc(rkt::launch_quantize_rows_fp8(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
                                         (int)x.size(1), reinterpret_cast<uint8_t*>(out.data_ptr()),
                                         (int)out.stride(0), row_scale.data_ptr<float>(), (int)rows, cur_stream()),
           "quantize_rows_fp8");
}

void device_stamp(Tensor& out, int64_t slot) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kLong && slot >= 0 && slot < out.numel(), "device_stamp: int64 slots");
  const c10::cuda::CUDAGuard g(out.device());
  check_rc(rkt::launch_stamp(reinterpret_cast<unsigned long long*>(out.data_ptr()), (int)slot, cur_stream()),
           "device_stamp");
}

void mem_bw(int64_t kind, Tensor& a, const Tensor& b, const optional<Tensor>& c, const optional<Tensor>& idx,
            int64_t bytes) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  const c10::cuda::CUDAGuard g(a.device());
  TORCH_CHECK(bytes % 64 == 0, "mem_bw: bytes must be a multiple of 64");
  const int64_t nb = b.numel() * b.element_size();
  if (kind == 3) {
    TORCH_CHECK(idx && idx->scalar_type() == at::kInt && idx->numel() >= bytes / 64, "mem_bw gather: int32 indices");
    TORCH_CHECK(a.numel() * a.element_size() >= bytes, "mem_bw gather: output too small");
  } else {
    TORCH_CHECK(nb >= bytes && (kind == 1 || a.numel() * a.element_size() >= bytes), "mem_bw: buffers too small");
    if (kind == 2) TORCH_CHECK(c && c->numel() * c->element_size() >= bytes, "mem_bw triad: c too small");
  }
  check_rc(rkt::launch_bw((int)kind, a.data_ptr(), b.data_ptr(), c ? c->data_ptr() : nullptr,
                          idx ? idx->data_ptr<int>() : nullptr, (size_t)bytes, cur_stream()),
           "mem_bw");
}

void rmsnorm(const Tensor& x, const Tensor& w, double eps, bool zero_centered, Tensor& out) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "x: bf16");
  const c10::cuda::CUDAGuard g(x.device());
  check_rc(rkt::launch_rmsnorm(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
                               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (int)x.size(0), (int)x.size(1),
                               (float)eps, zero_centered, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                               (int)out.stride(0), cur_stream()),
           "rmsnorm");
}

// A paged KV cache in fp8 (e4m3) holds one byte per value.
bool is_fp8_cache(const Tensor& t) {
  return t.scalar_type() == at::kFloat8_e4m3fn || t.scalar_type() == at::kByte;
}

void qk_rope_kv(const Tensor& qkv, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t rot, bool has_gate,
                const Tensor& positions, const Tensor& inv_freq, const optional<Tensor>& qn_w,
                const optional<Tensor>& kn_w, double eps, bool zero_centered, Tensor& q_out,
                const optional<Tensor>& gate_out, const optional<Tensor>& k_cache, const optional<Tensor>& v_cache,
                const optional<Tensor>& slot_mapping, int64_t page_size, double k_scale, double v_scale) {
  const c10::cuda::CUDAGuard g(qkv.device());
  const bool f8 = k_cache && k_cache->defined() && is_fp8_cache(*k_cache);
  if (k_cache && k_cache->defined() && v_cache && v_cache->defined())
    TORCH_CHECK(is_fp8_cache(*k_cache) == is_fp8_cache(*v_cache), "qk_rope_kv: K and V caches differ in dtype");
  check_rc(rkt::launch_qk_rope_kv(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), (int)qkv.stride(0), (int)T,
                                  (int)Hq, (int)Hkv, (int)D, (int)rot, has_gate, positions.data_ptr<int>(),
                                  inv_freq.data_ptr<float>(), ptr<__nv_bfloat16>(qn_w), ptr<__nv_bfloat16>(kn_w),
                                  (float)eps, zero_centered, reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
                                  ptr<__nv_bfloat16>(gate_out), ptr<void>(k_cache), ptr<void>(v_cache),
                                  ptr<int>(slot_mapping), (int)page_size, f8 ? 1 : 0, (float)k_scale, (float)v_scale,
                                  cur_stream()),
           "qk_rope_kv");
}

void embed(const Tensor& ids, const Tensor& table, int64_t vocab_lo, Tensor& out) {
  const c10::cuda::CUDAGuard g(ids.device());
  check_rc(rkt::launch_embed(ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                             (int)ids.size(0), (int)table.size(1), (int)vocab_lo, (int)(vocab_lo + table.size(0)),
                             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), cur_stream()),
           "embed");
}

void argmax_finalize(Tensor& keys, int64_t T, Tensor& out_ids, const optional<Tensor>& out_vals) {
  const c10::cuda::CUDAGuard g(keys.device());
  check_rc(rkt::launch_argmax_finalize(reinterpret_cast<unsigned long long*>(keys.data_ptr()), (int)T,
                                       out_ids.data_ptr<int>(), ptr<float>(out_vals), cur_stream()),
           "argmax_finalize");
}

void attention(const Tensor& q, Tensor& out, const optional<Tensor>& gate, const Tensor& k_cache,
               const Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t D, int64_t page_size, const Tensor& block_table,
               const Tensor& q_start, const Tensor& q_len, const Tensor& kv_len, const Tensor& w_seq,
               const Tensor& w_tok0, const Tensor& num_work, int64_t grid_work, double scale, int64_t num_splits,
               const optional<Tensor>& ws_o, const optional<Tensor>& ws_ml, const optional<Tensor>& err, bool decode,
               double k_scale, double v_scale, int64_t block_n) {
  CHECK_CUDA(q);
  const c10::cuda::CUDAGuard g(q.device());
  rkt::AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.gate = ptr<__nv_bfloat16>(gate);
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.page_size = (int)page_size;
  a.block_table = block_table.data_ptr<int>();
  a.max_pages = (int)block_table.size(1);
  a.q_start = q_start.data_ptr<int>();
  a.q_len = q_len.data_ptr<int>();
  a.kv_len = kv_len.data_ptr<int>();
  a.w_seq = w_seq.data_ptr<int>();
  a.w_tok0 = w_tok0.data_ptr<int>();
  a.num_work = num_work.data_ptr<int>();
  a.scale = (float)scale;
  a.num_splits = (int)num_splits;
  a.decode = decode ? 1 : 0;
  a.total_tokens = (int)q.size(0);
  a.ws_o = ptr<float>(ws_o);
  a.ws_ml = ptr<float>(ws_ml);
  a.err = ptr<int>(err);
  if (a.num_splits > 1) TORCH_CHECK(a.ws_o && a.ws_ml, "split attention needs workspaces");
  TORCH_CHECK(is_fp8_cache(k_cache) == is_fp8_cache(v_cache), "attention: K and V caches differ in dtype");
  a.kv_fp8 = is_fp8_cache(k_cache) ? 1 : 0;
  a.k_scale = (float)k_scale;
  a.v_scale = (float)v_scale;
  a.block_n = (int)block_n;
  const int num_pages = (int)(k_cache.numel() / (Hkv * page_size * D));
  check_rc(rkt::launch_attention(a, k_cache.data_ptr(), v_cache.data_ptr(), num_pages, (int)grid_work, cur_stream()),
           "attention");
}


void gdn(const Tensor& proj, const Tensor& conv_w, Tensor& conv_state, const Tensor& A_log, const Tensor& dt_bias,
         const Tensor& norm_w, Tensor& q, Tensor& k, Tensor& v, Tensor& beta, Tensor& g, Tensor& state, Tensor& out,
         const Tensor& positions, const Tensor& q_start, const Tensor& q_len, const Tensor& state_slot, int64_t Hk,
         int64_t Hv, int64_t conv_k, int64_t z_off, double eps, int64_t T, int64_t S, int64_t spec_rows,
         const optional<Tensor>& rk, const optional<Tensor>& rv, const optional<Tensor>& rg,
         const optional<Tensor>& rb, const optional<Tensor>& rx, int64_t gate_ch, double gate_lb, int64_t out_sig,
         Tensor& o_raw, int64_t one_token_kernel) {
  const c10::cuda::CUDAGuard g_(proj.device());
  rkt::GdnArgs a;
  TORCH_CHECK(o_raw.scalar_type() == at::kFloat && o_raw.is_contiguous() && o_raw.numel() >= T * Hv * 128,
              "gdn: o_raw [T, Hv, 128] fp32 scratch");
  a.o_raw = o_raw.data_ptr<float>();
  a.one_token_kernel = (int)one_token_kernel;
  a.err = err_ptr(proj.device());
  a.gate_ch = (int)gate_ch;
  a.gate_lb = (float)gate_lb;
  a.out_sig = (int)out_sig;
  TORCH_CHECK(g.numel() >= T * Hv * (gate_ch ? 128 : 1), "gdn: g buffer too small for the gate mode");
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ld_proj = (int)proj.stride(0);
  a.z_off = (int)z_off;
  a.conv_w = reinterpret_cast<const __nv_bfloat16*>(conv_w.data_ptr());
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.conv_k = (int)conv_k;
  a.Hk = (int)Hk;
  a.Hv = (int)Hv;
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.eps = (float)eps;
  a.q = q.data_ptr<float>();
  a.k = k.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.beta = beta.data_ptr<float>();
  a.g = g.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.positions = positions.data_ptr<int>();
  a.q_start = q_start.data_ptr<int>();
  a.q_len = q_len.data_ptr<int>();
  a.state_slot = state_slot.data_ptr<int>();
  a.n_seqs = (int)S;
  a.spec_rows = (int)spec_rows;
  if (spec_rows > 0) {
    TORCH_CHECK(rk && rv && rg && rb && rx, "gdn: spec_rows > 0 needs the retained buffers");
    a.rk = rk->data_ptr<float>();
    a.rv = rv->data_ptr<float>();
    a.rg = rg->data_ptr<float>();
    a.rb = rb->data_ptr<float>();
    a.rx = reinterpret_cast<__nv_bfloat16*>(rx->data_ptr());
  }
  check_rc(rkt::launch_gdn(a, (int)T, (int)S, cur_stream()), "gdn");
}

// state [L, slots, Hv, D, D] f32; conv_state [L, slots, K-1, C] bf16; retained rk [L, R, Hk, D],
// rv [L, R, Hv, D], rg/rb [L, R, Hv] f32, rx [L, R, C] bf16
void gdn_commit(Tensor& state, Tensor& conv_state, const Tensor& rk, const Tensor& rv, const Tensor& rg,
                const Tensor& rb, const Tensor& rx, const Tensor& q_start, const Tensor& state_slot,
                const Tensor& n_acc, int64_t n_verify, int64_t gate_ch) {
  const c10::cuda::CUDAGuard g_(state.device());
  rkt::GdnCommitArgs a;
  a.gate_ch = (int)gate_ch;
  a.n_layers = (int)state.size(0);
  a.Hv = (int)state.size(2);
  a.D = (int)state.size(3);
  a.Hk = (int)rk.size(2);
  a.conv_k = (int)conv_state.size(2) + 1;
  a.C = (int)conv_state.size(3);
  a.state = state.data_ptr<float>();
  a.state_layer_stride = (size_t)state.stride(0);
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.conv_layer_stride = (size_t)conv_state.stride(0);
  a.rk = rk.data_ptr<float>();
  a.rv = rv.data_ptr<float>();
  a.rg = rg.data_ptr<float>();
  a.rb = rb.data_ptr<float>();
  a.rx = reinterpret_cast<const __nv_bfloat16*>(rx.data_ptr());
  a.R = (int)rk.size(1);
  a.q_start = q_start.data_ptr<int>();
  a.state_slot = state_slot.data_ptr<int>();
  a.n_acc = n_acc.data_ptr<int>();
  a.n_verify = (int)n_verify;
  check_rc(rkt::launch_gdn_commit(a, cur_stream()), "gdn_commit");
}

void spec_accept(int64_t T, int64_t S, int64_t K, const Tensor& ids, const Tensor& q_start, const Tensor& q_len,
                 const Tensor& pos, const Tensor& verify, const Tensor& sample, const Tensor& y,
                 const Tensor& out_idx, const Tensor& next_tok, const Tensor& block_table, int64_t page_size,
                 int64_t dummy_page, Tensor& n_acc, Tensor& mtp_ids, Tensor& mtp_rows, Tensor& d_pos,
                 Tensor& d_slots, Tensor& d_kvlen) {
  const c10::cuda::CUDAGuard g_(ids.device());
  TORCH_CHECK(mtp_rows.scalar_type() == at::kLong, "spec_accept: mtp_rows must be int64");
  rkt::SpecAcceptArgs a;
  a.T = (int)T;
  a.S = (int)S;
  a.K = (int)K;
  a.ids = ids.data_ptr<int>();
  a.q_start = q_start.data_ptr<int>();
  a.q_len = q_len.data_ptr<int>();
  a.pos = pos.data_ptr<int>();
  a.verify = verify.data_ptr<int>();
  a.sample = sample.data_ptr<int>();
  a.y = y.data_ptr<int>();
  a.out_idx = out_idx.data_ptr<int>();
  a.next_tok = next_tok.data_ptr<int>();
  a.block_table = block_table.data_ptr<int>();
  a.max_pages = (int)block_table.size(1);
  a.page_size = (int)page_size;
  a.dummy_page = (int)dummy_page;
  a.n_acc = n_acc.data_ptr<int>();
  a.mtp_ids = mtp_ids.data_ptr<int>();
  a.mtp_rows = reinterpret_cast<long long*>(mtp_rows.data_ptr<int64_t>());
  a.d_pos = d_pos.data_ptr<int>();
  a.d_slots = d_slots.data_ptr<int>();
  a.d_kvlen = d_kvlen.data_ptr<int>();
  a.d_ld = (int)d_pos.stride(0);
  TORCH_CHECK(d_slots.stride(0) == d_pos.stride(0) && d_kvlen.stride(0) == d_pos.stride(0) &&
                  d_pos.size(0) >= K - 1 && d_pos.stride(0) >= S,
              "spec_accept: draft metadata must be [>=K-1][>=S] with one row stride");
  TORCH_CHECK(mtp_rows.numel() >= S && n_acc.numel() >= S && mtp_ids.numel() >= T, "spec_accept: outputs too small");
  check_rc(rkt::launch_spec_accept(a, cur_stream()), "spec_accept");
}

// ------------------------------------------------------------------ symmetric heap / IPC
Tensor symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, nbytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, nbytes) == cudaSuccess, "symm_alloc: memset failed");
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

Tensor ipc_handle(const Tensor& t) {
  auto h = torch::empty({64}, at::TensorOptions().dtype(at::kByte));
  check_rc(rkt::ipc_get_handle(t.data_ptr(), h.data_ptr()), "cudaIpcGetMemHandle");
  return h;
}

int64_t ipc_open(const Tensor& h, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  check_rc(rkt::ipc_open(h.data_ptr(), &p), "cudaIpcOpenMemHandle");
  return (int64_t)p;
}

void ipc_close(int64_t p) { rkt::ipc_close((void*)p); }

void p2p_copy(const Tensor& src, int64_t dst_ptr, int64_t bytes, int64_t blocks) {
  const c10::cuda::CUDAGuard g_(src.device());
  TORCH_CHECK(bytes <= src.numel() * src.element_size(), "p2p_copy: source too small");
  check_rc(rkt::launch_p2p_copy(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), (size_t)bytes, (int)blocks,
                                cur_stream()),
           "p2p_copy");
}

void flag_wait(const Tensor& flag, int64_t expect, int64_t limit_us, Tensor& err) {
  const c10::cuda::CUDAGuard g_(flag.device());
  TORCH_CHECK(flag.scalar_type() == at::kInt && err.scalar_type() == at::kInt, "flag_wait: int32 tensors");
  check_rc(rkt::launch_flag_wait(reinterpret_cast<const uint32_t*>(flag.data_ptr()), (uint32_t)expect,
                                 (unsigned long long)limit_us * 1000ull, err.data_ptr<int>(), cur_stream()),
           "flag_wait");
}

void peer_register(int64_t slot, std::vector<int64_t> bases, int64_t rank, int64_t world, int64_t flag_off,
                   const Tensor& counters) {
  std::vector<uint64_t> b(bases.begin(), bases.end());
  check_rc(rkt::peer_register((int)slot, b.data(), (int)rank, (int)world, (uint64_t)flag_off,
                              reinterpret_cast<uint32_t*>(counters.data_ptr())),
           "peer_register");
}

void sp_land(const Tensor& x, const Tensor& norm_w, double eps, bool zero_centered, int64_t t_r, int64_t mode,
             int64_t out, const optional<Tensor>& rs, int64_t n_part, const optional<Tensor>& comb,
             const optional<Tensor>& comb_w, int64_t k_out, const optional<Tensor>& xn_local, int64_t ag_off,
             int64_t agq_off, int64_t agsf_off, int64_t agrs_off, int64_t wait_site, int64_t signal_site,
             int64_t peer_slot, const optional<Tensor>& err) {
  const c10::cuda::CUDAGuard g(x.device());
  rkt::SpLandArgs a;
  a.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.d = (int)x.size(1);
  a.t_r = (int)t_r;
  a.mode = (int)mode;
  a.out = (int)out;
  a.zero_centered = zero_centered;
  a.eps = (float)eps;
  a.rs = ptr<float>(rs);
  a.n_part = (int)n_part;
  a.comb = ptr<__nv_bfloat16>(comb);
  a.comb_w = ptr<float>(comb_w);
  a.k_out = (int)k_out;
  a.xn_local = ptr<__nv_bfloat16>(xn_local);
  a.ag_off = (uint64_t)ag_off;
  a.agq_off = (uint64_t)agq_off;
  a.agsf_off = (uint64_t)agsf_off;
  a.agrs_off = (uint64_t)agrs_off;
  a.wait_site = (int)wait_site;
  a.signal_site = (int)signal_site;
  a.err = ptr<int>(err);
  check_rc(rkt::launch_sp_land(a, (int)peer_slot, (int)t_r, cur_stream()), "sp_land");
}

// Replicated-token landing: x[:T] (+)= fixed-order sum of the pushed partials / expert rows,
// then xn[:T] = RMSNorm(x) with norm_w (when given).  ar / comb are local views of the
// symmetric heap buffers; the wait is on `wait_site` of heap `peer_slot`.
void ar_land(const Tensor& x, int64_t T, int64_t mode, const optional<Tensor>& norm_w, const optional<Tensor>& xn,
             double eps, bool zero_centered, const optional<Tensor>& ar, int64_t ar_rows, int64_t world,
             const optional<Tensor>& comb, const optional<Tensor>& comb_w, int64_t k_out, int64_t wait_site,
             int64_t peer_slot, const optional<Tensor>& err) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x: contiguous bf16 CUDA");
  TORCH_CHECK(T <= x.size(0), "T exceeds x rows");
  const c10::cuda::CUDAGuard g(x.device());
  rkt::ArLandArgs a;
  a.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  a.norm_w = ptr<__nv_bfloat16>(norm_w);
  a.xn = ptr<__nv_bfloat16>(xn);
  if (xn.has_value()) TORCH_CHECK(xn->is_contiguous() && xn->size(1) == x.size(1) && xn->size(0) >= T, "xn");
  a.d = (int)x.size(1);
  a.mode = (int)mode;
  a.zero_centered = zero_centered;
  a.eps = (float)eps;
  a.ar = ptr<__nv_bfloat16>(ar);
  a.ar_rows = (int)ar_rows;
  a.world = (int)world;
  a.comb = ptr<__nv_bfloat16>(comb);
  a.comb_w = ptr<float>(comb_w);
  a.k_out = (int)k_out;
  a.wait_site = (int)wait_site;
  a.err = ptr<int>(err);
  check_rc(rkt::launch_ar_land(a, (int)peer_slot, (int)T, cur_stream()), "ar_land");
}

rkt::MoeSpArgs moe_sp_args(const py::dict& f) {
  rkt::MoeSpArgs a;
  auto gi = [&](const char* k, int64_t d) { return f.contains(k) ? f[k].cast<int64_t>() : d; };
  auto tp = [&](const char* k) -> void* { return f.contains(k) && !f[k].is_none() ? f[k].cast<Tensor>().data_ptr() : nullptr; };
  a.logits = (const float*)tp("logits");
  a.ld_logits = (int)gi("ld_logits", 0);
  a.E = (int)gi("E", 0);
  a.top_k = (int)gi("top_k", 0);
  a.n_shared = (int)gi("n_shared", 0);
  a.sigmoid = (int)gi("sigmoid", 0);
  a.norm_topk = (int)gi("norm_topk", 1);
  a.shared_gate_col = (int)gi("shared_gate_col", -1);
  a.scaling = f.contains("scaling") ? f["scaling"].cast<float>() : 1.f;
  a.bias = (const float*)tp("bias");
  a.xn = (const __nv_bfloat16*)tp("xn");
  a.k = (int)gi("k", 0);
  a.comb_w = (float*)tp("comb_w");
  a.cnt_local = (int*)tp("cnt_local");
  a.seg_rows = (int)gi("seg_rows", 0);
  a.cap = (int)gi("cap", 0);
  a.blk_rows = (int)gi("blk_rows", 128);
  a.xq_off = (uint64_t)gi("xq_off", 0);
  a.sf_off = (uint64_t)gi("sf_off", 0);
  a.rs_off = (uint64_t)gi("rs_off", 0);
  a.meta_off = (uint64_t)gi("meta_off", 0);
  a.cnt_off = (uint64_t)gi("cnt_off", 0);
  a.signal_site = (int)gi("signal_site", -1);
  a.blk_expert = (int*)tp("blk_expert");
  a.blk_row = (int*)tp("blk_row");
  a.blk_valid = (int*)tp("blk_valid");
  a.num_blocks = (int*)tp("num_blocks");
  a.row_list = (int*)tp("row_list");
  a.num_rows = (int*)tp("num_rows");
  a.err = (int*)tp("err");
  return a;
}

// y [rows, d] bf16 expert outputs, pos / weights [T, k]: this rank's partial MoE sums of
// T token rows pushed into slot `rank` of every rank's all-reduce buffer (byte offset
// ar_off of heap `peer_slot`), then the epoch of `signal_site`.
void moe_combine_push(const Tensor& y, const Tensor& pos, const Tensor& weights, int64_t k, int64_t T,
                      int64_t ar_off, int64_t ar_rows, int64_t peer_slot, int64_t signal_site) {
  CHECK_CUDA(y);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.stride(-1) == 1, "moe_combine_push: y bf16 rows");
  TORCH_CHECK(pos.scalar_type() == at::kInt && weights.scalar_type() == at::kFloat &&
                  pos.numel() >= T * k && weights.numel() >= T * k,
              "moe_combine_push: pos int32 / weights fp32 [T, k]");
  const c10::cuda::CUDAGuard g(y.device());
  rkt::MoeCombinePushArgs a;
  a.y = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  a.ldy = (int)y.stride(0);
  a.d = (int)y.size(-1);
  a.k = (int)k;
  a.pos = pos.data_ptr<int>();
  a.w = weights.data_ptr<float>();
  a.ar_off = (uint64_t)ar_off;
  a.ar_rows = (int)ar_rows;
  a.signal_site = (int)signal_site;
  check_rc(rkt::launch_moe_combine_push(a, (int)peer_slot, (int)T, cur_stream()), "moe_combine_push");
}

void moe_dispatch_sp(const py::dict& f, int64_t peer_slot, int64_t t_r) {
  check_rc(rkt::launch_moe_dispatch_sp(moe_sp_args(f), (int)peer_slot, (int)t_r, cur_stream()), "moe_dispatch_sp");
}

void moe_owner_plan_sp(const py::dict& f, int64_t peer_slot) {
  check_rc(rkt::launch_moe_owner_plan_sp(moe_sp_args(f), (int)peer_slot, cur_stream()), "moe_owner_plan_sp");
}

void quantize_rows_list(const Tensor& x, const Tensor& rows, const Tensor& n_rows, Tensor& packed, Tensor& sf,
                        Tensor& row_scale, int64_t sf_rows, int64_t max_rows) {
  const c10::cuda::CUDAGuard g(x.device());
  check_rc(rkt::launch_quantize_rows_list(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
                                          (int)x.size(1), rows.data_ptr<int>(), n_rows.data_ptr<int>(),
                                          packed.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(),
                                          row_scale.data_ptr<float>(), (int)sf_rows, (int)max_rows, cur_stream()),
           "quantize_rows_list");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "rocket_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("router_topk", &router_topk);
  m.def("moe_plan", &moe_plan);
  m.def("router_plan", &router_plan);
  m.def("moe_recount", &moe_recount);
  m.def("quantize_nvfp4", &quantize_nvfp4);
  m.def("moe_combine", &moe_combine);
  m.def("device_stamp", &device_stamp);
  m.def("set_err_flag", &set_err_flag);
  m.def("set_pdl", [](bool on) { rkt::set_pdl(on); });
  m.def("pdl_enabled", []() { return rkt::pdl_enabled(); });
  m.def("pdl_supported", []() { return rkt::pdl_supported(); });
  m.def("quantize_rows_fp8", &quantize_rows_fp8);
  m.def("dsa_index_kv", &dsa_index_kv);
  m.def("dsa_attention", &dsa_attention);
  m.def("dsa_select", &dsa_select);
  m.def("mla_latent_write", &mla_latent_write);
  m.def("mla_attention", &mla_attention);
  m.def("mem_bw", &mem_bw);
  m.def("hc_split", &hc_split);
  m.def("hc_combine", &hc_combine);
  m.def("hc_expand_mean", &hc_expand_mean);
  m.def("rmsnorm", &rmsnorm);
  m.def("qk_rope_kv", &qk_rope_kv);
  m.def("embed", &embed);
  m.def("argmax_finalize", &argmax_finalize);
  m.def("attention", &attention);
  m.def("gdn", &gdn);
  m.def("gdn_commit", &gdn_commit);
  m.def("flag_wait", &flag_wait);
  m.def("p2p_copy", &p2p_copy);
  m.def("spec_accept", &spec_accept);
  m.def("symm_alloc", &symm_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_register", &peer_register);
  m.def("sp_land", &sp_land);
  m.def("ar_land", &ar_land);
  m.def("moe_combine_push", &moe_combine_push);
  m.def("moe_dispatch_sp", &moe_dispatch_sp);
  m.def("moe_owner_plan_sp", &moe_owner_plan_sp);
  m.def("quantize_rows_list", &quantize_rows_list);
}
