// Reference-arm kernel controls: extern "C" entry points over the reference's own SIMT
// kernels, so kbench can time them on the same B200 next to this framework's kernels.
//
// The reference engine's kernel file (engines/glm5-moe-nvfp4-2b/src/kernels.cu with its
// headers) is compiled exactly as shipped; this file only forwards to its public host
// launchers (engines/glm5-moe-nvfp4-2b/src/kernels.h).  rocket_b200/refcontrols.py
// builds both into baseline/_ref/controls.so.  Nothing in the framework links it.
#include <cuda_runtime.h>

#include "kernels.h"

namespace re = rocket::engine;

extern "C" {

// rmsnorm over `batch` rows of n bf16 (kernels.h:69)
int ctl_rmsnorm(void* out, const void* x, const void* w, int batch, int n, float eps, void* stream) {
  re::rmsnorm(static_cast<re::bf16*>(out), static_cast<const re::bf16*>(x), static_cast<const re::bf16*>(w), batch,
              n, eps, static_cast<cudaStream_t>(stream));
  return (int)cudaGetLastError();
}

// sigmoid + bias top-k router, one block per token (kernels.h:212)
int ctl_moe_router(int* idx, float* w, const float* logits, const float* bias, int batch, int n_experts, int top_k,
                   int norm_topk, float scale, void* stream) {
  re::moe_router(idx, w, logits, bias, batch, n_experts, top_k, norm_topk != 0, scale,
                 static_cast<cudaStream_t>(stream));
  return (int)cudaGetLastError();
}

// NVFP4 quantization of gathered rows into the grouped-GEMM scale layout (kernels.h:250)
int ctl_nvfp4_quantize_rows(uint8_t* packed, uint8_t* sf, const void* x, const int* row_in_group,
                            const int* group_of_row, const long long* group_sf_base, int rows, int k, void* stream) {
  re::nvfp4_quantize_rows(packed, sf, static_cast<const re::bf16*>(x), row_in_group, group_of_row, group_sf_base,
                          rows, k, static_cast<cudaStream_t>(stream));
  return (int)cudaGetLastError();
}

// one KDA (per-channel gated delta rule) decode step on fp32 128x128 states, 64 heads
// (kernels.h:145)
int ctl_kda_step(float* state, void* o, const void* q, const void* k, const void* v, const void* g, const void* beta,
                 int batch, int heads, int head_dim, int row_stride, void* stream) {
  try {
    re::kda_recurrent_step(state, static_cast<re::bf16*>(o), static_cast<const re::bf16*>(q),
                           static_cast<const re::bf16*>(k), static_cast<const re::bf16*>(v),
                           static_cast<const re::bf16*>(g), static_cast<const re::bf16*>(beta), batch, heads,
                           head_dim, row_stride, static_cast<cudaStream_t>(stream));
  } catch (...) {
    return -2;
  }
  return (int)cudaGetLastError();
}

}  // extern "C"
