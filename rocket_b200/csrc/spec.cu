// Speculative decoding (MTP draft / verify) bookkeeping on the device.
//
// spec_accept_kernel runs between the target model's verify pass and the MTP
// draft pass of one engine step, so a whole speculative step stays on the GPU
// (and inside one CUDA graph for a pure-verify batch):
//
//   * greedy longest-prefix acceptance: a verify sequence fed
//     [last, d_1 .. d_K] at rows q0 .. q0+K; the target's argmax y_i at row q0+i
//     is the token that follows; d_{i+1} is accepted while d_{i+1} == y_i.
//     n_acc = number of accepted drafts; the step emits y_0 .. y_{n_acc}.
//   * the token paired with each row's hidden state in the MTP pass: the next
//     prompt token for prefill rows (known on the host), otherwise the row's
//     own y.  Rows past the accepted prefix get garbage pairs; their MTP KV
//     entries sit at positions the next step overwrites.
//   * the row whose MTP output proposes the next first draft (q0 + n_acc), and
//     the positions / KV slots / context lengths of the K-1 later draft steps.
//     Sequences that do not sample this step draft into the scratch page.
//
// Reference counterparts: greedy acceptance and transactional commit of the
// speculative round (engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:640-720,
// DecodeEngine::step_spec / commit_positions in src/model.h).
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rkt {

__global__ void spec_accept_kernel(SpecAcceptArgs a) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < a.T) {
    const int nt = a.next_tok[i];
    const int oi = a.out_idx[i];
    a.mtp_ids[i] = nt >= 0 ? nt : (oi >= 0 ? a.y[oi] : 0);
  }
  if (i < a.S) {
    const int q0 = a.q_start[i], ql = a.q_len[i];
    int acc = 0;
    if (a.verify[i]) {
      while (acc < a.K && acc + 1 < ql) {
        const int oi = a.out_idx[q0 + acc];
        if (oi < 0 || a.ids[q0 + acc + 1] != a.y[oi]) break;
        ++acc;
      }
    }
    a.n_acc[i] = acc;
    const int row = a.verify[i] ? q0 + acc : q0 + ql - 1;
    a.mtp_rows[i] = row;
    const int p = a.pos[row];
    for (int j = 1; j < a.K; ++j) {
      const int dp = p + j;
      int slot, kvl;
      if (a.sample[i]) {
        const int page = a.block_table[(size_t)i * a.max_pages + dp / a.page_size];
        slot = page * a.page_size + dp % a.page_size;
        kvl = dp + 1;
      } else {  // no draft wanted: write into the scratch page, attend to one key
        slot = a.dummy_page * a.page_size + (j % a.page_size);
        kvl = 1;
      }
      a.d_pos[(size_t)(j - 1) * a.d_ld + i] = a.sample[i] ? dp : 0;
      a.d_slots[(size_t)(j - 1) * a.d_ld + i] = slot;
      a.d_kvlen[(size_t)(j - 1) * a.d_ld + i] = kvl;
    }
  }
}

int launch_spec_accept(const SpecAcceptArgs& a, cudaStream_t st) {
  const int n = a.T > a.S ? a.T : a.S;
  if (n == 0) return 0;
  if (a.K < 1 || a.d_ld < a.S) return -2;
  launch_pdl(spec_accept_kernel, dim3((n + 255) / 256), dim3(256), 0, st, a);
  return (int)cudaGetLastError();
}

}  // namespace rkt
