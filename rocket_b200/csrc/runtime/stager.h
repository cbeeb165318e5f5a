// Native step staging: reserve KV slots for one engine step and write the step's int32
// metadata (token ids, positions, KV slots, per-sequence query ranges, attention work
// items, sampled rows, speculative verify / sample flags, next-token targets) into the
// engine's packed host buffer, plus the block-table rows -- the per-step host work that
// runs before every graph replay.
//
// Sequences arrive in the scheduler's order; a decode batch is padded to its graph bucket
// with dummy sequences on a scratch page (K + 1 rows each under speculation).  The field
// semantics are those of the engine's metadata buffer (engine/engine.py), and the Python
// restatement there is the test oracle for this code.
#pragma once
#include <cstdint>
#include <vector>

#include "kv_manager.h"

namespace rkt_rt {

struct StageItem {
  int64_t rid = 0;
  std::vector<int32_t> tokens;      // tokens fed this step
  int32_t start = 0;                // position of tokens[0]
  int32_t sample = 0, verify = 0, reserve = 0;
  int32_t state_slot = 0;
  std::vector<int32_t> next_prompt;  // prefill rows under speculation: the prompt tokens that follow
};

// Offsets (int32 elements) of the fields inside the packed metadata buffer; -1 = absent.
struct MetaLayout {
  int ids = -1, pos = -1, slots = -1, q_start = -1, q_len = -1, kv_len = -1, w_seq = -1, w_tok0 = -1,
      num_work = -1, out_rows = -1, state_slot = -1, verify = -1, sample = -1, out_idx = -1, next_tok = -1;
  // capacities (elements) checked before anything is written
  int max_tokens = 0, max_seqs = 0, max_work = 0, max_out = 0;
};

struct StageOut {
  int T = 0, S = 0, work = 0, n_out = 0;
};

// K: speculative drafts per verify (0 = off); tpb: query tokens per attention work item.
// pad_rows: rows of each padding sequence (B - items); -1 = K + 1 under speculation, else 1
StageOut stage_step(KvManager& kv, const std::vector<StageItem>& items, int B, int K, int tpb, int page_size,
                    int dummy_page, int dummy_slot, const MetaLayout& L, int32_t* meta, int32_t* bt, int bt_ld,
                    int pad_rows = -1);

}  // namespace rkt_rt
