#include "stager.h"

#include <stdexcept>

namespace rkt_rt {

StageOut stage_step(KvManager& kv, const std::vector<StageItem>& items, int B, int K, int tpb, int page_size,
                    int dummy_page, int dummy_slot, const MetaLayout& L, int32_t* meta, int32_t* bt, int bt_ld,
                    int pad_rows) {
  const int n = (int)items.size();
  if (pad_rows < 0) pad_rows = K ? K + 1 : 1;  // rows of a padding sequence: this step's verify width
  if (pad_rows < 1 || (!K && pad_rows != 1)) throw std::invalid_argument("stage_step: pad_rows");
  if (B < n) throw std::invalid_argument("stage_step: bucket smaller than the batch");
  if (tpb < 1) throw std::invalid_argument("stage_step: tpb < 1");
  if (K && (L.verify < 0 || L.sample < 0 || L.out_idx < 0 || L.next_tok < 0))
    throw std::invalid_argument("stage_step: speculative fields missing from the layout");
  {
    // capacities first: nothing is written (and no KV slot reserved) for a step that does not fit
    const int rows_pad = pad_rows;
    long T = 0, W = 0, O = 0;
    for (const StageItem& s : items) {
      const int k = (int)s.tokens.size();
      T += k;
      W += (k + tpb - 1) / tpb;
      O += (K && s.verify) ? k : (s.sample ? 1 : 0);
    }
    T += (long)(B - n) * rows_pad;
    W += (long)(B - n) * ((rows_pad + tpb - 1) / tpb);
    O += (long)(B - n) * rows_pad;
    if (T > L.max_tokens || B > L.max_seqs || W > L.max_work || O > L.max_out)
      throw std::length_error("stage_step: step exceeds the metadata buffers");
  }
  int32_t* ids = meta + L.ids;
  int32_t* pos = meta + L.pos;
  int32_t* slots = meta + L.slots;
  int32_t* qs = meta + L.q_start;
  int32_t* ql = meta + L.q_len;
  int32_t* kl = meta + L.kv_len;
  int32_t* ws = meta + L.w_seq;
  int32_t* wt = meta + L.w_tok0;
  int32_t* orow = meta + L.out_rows;
  int32_t* sslot = meta + L.state_slot;
  int32_t* ver = K ? meta + L.verify : nullptr;
  int32_t* smp = K ? meta + L.sample : nullptr;
  int32_t* oidx = K ? meta + L.out_idx : nullptr;
  int32_t* ntok = K ? meta + L.next_tok : nullptr;
  int t = 0, w = 0, n_out = 0;
  std::vector<int64_t> seq_ids;
  seq_ids.reserve(n);
  std::vector<int32_t> toks;
  for (int i = 0; i < n; ++i) {
    const StageItem& s = items[i];
    const int k = (int)s.tokens.size();
    toks.assign(s.tokens.begin(), s.tokens.end());
    toks.resize(k + s.reserve, 0);
    const std::vector<int32_t> sl = kv.append(s.rid, toks);
    for (int j = 0; j < k; ++j) {
      ids[t + j] = s.tokens[j];
      pos[t + j] = s.start + j;
      slots[t + j] = sl[j];
    }
    qs[i] = t;
    ql[i] = k;
    kl[i] = s.start + k;
    sslot[i] = s.state_slot;
    for (int t0 = 0; t0 < k; t0 += tpb) {
      ws[w] = i;
      wt[w] = t0;
      ++w;
    }
    if (K) {
      ver[i] = s.verify;
      smp[i] = s.sample;
      for (int j = 0; j < k; ++j) oidx[t + j] = -1;
      if (s.verify) {
        for (int j = 0; j < k; ++j) {
          orow[n_out + j] = t + j;
          oidx[t + j] = n_out + j;
          ntok[t + j] = -1;
        }
        n_out += k;
      } else {
        // prefill rows: the next prompt token; the last prompt row takes the sampled token
        const int nn = (int)s.next_prompt.size() < k ? (int)s.next_prompt.size() : k;
        for (int j = 0; j < nn; ++j) ntok[t + j] = s.next_prompt[j];
        for (int j = nn; j < k; ++j) ntok[t + j] = -1;
        if (s.sample) {
          orow[n_out] = t + k - 1;
          oidx[t + k - 1] = n_out;
          ++n_out;
        }
      }
    } else if (s.sample) {
      orow[n_out] = t + k - 1;
      ++n_out;
    }
    seq_ids.push_back(s.rid);
    t += k;
  }
  if (n) kv.block_table(seq_ids, bt, bt_ld);
  // pad a decode batch to its bucket with dummy sequences on the scratch page
  const int rows = pad_rows;
  for (int i = n; i < B; ++i) {
    for (int j = 0; j < rows; ++j) {
      ids[t + j] = 0;
      pos[t + j] = j;
      slots[t + j] = dummy_page * page_size + j;
    }
    qs[i] = t;
    ql[i] = rows;
    kl[i] = rows;
    sslot[i] = dummy_slot;
    for (int t0 = 0; t0 < rows; t0 += tpb) {
      ws[w] = i;
      wt[w] = t0;
      ++w;
    }
    for (int j = 0; j < rows; ++j) orow[n_out + j] = t + j;
    if (K) {
      ver[i] = 1;
      smp[i] = 1;
      for (int j = 0; j < rows; ++j) {
        oidx[t + j] = n_out + j;
        ntok[t + j] = -1;
      }
    }
    n_out += rows;
    bt[(size_t)i * bt_ld] = dummy_page;
    t += rows;
  }
  meta[L.num_work] = w;
  return StageOut{t, B, w, n_out};
}

}  // namespace rkt_rt
