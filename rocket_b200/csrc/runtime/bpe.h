// Byte-level BPE merge core (host side, C++).
//
// Symbols are raw byte strings.  encode_piece() splits one pre-tokenized piece
// into single bytes and applies merges in rank order (lowest rank first, the
// leftmost occurrence first among equal ranks), using a heap of candidate
// pairs over a doubly linked symbol list, so long pieces cost O(n log n).
// Pre-tokenization (the Split regex with Unicode classes) and special-token
// splitting happen in Python; this is the hot loop.
//
// Behavioural counterpart of the reference's Tokenizer::encode_piece
// (engines/glm5-moe-nvfp4-2b/src/tokenizer.cc:248; GPT-2 byte alphabet,
// `ignore_merges`); the data structures here are this build's own.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace rkt_rt {

class BpeModel {
 public:
  // vocab: byte string -> id; merges: (left, right) byte strings in rank order.
  BpeModel(const std::vector<std::pair<std::string, int32_t>>& vocab,
           const std::vector<std::pair<std::string, std::string>>& merges, bool ignore_merges);
  std::vector<int32_t> encode_piece(const std::string& piece);
  std::vector<int32_t> encode_pieces(const std::vector<std::string>& pieces);
  std::string decode(const std::vector<int32_t>& ids) const;
  int32_t token_id(const std::string& bytes) const;  // -1 if absent
  size_t vocab_size() const { return id_to_bytes_.size(); }
  size_t num_merges() const { return ranks_.size(); }

 private:
  struct PairHash {
    size_t operator()(const std::pair<int32_t, int32_t>& p) const {
      return std::hash<uint64_t>()(((uint64_t)(uint32_t)p.first << 32) | (uint32_t)p.second);
    }
  };
  std::unordered_map<std::string, int32_t> vocab_;
  std::vector<std::string> id_to_bytes_;
  // merge of symbol ids (a, b) -> (rank, merged id)
  std::unordered_map<std::pair<int32_t, int32_t>, std::pair<int32_t, int32_t>, PairHash> ranks_;
  int32_t byte_id_[256];
  bool ignore_merges_;
  std::unordered_map<std::string, std::vector<int32_t>> cache_;
};

}  // namespace rkt_rt
